"""CPU: the in-model swap logic (instance-level forward replacement, decode threshold, restore)."""

import pytest
import torch

from cernels_b200 import swaps


class DeepseekV2Experts(torch.nn.Module):  # name-matched stand-in for the transformers class
    def forward(self, h, idx, w):
        return "stock"


class Model(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.layers = torch.nn.ModuleList([DeepseekV2Experts(), torch.nn.Linear(2, 2), DeepseekV2Experts()])


def test_swap_dispatches_by_token_count_and_restores():
    m = Model()
    calls = []
    prefill = lambda h, i, w, mod: calls.append(("prefill", h.size(0))) or "prefill"  # noqa: E731
    decode = lambda h, i, w, mod: calls.append(("decode", h.size(0))) or "decode"  # noqa: E731
    assert swaps.swap_experts(m, "DeepseekV2Experts", prefill, decode) == 2
    e = m.layers[0]
    assert e(torch.zeros(4, 2), None, None) == "decode"
    assert e(torch.zeros(5, 2), None, None) == "prefill"
    assert calls == [("decode", 4), ("prefill", 5)]
    # prefill-only variant falls back to the class forward for decode shapes
    swaps.swap_experts(m, "DeepseekV2Experts", prefill, None)
    assert e(torch.zeros(1, 2), None, None) == "stock"
    # stock restores the class method
    swaps.swap_experts(m, "DeepseekV2Experts", None, None)
    assert "forward" not in vars(e)
    assert e(torch.zeros(9, 2), None, None) == "stock"


def test_swap_wrong_model_raises():
    with pytest.raises(RuntimeError, match="no GptOssExperts"):
        swaps.swap_experts(Model(), "GptOssExperts", lambda *a: None, None)


def test_swap_table_lists_stock_first():
    for name, (apply, variants) in swaps.SWAPS.items():
        assert variants[0] == "stock" and callable(apply)
    apply, _ = swaps.SWAPS["deepseek_v2"]
    m = Model()
    assert apply(m, "stock") == 2
