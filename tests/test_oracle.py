"""CPU: pins the numpy oracle against the golden fixtures made from the reference's
transformers modules, and its routing against torch.sort(stable=True)."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests import golden_io


@pytest.mark.parametrize("name", golden_io.NAMES)
def test_oracle_matches_transformers_fp32(name):
    g = golden_io.load(name)
    layout = O.LAYOUT_GPTOSS if g["kind"] == "gpt_oss" else O.LAYOUT_LINEAR
    out = O.moe_experts(g["x"].float().numpy(), g["w1"].float().numpy(), g["w2"].float().numpy(),
                        g["indices"].numpy(), g["weights"].numpy(), layout,
                        g["b1"].numpy() if "b1" in g else None, g["b2"].numpy() if "b2" in g else None)
    if g["kind"] == "qwen3_next":
        out = out + O.shared_expert(g["x"].float().numpy(), g["shared_gate_proj"].float().numpy(),
                                    g["shared_up_proj"].float().numpy(), g["shared_down_proj"].float().numpy(),
                                    g["shared_gate"].float().numpy())
    # fp32 vs fp32 (different summation order only)
    assert O.rel_err(out, g["ref_fp32"].numpy()) < 1e-5
    # and the reference's own verify() tolerance against its bf16 eager output
    assert np.allclose(out, g["ref_bf16"].float().numpy(), atol=2e-2, rtol=2e-2)


def _torch_route(indices: torch.Tensor, E: int):
    flat = indices.reshape(-1).long()
    valid = (flat >= 0) & (flat < E)
    key = torch.where(valid, flat, torch.full_like(flat, E))
    order = torch.sort(key, stable=True).indices
    n = int(valid.sum())
    counts = torch.bincount(flat[valid], minlength=E)
    offsets = torch.zeros(E + 1, dtype=torch.long)
    offsets[1:] = torch.cumsum(counts, 0)
    return offsets, order[:n]


@pytest.mark.parametrize("T,k,E,seed", [(1, 1, 4, 0), (7, 3, 5, 1), (128, 8, 128, 2), (1000, 10, 512, 3),
                                        (333, 6, 64, 4)])
def test_route_matches_stable_sort(T, k, E, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(-1, E + 1, (T, k), generator=g)  # includes invalid ids -1 and E
    offsets, order, inv = O.route(idx.numpy(), E)
    t_off, t_order = _torch_route(idx, E)
    assert np.array_equal(offsets, t_off.numpy())
    assert np.array_equal(order, t_order.numpy())
    flat = idx.reshape(-1).numpy()
    for i in range(flat.shape[0]):
        if 0 <= flat[i] < E:
            assert order[inv[i]] == i
        else:
            assert inv[i] == -1


def test_route_expert_sets_match_eager_loop():
    """Per-expert token sets equal the transformers eager loop's torch.where(mask[e])."""
    g = torch.Generator().manual_seed(5)
    T, k, E = 50, 4, 9
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    offsets, order, _ = O.route(idx.numpy(), E)
    mask = torch.nn.functional.one_hot(idx, num_classes=E).permute(2, 1, 0)
    for e in range(E):
        _, token_idx = torch.where(mask[e])
        ours = order[offsets[e]:offsets[e + 1]] // k
        assert sorted(token_idx.tolist()) == sorted(ours.tolist())


@pytest.mark.parametrize("name,mode,renorm", [("gpt_oss_small", 0, False), ("qwen3_next_small", 1, True)])
def test_router_tail_oracle_matches_transformers_router(name, mode, renorm):
    """The router-tail restatement reproduces the transformers routers' selections and weights
    (logits recomputed with the same bf16 linear the module ran)."""
    g = golden_io.load(name)
    x, W = g["x"], g["router_w"]
    logits = torch.nn.functional.linear(x, W, g["router_b"] if "router_b" in g else None).float().numpy()
    k = g["indices"].shape[1]
    idx, w = O.router_tail(logits, k, mode, renorm)
    ref_idx = g["indices"].numpy()
    # same expert sets per token (transformers' top-k order among equal values is unspecified)
    assert all(set(a) == set(b) for a, b in zip(idx.tolist(), ref_idx.tolist()))
    ref_w = g["weights"].numpy()
    for t in range(idx.shape[0]):
        mine = dict(zip(idx[t].tolist(), w[t].tolist()))
        theirs = dict(zip(ref_idx[t].tolist(), ref_w[t].tolist()))
        for e, v in theirs.items():
            assert abs(mine[e] - v) <= 1e-2 * max(1.0, abs(v))
