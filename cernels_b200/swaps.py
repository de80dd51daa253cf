"""In-model swaps: replace the forward of every transformers experts module of a class with
this library's operators — the reference's swap point #2 (src/modeling/swaps.py).

As in the reference, the replacement is an instance attribute (``mod.forward``), so deleting it
("stock") restores the class method, and the forward picks the decode entry point at or below
DECODE_MAX_TOKENS tokens and the prefill entry point above (src/modeling/swaps.py:13,20-42).
The ops take no host synchronisation, so a swapped model can be captured in a CUDA graph.

SWAPS maps a model name to (apply(model, variant), variants), stock first.
"""

from __future__ import annotations

from typing import Callable

import torch

DECODE_MAX_TOKENS = 4  # at or below this many tokens the decode entry point handles the op


def _experts_fwd(mod, kernel: Callable | None, decode_kernel: Callable | None):
    def fwd(h, idx, w, _m=mod):
        op = decode_kernel if h.size(0) <= DECODE_MAX_TOKENS else kernel
        if op is None:  # this shape's entry point is not enabled in this variant
            return type(_m).forward(_m, h, idx, w)
        return op(h, idx, w, _m)

    return fwd


def swap_experts(model: torch.nn.Module, cls_name: str, kernel: Callable | None,
                 decode_kernel: Callable | None) -> int:
    """Sets (or, with both kernels None, restores) the forward of every `cls_name` instance.
    Returns the number of modules touched; raises when the model has none."""
    n = 0
    for mod in model.modules():
        if type(mod).__name__ != cls_name:
            continue
        n += 1
        if "forward" in vars(mod):
            del mod.forward
        if kernel is not None or decode_kernel is not None:
            mod.forward = _experts_fwd(mod, kernel, decode_kernel)
    if not n:
        raise RuntimeError(f"no {cls_name} modules found — wrong model for this swap")
    return n


# ---------------------------------------------------------------- per-family kernels
def _linear_kernels():
    from .registry import cohere2_moe_experts as c2

    return c2.kernel, c2.decode_kernel


def _gpt_oss_kernels():
    """GptOssExperts.forward(hidden, router_indices, routing_weights) with its biases."""
    from . import ops
    from .registry import gpt_oss_moe_experts as go

    def prefill(h, idx, w, mod):
        w1, b1, w2, b2 = go._weights(mod)
        with torch.no_grad():
            return ops.gpt_oss_moe_experts(h.contiguous(), w1, b1, w2, b2, idx.to(torch.int32).contiguous(),
                                           w.float().contiguous(), int(idx.size(1)))

    def decode(h, idx, w, mod):
        w1, b1, w2, b2 = go._weights(mod)
        with torch.no_grad():
            return ops.gpt_oss_moe_experts_decode(h.contiguous(), w1, b1, w2, b2, idx.to(torch.int32).contiguous(),
                                                  w.float().contiguous(), int(idx.size(1)))

    return prefill, decode


def _family(cls_name: str, kernels: Callable):
    def apply(model, variant: str):
        if variant == "stock":
            return swap_experts(model, cls_name, None, None)
        kernel, decode_kernel = kernels()
        return swap_experts(model, cls_name, kernel, decode_kernel if variant == "custom" else None)

    return apply


SWAPS = {
    # the reference's two models (their experts classes need transformers >= 5.10)
    "north_mini_code": (_family("Cohere2MoeExperts", _linear_kernels), ("stock", "custom_prefill", "custom")),
    "deepseek_ocr_2": (_family("DeepseekOcr2TextExperts", _linear_kernels), ("stock", "custom_prefill", "custom")),
    # experts classes of the installed transformers with the same contracts
    "deepseek_v2": (_family("DeepseekV2Experts", _linear_kernels), ("stock", "custom_prefill", "custom")),
    "qwen3_next": (_family("Qwen3NextExperts", _linear_kernels), ("stock", "custom_prefill", "custom")),
    "gpt_oss": (_family("GptOssExperts", _gpt_oss_kernels), ("stock", "custom_prefill", "custom")),
}
