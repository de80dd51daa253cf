"""Shared preparation for the loaders (the reference's per-call casts, cached where the
reference caches them: src/kops/registry/gpt_oss_moe_experts.py:14-26)."""

from __future__ import annotations

import torch


def routing_tensors(top_k_index: torch.Tensor, top_k_weights: torch.Tensor):
    """int64 -> int32 indices and any-float -> fp32 weights, contiguous
    (src/kops/registry/cohere2_moe_experts.py:25-26)."""
    idx = top_k_index if top_k_index.dtype == torch.int32 else top_k_index.to(torch.int32)
    w = top_k_weights if top_k_weights.dtype == torch.float32 else top_k_weights.float()
    return idx.contiguous(), w.contiguous()


def module_cache(mod: torch.nn.Module, key: str, stamp, build):
    """Per-module cache of static derived tensors. ``stamp`` is a tuple identifying the
    source tensors (storage pointers and versions); ``build()`` runs only when it changes."""
    cache = getattr(mod, "_cernels_cache", None)
    if cache is None:
        cache = {}
        mod._cernels_cache = cache
    hit = cache.get(key)
    if hit is not None and hit[1] == stamp:
        return hit[0]
    value = build()
    cache[key] = (value, stamp)
    return value
