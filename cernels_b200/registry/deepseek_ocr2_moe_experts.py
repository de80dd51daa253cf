"""deepseek_ocr2_moe_experts loader — drop-in for src/kops/registry/deepseek_ocr2_moe_experts.py.

Receives what the transformers experts module's forward receives — flat hidden states,
top_k_index, top_k_weights — plus the experts module for weight storage. Routing,
gather, both grouped GEMMs, the SwiGLU, the router-weight scale and the combine run in
the CUDA op. Weights are consumed in place in the F.linear layout: gate_up_proj [E, 2F, H],
down_proj [E, H, F].
"""

import torch

from .. import ops
from ._common import routing_tensors


def kernel(x, top_k_index, top_k_weights, experts):
    if experts is None:
        raise RuntimeError("experts module not available (meta device)")
    with torch.no_grad():
        idx, w = routing_tensors(top_k_index, top_k_weights)
        return ops.deepseek_ocr2_moe_experts(x.contiguous(), experts.gate_up_proj.data.contiguous(),
                                      experts.down_proj.data.contiguous(), idx, w, int(top_k_index.size(1)))


def decode_kernel(x, top_k_index, top_k_weights, experts):
    """Fused gather-GEMV entry point for decode (a few tokens); same contract."""
    if experts is None:
        raise RuntimeError("experts module not available (meta device)")
    with torch.no_grad():
        idx, w = routing_tensors(top_k_index, top_k_weights)
        return ops.deepseek_ocr2_moe_experts_decode(x.contiguous(), experts.gate_up_proj.data.contiguous(),
                                             experts.down_proj.data.contiguous(), idx, w,
                                             int(top_k_index.size(1)))
