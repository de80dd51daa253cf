"""gpt_oss_moe_experts loader — drop-in for src/kops/registry/gpt_oss_moe_experts.py.

``kernel(x, mlp)`` takes hidden states [B, S, H] and a GptOssMLP. The router runs in the
timed path, as in the reference loader: its linear, top-k and softmax in one tensor-core
kernel (cernels_router); the CUDA op does routing, both grouped GEMMs (with biases) and the
clamped interleaved SwiGLU. Weights are consumed in place in the transformers layout
([E, H, 2F] interleaved gate/up, [E, F, H]); only the fp32 bias casts are cached on the
module, as the reference does (its ``_kops_weights``).
"""

import torch

from .. import ops
from ._common import module_cache


def _weights(experts):
    gb, db = experts.gate_up_proj_bias, experts.down_proj_bias
    stamp = (gb.data_ptr(), gb._version, db.data_ptr(), db._version)
    b1, b2 = module_cache(experts, "bias_f32", stamp,
                          lambda: (gb.data.float().contiguous(), db.data.float().contiguous()))
    return experts.gate_up_proj.data.contiguous(), b1, experts.down_proj.data.contiguous(), b2


def route(xf, mlp, out=None):
    """transformers GptOssTopKRouter in one kernel (cernels_router): logits = x W^T + b on the
    tensor cores, rounded to bf16, top-k and the softmax over the k logits in its epilogue
    (int32 ids, fp32 weights)."""
    r = mlp.router
    k = int(r.top_k)
    if k > ops.ROUTER_MAX_TOPK:  # beyond the fused kernel's limit: linear, then the tail kernel
        logits = torch.nn.functional.linear(xf, r.weight, r.bias)
        return ops.router_topk(logits, k, ops.ROUTER_TOPK_SOFTMAX)
    return ops.router(xf, r.weight.data, None if r.bias is None else r.bias.data, int(r.weight.shape[0]), k,
                      ops.ROUTER_TOPK_SOFTMAX, out=out)


def kernel(x, mlp):
    if mlp is None:
        raise RuntimeError("mlp module not available (meta device)")
    bsz, seqlen, hidden = x.shape
    xf = x.reshape(-1, hidden).contiguous()
    with torch.no_grad():
        idx, w = route(xf, mlp)
        w1, b1, w2, b2 = _weights(mlp.experts)
        out = ops.gpt_oss_moe_experts(xf, w1, b1, w2, b2, idx, w, int(mlp.router.top_k))
    return out.reshape(bsz, seqlen, hidden)


def decode_kernel(x, mlp):
    if mlp is None:
        raise RuntimeError("mlp module not available (meta device)")
    bsz, seqlen, hidden = x.shape
    xf = x.reshape(-1, hidden).contiguous()
    with torch.no_grad():
        idx, w = route(xf, mlp)
        w1, b1, w2, b2 = _weights(mlp.experts)
        out = ops.gpt_oss_moe_experts_decode(xf, w1, b1, w2, b2, idx, w, int(mlp.router.top_k))
    return out.reshape(bsz, seqlen, hidden)
