"""qwen3_next_moe_experts loader — drop-in for src/kops/registry/qwen3_next_moe_experts.py.

``kernel(x, block)`` takes the raw hidden states [B, S, H] and a
Qwen3NextSparseMoeBlock. As in the reference loader, the router runs in the timed path:
its linear, softmax, top-k and renorm in one tensor-core kernel (cernels_router); the routed
experts run in the CUDA op; the always-on shared expert ``sigmoid(shared_expert_gate(x)) *
shared_expert(x)`` runs through the same CUDA grouped-GEMM path as a one-expert,
one-slot problem whose router weight is the sigmoid gate (its gate/up weights are
concatenated once into the [1, 2Fs, H] layout and cached on the block). When the shared
intermediate size equals the routed one (Qwen3-Next: 512), ``kernel`` instead folds the shared
expert into the routed call: one router kernel over [W_router; g_shared] that appends a
(E, sigmoid(gate)) slot to every token, and the shared expert as an always-on
group of the same grouped GEMMs (cernels_moe_experts_shared).
"""

import os

import torch

from .. import ops
from ._common import module_cache


def _shared_weights(block):
    se = block.shared_expert

    g, u, d = se.gate_proj.weight, se.up_proj.weight, se.down_proj.weight
    stamp = (g.data_ptr(), g._version, u.data_ptr(), u._version, d.data_ptr(), d._version)

    def build():
        w1 = torch.cat([g.data, u.data], dim=0).unsqueeze(0).contiguous()  # [1, 2Fs, H]
        w2 = d.data.unsqueeze(0).contiguous()                               # [1, H, Fs]
        return w1, w2

    return module_cache(block, "shared", stamp, build)


def shared_expert(xf: torch.Tensor, block) -> torch.Tensor:
    """sigmoid(x @ g^T) * shared_mlp(x) via the CUDA op (one expert, topk = 1)."""
    w1, w2 = _shared_weights(block)
    T = xf.shape[0]
    gate = torch.sigmoid(torch.nn.functional.linear(xf, block.shared_expert_gate.weight).float()).contiguous()
    idx = torch.zeros(T, 1, dtype=torch.int32, device=xf.device)
    return ops.qwen3_next_moe_experts(xf, w1, w2, idx, gate, 1)


def route(xf, block):
    """transformers Qwen3NextTopKRouter in one kernel (cernels_router): logits = x W^T on the
    tensor cores, rounded to bf16, then fp32 softmax, top-k and renormalisation in its epilogue
    (int32 ids, fp32 weights)."""
    k = int(block.gate.top_k)
    renorm = bool(block.gate.norm_topk_prob)
    if k > ops.ROUTER_MAX_TOPK:
        logits = torch.nn.functional.linear(xf, block.gate.weight)
        return ops.router_topk(logits, k, ops.ROUTER_SOFTMAX_TOPK, renorm)
    return ops.router(xf, block.gate.weight.data, None, int(block.gate.weight.shape[0]), k, ops.ROUTER_SOFTMAX_TOPK,
                      renorm)


def _router_and_gate(block):
    """[pad8(E + 1), H]: router weight, the shared-expert gate row, zero rows up to a multiple of
    8 (so the router GEMM's output rows stay 16-byte aligned). Cached on the block."""
    g, sg = block.gate.weight, block.shared_expert_gate.weight
    stamp = (g.data_ptr(), g._version, sg.data_ptr(), sg._version)

    def build():
        E = g.shape[0]
        rows = (E + 1 + 7) // 8 * 8
        w = torch.zeros(rows, g.shape[1], dtype=g.dtype, device=g.device)
        w[:E] = g.data
        w[E] = sg.data[0]
        return w

    return module_cache(block, "router_gate", stamp, build)


FUSE_SHARED = os.environ.get("CERNELS_QWEN3_FUSE_SHARED", "1") != "0"


def fused_shared_supported(block) -> bool:
    se = block.shared_expert
    return FUSE_SHARED and se.gate_proj.weight.shape[0] == block.experts.gate_up_proj.shape[1] // 2


def _fused_route(xf, block, return_logits=False, out=None):
    """Router + shared-expert gate in one kernel: ids / weights [T, k + 1], the last column
    (E, sigmoid(gate)); with return_logits also the bf16 logits [T, pad8(E + 1)]."""
    E = int(block.experts.gate_up_proj.shape[0])
    k = int(block.gate.top_k)
    renorm = bool(block.gate.norm_topk_prob)
    wg = _router_and_gate(block)
    if k > ops.ROUTER_MAX_TOPK:
        logits = torch.nn.functional.linear(xf, wg)
        idx, w = ops.router_topk(logits, k, ops.ROUTER_SOFTMAX_TOPK, renorm, shared_gate=E)
        return (logits, idx, w) if return_logits else (idx, w)
    r = ops.router(xf, wg, None, E, k, ops.ROUTER_SOFTMAX_TOPK, renorm, shared_gate=True, return_logits=return_logits,
                   out=out)
    return (r[2], r[0], r[1]) if return_logits else r


def route_debug(xf, block):
    """The routing kernel() uses when the shared expert is fused: returns (logits [T, pad8(E + 1)],
    ids [T, k + 1] int32, weights [T, k + 1] fp32), the last column being (E, sigmoid(gate))."""
    with torch.no_grad():
        return _fused_route(xf, block, return_logits=True)


def kernel(x, block):
    if block is None:
        raise RuntimeError("block module not available (meta device)")
    bsz, seqlen, hidden = x.shape
    xf = x.reshape(-1, hidden).contiguous()
    with torch.no_grad():
        e = block.experts
        k = int(block.gate.top_k)
        if fused_shared_supported(block):
            # router + shared gate in one GEMM, top-k + renorm + sigmoid gate in one kernel, and
            # the shared expert as an always-on group of the same grouped GEMMs
            idx, w = _fused_route(xf, block)
            sw1, sw2 = _shared_weights(block)
            out = ops.run_experts_shared(xf, e.gate_up_proj.data.contiguous(), e.down_proj.data.contiguous(), sw1,
                                         sw2, idx, w, k)
        else:
            idx, w = route(xf, block)
            routed = ops.qwen3_next_moe_experts(xf, e.gate_up_proj.data.contiguous(), e.down_proj.data.contiguous(),
                                                idx, w, k)
            out = routed + shared_expert(xf, block)
    return out.reshape(bsz, seqlen, hidden)


def decode_kernel(x, block):
    """Decode-shape variant (a few tokens): routed experts through the gather-GEMV path."""
    if block is None:
        raise RuntimeError("block module not available (meta device)")
    bsz, seqlen, hidden = x.shape
    xf = x.reshape(-1, hidden).contiguous()
    with torch.no_grad():
        idx, w = route(xf, block)
        e = block.experts
        routed = ops.qwen3_next_moe_experts_decode(xf, e.gate_up_proj.data.contiguous(),
                                                   e.down_proj.data.contiguous(), idx, w, int(block.gate.top_k))
        out = routed + shared_expert(xf, block)
    return out.reshape(bsz, seqlen, hidden)
