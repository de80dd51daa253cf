"""torch.library operators with the reference schemas, implemented over the C ABI.

Each op keeps the schema of the reference's kernel-builder binding, e.g.
``cohere2_moe_experts(Tensor x, Tensor gate_up_proj, Tensor down_proj, Tensor indices,
Tensor weights, int topk) -> Tensor`` (src/kops/cohere2_moe_experts/torch-ext/torch_binding.cpp:7-12),
registered here under the ``cernels_b200`` namespace for CUDA (and Meta, for shape
propagation). The CUDA implementation runs on the current stream of x's device, takes
scratch from torch's caching allocator and launches through ctypes; it never
synchronises, so calls can be captured in CUDA graphs.

Errors mirror the reference's TORCH_CHECKs: wrong dtype, device, rank or contiguity
raise RuntimeError before any launch; expert ids outside [0, E) are skipped silently
(src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:35,49-50).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_NS = "cernels_b200"
_defined = False
_LIBS: list = []  # keep torch.library.Library objects alive

SCHEMA_PLAIN = "(Tensor x, Tensor gate_up_proj, Tensor down_proj, Tensor indices, Tensor weights, int topk) -> Tensor"
SCHEMA_GPTOSS = (
    "(Tensor x, Tensor gate_up_proj, Tensor gate_up_bias, Tensor down_proj, Tensor down_bias, "
    "Tensor indices, Tensor weights, int topk) -> Tensor"
)

# Reference op name -> (schema, layout, decode)
OPS = {
    "cohere2_moe_experts": (SCHEMA_PLAIN, _lib.LAYOUT_LINEAR, False),
    "cohere2_moe_experts_decode": (SCHEMA_PLAIN, _lib.LAYOUT_LINEAR, True),
    "deepseek_ocr2_moe_experts": (SCHEMA_PLAIN, _lib.LAYOUT_LINEAR, False),
    "deepseek_ocr2_moe_experts_decode": (SCHEMA_PLAIN, _lib.LAYOUT_LINEAR, True),
    "qwen3_next_moe_experts": (SCHEMA_PLAIN, _lib.LAYOUT_LINEAR, False),
    "qwen3_next_moe_experts_decode": (SCHEMA_PLAIN, _lib.LAYOUT_LINEAR, True),
    "gpt_oss_moe_experts": (SCHEMA_GPTOSS, _lib.LAYOUT_GPTOSS, False),
    "gpt_oss_moe_experts_decode": (SCHEMA_GPTOSS, _lib.LAYOUT_GPTOSS, True),
}

DECODE_MAX_PAIRS = 1024


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def shape_of(x: torch.Tensor, gate_up_proj: torch.Tensor, down_proj: torch.Tensor, topk: int, layout: int) -> _lib.MoeShape:
    T, H = x.shape
    E = gate_up_proj.shape[0]
    if layout == _lib.LAYOUT_LINEAR:
        F = gate_up_proj.shape[1] // 2
    else:
        F = gate_up_proj.shape[2] // 2
    return _lib.MoeShape(int(T), int(H), int(E), int(F), int(topk), int(layout))


def validate(x, gate_up_proj, down_proj, indices, weights, topk, layout, b1=None, b2=None) -> None:
    """The reference's TORCH_CHECKs plus the dtype / rank checks its kernels assume."""
    tensors = [("x", x), ("gate_up_proj", gate_up_proj), ("down_proj", down_proj), ("indices", indices),
               ("weights", weights)]
    if b1 is not None:
        tensors.append(("gate_up_bias", b1))
    if b2 is not None:
        tensors.append(("down_bias", b2))
    for name, t in tensors:
        _check(t.is_cuda, f"{name} must be a CUDA tensor")
        _check(t.device == x.device, f"{name} must be on {x.device}")
        _check(t.is_contiguous(), f"{name} must be contiguous")
    _check(x.dim() == 2 and x.dtype == torch.bfloat16, "x must be [T, H] bf16")
    _check(gate_up_proj.dim() == 3 and gate_up_proj.dtype == torch.bfloat16, "gate_up_proj must be 3-D bf16")
    _check(down_proj.dim() == 3 and down_proj.dtype == torch.bfloat16, "down_proj must be 3-D bf16")
    _check(indices.dtype == torch.int32, "indices must be int32")
    _check(weights.dtype == torch.float32, "weights must be fp32")
    T, H = x.shape
    E = gate_up_proj.shape[0]
    _check(indices.dim() == 2 and tuple(indices.shape) == (T, topk), "indices must be [T, topk]")
    _check(weights.dim() == 2 and tuple(weights.shape) == (T, topk), "weights must be [T, topk]")
    if layout == _lib.LAYOUT_LINEAR:
        _check(gate_up_proj.shape[2] == H and gate_up_proj.shape[1] % 2 == 0, "gate_up_proj must be [E, 2F, H]")
        F = gate_up_proj.shape[1] // 2
        _check(tuple(down_proj.shape) == (E, H, F), "down_proj must be [E, H, F]")
    else:
        _check(gate_up_proj.shape[1] == H and gate_up_proj.shape[2] % 2 == 0, "gate_up_proj must be [E, H, 2F]")
        F = gate_up_proj.shape[2] // 2
        _check(tuple(down_proj.shape) == (E, F, H), "down_proj must be [E, F, H]")
        if b1 is not None:
            _check(b1.dtype == torch.float32 and tuple(b1.shape) == (E, 2 * F), "gate_up_bias must be [E, 2F] fp32")
        if b2 is not None:
            _check(b2.dtype == torch.float32 and tuple(b2.shape) == (E, H), "down_bias must be [E, H] fp32")
    _check(H % 8 == 0 and F % 8 == 0, "H and F must be multiples of 8")


def run_experts(x, gate_up_proj, down_proj, indices, weights, topk, layout, decode, b1=None, b2=None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Validates, allocates output + workspace, and calls the C ABI on x's current stream."""
    validate(x, gate_up_proj, down_proj, indices, weights, topk, layout, b1, b2)
    shape = shape_of(x, gate_up_proj, down_proj, topk, layout)
    if decode and shape.tokens * shape.topk > DECODE_MAX_PAIRS:
        decode = False  # the grouped-GEMM path covers any size, on the GPU
    if out is None:
        out = torch.empty_like(x)
    if shape.tokens == 0:
        return out
    lib = _lib.load()
    ws_bytes = _lib.workspace_bytes(shape, decode)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    fn = lib.cernels_moe_experts_decode if decode else lib.cernels_moe_experts
    with torch.cuda.device(x.device):
        rc = fn(ctypes.byref(shape), x.data_ptr(), gate_up_proj.data_ptr(), _ptr(b1), down_proj.data_ptr(), _ptr(b2),
                indices.data_ptr(), weights.data_ptr(), out.data_ptr(), ws.data_ptr(), ws_bytes,
                _stream_handle(x.device))
    _lib.check(rc, "cernels_moe_experts_decode" if decode else "cernels_moe_experts")
    return out


def _make_impl(layout: int, decode: bool, has_bias: bool):
    if has_bias:
        def impl(x, gate_up_proj, gate_up_bias, down_proj, down_bias, indices, weights, topk):
            return run_experts(x, gate_up_proj, down_proj, indices, weights, topk, layout, decode,
                               gate_up_bias, down_bias)
    else:
        def impl(x, gate_up_proj, down_proj, indices, weights, topk):
            return run_experts(x, gate_up_proj, down_proj, indices, weights, topk, layout, decode)
    return impl


def _meta_impl(has_bias: bool):
    if has_bias:
        def meta(x, gate_up_proj, gate_up_bias, down_proj, down_bias, indices, weights, topk):
            return torch.empty_like(x)
    else:
        def meta(x, gate_up_proj, down_proj, indices, weights, topk):
            return torch.empty_like(x)
    return meta


def register() -> None:
    """Defines the ``cernels_b200::*`` operators (idempotent)."""
    global _defined
    if _defined:
        return
    lib_def = torch.library.Library(_NS, "DEF")
    lib_cuda = torch.library.Library(_NS, "IMPL", "CUDA")
    lib_meta = torch.library.Library(_NS, "IMPL", "Meta")
    for name, (schema, layout, decode) in OPS.items():
        has_bias = schema is SCHEMA_GPTOSS
        lib_def.define(name + schema)
        lib_cuda.impl(name, _make_impl(layout, decode, has_bias))
        lib_meta.impl(name, _meta_impl(has_bias))
    _LIBS.extend([lib_def, lib_cuda, lib_meta])
    _defined = True


register()
ops = getattr(torch.ops, _NS)


# Python re-exports with the reference's function names
# (src/kops/cohere2_moe_experts/torch-ext/cohere2_moe_experts/__init__.py:1-12).
def cohere2_moe_experts(x, gate_up_proj, down_proj, indices, weights, topk):
    return ops.cohere2_moe_experts(x, gate_up_proj, down_proj, indices, weights, topk)


def cohere2_moe_experts_decode(x, gate_up_proj, down_proj, indices, weights, topk):
    return ops.cohere2_moe_experts_decode(x, gate_up_proj, down_proj, indices, weights, topk)


def deepseek_ocr2_moe_experts(x, gate_up_proj, down_proj, indices, weights, topk):
    return ops.deepseek_ocr2_moe_experts(x, gate_up_proj, down_proj, indices, weights, topk)


def deepseek_ocr2_moe_experts_decode(x, gate_up_proj, down_proj, indices, weights, topk):
    return ops.deepseek_ocr2_moe_experts_decode(x, gate_up_proj, down_proj, indices, weights, topk)


def qwen3_next_moe_experts(x, gate_up_proj, down_proj, indices, weights, topk):
    return ops.qwen3_next_moe_experts(x, gate_up_proj, down_proj, indices, weights, topk)


def qwen3_next_moe_experts_decode(x, gate_up_proj, down_proj, indices, weights, topk):
    return ops.qwen3_next_moe_experts_decode(x, gate_up_proj, down_proj, indices, weights, topk)


def gpt_oss_moe_experts(x, gate_up_proj, gate_up_bias, down_proj, down_bias, indices, weights, topk):
    return ops.gpt_oss_moe_experts(x, gate_up_proj, gate_up_bias, down_proj, down_bias, indices, weights, topk)


def gpt_oss_moe_experts_decode(x, gate_up_proj, gate_up_bias, down_proj, down_bias, indices, weights, topk):
    return ops.gpt_oss_moe_experts_decode(x, gate_up_proj, gate_up_bias, down_proj, down_bias, indices, weights, topk)


def run_experts_shared(x, gate_up_proj, down_proj, shared_gate_up, shared_down, indices, weights, topk):
    """Routed experts (LINEAR layout) + one always-on shared expert in the same launches.
    indices / weights: [T, topk + 1], last column = (E, shared gate weight)."""
    for name, t in (("x", x), ("gate_up_proj", gate_up_proj), ("down_proj", down_proj), ("indices", indices),
                    ("weights", weights), ("shared_gate_up", shared_gate_up), ("shared_down", shared_down)):
        _check(t.is_cuda and t.device == x.device and t.is_contiguous(), f"{name} must be a contiguous CUDA tensor on x's device")
    _check(x.dtype == torch.bfloat16 and x.dim() == 2, "x must be [T, H] bf16")
    _check(indices.dtype == torch.int32 and weights.dtype == torch.float32, "indices int32, weights fp32")
    _check(tuple(indices.shape) == (x.shape[0], topk + 1) and tuple(weights.shape) == (x.shape[0], topk + 1),
           "indices / weights must be [T, topk + 1]")
    E, F = gate_up_proj.shape[0], gate_up_proj.shape[1] // 2
    _check(tuple(shared_gate_up.shape) == (1, 2 * F, x.shape[1]) and tuple(shared_down.shape) == (1, x.shape[1], F),
           "shared expert weights must be [1, 2F, H] and [1, H, F]")
    out = torch.empty_like(x)
    if x.shape[0] == 0:
        return out
    shape = shape_of(x, gate_up_proj, down_proj, topk, _lib.LAYOUT_LINEAR)
    ws_shape = _lib.MoeShape(shape.tokens, shape.hidden, shape.experts + 1, shape.intermediate, shape.topk + 1,
                             shape.layout)
    ws_bytes = _lib.workspace_bytes(ws_shape, False)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.load().cernels_moe_experts_shared(
            ctypes.byref(shape), x.data_ptr(), gate_up_proj.data_ptr(), down_proj.data_ptr(), shared_gate_up.data_ptr(),
            shared_down.data_ptr(), indices.data_ptr(), weights.data_ptr(), out.data_ptr(), ws.data_ptr(), ws_bytes,
            _stream_handle(x.device))
    _lib.check(rc, "cernels_moe_experts_shared")
    return out


# ---------------------------------------------------------------- stage entry points
class RouteBuffers:
    """Output and scratch tensors of `route`, kept between calls of the same shape (a caller that
    routes every step, like the expert-parallel forward, then allocates nothing per step). The
    results of one call are overwritten by the next call on the same buffers."""

    def __init__(self):
        self._key = None
        self._bufs = None

    def get(self, T: int, k: int, experts: int, dev):
        key = (T, k, experts, dev)
        if key != self._key:
            shape = _lib.MoeShape(int(T), 8, int(experts), 8, int(k), _lib.LAYOUT_LINEAR)
            ws_bytes = _lib.workspace_bytes(shape, False)
            self._bufs = (shape, torch.empty(experts + 1, dtype=torch.int32, device=dev),
                          torch.zeros(T * k, dtype=torch.int32, device=dev),
                          torch.zeros(T * k, dtype=torch.float32, device=dev),
                          torch.empty(T * k, dtype=torch.int32, device=dev),
                          torch.empty(ws_bytes, dtype=torch.uint8, device=dev), ws_bytes)
            self._key = key
        return self._bufs


def route(indices: torch.Tensor, weights: torch.Tensor, experts: int, buffers: RouteBuffers | None = None):
    """Routing only: returns (offsets [E+1], perm_token [Tk], perm_weight [Tk], inv [Tk]).

    Stable in the flat index t*topk+j; ids outside [0, E) are skipped (inv = -1). With `buffers`
    the results live in (and are overwritten by the next call on) those buffers.
    """
    _check(indices.is_cuda and indices.dtype == torch.int32 and indices.is_contiguous() and indices.dim() == 2,
           "indices must be a contiguous [T, topk] int32 CUDA tensor")
    _check(weights.dtype == torch.float32 and weights.shape == indices.shape and weights.is_contiguous(),
           "weights must be contiguous fp32 [T, topk]")
    T, k = indices.shape
    dev = indices.device
    shape, offsets, perm_token, perm_weight, inv, ws, ws_bytes = (buffers or RouteBuffers()).get(T, k, experts, dev)
    with torch.cuda.device(dev):
        rc = _lib.load().cernels_moe_route(ctypes.byref(shape), indices.data_ptr(), weights.data_ptr(),
                                           offsets.data_ptr(), perm_token.data_ptr(), perm_weight.data_ptr(),
                                           inv.data_ptr(), ws.data_ptr(), ws_bytes, _stream_handle(dev))
    _lib.check(rc, "cernels_moe_route")
    return offsets, perm_token, perm_weight, inv


def grouped_experts(rows: torch.Tensor, group_counts: torch.Tensor, gate_up_proj: torch.Tensor,
                    down_proj: torch.Tensor, layout: int, b1: torch.Tensor | None = None,
                    b2: torch.Tensor | None = None) -> torch.Tensor:
    """Expert outputs (+ down bias, unweighted) for rows grouped into contiguous runs:
    run g has group_counts[g] rows and uses expert g % E of the weights."""
    _check(rows.is_cuda and rows.dtype == torch.bfloat16 and rows.is_contiguous() and rows.dim() == 2,
           "rows must be a contiguous [N, H] bf16 CUDA tensor")
    counts = group_counts.to(device=rows.device, dtype=torch.int32).contiguous()
    N, H = rows.shape
    E = gate_up_proj.shape[0]
    F = gate_up_proj.shape[1] // 2 if layout == _lib.LAYOUT_LINEAR else gate_up_proj.shape[2] // 2
    G = counts.numel()
    out = torch.empty_like(rows)
    if N == 0:
        return out
    shape = _lib.MoeShape(int(N), int(H), int(E), int(F), 1, int(layout))
    ws_shape = _lib.MoeShape(int(N), int(H), int(G), int(F), 1, int(layout))
    ws_bytes = _lib.workspace_bytes(ws_shape, False)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=rows.device)
    with torch.cuda.device(rows.device):
        rc = _lib.load().cernels_moe_grouped_experts(
            ctypes.byref(shape), G, counts.data_ptr(), rows.data_ptr(), gate_up_proj.data_ptr(), _ptr(b1),
            down_proj.data_ptr(), _ptr(b2), out.data_ptr(), ws.data_ptr(), ws_bytes, _stream_handle(rows.device))
    _lib.check(rc, "cernels_moe_grouped_experts")
    return out


ROUTER_TOPK_SOFTMAX = 0
ROUTER_SOFTMAX_TOPK = 1


def router_topk(logits: torch.Tensor, topk: int, mode: int, renorm: bool = False, shared_gate=False):
    """Top-k expert ids (int32) and fp32 routing weights from router logits [T, E] in one launch
    (see cernels_router_topk in include/cernels_b200.h). With shared_gate = E (the routed expert
    count), logits are [T, pad8(E + 1)] with column E a shared expert's gate: outputs get an
    (E, sigmoid(gate)) slot appended."""
    _check(logits.is_cuda and logits.dim() == 2 and logits.dtype in (torch.bfloat16, torch.float32),
           "logits must be a [T, E] bf16 or fp32 CUDA tensor")
    logits = logits.contiguous()
    T, E = logits.shape
    if shared_gate:  # [T, pad8(E + 1)]: E routed logits, the gate logit, zero padding
        E = int(shared_gate) if not isinstance(shared_gate, bool) else E - 1
        _check(logits.shape[1] == (E + 1 + 7) // 8 * 8, "shared-gate logits must have pad8(E + 1) columns")
    cols = topk + int(bool(shared_gate))
    idx = torch.empty(T, cols, dtype=torch.int32, device=logits.device)
    w = torch.empty(T, cols, dtype=torch.float32, device=logits.device)
    with torch.cuda.device(logits.device):
        rc = _lib.load().cernels_router_topk(logits.data_ptr(), int(logits.dtype == torch.bfloat16), T, E, int(topk),
                                             int(mode), int(bool(renorm)), int(bool(shared_gate)), idx.data_ptr(),
                                             w.data_ptr(), _stream_handle(logits.device))
    _lib.check(rc, "cernels_router_topk")
    return idx, w


def router(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, experts: int, topk: int, mode: int,
           renorm: bool = False, shared_gate: bool = False, return_logits: bool = False, out=None):
    """Fused router (cernels_router): logits = x weight^T (+ bias) on the tensor cores with the
    top-k / softmax tail in the same kernel; returns int32 ids and fp32 weights [T, topk (+1)]
    (and, with return_logits, the bf16 logits [T, weight.shape[0]] the selection used; only the
    first experts (+1) columns are written). weight: [rows >= experts (+1), H] bf16; with
    shared_gate, row `experts` is a shared expert's gate and an (experts, sigmoid(gate)) slot is
    appended to every token. out: (ids, weights) tensors of that shape to write into."""
    _check(x.is_cuda and x.dim() == 2 and x.dtype == torch.bfloat16, "x must be a [T, H] bf16 CUDA tensor")
    _check(weight.is_cuda and weight.dim() == 2 and weight.dtype == torch.bfloat16 and weight.shape[1] == x.shape[1],
           "router weight must be [rows, H] bf16")
    _check(bias is None or (bias.dtype == torch.bfloat16 and bias.numel() >= experts), "router bias must be bf16 [E]")
    x = x.contiguous()
    weight = weight.contiguous()
    bias = None if bias is None else bias.contiguous()
    T = x.shape[0]
    cols = topk + int(bool(shared_gate))
    if out is not None and tuple(out[0].shape) == (T, cols) and out[0].device == x.device:
        idx, w = out  # reused output buffers (overwritten)
    else:
        idx = torch.empty(T, cols, dtype=torch.int32, device=x.device)
        w = torch.empty(T, cols, dtype=torch.float32, device=x.device)
    logits = torch.zeros(T, weight.shape[0], dtype=torch.bfloat16, device=x.device) if return_logits else None
    with torch.cuda.device(x.device):
        rc = _lib.load().cernels_router(x.data_ptr(), T, x.shape[1], weight.data_ptr(), weight.shape[0], _ptr(bias),
                                        int(experts), int(topk), int(mode), int(bool(renorm)), int(bool(shared_gate)),
                                        idx.data_ptr(), w.data_ptr(), _ptr(logits), _stream_handle(x.device))
    _lib.check(rc, "cernels_router")
    return (idx, w, logits) if return_logits else (idx, w)


ROUTER_MAX_TOPK = 16


def gather_rows(x: torch.Tensor, perm_token: torch.Tensor, rows: int | None = None) -> torch.Tensor:
    """rows_out[i] = x[perm_token[i]] for i < rows (bf16 [rows, H])."""
    _check(x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.dim() == 2, "x must be [T, H] bf16")
    _check(perm_token.dtype == torch.int32 and perm_token.is_contiguous(), "perm_token must be int32")
    n = perm_token.numel() if rows is None else int(rows)
    out = torch.empty(n, x.shape[1], dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.load().cernels_moe_gather(x.data_ptr(), perm_token.data_ptr(), n, x.shape[1], out.data_ptr(),
                                            _stream_handle(x.device))
    _lib.check(rc, "cernels_moe_gather")
    return out


def combine_rows(rows: torch.Tensor, inv: torch.Tensor, weights: torch.Tensor, out: torch.Tensor | None = None):
    """out[t] = bf16(sum_j weights[t, j] * rows[inv[t*topk + j]]) in fp32, slot order."""
    T, k = weights.shape
    H = rows.shape[1]
    _check(rows.dtype == torch.bfloat16 and rows.is_contiguous(), "rows must be contiguous bf16")
    _check(inv.dtype == torch.int32 and inv.numel() == T * k, "inv must be int32 [T*topk]")
    _check(weights.dtype == torch.float32 and weights.is_contiguous(), "weights must be fp32")
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=rows.device)
    with torch.cuda.device(rows.device):
        rc = _lib.load().cernels_moe_combine(rows.data_ptr(), inv.data_ptr(), weights.data_ptr(), T, k, H,
                                             out.data_ptr(), _stream_handle(rows.device))
    _lib.check(rc, "cernels_moe_combine")
    return out
