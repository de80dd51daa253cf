"""CPU: the C-ABI library loads, exports every function declared in include/*.h, and
rejects invalid arguments with the documented codes (no GPU work is issued)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from cernels_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(cernels_\w+)\s*\(", text, flags=re.M)
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.PROTOTYPES, f"{n} has no ctypes prototype"


def test_version_and_error_strings():
    lib = _lib.load()
    assert lib.cernels_version() >= 100
    for code in range(7):
        assert lib.cernels_error_string(code)
    assert lib.cernels_error_string(99) == b"unknown error"


def shape(T=8, H=64, E=4, F=32, k=2, layout=0):
    return _lib.MoeShape(T, H, E, F, k, layout)


def test_workspace_sizes_grow_with_tokens():
    a = _lib.workspace_bytes(shape(T=8), False)
    b = _lib.workspace_bytes(shape(T=800), False)
    assert 0 < a < b
    assert _lib.workspace_bytes(shape(T=8), True) > 0


def test_gptoss_decode_workspace_holds_k_split_slabs():
    """GPTOSS decode at a few tokens splits K across CTAs (gpt-oss-20b at T=1: 4 touched experts
    x 23 gate/up column blocks -> 7 splits; x 12 down column blocks -> 8 splits, capped); the
    workspace query covers the gate/up split sums and the down split slabs, and the LINEAR
    layout keeps one slab."""
    T, H, E, F, k = 1, 2880, 32, 2880, 4
    tk = T * k
    gptoss = _lib.workspace_bytes(_lib.MoeShape(T, H, E, F, k, _lib.LAYOUT_GPTOSS), True)
    linear = _lib.workspace_bytes(_lib.MoeShape(T, H, E, F, k, _lib.LAYOUT_LINEAR), True)
    assert linear >= tk * (F + H) * 4
    assert gptoss >= tk * F * 4 + 8 * tk * H * 4 + 7 * tk * 2 * F * 4
    assert gptoss - linear >= 7 * tk * H * 4 + 7 * tk * 2 * F * 4
    # 64 tokens: 32 groups x 23 gate/up blocks fill the machine (no gate/up split); 32 x 12 down
    # blocks do not (2 down splits): exactly one extra [T*topk, H] fp32 slab, up to alignment
    big = (64, H, E, F, k)
    extra = (_lib.workspace_bytes(_lib.MoeShape(*big, _lib.LAYOUT_GPTOSS), True)
             - _lib.workspace_bytes(_lib.MoeShape(*big, _lib.LAYOUT_LINEAR), True))
    assert 64 * k * H * 4 <= extra <= 64 * k * H * 4 + 1024


@pytest.mark.parametrize("bad,code", [
    (dict(H=60), 2), (dict(F=12), 2), (dict(E=0), 1), (dict(k=0), 1), (dict(T=-1), 1), (dict(layout=7), 1),
    (dict(E=4096), 5),
])
def test_invalid_shapes_rejected(bad, code):
    lib = _lib.load()
    s = shape(**bad)
    n = ctypes.c_size_t(0)
    assert lib.cernels_moe_workspace_bytes(ctypes.byref(s), 0, ctypes.byref(n)) == code


def test_null_and_workspace_errors_before_any_launch():
    lib = _lib.load()
    s = shape()
    # NULL inputs
    rc = lib.cernels_moe_experts(ctypes.byref(s), None, None, None, None, None, None, None, None, None, 0, None)
    assert rc == 6
    # workspace too small (non-null, aligned fake pointers; rejected before touching them)
    p = 1 << 20
    rc = lib.cernels_moe_experts(ctypes.byref(s), p, p, None, p, None, p, p, p, p, 16, None)
    assert rc == 3
    # misaligned x
    rc = lib.cernels_moe_experts(ctypes.byref(s), p + 2, p, None, p, None, p, p, p, p, 1 << 30, None)
    assert rc == 2
    # decode pair limit
    big = shape(T=600, k=2)
    rc = lib.cernels_moe_experts_decode(ctypes.byref(big), p, p, None, p, None, p, p, p, p, 1 << 40, None)
    assert rc == 5
    assert lib.cernels_moe_gather(p, p, 4, 12, p, None) == 2
    assert lib.cernels_moe_combine(p, p, p, 4, 0, 64, p, None) == 1


def test_empty_token_batch_is_a_noop():
    lib = _lib.load()
    s = shape(T=0)
    assert lib.cernels_moe_experts(ctypes.byref(s), None, None, None, None, None, None, None, None, None, 0, None) == 0


def test_torch_shim_rejects_cpu_tensors_like_torch_check():
    from cernels_b200 import ops
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    w1 = torch.zeros(2, 64, 64, dtype=torch.bfloat16)
    w2 = torch.zeros(2, 64, 32, dtype=torch.bfloat16)
    idx = torch.zeros(4, 1, dtype=torch.int32)
    w = torch.zeros(4, 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.run_experts(x, w1, w2, idx, w, 1, 0, False)


def test_torch_ops_registered_with_reference_schemas():
    from cernels_b200 import ops
    for name in ["cohere2_moe_experts", "cohere2_moe_experts_decode", "deepseek_ocr2_moe_experts",
                 "deepseek_ocr2_moe_experts_decode", "qwen3_next_moe_experts", "gpt_oss_moe_experts"]:
        schema = str(getattr(torch.ops.cernels_b200, name).default._schema)
        assert "int topk" in schema and schema.endswith("-> Tensor")
    # meta propagation works without a GPU
    x = torch.empty(5, 64, dtype=torch.bfloat16, device="meta")
    out = torch.ops.cernels_b200.cohere2_moe_experts(
        x, torch.empty(2, 64, 64, dtype=torch.bfloat16, device="meta"),
        torch.empty(2, 64, 32, dtype=torch.bfloat16, device="meta"),
        torch.empty(5, 1, dtype=torch.int32, device="meta"), torch.empty(5, 1, device="meta"), 1)
    assert out.shape == (5, 64)


def test_router_and_ep_argument_checks_before_any_launch():
    """cernels_router / cernels_ep_* reject bad arguments with the documented codes before touching
    the device (no GPU needed)."""
    lib = _lib.load()
    p = 1 << 20
    # topk above the fused kernel's 16, topk > E, rows < E (+ gate), bad mode, H not a multiple of 8
    assert lib.cernels_router(p, 8, 64, p, 32, None, 32, 17, 0, 0, 0, p, p, None, None) == 1
    assert lib.cernels_router(p, 8, 64, p, 4, None, 4, 5, 0, 0, 0, p, p, None, None) == 1
    assert lib.cernels_router(p, 8, 64, p, 32, None, 32, 4, 0, 0, 1, p, p, None, None) == 1
    assert lib.cernels_router(p, 8, 64, p, 32, None, 32, 4, 9, 0, 0, p, p, None, None) == 1
    assert lib.cernels_router(p, 8, 60, p, 32, None, 32, 4, 0, 0, 0, p, p, None, None) == 2
    # empty batch: nothing to do; NULL outputs
    assert lib.cernels_router(None, 0, 64, None, 32, None, 32, 4, 0, 0, 0, None, None, None, None) == 0
    assert lib.cernels_router(p, 8, 64, p, 32, None, 32, 4, 0, 0, 0, None, p, None, None) == 6
    # misaligned x
    assert lib.cernels_router(p + 4, 8, 64, p, 32, None, 32, 4, 0, 0, 0, p, p, None, None) == 2
    # EP: world / rank / sizes / shared rows
    ctx = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    assert lib.cernels_ep_create(0, 0, 64, 4, 16, 0, ctypes.byref(ctx), h) == 1
    assert lib.cernels_ep_create(2, 2, 64, 4, 16, 0, ctypes.byref(ctx), h) == 1
    assert lib.cernels_ep_create(0, 2, 60, 4, 16, 0, ctypes.byref(ctx), h) == 1
    assert lib.cernels_ep_create(0, 2, 64, 4, 16, -1, ctypes.byref(ctx), h) == 1
    assert lib.cernels_ep_create(0, 16, 64, 256, 16, 0, ctypes.byref(ctx), h) == 5  # 4096 experts
    # a NULL / unconnected context
    assert lib.cernels_ep_dispatch(None, p, p, p, 4, 0, 0, None) == 6
    assert lib.cernels_ep_combine(None, p, p, 4, 2, 0, p, 0, None) == 6
    # the wait limit is a plain setting
    assert lib.cernels_set_wait_limit_ns(1_000_000) == 0
    assert lib.cernels_set_wait_limit_ns(0) == 0
