"""GPU: the no-allocation decode entry point (cernels_moe_experts_decode_noalloc).

It exists for callers that cannot allocate device memory themselves — runtimes that
forbid cudaMalloc or plan every device byte at start-up — and takes its scratch from a
static device array inside the library. This file checks, through the C ABI, that two
calls in a row give the same result as the workspace-based decode entry point (the same
deterministic kernels, so the bits must match; the parity tolerance used by the other GPU
tests is checked too), that the status word the no-alloc call leaves behind reads zero, and
that every decode kernel family runs on the static scratch: the cooperative streaming
kernel (a few (token, slot) pairs), the two-kernel LINEAR path and the split-K GPTOSS path.
It is named to be collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

from cernels_b200 import _lib
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _case(seed, T, H, E, F, k, layout):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    if layout == _lib.LAYOUT_LINEAR:
        w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(E, H, F, generator=g) * 0.02).to(torch.bfloat16)
        b1 = b2 = None
    else:
        w1 = (torch.randn(E, H, 2 * F, generator=g) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(E, F, H, generator=g) * 0.02).to(torch.bfloat16)
        b1 = torch.randn(E, 2 * F, generator=g) * 0.01
        b2 = torch.randn(E, H, generator=g) * 0.01
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, k, generator=g)
    dev = [None if t is None else t.cuda().contiguous() for t in (x, w1, w2, idx, w, b1, b2)]
    return dev


def _ptr(t):
    return None if t is None else t.data_ptr()


@pytest.mark.parametrize("layout,dims", [(_lib.LAYOUT_LINEAR, (1, 2048, 64, 1408, 6)),   # streaming kernel
                                         (_lib.LAYOUT_LINEAR, (8, 2048, 64, 1408, 6)),   # two-kernel path
                                         (_lib.LAYOUT_GPTOSS, (4, 2880, 32, 2880, 4))])  # split-K GPTOSS
def test_noalloc_decode_matches_workspace_decode(layout, dims):
    T, H, E, F, k = dims
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    shape = _lib.MoeShape(T, H, E, F, k, layout)
    outs = []
    for seed in (1, 2):  # two calls in a row, different inputs
        x, w1, w2, idx, w, b1, b2 = _case(seed, T, H, E, F, k, layout)
        ref_out = torch.empty_like(x)
        nbytes = _lib.workspace_bytes(shape, True)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        rc = lib.cernels_moe_experts_decode(ctypes.byref(shape), x.data_ptr(), w1.data_ptr(), _ptr(b1),
                                            w2.data_ptr(), _ptr(b2), idx.data_ptr(), w.data_ptr(),
                                            ref_out.data_ptr(), ws.data_ptr(), nbytes, stream)
        assert rc == 0
        out = torch.full_like(x, float("nan"))
        rc = lib.cernels_moe_experts_decode_noalloc(ctypes.byref(shape), x.data_ptr(), w1.data_ptr(), _ptr(b1),
                                                    w2.data_ptr(), _ptr(b2), idx.data_ptr(), w.data_ptr(),
                                                    out.data_ptr(), stream)
        assert rc == 0
        torch.cuda.synchronize()
        err = O.rel_err(out.float().cpu().numpy(), ref_out.float().cpu().numpy())
        assert np.isfinite(out.float().cpu().numpy()).all()
        assert err <= TOL, f"call {seed}: rel err {err:.3e}"
        assert torch.equal(out, ref_out), f"call {seed}: differs from the workspace decode"
        status = ctypes.c_int(-1)
        assert lib.cernels_workspace_status(ctypes.byref(shape), 1, None, ctypes.byref(status), stream) == 0
        assert status.value == 0
        outs.append(out)
    assert not torch.equal(outs[0], outs[1])  # the second call really recomputed


def test_noalloc_rejects_problems_beyond_static_scratch():
    lib = _lib.load()
    # 1000 pairs x (F + H) x 4 bytes is far above the 4 MiB static scratch.
    shape = _lib.MoeShape(250, 4096, 64, 4096, 4, _lib.LAYOUT_LINEAR)
    p = 1 << 20
    rc = lib.cernels_moe_experts_decode_noalloc(ctypes.byref(shape), p, p, None, p, None, p, p, p,
                                                torch.cuda.current_stream().cuda_stream)
    assert rc == 5
