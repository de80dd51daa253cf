"""GPU: a bounded wait inside a kernel that runs out returns, and says so in a status word.

Every spin inside this library's kernels (pipeline mbarriers, grid barriers, peer-rank
flags) gives up after a limit, records a nonzero status and lets the kernel return, so a
logic error or a dead peer never leaves the GPU spinning. This test makes one such wait
run out on purpose, without any fault: a one-rank expert-parallel context is asked to run
its experts for a step whose rows were never dispatched, so the wait for the source's
arrival flag can only time out. The limit is lowered to 50 ms for the test.
"""

import ctypes
import time

import pytest
import torch

from cernels_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_ep_wait_for_missing_dispatch_times_out_and_reports():
    lib = _lib.load()
    H, El, F, cap = 256, 2, 128, 64
    ctx = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    _lib.check(lib.cernels_ep_create(0, 1, H, El, cap, 0, ctypes.byref(ctx), handle), "cernels_ep_create")
    try:
        _lib.check(lib.cernels_ep_connect(ctx, handle.raw), "cernels_ep_connect")
        w1 = torch.zeros(El, 2 * F, H, dtype=torch.bfloat16, device="cuda")
        w2 = torch.zeros(El, H, F, dtype=torch.bfloat16, device="cuda")
        shape = _lib.MoeShape(cap, H, El, F, 1, _lib.LAYOUT_LINEAR)
        n = ctypes.c_size_t(0)
        _lib.check(lib.cernels_ep_experts_workspace_bytes(ctx, ctypes.byref(shape), ctypes.byref(n)), "ws")
        ws = torch.empty(n.value, dtype=torch.uint8, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        status = ctypes.c_int(-1)
        _lib.check(lib.cernels_ep_status(ctx, ctypes.byref(status)), "cernels_ep_status")
        assert status.value == 0
        _lib.check(lib.cernels_set_wait_limit_ns(50_000_000), "cernels_set_wait_limit_ns")
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        # epoch 7 was never dispatched: the experts step's wait for it must give up
        _lib.check(lib.cernels_ep_experts(ctx, ctypes.byref(shape), w1.data_ptr(), None, w2.data_ptr(), None, None,
                                          None, 0, 7, ws.data_ptr(), n.value, stream), "cernels_ep_experts")
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        _lib.check(lib.cernels_ep_status(ctx, ctypes.byref(status)), "cernels_ep_status")
        assert status.value != 0, "the timed-out wait did not record a status"
        assert elapsed < 1.5, f"kernel returned after {elapsed:.2f} s, limit was 50 ms"
    finally:
        lib.cernels_set_wait_limit_ns(0)
        lib.cernels_ep_destroy(ctx)
    # the context stays usable: a regular operator call afterwards is correct
    g = torch.Generator().manual_seed(0)
    x = torch.randn(16, 64, generator=g).to(torch.bfloat16).cuda()
    w1 = (torch.randn(2, 64, 64, generator=g) * 0.05).to(torch.bfloat16).cuda()
    w2 = (torch.randn(2, 64, 32, generator=g) * 0.05).to(torch.bfloat16).cuda()
    idx = torch.zeros(16, 1, dtype=torch.int32, device="cuda")
    w = torch.ones(16, 1, device="cuda")
    out = ops.cohere2_moe_experts(x, w1, w2, idx, w, 1)
    xf = x.float()
    gu = xf @ w1[0].float().T
    ref = (torch.nn.functional.silu(gu[:, :32]) * gu[:, 32:]) @ w2[0].float().T
    assert torch.allclose(out.float(), ref, atol=2e-2, rtol=2e-2)


def test_prefill_status_word_reads_zero_after_a_normal_call():
    lib = _lib.load()
    g = torch.Generator().manual_seed(1)
    T, H, E, F, k = 64, 128, 4, 64, 2
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.05).to(torch.bfloat16).cuda()
    w2 = (torch.randn(E, H, F, generator=g) * 0.05).to(torch.bfloat16).cuda()
    idx = torch.randint(0, E, (T, k), generator=g).to(torch.int32).cuda()
    w = torch.rand(T, k, generator=g).cuda()
    for decode in (0, 1):
        shape = _lib.MoeShape(T if not decode else 4, H, E, F, k, _lib.LAYOUT_LINEAR)
        n = _lib.workspace_bytes(shape, bool(decode))
        ws = torch.full((n,), 0xFF, dtype=torch.uint8, device="cuda")  # stale nonzero garbage
        out = torch.empty(shape.tokens, H, dtype=torch.bfloat16, device="cuda")
        fn = lib.cernels_moe_experts_decode if decode else lib.cernels_moe_experts
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(fn(ctypes.byref(shape), x.data_ptr(), w1.data_ptr(), None, w2.data_ptr(), None, idx.data_ptr(),
                      w.data_ptr(), out.data_ptr(), ws.data_ptr(), n, stream), "op")
        st = ctypes.c_int(-1)
        _lib.check(lib.cernels_workspace_status(ctypes.byref(shape), decode, ws.data_ptr(), ctypes.byref(st), stream),
                   "status")
        assert st.value == 0
