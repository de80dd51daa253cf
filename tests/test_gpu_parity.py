"""GPU parity: the CUDA path (through the C ABI / torch ops) against the CPU oracle.

Bars: routing offsets / permutation / inverse map bit-exact; expert outputs
max|out - ref| / max|ref| <= 1e-2 against the fp32 oracle (bf16 in, fp32 accumulate),
plus the reference's own verify() (allclose atol = rtol = 2e-2).
"""

import numpy as np
import pytest
import torch

from cernels_b200 import ops
from cernels_b200.configs import CONFIGS, LAYOUT_GPTOSS, LAYOUT_LINEAR, make_case
from oracle import moe_oracle as O
from tests import golden_io

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda"


def run_op(x, w1, w2, idx, w, k, layout, decode=False, b1=None, b2=None):
    return ops.run_experts(x.to(DEV).contiguous(), w1.to(DEV).contiguous(), w2.to(DEV).contiguous(),
                           idx.to(DEV).to(torch.int32).contiguous(), w.to(DEV).float().contiguous(), k, layout, decode,
                           None if b1 is None else b1.to(DEV).float().contiguous(),
                           None if b2 is None else b2.to(DEV).float().contiguous())


def oracle_out(x, w1, w2, idx, w, layout, b1=None, b2=None, token_subset=None):
    return O.moe_experts(x.float().cpu().numpy(), w1.float().cpu().numpy(), w2.float().cpu().numpy(),
                         idx.cpu().numpy(), w.float().cpu().numpy(), layout,
                         None if b1 is None else b1.float().cpu().numpy(),
                         None if b2 is None else b2.float().cpu().numpy(), token_subset=token_subset)


def assert_close(out, ref, tol=TOL):
    out = out.float().cpu().numpy()
    err = O.rel_err(out, ref)
    assert np.isfinite(out).all()
    assert err <= tol, f"rel err {err:.3e} > {tol}"
    return err


# ---------------------------------------------------------------- routing
@pytest.mark.parametrize("T,k,E,seed", [(1, 1, 1, 0), (3, 2, 5, 1), (512, 6, 64, 2), (2048, 8, 128, 3),
                                        (4096, 10, 512, 4), (16384, 4, 32, 5), (1500, 7, 2048, 6), (257, 3, 33, 7)])
def test_route_bit_exact(T, k, E, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(-1, E + 1, (T, k), generator=g).to(torch.int32)  # -1 and E are skipped
    w = torch.rand(T, k, generator=g)
    offsets, perm_token, perm_weight, inv = ops.route(idx.to(DEV), w.to(DEV), E)
    r_off, r_order, r_inv = O.route(idx.numpy(), E)
    n = int(r_off[-1])
    assert np.array_equal(offsets.cpu().numpy(), r_off)
    assert np.array_equal(perm_token.cpu().numpy()[:n], (r_order // k).astype(np.int32))
    assert np.array_equal(perm_weight.cpu().numpy()[:n], w.reshape(-1).numpy()[r_order])
    assert np.array_equal(inv.cpu().numpy(), r_inv)


def test_route_is_deterministic_across_calls():
    g = torch.Generator().manual_seed(9)
    idx = torch.randint(0, 64, (4096, 6), generator=g).to(torch.int32).to(DEV)
    w = torch.rand(4096, 6, generator=g).to(DEV)
    a = ops.route(idx, w, 64)
    b = ops.route(idx, w, 64)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


# ---------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("name", golden_io.NAMES)
@pytest.mark.parametrize("decode", [False, True])
def test_golden_fixtures(name, decode):
    g = golden_io.load(name)
    layout = LAYOUT_GPTOSS if g["kind"] == "gpt_oss" else LAYOUT_LINEAR
    k = g["indices"].shape[1]
    out = run_op(g["x"], g["w1"], g["w2"], g["indices"], g["weights"], k, layout, decode, g.get("b1"), g.get("b2"))
    ref = O.moe_experts(g["x"].float().numpy(), g["w1"].float().numpy(), g["w2"].float().numpy(),
                        g["indices"].numpy(), g["weights"].numpy(), layout,
                        g["b1"].numpy() if "b1" in g else None, g["b2"].numpy() if "b2" in g else None)
    assert_close(out, ref)
    if g["kind"] != "qwen3_next":  # qwen3 golden output includes the shared expert
        assert torch.allclose(out.float().cpu(), g["ref_bf16"].float(), atol=2e-2, rtol=2e-2)


# ---------------------------------------------------------------- shapes and edge cases
SHAPES = [
    # T, H, E, F, k  (covers F % 128 != 0, H % 64 != 0, one expert, > 128 rows per expert, many experts)
    (1, 64, 4, 32, 2),
    (5, 72, 3, 40, 3),
    (64, 256, 8, 128, 2),
    (300, 192, 4, 136, 1),
    (513, 512, 16, 264, 4),
    (200, 2048, 64, 1408, 6),
    (1024, 2048, 512, 512, 10),
    (777, 2880, 8, 2880, 4),
]


@pytest.mark.parametrize("layout", [LAYOUT_LINEAR, LAYOUT_GPTOSS])
@pytest.mark.parametrize("T,H,E,F,k", SHAPES)
def test_prefill_shapes(T, H, E, F, k, layout):
    g = torch.Generator().manual_seed(T * 31 + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    if layout == LAYOUT_LINEAR:
        w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.05).to(torch.bfloat16)
        w2 = (torch.randn(E, H, F, generator=g) * 0.05).to(torch.bfloat16)
        b1 = b2 = None
    else:
        w1 = (torch.randn(E, H, 2 * F, generator=g) * 0.05).to(torch.bfloat16)
        w2 = (torch.randn(E, F, H, generator=g) * 0.05).to(torch.bfloat16)
        b1 = torch.randn(E, 2 * F, generator=g) * 0.1
        b2 = torch.randn(E, H, generator=g) * 0.1
    k = min(k, E)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.rand(T, k, generator=g)
    out = run_op(x, w1, w2, idx, w, k, layout, False, b1, b2)
    assert_close(out, oracle_out(x, w1, w2, idx, w, layout, b1, b2))


def test_skewed_routing_many_rows_one_expert():
    """Most entries on expert 0 (many m-tiles), some experts empty, invalid ids mixed in."""
    g = torch.Generator().manual_seed(11)
    T, H, E, F, k = 1000, 256, 6, 96, 3
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E, H, F, generator=g) * 0.05).to(torch.bfloat16)
    idx = torch.zeros(T, k, dtype=torch.int64)
    idx[:, 1] = torch.where(torch.rand(T, generator=g) < 0.5, 2, -1)
    idx[:, 2] = torch.where(torch.rand(T, generator=g) < 0.1, 5, E)  # E is out of range -> skipped
    w = torch.rand(T, k, generator=g)
    for decode in (False,):
        out = run_op(x, w1, w2, idx, w, k, LAYOUT_LINEAR, decode)
        assert_close(out, oracle_out(x, w1, w2, idx, w, LAYOUT_LINEAR))


def test_all_slots_invalid_gives_zeros():
    T, H, E, F, k = 9, 64, 4, 32, 2
    x = torch.randn(T, H).to(torch.bfloat16)
    w1 = torch.randn(E, 2 * F, H).to(torch.bfloat16)
    w2 = torch.randn(E, H, F).to(torch.bfloat16)
    idx = torch.full((T, k), -1)
    w = torch.rand(T, k)
    for decode in (False, True):
        out = run_op(x, w1, w2, idx, w, k, LAYOUT_LINEAR, decode)
        assert torch.count_nonzero(out) == 0


def test_empty_batch():
    x = torch.empty(0, 64, dtype=torch.bfloat16)
    out = run_op(x, torch.zeros(2, 64, 64, dtype=torch.bfloat16), torch.zeros(2, 64, 32, dtype=torch.bfloat16),
                 torch.empty(0, 1, dtype=torch.int64), torch.empty(0, 1), 1, LAYOUT_LINEAR)
    assert out.shape == (0, 64)


# ---------------------------------------------------------------- decode
@pytest.mark.parametrize("layout", [LAYOUT_LINEAR, LAYOUT_GPTOSS])
@pytest.mark.parametrize("T", [1, 2, 3, 4, 8, 33, 60])
def test_decode_matches_oracle_and_prefill(T, layout):
    g = torch.Generator().manual_seed(100 + T)
    H, E, F, k = (2048, 64, 1408, 6) if layout == LAYOUT_LINEAR else (2880, 32, 2880, 4)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    if layout == LAYOUT_LINEAR:
        w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(E, H, F, generator=g) * 0.02).to(torch.bfloat16)
        b1 = b2 = None
    else:
        w1 = (torch.randn(E, H, 2 * F, generator=g) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(E, F, H, generator=g) * 0.02).to(torch.bfloat16)
        b1 = torch.randn(E, 2 * F, generator=g) * 0.01
        b2 = torch.randn(E, H, generator=g) * 0.01
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.rand(T, k, generator=g)
    ref = oracle_out(x, w1, w2, idx, w, layout, b1, b2)
    out_d = run_op(x, w1, w2, idx, w, k, layout, True, b1, b2)
    assert_close(out_d, ref)
    out_p = run_op(x, w1, w2, idx, w, k, layout, False, b1, b2)
    assert_close(out_p, ref)


def test_decode_deterministic():
    g = torch.Generator().manual_seed(7)
    T, H, E, F, k = 8, 2048, 64, 1408, 6
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, F, generator=g) * 0.02).to(torch.bfloat16)
    idx = torch.randint(0, E, (T, k), generator=g)
    w = torch.rand(T, k, generator=g)
    a = run_op(x, w1, w2, idx, w, k, LAYOUT_LINEAR, True)
    b = run_op(x, w1, w2, idx, w, k, LAYOUT_LINEAR, True)
    assert torch.equal(a, b)


@pytest.mark.parametrize("T,H,E,F,k", [(1, 200, 8, 136, 2), (3, 1000, 16, 520, 4), (5, 2880, 32, 2880, 4),
                                       (2, 4096, 128, 1024, 8)])
def test_decode_gptoss_split_k_shapes(T, H, E, F, k):
    """GPTOSS decode splits K across CTAs when few experts are touched (split count from the
    shape; ragged splits when H or F is not a multiple of it): matches the oracle, and two
    calls give identical bits."""
    g = torch.Generator().manual_seed(11 * T + H)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(E, H, 2 * F, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, F, H, generator=g) * 0.02).to(torch.bfloat16)
    b1 = torch.randn(E, 2 * F, generator=g) * 0.01
    b2 = torch.randn(E, H, generator=g) * 0.01
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.rand(T, k, generator=g)
    ref = oracle_out(x, w1, w2, idx, w, LAYOUT_GPTOSS, b1, b2)
    a = run_op(x, w1, w2, idx, w, k, LAYOUT_GPTOSS, True, b1, b2)
    b = run_op(x, w1, w2, idx, w, k, LAYOUT_GPTOSS, True, b1, b2)
    assert_close(a, ref)
    assert torch.equal(a, b)


# ---------------------------------------------------------------- benchmark configurations
@pytest.mark.parametrize("name", ["deepseek_v2_lite", "qwen3_30b_a3b", "qwen3_next"])
def test_benchmark_configs_full_size(name):
    case = make_case(CONFIGS[name], device=DEV)
    out = run_op(case.x, case.w1, case.w2, case.indices, case.weights, case.cfg.topk, case.cfg.layout)
    ref = oracle_out(case.x, case.w1, case.w2, case.indices, case.weights, case.cfg.layout)
    err = assert_close(out, ref)
    print(f"{name}: rel err {err:.2e}")
    assert torch.allclose(out.float().cpu(), torch.from_numpy(ref), atol=2e-2, rtol=2e-2)


def test_gpt_oss_full_size_token_sample():
    """C5 at full size on the GPU; each token's output depends only on its own row, so a
    seeded sample of 96 tokens is checked against the oracle restricted to them."""
    case = make_case(CONFIGS["gpt_oss_20b"], device=DEV)
    out = run_op(case.x, case.w1, case.w2, case.indices, case.weights, 4, LAYOUT_GPTOSS, False, case.b1, case.b2)
    sample = np.sort(np.random.default_rng(0).choice(case.cfg.tokens, 96, replace=False))
    ref = oracle_out(case.x, case.w1, case.w2, case.indices, case.weights, LAYOUT_GPTOSS, case.b1, case.b2,
                     token_subset=sample)
    assert_close(out[torch.from_numpy(sample).to(DEV)], ref[sample])
    # whole-output sanity: every row finite
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("name", ["qwen3_30b_a3b", "qwen3_next", "gpt_oss_20b"])
def test_benchmark_config_decode_t8(name):
    """Decode at T=8 with each benchmark configuration's weights and routing (C3 is the
    "also run at decode T=8" case: 64 pairs through the two-kernel LINEAR path; C4: 80 pairs
    over 512 experts; C5: the split-K GPTOSS path at 8 tokens)."""
    case = make_case(CONFIGS[name].with_tokens(8), device=DEV)
    cfg = case.cfg
    out = run_op(case.x, case.w1, case.w2, case.indices, case.weights, cfg.topk, cfg.layout, True, case.b1, case.b2)
    ref = oracle_out(case.x, case.w1, case.w2, case.indices, case.weights, cfg.layout, case.b1, case.b2)
    assert_close(out, ref)


def test_qwen3_next_full_kernel_full_size():
    """C4 at full size through kernel(x, block): router, fused shared expert and routed experts.
    The routing the kernel used must equal the router-tail oracle on the same logits bit for bit,
    and the output must match the oracle's routed experts plus its gated shared expert on those
    ids, over every row (no row allowance)."""
    from cernels_b200.hf_modules import build_module
    from cernels_b200.registry import qwen3_next_moe_experts as qn
    case = make_case(CONFIGS["qwen3_next"], device=DEV)
    cfg = case.cfg
    _, blk = build_module(case)
    x3 = case.x.unsqueeze(0)
    with torch.no_grad():
        out = qn.kernel(x3, blk).squeeze(0)
        logits, idx, w = qn.route_debug(case.x, blk)
    E, k = cfg.experts, cfg.topk
    r_idx, r_w = O.router_tail(logits[:, :E].float().cpu().numpy(), k, 1, True)
    assert np.array_equal(idx[:, :k].cpu().numpy(), r_idx)
    assert np.allclose(w[:, :k].cpu().numpy(), r_w, atol=1e-6, rtol=1e-4)
    gate = 1.0 / (1.0 + np.exp(-logits[:, E].float().cpu().numpy()))
    assert np.allclose(w[:, k].cpu().numpy(), gate, atol=1e-6, rtol=1e-4)
    ref = O.moe_experts(case.x.float().cpu().numpy(), case.w1.float().cpu().numpy(), case.w2.float().cpu().numpy(),
                        r_idx, r_w, LAYOUT_LINEAR)
    sh = case.shared
    xs = case.x.float().cpu().numpy()
    g = xs @ sh["gate_proj"].float().cpu().numpy().T
    u = xs @ sh["up_proj"].float().cpu().numpy().T
    y = ((g / (1.0 + np.exp(-g))) * u) @ sh["down_proj"].float().cpu().numpy().T
    ref = ref + y * gate[:, None]
    assert_close(out, ref)


@pytest.mark.parametrize("T", [1, 4, 8])
def test_decode_config(T):
    case = make_case(CONFIGS["decode"].with_tokens(T), device=DEV)
    out = run_op(case.x, case.w1, case.w2, case.indices, case.weights, 6, LAYOUT_LINEAR, True)
    ref = oracle_out(case.x, case.w1, case.w2, case.indices, case.weights, LAYOUT_LINEAR)
    assert_close(out, ref)


@pytest.mark.parametrize("decode", [False, True])
def test_cuda_graph_capture_and_replay(decode):
    """No host sync inside the op: it captures into a CUDA graph, and replays see new inputs."""
    g = torch.Generator().manual_seed(21)
    T, H, E, F, k = 8, 2048, 64, 1408, 6
    w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    w2 = (torch.randn(E, H, F, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    idx = torch.randint(0, E, (T, k), generator=g).to(torch.int32).to(DEV)
    w = torch.rand(T, k, generator=g).to(DEV)
    fn = ops.cohere2_moe_experts_decode if decode else ops.cohere2_moe_experts
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(x, w1, w2, idx, w, k)  # warm-up (sets kernel attributes outside capture)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fn(x, w1, w2, idx, w, k)
    for seed in (1, 2):
        gg = torch.Generator().manual_seed(seed)
        x.copy_(torch.randn(T, H, generator=gg).to(torch.bfloat16))
        idx.copy_(torch.randint(0, E, (T, k), generator=gg).to(torch.int32))
        graph.replay()
        torch.cuda.synchronize()
        eager = fn(x, w1, w2, idx, w, k)
        assert torch.equal(out, eager)


@pytest.mark.parametrize("T,H,E,F,k", [(1, 64, 4, 32, 2), (2, 72, 3, 40, 3), (1, 2880, 16, 768, 6), (2, 512, 512, 512, 6),
                                       (1, 4096, 8, 1536, 4)])
def test_decode_streaming_shapes(T, H, E, F, k):
    """Small decode batches (<= 12 pairs) take the bulk-copy streaming kernel."""
    g = torch.Generator().manual_seed(T * 7 + H)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E, H, F, generator=g) * 0.05).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    idx[0, 0] = -1  # one skipped slot
    w = torch.rand(T, k, generator=g)
    out = run_op(x, w1, w2, idx, w, k, LAYOUT_LINEAR, True)
    assert_close(out, oracle_out(x, w1, w2, idx, w, LAYOUT_LINEAR))
    none = run_op(x, w1, w2, torch.full_like(idx, -1), w, k, LAYOUT_LINEAR, True)
    assert torch.count_nonzero(none) == 0


@pytest.mark.parametrize("layout", [LAYOUT_LINEAR, LAYOUT_GPTOSS])
def test_grouped_experts_segments(layout):
    """cernels_moe_grouped_experts: rows in runs ordered (source rank, local expert)."""
    g = torch.Generator().manual_seed(5)
    R, E, H, F = 4, 3, 256, 136
    counts = torch.randint(0, 200, (R * E,), generator=g)
    counts[1] = 0
    counts[5] = 300  # several m-tiles in one run
    N = int(counts.sum())
    rows = torch.randn(N, H, generator=g).to(torch.bfloat16)
    if layout == LAYOUT_LINEAR:
        w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.05).to(torch.bfloat16)
        w2 = (torch.randn(E, H, F, generator=g) * 0.05).to(torch.bfloat16)
        b1 = b2 = None
    else:
        w1 = (torch.randn(E, H, 2 * F, generator=g) * 0.05).to(torch.bfloat16)
        w2 = (torch.randn(E, F, H, generator=g) * 0.05).to(torch.bfloat16)
        b1 = torch.randn(E, 2 * F, generator=g) * 0.1
        b2 = torch.randn(E, H, generator=g) * 0.1
    out = ops.grouped_experts(rows.to(DEV), counts.to(DEV), w1.to(DEV), w2.to(DEV), layout,
                              None if b1 is None else b1.to(DEV), None if b2 is None else b2.to(DEV))
    ref = np.zeros((N, H), np.float32)
    start = 0
    for gi, c in enumerate(counts.tolist()):
        e = gi % E
        if c:
            ref[start:start + c] = O.expert_rows(rows[start:start + c].float().numpy(), w1[e].float().numpy(),
                                                 w2[e].float().numpy(), layout,
                                                 None if b1 is None else b1[e].numpy(),
                                                 None if b2 is None else b2[e].numpy())
        start += c
    assert_close(out, ref)


@pytest.mark.parametrize("mode,E,k,renorm", [(0, 32, 4, False), (1, 512, 10, True), (1, 128, 8, False),
                                             (0, 64, 6, False), (1, 1000, 32, True)])
def test_router_topk_matches_torch(mode, E, k, renorm):
    g = torch.Generator().manual_seed(E + k)
    T = 777
    logits32 = torch.randn(T, E, generator=g).to(DEV)
    idx, w = ops.router_topk(logits32, k, mode, renorm)
    if mode == 0:
        v, i = torch.topk(logits32, k, dim=-1)
        ref_w = torch.softmax(v, dim=-1).to(torch.bfloat16).float()
    else:
        p = torch.softmax(logits32, dim=-1)
        v, i = torch.topk(p, k, dim=-1)
        ref_w = v / v.sum(-1, keepdim=True) if renorm else v
    assert torch.equal(idx.long(), i)  # fp32 random logits: no ties
    assert torch.allclose(w, ref_w, atol=1e-5, rtol=1e-2)
    # bf16 logits: the selected values equal torch's sorted top-k (ties may permute ids)
    lb = logits32.to(torch.bfloat16)
    idx_b, _ = ops.router_topk(lb, k, mode, renorm)
    got = torch.gather(lb.float(), 1, idx_b.long())
    assert torch.equal(got, torch.topk(lb.float(), k, dim=-1).values)


@pytest.mark.parametrize("name", ["qwen3_next", "gpt_oss_20b"])
def test_loader_matches_transformers_module(name):
    """kernel(x, block) / kernel(x, mlp) against the transformers module the reference
    benchmarks (op_eager), at reduced size, with the reference's verify() tolerance."""
    from cernels_b200.hf_modules import build_module, reference_forward
    from cernels_b200.registry import gpt_oss_moe_experts as go
    from cernels_b200.registry import qwen3_next_moe_experts as qn
    cfg = CONFIGS[name].scaled(tokens=256, experts=32 if name == "qwen3_next" else 8,
                                hidden=512, inter=256, **({"shared_inter": 256} if name == "qwen3_next" else {}))
    case = make_case(cfg, device=DEV)
    kind, mod = build_module(case)
    ref = reference_forward(kind, mod, case)
    out = (qn.kernel if kind == "qwen3_next" else go.kernel)(case.x.unsqueeze(0), mod).squeeze(0)
    close = torch.isclose(out.float(), ref.float(), atol=2e-2, rtol=2e-2)
    # a bf16 tie in the router logits may pick a different expert for a token: allow <= 1% of rows
    bad_rows = (~close).any(dim=1).float().mean().item()
    assert bad_rows <= 0.01, bad_rows


def test_host_pipeline_matches_direct_call():
    """cernels_b200.pipeline.HostPipeline: chunked host->device->host run equals one call."""
    from cernels_b200.pipeline import HostPipeline
    g = torch.Generator().manual_seed(3)
    T, H, E, F, k = 1000, 512, 16, 256, 4
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    w2 = (torch.randn(E, H, F, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, k, generator=g)
    step = lambda xx, ii, ww: ops.cohere2_moe_experts(xx, w1, w2, ii, ww, k)  # noqa: E731
    direct = step(x.to(DEV), idx.to(DEV), w.to(DEV)).cpu()
    out = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    HostPipeline().run(step, [x.pin_memory(), idx.pin_memory(), w.pin_memory()], out, chunks=3)
    torch.cuda.synchronize()
    assert torch.equal(out, direct)


def test_shared_expert_fused_path_matches_separate_path():
    """cernels_moe_experts_shared (shared expert as an always-on group) vs the routed op plus the
    shared expert run as its own one-expert problem, on the same routing (fused router output)."""
    from cernels_b200.hf_modules import build_module
    from cernels_b200.registry import qwen3_next_moe_experts as qn
    cfg = CONFIGS["qwen3_next"].scaled(tokens=300, experts=64, hidden=512, inter=256, shared_inter=256)
    case = make_case(cfg, device=DEV)
    _, blk = build_module(case)
    xf = case.x
    k = cfg.topk
    assert qn.fused_shared_supported(blk)
    with torch.no_grad():
        logits = torch.nn.functional.linear(xf, qn._router_and_gate(blk))
        idx, w = ops.router_topk(logits, k, ops.ROUTER_SOFTMAX_TOPK, True, shared_gate=cfg.experts)
        assert torch.all(idx[:, k] == cfg.experts)
        sw1, sw2 = qn._shared_weights(blk)
        e = blk.experts
        fused = ops.run_experts_shared(xf, e.gate_up_proj.data, e.down_proj.data, sw1, sw2, idx, w, k)
        routed = ops.qwen3_next_moe_experts(xf, e.gate_up_proj.data, e.down_proj.data, idx[:, :k].contiguous(),
                                            w[:, :k].contiguous(), k)
        shared = ops.qwen3_next_moe_experts(xf, sw1, sw2, torch.zeros_like(idx[:, :1]), w[:, k:].contiguous(), 1)
        ref = (routed.float() + shared.float()).cpu().numpy()
    assert_close(fused, ref)


@pytest.mark.parametrize("name", ["deepseek_v2_lite", "gpt_oss_20b"])
def test_in_model_swap_matches_module(name):
    """swaps.SWAPS on transformers experts modules: decode (<= 4 tokens) and prefill shapes."""
    from cernels_b200 import swaps
    from cernels_b200.hf_modules import build_module
    cfg = CONFIGS[name].scaled(tokens=64, experts=8, hidden=512, inter=256)
    case = make_case(cfg, device=DEV)
    kind, mod = build_module(case)
    experts = mod.experts if kind == "gpt_oss" else mod
    family = "gpt_oss" if kind == "gpt_oss" else "deepseek_v2"
    for T in (3, 64):
        x = case.x[:T].contiguous()
        idx = case.indices[:T].contiguous()
        w = case.weights[:T].to(torch.bfloat16 if kind != "gpt_oss" else torch.float32).contiguous()
        with torch.no_grad():
            swaps.SWAPS[family][0](experts, "stock")
            ref = experts(x, idx, w)
            swaps.SWAPS[family][0](experts, "custom")
            out = experts(x, idx, w)
            swaps.SWAPS[family][0](experts, "stock")
        assert torch.allclose(out.float(), ref.float(), atol=2e-2, rtol=2e-2)



@pytest.mark.parametrize("mode,E,k,renorm", [(0, 32, 4, False), (1, 512, 10, True), (0, 64, 6, False)])
def test_router_topk_matches_oracle(mode, E, k, renorm):
    """router_topk kernel vs the numpy router-tail oracle (fp32 logits, no ties)."""
    g = torch.Generator().manual_seed(100 + E)
    logits = torch.randn(513, E, generator=g)
    idx, w = ops.router_topk(logits.to(DEV), k, mode, renorm)
    r_idx, r_w = O.router_tail(logits.numpy(), k, mode, renorm)
    assert np.array_equal(idx.cpu().numpy(), r_idx)
    if mode == 0:  # the kernel rounds gpt-oss scores to bf16 as transformers does
        r_w = torch.from_numpy(r_w).to(torch.bfloat16).float().numpy()
    assert np.allclose(w.cpu().numpy(), r_w, atol=1e-5, rtol=1e-2)


def _bf16_np(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


@pytest.mark.parametrize("mode,T,H,E,k,renorm,gate,bias", [
    (0, 777, 2880, 32, 4, False, False, True),     # gpt-oss router (C5 shape, fewer tokens)
    (1, 300, 2048, 512, 10, True, True, False),    # qwen3-next router + shared gate, 4-CTA cluster
    (1, 1000, 2048, 512, 10, True, False, False),  # qwen3-next router alone
    (1, 129, 512, 128, 8, False, False, False),
    (0, 5, 64, 8, 2, False, False, True),
    (1, 40, 256, 1000, 16, True, True, False),     # many experts: cluster of 4 over 1001 columns
])
def test_fused_router_matches_oracle(mode, T, H, E, k, renorm, gate, bias):
    """cernels_router: the bf16 logits it selected from equal the fp32 product rounded to bf16
    (within one bf16 step: the summation order differs), and its ids / weights equal the
    router-tail oracle applied to those logits (ids bit-exact, ties to the lower id)."""
    g = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    rows = (E + 1 + 7) // 8 * 8 if gate else E
    wt = (torch.randn(rows, H, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(E, generator=g) * 0.02).to(torch.bfloat16) if bias else None
    idx, w, logits = ops.router(x.to(DEV), wt.to(DEV), None if b is None else b.to(DEV), E, k, mode, renorm,
                                shared_gate=gate, return_logits=True)
    cols = E + int(gate)
    lg = logits.float().cpu().numpy()[:, :cols]
    ref = x.float().numpy() @ wt.float().numpy()[:cols].T
    if b is not None:
        ref[:, :E] += b.float().numpy()
    step = np.maximum(np.abs(ref), 1e-30) * 2.0 ** -7
    assert np.all(np.abs(lg - ref) <= step + 1e-4)  # absolute slack: cancellation near zero
    assert np.mean(lg == _bf16_np(ref)) > 0.99
    r_idx, r_w = O.router_tail(lg[:, :E], k, mode, renorm)
    assert np.array_equal(idx[:, :k].cpu().numpy(), r_idx)
    if mode == 0:  # gpt-oss weights are rounded to bf16: one bf16 step apart at a rounding boundary
        assert np.allclose(w[:, :k].cpu().numpy(), _bf16_np(r_w), atol=1e-6, rtol=2.0 ** -8)
    else:
        assert np.allclose(w[:, :k].cpu().numpy(), r_w, atol=1e-6, rtol=1e-5)
    if gate:
        assert np.all(idx[:, k].cpu().numpy() == E)
        assert np.allclose(w[:, k].cpu().numpy(), 1.0 / (1.0 + np.exp(-lg[:, E])), atol=1e-6, rtol=1e-5)
    # without the debug logits output the kernel takes the same decisions
    idx2, w2 = ops.router(x.to(DEV), wt.to(DEV), None if b is None else b.to(DEV), E, k, mode, renorm,
                          shared_gate=gate)
    assert torch.equal(idx, idx2) and torch.equal(w, w2)


def test_fused_router_gpt_oss_full_batch_matches_torch_linear():
    """C5's router on its full 16,384-token batch: the ids equal a torch (cuBLAS) linear + the
    router-tail oracle wherever the top-k margin exceeds one bf16 step of the logits."""
    from cernels_b200.hf_modules import build_module
    from cernels_b200.registry import gpt_oss_moe_experts as go
    case = make_case(CONFIGS["gpt_oss_20b"], device=DEV)
    _, mlp = build_module(case)
    with torch.no_grad():
        idx, w = go.route(case.x, mlp)
        lt = torch.nn.functional.linear(case.x, mlp.router.weight, mlp.router.bias).float().cpu().numpy()
    r_idx, r_w = O.router_tail(lt, 4, 0)
    srt = -np.sort(-lt, axis=1)
    margin = srt[:, 3] - srt[:, 4]
    clear = margin > np.abs(srt[:, 3]) * 2.0 ** -7
    assert clear.mean() > 0.9
    assert np.array_equal(idx.cpu().numpy()[clear], r_idx[clear])
