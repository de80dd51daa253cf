"""Benchmark of the MoE-experts hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

A "step" is one call of the reference benchmark's timed operation on one batch:
  * experts configs (deepseek_v2_lite, qwen3_30b_a3b, decode): the op on (x, top_k_index,
    top_k_weights, experts) — the reference's ``kernel(x, idx, w, experts)``;
  * qwen3_next: ``kernel(x, block)`` — router + routed experts + gated shared expert;
  * gpt_oss_20b (default): ``kernel(x, mlp)`` — router + routed experts with biases.
``value`` is tokens/s over the whole job with inputs resident in HBM (CUDA events on the
launch stream, L2 flushed with a 256 MB write before every timed step, max over ranks);
``e2e`` is the same metric through the same public API from pinned host buffers
(host->device copy of the step's inputs and device->host copy of its output inside the
timed region). Multi-GPU runs (torchrun, one rank per GPU) use expert parallelism for
the EP configs (qwen3_next, gpt_oss_20b): tokens and experts sharded contiguously, rows
dispatched to and returned from their experts' owners through NVLink peer memory by this
library's own kernels (cernels_ep_*; NCCL all-to-all is the optional transport); total
tokens fixed ("strong" scaling). At N = 1 the line also carries ``configs``: every other
benchmark configuration (C1, C3, C4, decode shapes) timed the same way.

``--impl reference`` times the reference's own CPU path — the transformers op_eager
module the reference benchmarks against — on a bounded token sample on this host's cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import faulthandler

faulthandler.enable()  # a native crash prints the Python stack of every thread to stderr

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

DEFAULT_CONFIG = "gpt_oss_20b"
CONFIGS_TOKENS = {"gpt_oss_20b": 16384}  # workloads whose ncu traffic is recorded below
EP_CONFIGS = ("qwen3_next", "gpt_oss_20b")
L2_FLUSH_BYTES = 256 << 20


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default=DEFAULT_CONFIG)
    p.add_argument("--tokens", type=int, default=None, help="override T of the config")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--cpu-sample-s", type=float, default=15.0, help="target seconds of the CPU baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--graph", action="store_true", help="replay the step as a CUDA graph (decode)")
    p.add_argument("--no-configs", action="store_true", help="skip the sweep over the other configurations")
    p.add_argument("--align", action="store_true", help="multi-GPU: barrier before each timed step (outside it)")
    return p.parse_args(argv)


# ---------------------------------------------------------------- distributed plumbing
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def init_dist(world: int, backend: str):
    import torch.distributed as dist

    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group(backend=backend)
    return dist


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock, power and clock-event reasons of this rank's GPU through NVML (read
    only) every millisecond on a background thread while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self.error = None

    def __enter__(self):
        import threading

        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            # match this CUDA device to its NVML handle by PCI location (NVML order may differ)
            props = torch.cuda.get_device_properties(self.cuda_index)
            want = (int(getattr(props, "pci_domain_id", 0)), int(props.pci_bus_id), int(props.pci_device_id))
            h = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                cand = pynvml.nvmlDeviceGetHandleByIndex(i)
                info = pynvml.nvmlDeviceGetPciInfo(cand)
                if (int(info.domain), int(info.bus), int(info.device)) == want:
                    h = cand
                    break
            if h is None:
                raise RuntimeError(f"no NVML device with PCI bus id {want}")
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._stop = threading.Event()

            def run():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((mhz, pw, rs))
                    except Exception as e:  # keep the benchmark running
                        self.error = str(e)
                    self._stop.wait(0.001)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception as e:
            self.error = f"nvml unavailable: {e}"
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [self.error or "no samples"]}
        loaded = [s for s in self.samples if s[1] > 300.0] or self.samples
        reasons = sorted({n for s in loaded for n, bit in self.REASONS.items() if s[2] & bit})
        return {"sm_mhz": statistics.median(s[0] for s in loaded), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(loaded), "power_w_median": round(statistics.median(s[1] for s in loaded), 1),
                "sm_mhz_min": min(s[0] for s in loaded), "power_w_max": round(max(s[1] for s in loaded), 1)}


# ---------------------------------------------------------------- workload
def build_workload(args, device, rank, world):
    import torch

    from cernels_b200.configs import CONFIGS, make_case
    from cernels_b200.hf_modules import build_module

    cfg = CONFIGS[args.config]
    if args.tokens:
        cfg = cfg.with_tokens(args.tokens)
    case = make_case(cfg, device=device)
    kind, module = build_module(case, device=device)
    return cfg, case, kind, module


def make_step(cfg, case, kind, module, world, rank):
    """Returns (step(x) -> out, input tensors of one step, launches per step)."""
    import torch

    from cernels_b200.registry import cohere2_moe_experts as c2
    from cernels_b200.registry import gpt_oss_moe_experts as go
    from cernels_b200.registry import qwen3_next_moe_experts as qn

    decode = cfg.name == "decode"
    if world > 1 and cfg.name in EP_CONFIGS:
        from cernels_b200 import ep

        planner = ep.ExpertParallelMoe.from_module(kind, module, rank, world)
        shard = ep.token_shard(cfg.tokens, rank, world)
        x = case.x[shard].contiguous()
        step = lambda xx: planner.forward(xx)  # noqa: E731
        step.planner = planner
        return step, [x], planner.launches_per_step
    # launches of this library's kernels per step (router tail 1 + route 3 + gather 1 + 2 GEMMs
    # + combine 1); the router GEMM runs in cuBLAS through torch
    if kind == "gpt_oss":
        return (lambda xx: go.kernel(xx.unsqueeze(0), module).squeeze(0)), [case.x], 8
    if kind == "qwen3_next":
        return (lambda xx: qn.kernel(xx.unsqueeze(0), module).squeeze(0)), [case.x], 8
    idx, w = case.indices, case.weights.to(torch.bfloat16)
    fn = c2.decode_kernel if decode else c2.kernel
    return (lambda xx, ii, ww: fn(xx, ii, ww, module)), [case.x, idx, w], (2 if decode else 7)


def time_device(step, inputs, steps, warmup, flush, graph=False, align=None):
    """CUDA-event time of `steps` calls (ms total, per-step list): events on the launch stream
    around each step, the L2 flush between steps outside them, one synchronisation after the last
    step (the host enqueues ahead, as a serving loop does, so Python launch overhead stays off the
    device timeline). `align` (multi-GPU) runs before each step, outside its timed interval, so
    that every rank starts the step together; it synchronises the host every step."""
    import torch

    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        step(*inputs)
    torch.cuda.synchronize()
    g = None
    if graph:
        s = torch.cuda.Stream()
        s.wait_stream(stream)
        with torch.cuda.stream(s):
            step(*inputs)
        stream.wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step(*inputs)
        torch.cuda.synchronize()
    marks = []
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        if align is not None:
            align()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        if g is not None:
            g.replay()
        else:
            step(*inputs)
        b.record(stream)
        marks.append((a, b))
    torch.cuda.synchronize()
    per = [a.elapsed_time(b) for a, b in marks]
    return sum(per), per


def time_e2e(step, inputs, steps, warmup, flush, chunks=1, taper=False):
    """Pinned host inputs -> device -> step -> host output, per step, CUDA events. With
    chunks > 1 the public HostPipeline overlaps the copies of one token chunk with the compute
    of another (the result is identical: tokens are independent)."""
    import torch

    from cernels_b200.pipeline import HostPipeline

    stream = torch.cuda.current_stream()
    host_in = [t.cpu().pin_memory() for t in inputs]
    out_sample = step(*inputs)
    host_out = torch.empty(out_sample.shape, dtype=out_sample.dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = host_out.numel() * host_out.element_size()
    pipe = HostPipeline()

    def one():
        pipe.run(step, host_in, host_out, chunks, taper)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(steps):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        one()
        b.record(stream)
        b.synchronize()
        total += a.elapsed_time(b)
    return total, h2d, d2h


def stage_profile(case, steps):
    """Per-stage device times (ms) of the experts op via the C-ABI profiling entry."""
    import ctypes

    import torch

    from cernels_b200 import _lib, ops

    cfg = case.cfg
    idx = case.indices.to(torch.int32).contiguous()
    w = case.weights.float().contiguous()
    shape = ops.shape_of(case.x, case.w1, case.w2, cfg.topk, cfg.layout)
    nbytes = _lib.workspace_bytes(shape, False)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=case.x.device)
    out = torch.empty_like(case.x)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=case.x.device)
    acc = [0.0] * 5
    stage = (ctypes.c_float * 5)()
    n = 0
    for i in range(steps + 2):
        flush.zero_()
        rc = _lib.load().cernels_moe_experts_profiled(
            ctypes.byref(shape), case.x.data_ptr(), case.w1.data_ptr(), ops._ptr(case.b1), case.w2.data_ptr(),
            ops._ptr(case.b2), idx.data_ptr(), w.data_ptr(), out.data_ptr(), ws.data_ptr(), nbytes,
            torch.cuda.current_stream().cuda_stream, stage)
        _lib.check(rc, "cernels_moe_experts_profiled")
        if i >= 2:
            for j in range(5):
                acc[j] += stage[j]
            n += 1
    return [a / n for a in acc]


def decode_roofline(case, steps):
    """Decode op (its kernels only: int32/fp32 routing inputs prepared outside) timed with CUDA
    events, L2 flushed before each call; bound = HBM on the touched experts' weights."""
    import torch

    from cernels_b200 import ops
    from cernels_b200.configs import LAYOUT_GPTOSS, touched_experts

    cfg = case.cfg
    idx = case.indices.to(torch.int32).contiguous()
    w = case.weights.float().contiguous()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=case.x.device)
    stream = torch.cuda.current_stream()
    total = 0.0
    for i in range(steps + 3):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        ops.run_experts(case.x, case.w1, case.w2, idx, w, cfg.topk, cfg.layout, True, case.b1, case.b2)
        b.record(stream)
        b.synchronize()
        if i >= 3:
            total += a.elapsed_time(b)
    ms = total / steps
    hbm, _, src = load_peaks()
    e = touched_experts(case.indices, cfg.experts)
    bytes_ = 3.0 * cfg.hidden * cfg.inter * 2 * e + 2.0 * cfg.tokens * cfg.hidden * 2
    achieved = bytes_ / (ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(achieved / hbm, 4),
            "kernel": "decode op (" + ("split-K GPTOSS decode kernels" if cfg.layout == LAYOUT_GPTOSS else
                                       "streaming LINEAR decode kernel" if cfg.tokens * cfg.topk <= 12 else
                                       "two-kernel LINEAR decode") + ")",
            "peak_source": src,
            "traffic": None, "op_ms": round(ms, 4), "algorithmic": {"bytes": bytes_, "touched_experts": e}}


def load_peaks(sustained=False):
    """(HBM GB/s, bf16 TFLOP/s, source) from MEASURED_PEAKS.json: the burst bf16 figure for a kernel
    timed alone, the sustained one (power-capped, seconds-long cuBLAS loop) with sustained=True."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        tf = float(p["bf16_tflops_sustained"] if sustained else p["bf16_tflops"])
        return float(p["hbm_gbs"]), tf, "measured" + (" sustained" if sustained else " burst")
    except Exception:
        return 6650.0, (1400.0 if sustained else 1590.0), "fallback" + (" sustained" if sustained else " burst")


# dram__bytes_read.sum + dram__bytes_write.sum per launch from one ncu capture at the full
# workload (profiles/grouped_gemm_gpt_oss_20b.md): (config, kernel) -> bytes
NCU_TRAFFIC = {
    ("gpt_oss_20b", "gate_up_gemm"): 1.440748e9 + 0.361273e9,
    ("gpt_oss_20b", "down_gemm"): 0.909377e9 + 0.354875e9,
}


def roofline(cfg, case, stage_ms):
    """Dominant kernel's achieved rate vs the measured peak."""
    from cernels_b200.configs import LAYOUT_GPTOSS, touched_experts

    hbm, tflops, src = load_peaks()
    T, H, F, k = cfg.tokens, cfg.hidden, cfg.inter, cfg.topk
    tk = T * k
    e = touched_experts(case.indices, cfg.experts)
    names = ["route", "gather", "gate_up_gemm", "down_gemm", "combine"]
    dom = max(range(5), key=lambda i: stage_ms[i])
    if dom == 3:
        flops = 2.0 * tk * F * H
        bytes_ = e * H * F * 2 + tk * F * 2 + tk * H * 2 + (e * H * 4 if cfg.layout == LAYOUT_GPTOSS else 0)
    else:
        flops = 4.0 * tk * H * F
        bytes_ = e * 2 * F * H * 2 + tk * H * 2 + tk * F * 2 + (e * 2 * F * 4 if cfg.layout == LAYOUT_GPTOSS else 0)
    if dom not in (2, 3):
        flops = 0.0
        bytes_ = {0: tk * 8 * 3, 1: tk * H * 4, 4: tk * H * 2 + T * H * 2}[dom]
    sec = stage_ms[dom] / 1e3
    intensity = flops / bytes_ if bytes_ else 0.0
    ridge = tflops * 1e12 / (hbm * 1e9)
    if flops and intensity >= ridge:
        # the grouped GEMMs of a step run back to back for milliseconds, step after step: the
        # power-capped sustained peak is their denominator (the burst fraction is reported too)
        _, tf_sus, src = load_peaks(sustained=True)
        achieved = flops / sec / 1e12
        r = {"bound": "tensor", "achieved": round(achieved, 1), "peak": tf_sus, "unit": "TFLOP/s",
             "frac_of_burst": round(achieved / tflops, 4), "burst_peak": tflops}
    else:
        achieved = bytes_ / sec / 1e9
        r = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s"}
    r["frac"] = round(achieved / r["peak"], 4)
    r["kernel"] = names[dom]
    r["peak_source"] = src
    r["traffic"] = NCU_TRAFFIC.get((cfg.name, names[dom])) if cfg.tokens == CONFIGS_TOKENS.get(cfg.name) else None
    r["stage_ms"] = {n: round(v, 4) for n, v in zip(names, stage_ms)}
    r["algorithmic"] = {"flops": flops, "bytes": bytes_}
    return r


# ---------------------------------------------------------------- CPU baselines
def cpu_oracle_baseline(case, target_s):
    """numpy oracle (oracle/moe_oracle.py, a port of the reference algorithm) on a token sample."""
    import numpy as np

    from oracle import moe_oracle as O

    cfg = case.cfg
    x = case.x.float().cpu().numpy()
    w1 = case.w1.float().cpu().numpy()
    w2 = case.w2.float().cpu().numpy()
    b1 = None if case.b1 is None else case.b1.cpu().numpy()
    b2 = None if case.b2 is None else case.b2.cpu().numpy()
    idx = case.indices.cpu().numpy()
    wts = case.weights.float().cpu().numpy()
    n = min(cfg.tokens, 64)
    while True:
        t0 = time.perf_counter()
        O.moe_experts(x[:n], w1, w2, idx[:n], wts[:n], cfg.layout, b1, b2)
        dt = time.perf_counter() - t0
        if dt * 4 > target_s or n >= cfg.tokens:
            break
        n = min(cfg.tokens, n * 4)
    return {"value": round(n / dt, 2), "unit": "tokens/s", "cores": _threads(), "kind": "port",
            "sample": f"numpy fp32 oracle, first {n} of {cfg.tokens} tokens, 1 call, {dt:.2f} s"}


def _threads():
    import torch

    return int(torch.get_num_threads())


def run_reference(args):
    """The reference's op_eager module (transformers, bf16) on this host's CPU cores."""
    import torch

    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    from cernels_b200.configs import CONFIGS, make_case
    from cernels_b200.hf_modules import build_module, reference_forward

    cfg = CONFIGS[args.config]
    if args.tokens:
        cfg = cfg.with_tokens(args.tokens)
    case = make_case(cfg, device="cpu")
    kind, module = build_module(case, device="cpu")
    # bounded sample: grow the token count until one call takes ~target/ (steps)
    per_step = max(0.5, args.cpu_sample_s / max(1, args.steps + args.warmup))
    n = min(cfg.tokens, 16)
    while True:
        xs = case.x[:n]
        t0 = time.perf_counter()
        reference_forward(kind, module, case, xs, case.indices[:n], case.weights[:n])
        dt = time.perf_counter() - t0
        if dt * 2 > per_step or n >= cfg.tokens:
            break
        n = min(cfg.tokens, n * 2)
    xs = case.x[:n]
    for _ in range(args.warmup):
        reference_forward(kind, module, case, xs, case.indices[:n], case.weights[:n])
    total = 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        reference_forward(kind, module, case, xs, case.indices[:n], case.weights[:n])
        total += time.perf_counter() - t0
    value = n * args.steps / total
    line = {
        "impl": "reference", "metric": "MoE-experts tokens/s", "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if cfg.name in EP_CONFIGS else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, reference config distributions)",
        "config": {"workload": cfg.name, "tokens": cfg.tokens, "hidden": cfg.hidden, "experts": cfg.experts,
                   "intermediate": cfg.inter, "topk": cfg.topk, "reference_op": f"transformers {type(module).__name__}",
                   "sample_tokens_per_step": n,
                   "note": "a bounded token sample per step, reported as a per-token rate; the CPU arm "
                           "does not scale with N"},
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": _threads(), "kind": "reference",
                         "sample": f"first {n} of {cfg.tokens} tokens per step, transformers {type(module).__name__} "
                                   f"bf16 eager on CPU"},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm
def log(msg: str) -> None:
    print(f"[bench] {msg}", file=sys.stderr, flush=True)


def run_ours(args):
    import torch

    rank, world, local = dist_env()
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = init_dist(world, "nccl")
    import cernels_b200  # noqa: F401  (loads the CUDA library; raises if missing)

    log("building workload")
    cfg, case, kind, module = build_workload(args, device, rank, world)
    step, inputs, launches = make_step(cfg, case, kind, module, world, rank)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    warmup = max(3, args.warmup)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    log("timed region")
    use_graph = args.graph
    align = None
    if world > 1 and args.align:
        def align():
            dist.barrier(device_ids=[local])
    with ClockSampler(local) as clocks:
        total_ms, per = time_device(step, inputs, args.steps, warmup, flush, graph=use_graph, align=align)
    log(f"clock samples: {len(clocks.samples)} ({clocks.error})")
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([total_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        dist.barrier()
    # token-chunked copy/compute overlap for large single-GPU batches (EP steps are collective)
    # token chunks of the host pipeline: for large single-GPU batches 4 and 8 equal chunks and 4
    # tapered ones (half-size first and last) are tried, the fastest kept
    chunk_options = ((4, False), (8, False), (4, True)) if (world == 1 and cfg.tokens >= 4096) else ((1, False),)
    log("e2e")
    e2e_tried = {}
    for ch, taper in chunk_options:
        e2e_tried[f"{ch}{'t' if taper else ''}"] = time_e2e(step, inputs, args.steps, warmup, flush, ch, taper)
    e2e_chunks = min(e2e_tried, key=lambda ch: e2e_tried[ch][0])
    e2e_ms, h2d, d2h = e2e_tried[e2e_chunks]
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    hot = None
    if world == 1:
        # the reference's own methodology: back-to-back calls, no L2 flush (hot L2)
        log("hot-L2 timing")
        hot_ms, _ = time_device(step, inputs, args.steps, 1, None, graph=args.graph)
        hot = {"ms_per_step": round(hot_ms / args.steps, 4),
               "value": round(cfg.tokens * args.steps / (hot_ms / 1e3), 1), "unit": "tokens/s"}

    phases = None
    if world > 1 and hasattr(step, "planner"):
        # per-phase device times of the EP step (CUDA events between the phases' launches, L2
        # flushed before each step), median over steps, max over ranks
        planner = step.planner
        kept = []
        for _ in range(max(3, min(args.steps, 10))):  # no host sync between steps (as in the timed loop)
            flush.zero_()
            planner.timing = []
            step(*inputs)
            kept.append(planner.timing)
        rows = [planner.phase_ms(ev) for ev in kept]
        planner.timing = None
        names = list(rows[0].keys())
        med = torch.tensor([statistics.median(r[n] for r in rows) for n in names], device=device)
        dist.all_reduce(med, op=dist.ReduceOp.MAX)
        phases = {n: round(float(v), 4) for n, v in zip(names, med.tolist())}
    ep_extra = None
    if world > 1 and cfg.name == "gpt_oss_20b" and not args.no_configs:
        # the other expert-parallel configuration (qwen3_next: 512 experts, shared expert inside
        # the EP step), timed the same way at this N
        ep_extra = measure_ep_config("qwen3_next", device, rank, world, min(args.steps, 10), flush, dist)
    tokens = cfg.tokens
    ms_per_step = total_ms / args.steps
    value = tokens * args.steps / (total_ms / 1e3)
    e2e_value = tokens * args.steps / (e2e_ms / 1e3)
    roof = None
    cpu = None
    if rank == 0:
        if cfg.name == "decode":
            roof = decode_roofline(case, min(args.steps, 20))
        elif world == 1 or cfg.name not in EP_CONFIGS:
            log("stage profile")
            roof = roofline(cfg, case, stage_profile(case, min(args.steps, 10)))
        elif phases is not None:
            roof = ep_roofline(cfg, world, phases)
        if world == 1 and not args.no_cpu_baseline:
            log("cpu baseline")
            cpu = cpu_oracle_baseline(case, args.cpu_sample_s)
    configs = None
    if world == 1 and not args.no_configs:
        log("configuration sweep")
        configs = measure_configs(min(args.steps, 10), device)
    if rank == 0:
        line = {
            "metric": "MoE-experts tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "strong" if cfg.name in EP_CONFIGS else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; reference config shapes and distributions)",
            "config": {"workload": cfg.name, "tokens": cfg.tokens, "hidden": cfg.hidden, "experts": cfg.experts,
                       "intermediate": cfg.inter, "topk": cfg.topk, "shared_intermediate": cfg.shared_inter,
                       "parallelism": f"ep{world}" if (world > 1 and cfg.name in EP_CONFIGS) else f"replica{world}",
                       "l2": "flushed (256 MB write) before every timed step", "graph": bool(use_graph),
                       "step_barrier": align is not None},
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "token_chunks": e2e_chunks,
                    "chunk_options_ms_per_step": {ch: round(v[0] / args.steps, 4) for ch, v in e2e_tried.items()}},
            "hot_l2": hot,
            "gpu_launches": launches * args.steps,
            "clocks": clocks.summary(),
            "op_roofline_ms": round(op_roofline_ms(cfg, case), 4),
            "configs": configs,
            "ep_phases_ms": phases,
            "ep_configs": ep_extra,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# Every benchmark configuration other than the headline one, measured in the same run
# (N = 1): (label, config, tokens override, decode entry point)
CONFIG_SWEEP = [
    ("deepseek_v2_lite", "deepseek_v2_lite", None, False),
    ("qwen3_30b_a3b", "qwen3_30b_a3b", None, False),
    ("qwen3_next", "qwen3_next", None, False),
    ("decode_t1", "decode", 1, True),
    ("decode_t4", "decode", 4, True),
    ("decode_t8", "decode", 8, True),
    ("qwen3_30b_a3b_decode_t8", "qwen3_30b_a3b", 8, True),
    ("gpt_oss_20b_decode_t1", "gpt_oss_20b", 1, True),
    ("gpt_oss_20b_decode_t8", "gpt_oss_20b", 8, True),
]


def config_step(kind, module, case, decode):
    """The reference-facing call of one configuration: (step, inputs)."""
    import torch

    from cernels_b200.registry import cohere2_moe_experts as c2
    from cernels_b200.registry import gpt_oss_moe_experts as go
    from cernels_b200.registry import qwen3_next_moe_experts as qn

    if kind in ("gpt_oss", "qwen3_next"):
        mod = go if kind == "gpt_oss" else qn
        fn = mod.decode_kernel if decode else mod.kernel
        return (lambda xx: fn(xx.unsqueeze(0), module).squeeze(0)), [case.x]
    fn = c2.decode_kernel if decode else c2.kernel
    return (lambda xx, ii, ww: fn(xx, ii, ww, module)), [case.x, case.indices, case.weights.to(torch.bfloat16)]


def measure_configs(steps, device):
    """ms/step, tokens/s, op roofline and the dominant kernel's roofline fraction of every
    configuration in CONFIG_SWEEP, timed like the headline (CUDA events on the launch stream,
    L2 flushed before every timed step; decode steps replayed as CUDA graphs), with clocks
    sampled over the whole sweep."""
    import torch

    from cernels_b200.configs import CONFIGS, make_case
    from cernels_b200.hf_modules import build_module

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    out = {}
    with ClockSampler(device.index or 0) as clocks:
        for label, name, tokens, decode in CONFIG_SWEEP:
            try:
                cfg = CONFIGS[name] if tokens is None else CONFIGS[name].with_tokens(tokens)
                case = make_case(cfg, device=device)
                kind, module = build_module(case, device=device)
                step, inputs = config_step(kind, module, case, decode)
                total_ms, _ = time_device(step, inputs, steps, 3, flush, graph=decode)
                ms = total_ms / steps
                roof = decode_roofline(case, steps) if decode else roofline(cfg, case, stage_profile(case, steps))
                op_ms = op_roofline_ms(cfg, case)
                out[label] = {
                    "tokens": cfg.tokens, "entry": ("decode_kernel" if decode else "kernel"),
                    "ms_per_step": round(ms, 4), "tokens_per_s": round(cfg.tokens / (ms / 1e3), 1),
                    "op_roofline_ms": round(op_ms, 4), "frac_of_op_roofline": round(op_ms / ms, 4),
                    "graph": decode,
                    "roofline": {k: roof[k] for k in ("bound", "kernel", "achieved", "peak", "unit", "frac")},
                }
                del case, module
            except Exception as e:  # one failing entry must not lose the others
                out[label] = {"error": f"{type(e).__name__}: {e}"}
            torch.cuda.synchronize()
    out["clocks"] = clocks.summary()
    out["method"] = ("CUDA events on the launch stream, 256 MB L2 flush before every timed step, "
                     f"{steps} timed steps after 3 warm-up; decode entries replayed as CUDA graphs")
    return out


def ep_roofline(cfg, world, phases):
    """Expert-parallel step, per rank: the grouped GEMMs' FLOPs of this rank's share of the rows
    (total / world) over the "experts" phase (its GEMMs, plus the wait for rows still arriving),
    against the sustained bf16 peak; with the NVLink bytes each rank sends (its routed rows that
    leave the GPU, each way) for context."""
    _, tf_sus, src = load_peaks(sustained=True)
    flops = cfg.flops() / world
    sec = phases["experts"] / 1e3
    achieved = flops / sec / 1e12
    row_bytes = cfg.hidden * 2
    remote_rows = cfg.tokens * cfg.topk / world * (world - 1) / world
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": tf_sus, "unit": "TFLOP/s",
            "frac": round(achieved / tf_sus, 4), "kernel": "grouped GEMMs of the EP step (experts phase, per rank)",
            "peak_source": src, "traffic": None,
            "algorithmic": {"flops_per_rank": flops, "nvlink_bytes_per_rank_each_way": remote_rows * row_bytes},
            "phases_ms": phases}


def measure_ep_config(name, device, rank, world, steps, flush, dist):
    """ms/step (max over ranks), tokens/s and per-phase times of one more EP configuration."""
    import torch

    from cernels_b200.configs import CONFIGS, make_case
    from cernels_b200.hf_modules import build_module

    try:
        cfg = CONFIGS[name]
        case = make_case(cfg, device=device)
        kind, module = build_module(case, device=device)
        step, inputs, _ = make_step(cfg, case, kind, module, world, rank)
        dist.barrier()
        total_ms, _ = time_device(step, inputs, steps, 3, flush)
        t = torch.tensor([total_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item()) / steps
        planner = step.planner
        kept = []
        for _ in range(3):  # no host sync between steps (as in the timed loop)
            flush.zero_()
            planner.timing = []
            step(*inputs)
            kept.append(planner.timing)
        rows = [planner.phase_ms(ev) for ev in kept]
        planner.timing = None
        names = list(rows[0].keys())
        med = torch.tensor([statistics.median(r[n] for r in rows) for n in names], device=device)
        dist.all_reduce(med, op=dist.ReduceOp.MAX)
        return {name: {"ms_per_step": round(ms, 4), "tokens_per_s": round(cfg.tokens / (ms / 1e3), 1),
                       "tokens": cfg.tokens, "scaling": "strong", "shared_expert": "inside the EP step",
                       "phases_ms": {n: round(float(v), 4) for n, v in zip(names, med.tolist())}}}
    except Exception as e:  # keep the headline line
        return {name: {"error": f"{type(e).__name__}: {e}"}}


def op_roofline_ms(cfg, case):
    from cernels_b200.configs import touched_experts

    hbm, tflops, _ = load_peaks()
    e = touched_experts(case.indices, cfg.experts)
    return max(cfg.flops() / (tflops * 1e12), cfg.bytes_moved(e) / (hbm * 1e9)) * 1e3


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
