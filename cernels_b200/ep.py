"""Expert parallelism for the MoE-experts operators (one process per GPU).

The reference is single-GPU; expert parallelism is the north star's multi-GPU scheme for
the large-token configurations (qwen3_next, gpt_oss). Rank r of R owns the contiguous
expert slice [r*E/R, (r+1)*E/R) and the contiguous token slice of its batch.

Default transport: NVLink peer memory (``P2PTransport`` over ``cernels_ep_*``, see
csrc/ep_p2p.cu). One forward, without any host synchronisation:

  1. router on the local tokens (one tensor-core kernel: linear + top-k + softmax)
  2. routing kernel over the GLOBAL expert ids: offsets, stable permutation, inverse map
  3. per-expert row counts exchanged through the peers' windows; every rank learns where its
     rows go in each owner's expert-contiguous receive region
  4. rows for the other ranks copied straight into their windows on a side stream, expert by
     expert, with a per-(rank, expert) arrival flag; this rank's own rows copied in order
  5. owner side: grouped tcgen05 GEMMs on the received rows in place; the gate/up GEMM waits per
     expert for the arrival flags (so it overlaps the transfer), the down GEMM's epilogue stores
     every result row into its source's return region over NVLink
  6. combine kernel: out[t] = sum_j w[t, j] * row[inv[t, j]] in fp32, slot order
  qwen3_next runs its shared expert inside the same GEMMs, as one more group on the local tokens.

``transport="nccl"`` (and the CPU path the tests run on gloo ranks): counts and rows exchanged
with all_to_all_single, the received rows (runs per (source rank, local expert)) through
``cernels_moe_grouped_experts``, results returned by a second all-to-all; optional chunking
pipelines dispatch, GEMMs and return. All device work goes through a ``Backend``.
"""

from __future__ import annotations

import dataclasses
from typing import Callable

import numpy as np
import torch
import torch.distributed as dist


def token_shard(tokens: int, rank: int, world: int) -> slice:
    """Contiguous token slice of rank `rank` (first `tokens % world` ranks get one more)."""
    base, rem = divmod(tokens, world)
    start = rank * base + min(rank, rem)
    return slice(start, start + base + (1 if rank < rem else 0))


def expert_shard(experts: int, rank: int, world: int) -> tuple[int, int]:
    if experts % world:
        raise ValueError(f"{experts} experts do not split evenly over {world} ranks")
    per = experts // world
    return rank * per, (rank + 1) * per


@dataclasses.dataclass
class Backend:
    """Device operations the EP forward needs.

    route(indices int32 [T,k], weights fp32 [T,k], E) -> (offsets [E+1], perm_token, perm_weight, inv)
    gather(x [T,H], perm_token, rows) -> [rows, H]
    experts(rows [N,H], counts [R * E_local]) -> [N,H]: rows arrive as contiguous runs ordered
        (source rank, local expert); run g uses local expert g % E_local (unweighted, + bias)
    combine(rows [M,H], inv int32 [T*k], weights fp32 [T,k]) -> [T,H]
    """

    route: Callable
    gather: Callable
    experts: Callable
    combine: Callable


def cuda_backend(layout: int, w1: torch.Tensor, w2: torch.Tensor, b1=None, b2=None) -> Backend:
    from . import ops

    def experts(rows, counts):
        return ops.grouped_experts(rows, counts, w1, w2, layout, b1, b2)

    return Backend(route=ops.route, gather=ops.gather_rows, experts=experts, combine=ops.combine_rows)


class P2PTransport:
    """Device-side dispatch / return over NVLink peer memory (include/cernels_b200.h,
    cernels_ep_*): one IPC-shared window per rank, no NCCL and no host sync per step."""

    def __init__(self, rank: int, world: int, hidden: int, local_experts: int, max_rows: int, device, group=None,
                 shared_rows: int = 0):
        import ctypes

        from . import _lib

        self._lib = _lib
        lib = _lib.load()
        self.ctx = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(device):
            _lib.check(lib.cernels_ep_create(rank, world, hidden, local_experts, max_rows, shared_rows,
                                             ctypes.byref(self.ctx), handle), "cernels_ep_create")
            handles = [None] * world
            dist.all_gather_object(handles, handle.raw, group=group)
            _lib.check(lib.cernels_ep_connect(self.ctx, b"".join(handles)), "cernels_ep_connect")
        dist.barrier(group=group)
        self.device = device
        self.max_rows = max_rows
        self.shared_rows = shared_rows
        self._ws = None  # epochs are counted on the device (epoch argument 0): steps replay from CUDA graphs

    def status(self) -> int:
        import ctypes

        st = ctypes.c_int(0)
        self._lib.check(self._lib.load().cernels_ep_status(self.ctx, ctypes.byref(st)), "cernels_ep_status")
        return int(st.value)

    def step(self, x, perm_token, offsets, inv, w, weights, shape, mark=lambda: None, shared=None):
        """dispatch -> grouped experts (results stored back into the sources' windows) -> combine
        for one batch; returns [T, H] bf16. shared = (w1 [1, 2F, H], w2 [1, H, F]): an always-on
        expert on this rank's tokens, weighted by the last column of w."""
        import ctypes

        lib = self._lib.load()
        T, k = w.shape
        if T * k > self.max_rows:
            raise RuntimeError(f"expert-parallel window holds {self.max_rows} routed rows, batch has {T * k}")
        if shared is not None and T > self.shared_rows:
            raise RuntimeError(f"expert-parallel window holds {self.shared_rows} shared-expert rows, batch has {T}")
        layout, w1, b1, w2, b2 = weights
        n_shared = T if shared is not None else 0
        stream = torch.cuda.current_stream(self.device).cuda_stream
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        self._lib.check(lib.cernels_ep_dispatch(self.ctx, x.data_ptr(), perm_token.data_ptr(), offsets.data_ptr(),
                                                T * k, n_shared, 0, stream), "cernels_ep_dispatch")
        mark()
        key = (shape.hidden, shape.intermediate, shape.experts, shape.layout)
        if getattr(self, "_ws_key", None) != key:  # workspace sized once per shape
            n = ctypes.c_size_t(0)
            self._lib.check(lib.cernels_ep_experts_workspace_bytes(self.ctx, ctypes.byref(shape), ctypes.byref(n)),
                            "cernels_ep_experts_workspace_bytes")
            if self._ws is None or self._ws.numel() < n.value:
                self._ws = torch.empty(n.value, dtype=torch.uint8, device=self.device)
            self._ws_key = key
        n = ctypes.c_size_t(self._ws.numel())
        sw1, sw2 = shared if shared is not None else (None, None)
        self._lib.check(lib.cernels_ep_experts(self.ctx, ctypes.byref(shape), w1.data_ptr(), ptr(b1), w2.data_ptr(),
                                               ptr(b2), ptr(sw1), ptr(sw2), n_shared, 0, self._ws.data_ptr(), n.value,
                                               stream), "cernels_ep_experts")
        mark()
        out = torch.empty(T, x.shape[1], dtype=x.dtype, device=x.device)
        self._lib.check(lib.cernels_ep_combine(self.ctx, inv.data_ptr(), w.data_ptr(), T, k, int(n_shared > 0),
                                               out.data_ptr(), 0, stream), "cernels_ep_combine")
        mark()
        return out

    def __del__(self):
        try:
            if self.ctx:
                self._lib.load().cernels_ep_destroy(self.ctx)
        except Exception:
            pass


class ExpertParallelMoe:
    """EP forward over a process group; weights of the local expert slice only."""

    def __init__(self, experts: int, topk: int, rank: int, world: int, router: Callable, backend: Backend,
                 shared: Callable | None = None, group=None, chunks: int | None = None,
                 local_weights: tuple | None = None, transport: str = "auto",
                 fused_shared: tuple | None = None):
        self.E = experts
        self.k = topk
        self.rank = rank
        self.world = world
        self.e0, self.e1 = expert_shard(experts, rank, world)
        self.router = router
        self.backend = backend
        self.shared = shared
        self.group = group
        self.chunks = chunks  # None: chosen from the row count
        # (layout, w1, b1, w2, b2) of the local expert slice; needed by the peer-memory transport
        self.local_weights = local_weights
        self.transport = transport  # "p2p" (CUDA peer memory), "nccl", or "auto"
        # (router_with_shared_slot, (shared w1, shared w2)): the peer-memory path runs the shared
        # expert inside the EP step as one more grouped-GEMM group; the router then returns
        # topk + 1 columns, the last one (E, shared gate weight)
        self.fused_shared = fused_shared
        self._p2p = None
        # router(1) + route(3) + counts(1) + 2 copies + segments(1) + rowmap(1) + 2 GEMMs + results(1)
        # + combine(1)
        self.launches_per_step = 13

    # ------------------------------------------------------------ construction
    @classmethod
    def from_module(cls, kind: str, module, rank: int, world: int, group=None) -> "ExpertParallelMoe":
        from .configs import LAYOUT_GPTOSS, LAYOUT_LINEAR

        if kind == "gpt_oss":
            ex = module.experts
            E = ex.gate_up_proj.shape[0]
            e0, e1 = expert_shard(E, rank, world)
            w1 = ex.gate_up_proj.data[e0:e1].contiguous()
            w2 = ex.down_proj.data[e0:e1].contiguous()
            b1 = ex.gate_up_proj_bias.data[e0:e1].float().contiguous()
            b2 = ex.down_proj_bias.data[e0:e1].float().contiguous()
            backend = cuda_backend(LAYOUT_GPTOSS, w1, w2, b1, b2)
            local = (LAYOUT_GPTOSS, w1, b1, w2, b2)

            from .registry import gpt_oss_moe_experts as go

            def router(x, out=None):
                return go.route(x, module, out=out)

            return cls(E, int(module.router.top_k), rank, world, router, backend, None, group, local_weights=local)
        if kind == "qwen3_next":
            from .registry import qwen3_next_moe_experts as qn

            ex = module.experts
            E = ex.gate_up_proj.shape[0]
            e0, e1 = expert_shard(E, rank, world)
            w1 = ex.gate_up_proj.data[e0:e1].contiguous()
            w2 = ex.down_proj.data[e0:e1].contiguous()
            backend = cuda_backend(LAYOUT_LINEAR, w1, w2)
            local = (LAYOUT_LINEAR, w1, None, w2, None)

            def router(x, out=None):
                return qn.route(x, module)

            fused = None
            if qn.fused_shared_supported(module):
                fused = (lambda x, out=None: qn._fused_route(x, module, out=out), qn._shared_weights(module))
            return cls(E, int(module.gate.top_k), rank, world, router, backend, lambda x: qn.shared_expert(x, module),
                       group, local_weights=local, fused_shared=fused)
        raise ValueError(f"expert parallelism is not used for {kind}")

    # ------------------------------------------------------------ forward
    @staticmethod
    def piece_counts(counts: np.ndarray, chunks: int) -> np.ndarray:
        """Splits one destination segment (rows of consecutive experts with `counts` rows each)
        into `chunks` contiguous row pieces; returns [chunks, len(counts)] rows per expert per piece."""
        n = int(counts.sum())
        bounds = (np.arange(chunks + 1, dtype=np.int64) * n) // chunks
        starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
        ends = starts + counts
        lo = np.maximum(starts[None, :], bounds[:-1, None])
        hi = np.minimum(ends[None, :], bounds[1:, None])
        return np.maximum(hi - lo, 0)

    def chunks_for(self, rows: int = 0) -> int:
        # One chunk by default: on B200 the host-side chunk bookkeeping and the smaller GEMM
        # calls cost more than the overlap gains at 2 ranks (measured); callers can opt in.
        return 1 if self.chunks is None else max(1, int(self.chunks))

    def use_p2p(self, x: torch.Tensor) -> bool:
        if self.transport == "nccl" or not x.is_cuda or self.local_weights is None:
            return False
        return True

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.use_p2p(x):
            return self.forward_p2p(x)
        return self.forward_nccl(x)

    PHASES = ("router", "route", "dispatch", "experts", "combine", "shared")

    def _mark(self):
        """Records a CUDA event on the current stream when phase timing is on (self.timing)."""
        if getattr(self, "timing", None) is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.timing.append(ev)

    def phase_ms(self, events=None):
        """Per-phase device times (ms) of the last timed forward, or of the event list `events` kept
        from an earlier one (PHASES order; the shared expert's phase is 0 when there is none).
        Synchronises."""
        ev = self.timing if events is None else events
        torch.cuda.synchronize()
        out = [a.elapsed_time(b) for a, b in zip(ev[:-1], ev[1:])]
        return dict(zip(self.PHASES, out + [0.0] * (len(self.PHASES) - len(out))))

    def forward_p2p(self, x: torch.Tensor) -> torch.Tensor:
        from . import _lib

        if getattr(self, "timing", None) is not None:
            self.timing = []
        fused = self.fused_shared
        with torch.no_grad():
            self._mark()
            # router outputs and routing tables live in buffers reused from step to step
            if not hasattr(self, "_route_bufs"):
                from . import ops

                self._route_bufs = ops.RouteBuffers()
                self._router_out = None
            idx, w = (fused[0] if fused is not None else self.router)(x, out=self._router_out)
            self._router_out = (idx, w)
            self._mark()
            # the shared slot's id E is outside [0, E): routing skips it (inv = -1)
            offsets, perm_token, _perm_weight, inv = self.backend.route(idx, w, self.E, self._route_bufs)
            self._mark()
            if self._p2p is None:
                # window capacity: the most routed rows (and tokens) any rank has (all ranks agree)
                cap = torch.tensor([idx.numel(), x.shape[0]], dtype=torch.int64, device=x.device)
                dist.all_reduce(cap, op=dist.ReduceOp.MAX, group=self.group)
                self._p2p = P2PTransport(self.rank, self.world, x.shape[1], self.E // self.world, int(cap[0].item()),
                                         x.device, self.group, shared_rows=int(cap[1].item()) if fused else 0)
            layout, w1, b1, w2, b2 = self.local_weights
            F = w1.shape[1] // 2 if layout == 0 else w1.shape[2] // 2
            shape = _lib.MoeShape(int(self._p2p.max_rows), int(x.shape[1]), int(self.E // self.world), int(F), 1,
                                  int(layout))
            out = self._p2p.step(x.contiguous(), perm_token, offsets, inv, w, self.local_weights, shape,
                                 mark=self._mark, shared=None if fused is None else fused[1])
            if self.shared is not None and fused is None:
                out = out + self.shared(x)
                self._mark()
            return out

    def forward_nccl(self, x: torch.Tensor) -> torch.Tensor:
        R, E, k = self.world, self.E, self.k
        per = E // R
        dev = x.device
        with torch.no_grad():
            idx, w = self.router(x)
            idx = idx.to(torch.int32).contiguous()
            w = w.float().contiguous()
            H = x.shape[1]
            offsets, perm_token, _perm_weight, inv = self.backend.route(idx, w, E)
            # per-expert counts, grouped by destination rank -> [R, per]
            send_counts = (offsets[1:] - offsets[:-1]).to(torch.int64).reshape(R, per)
            recv_counts = torch.empty_like(send_counts)
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
            C = self.chunks_for(0)
            if C == 1:
                # Enqueue the gather before the host copy below so it runs while the host waits;
                # rows past the valid count gather token 0 (route zero-fills) and are not sent.
                tk = idx.numel()
                send_all = self.backend.gather(x, perm_token, tk) if tk else x.new_empty(0, H)
            host = torch.stack([send_counts, recv_counts]).cpu().numpy()  # the one device->host copy
            sc, rc = host[0], host[1]
            n_send = int(sc.sum())
            if C == 1:
                inv2 = inv
                send_buf = send_all[:n_send]
                send_rows = sc.sum(1)[None, :]
                recv_rows = rc.sum(1)[None, :]
                recv_p = None
            else:
                send_p = np.stack([self.piece_counts(sc[d], C) for d in range(R)], axis=1)
                recv_p = np.stack([self.piece_counts(rc[s_], C) for s_ in range(R)], axis=1)
                # chunk-major order of the routed rows: for c: for d: piece (c, d)
                seg_start = np.concatenate([[0], np.cumsum(sc.sum(1))[:-1]])
                piece_start = np.zeros((C, R), dtype=np.int64)
                for d in range(R):
                    piece_start[:, d] = seg_start[d] + np.concatenate([[0], np.cumsum(send_p[:, d].sum(1))[:-1]])
                order = np.concatenate([np.arange(piece_start[c, d], piece_start[c, d] + send_p[c, d].sum())
                                        for c in range(C) for d in range(R)]) if n_send else np.zeros(0, np.int64)
                order_t = torch.from_numpy(order).to(dev)
                pos = torch.empty(max(n_send, 1), dtype=torch.int64, device=dev)
                pos[order_t] = torch.arange(n_send, device=dev)
                inv2 = torch.where(inv >= 0, pos[inv.clamp(min=0).long()], -1).to(torch.int32).contiguous()
                send_buf = (self.backend.gather(x, perm_token[order_t].contiguous(), n_send) if n_send
                            else x.new_empty(0, H))
                send_rows = send_p.sum(2)   # [C, R]
                recv_rows = recv_p.sum(2)   # [C, R]
            # pipeline: dispatch all chunks, then per chunk: wait, experts, return
            recv_bufs, handles, s_off = [], [], 0
            for c in range(C):
                ns, nr = int(send_rows[c].sum()), int(recv_rows[c].sum())
                rb = x.new_empty(nr, H)
                handles.append(dist.all_to_all_single(rb, send_buf[s_off:s_off + ns], recv_rows[c].tolist(),
                                                      send_rows[c].tolist(), group=self.group, async_op=True))
                recv_bufs.append(rb)
                s_off += ns
            back = x.new_empty(n_send, H)
            ret_handles, s_off = [], 0
            for c in range(C):
                ns, nr = int(send_rows[c].sum()), int(recv_rows[c].sum())
                handles[c].wait()
                if nr:
                    counts_c = (recv_counts.reshape(-1) if recv_p is None else
                                torch.from_numpy(recv_p[c].reshape(-1).astype(np.int32)).to(dev))
                    rows_out = self.backend.experts(recv_bufs[c], counts_c)
                else:
                    rows_out = x.new_empty(0, H)
                ret_handles.append(dist.all_to_all_single(back[s_off:s_off + ns], rows_out, send_rows[c].tolist(),
                                                          recv_rows[c].tolist(), group=self.group, async_op=True))
                s_off += ns
            for h in ret_handles:
                h.wait()
            out = self.backend.combine(back, inv2, w)
            if self.shared is not None:
                out = out + self.shared(x)
            return out
