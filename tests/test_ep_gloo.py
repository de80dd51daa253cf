"""CPU (gloo) tests of the expert-parallel exchange logic in cernels_b200.ep.

Each rank runs ExpertParallelMoe.forward on its token shard with a CPU backend built from
the oracle; the concatenated outputs must equal the single-process oracle on all tokens.
Also checks that a rank that never joins makes the others fail with a timeout error
(failure detected on the host, no GPU involved).
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cernels_b200 import ep
from oracle import moe_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def make_problem(layout, T=40, H=32, E=8, F=24, k=3, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    router_w = torch.randn(E, H, generator=g)
    if layout == O.LAYOUT_LINEAR:
        w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.1).to(torch.bfloat16)
        w2 = (torch.randn(E, H, F, generator=g) * 0.1).to(torch.bfloat16)
        b1 = b2 = None
    else:
        w1 = (torch.randn(E, H, 2 * F, generator=g) * 0.1).to(torch.bfloat16)
        w2 = (torch.randn(E, F, H, generator=g) * 0.1).to(torch.bfloat16)
        b1 = torch.randn(E, 2 * F, generator=g) * 0.1
        b2 = torch.randn(E, H, generator=g) * 0.1
    return dict(x=x, router_w=router_w, w1=w1, w2=w2, b1=b1, b2=b2, k=k, layout=layout)


def router_fn(p):
    def router(x):
        logits = x.float() @ p["router_w"].T
        v, i = torch.topk(logits, p["k"], dim=-1)
        return i, torch.softmax(v, dim=-1)
    return router


def cpu_backend(p, e0, e1):
    layout = p["layout"]

    def route(idx, w, E):
        offsets, order, inv = O.route(idx.numpy(), E)
        k = idx.shape[1]
        perm_token = torch.zeros(idx.numel(), dtype=torch.int32)
        perm_token[:order.size] = torch.from_numpy((order // k).astype(np.int32))
        perm_w = w.reshape(-1)[torch.from_numpy(order)]
        return torch.from_numpy(offsets), perm_token, perm_w, torch.from_numpy(inv)

    def gather(x, perm_token, rows):
        return x[perm_token[:rows].long().clamp(0, x.shape[0] - 1)].contiguous()

    def experts(rows, counts):
        out = np.zeros((rows.shape[0], rows.shape[1]), np.float32)
        per = e1 - e0
        li = np.repeat(np.arange(counts.numel()) % per, counts.numpy())
        for le in range(e1 - e0):
            sel = np.nonzero(li == le)[0]
            if sel.size == 0:
                continue
            e = e0 + le
            out[sel] = O.expert_rows(rows[sel].float().numpy(), p["w1"][e].float().numpy(),
                                     p["w2"][e].float().numpy(), layout,
                                     None if p["b1"] is None else p["b1"][e].numpy(),
                                     None if p["b2"] is None else p["b2"][e].numpy())
        return torch.from_numpy(out).to(torch.bfloat16)

    def combine(rows, inv, w):
        T, k = w.shape
        out = torch.zeros(T, rows.shape[1])
        for t in range(T):
            for j in range(k):
                s = int(inv[t * k + j])
                if s >= 0:
                    out[t] += w[t, j] * rows[s].float()
        return out.to(torch.bfloat16)

    return ep.Backend(route=route, gather=gather, experts=experts, combine=combine)


def _worker(rank, world, port, layout, result_q, chunks=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p = make_problem(layout)
        E = p["w1"].shape[0]
        e0, e1 = ep.expert_shard(E, rank, world)
        moe = ep.ExpertParallelMoe(E, p["k"], rank, world, router_fn(p), cpu_backend(p, e0, e1), chunks=chunks)
        shard = ep.token_shard(p["x"].shape[0], rank, world)
        out = moe.forward(p["x"][shard].contiguous())
        result_q.put((rank, out.float().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,chunks", [(2, None), (2, 3), (4, 2)])
@pytest.mark.parametrize("layout", [O.LAYOUT_LINEAR, O.LAYOUT_GPTOSS])
def test_ep_matches_single_process_oracle(world, chunks, layout):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, layout, q, chunks)) for r in range(world)]
    for pr in procs:
        pr.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    out = np.concatenate([results[r] for r in range(world)])
    p = make_problem(layout)
    idx, w = router_fn(p)(p["x"])
    ref = O.moe_experts(p["x"].float().numpy(), p["w1"].float().numpy(), p["w2"].float().numpy(), idx.numpy(),
                        w.numpy(), layout, None if p["b1"] is None else p["b1"].numpy(),
                        None if p["b2"] is None else p["b2"].numpy())
    assert O.rel_err(out, ref) <= 1e-2


def test_piece_counts_partition_each_segment():
    rng = np.random.default_rng(0)
    for _ in range(50):
        counts = rng.integers(0, 40, size=rng.integers(1, 9))
        for C in (1, 2, 3, 5):
            p = ep.ExpertParallelMoe.piece_counts(counts, C)
            assert p.shape == (C, counts.size)
            assert np.array_equal(p.sum(0), counts)
            sizes = p.sum(1)
            assert sizes.max() - sizes.min() <= 1


def test_shards_cover_tokens_and_experts():
    for T, R in [(16384, 8), (10, 3), (3, 4)]:
        covered = []
        for r in range(R):
            s = ep.token_shard(T, r, R)
            covered += list(range(T))[s]
        assert covered == list(range(T))
    assert ep.expert_shard(32, 7, 8) == (28, 32)
    with pytest.raises(ValueError):
        ep.expert_shard(30, 0, 8)


def _absent_peer_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if rank == 1:
        return  # never joins the group
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
        q.put((rank, "joined"))
    except Exception as e:  # the store / rendezvous times out on the host
        q.put((rank, f"error: {type(e).__name__}"))


def test_missing_rank_is_detected_on_host():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    rank, msg = q.get(timeout=60)
    for pr in procs:
        pr.join(timeout=30)
    assert rank == 0 and msg.startswith("error")
