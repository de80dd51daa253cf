"""GPU: expert parallelism over NCCL on every visible GPU (skipped with fewer than 2).

Each rank runs the EP forward on its token shard. Its rows must match (1) the fp32 CPU
oracle on a seeded sample of 64 of its tokens, routed by the same router call the EP step
makes, and (2) the single-GPU operator on the full batch. The parity tolerance applies.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cfg_name, tokens, transport, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from cernels_b200 import ep
        from cernels_b200.configs import CONFIGS, make_case
        from cernels_b200.hf_modules import build_module
        from cernels_b200.registry import gpt_oss_moe_experts as go
        from cernels_b200.registry import qwen3_next_moe_experts as qn
        from oracle import moe_oracle as O

        cfg = CONFIGS[cfg_name].with_tokens(tokens)
        case = make_case(cfg, device=f"cuda:{rank}")
        kind, module = build_module(case)
        moe = ep.ExpertParallelMoe.from_module(kind, module, rank, world)
        moe.transport = transport
        shard = ep.token_shard(cfg.tokens, rank, world)
        out = moe.forward(case.x[shard].contiguous())
        out2 = moe.forward(case.x[shard].contiguous())  # a second step (reused windows / epochs)
        full = (go.kernel if kind == "gpt_oss" else qn.kernel)(case.x.unsqueeze(0), module).squeeze(0)
        torch.cuda.synchronize()
        err = max(O.rel_err(out.float().cpu().numpy(), full[shard].float().cpu().numpy()),
                  O.rel_err(out2.float().cpu().numpy(), full[shard].float().cpu().numpy()))
        # against the oracle: a seeded sample of this rank's tokens
        xs = case.x[shard].contiguous()
        with torch.no_grad():
            idx, w = moe.router(xs)
        n = xs.shape[0]
        sample = np.sort(np.random.default_rng(rank).choice(n, min(64, n), replace=False))
        xn = xs.float().cpu().numpy()
        ref = O.moe_experts(xn, case.w1.float().cpu().numpy(), case.w2.float().cpu().numpy(), idx.cpu().numpy(),
                            w.float().cpu().numpy(), cfg.layout,
                            None if case.b1 is None else case.b1.cpu().numpy(),
                            None if case.b2 is None else case.b2.cpu().numpy(), token_subset=sample)[sample]
        if case.shared is not None:
            sh = {k_: v.float().cpu().numpy() for k_, v in case.shared.items()}
            ref = ref + O.shared_expert(xn[sample], sh["gate_proj"], sh["up_proj"], sh["down_proj"], sh["gate"])
        err = max(err, O.rel_err(out.float().cpu().numpy()[sample], ref),
                  O.rel_err(out2.float().cpu().numpy()[sample], ref))
        if transport == "p2p":
            assert moe._p2p is not None and moe._p2p.status() == 0
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["p2p", "nccl"])
@pytest.mark.parametrize("cfg_name,tokens", [("gpt_oss_20b", 2048), ("qwen3_next", 1024)])
def test_ep_matches_single_gpu(cfg_name, tokens, transport):
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    world = 2 if world < 4 else (4 if world < 8 else 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg_name, tokens, transport, q)) for r in range(world)]
    for p in procs:
        p.start()
    errs = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert max(errs.values()) <= 1e-2, errs
