"""Host logic of the (b, h)-sharded multi-GPU path on CPU with world_size-2 gloo
process groups: the plan partitions the units exactly, per-shard oracle results
gathered from the ranks equal the single-process result (so the shard's global
head slopes are right), and the max-over-ranks timing reduction works."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, B, Hq, Hkv, S, D, out):
    import sys
    for p in (ROOT, os.path.join(ROOT, "co-alibi_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from co_alibi_attn.sharding import shard_plan
    from oracle import coalibi_oracle as orc
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = shard_plan(B, Hq, Hkv, world, rank)
        g = torch.Generator().manual_seed(0)
        q = torch.randn(B, Hq, S, D, generator=g, dtype=torch.float64)
        k = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64)
        v = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64)
        sl = orc.api_slopes(Hq, 8.0, torch.float64)[sh.h0:sh.h1]
        o, _, _ = orc.forward(q[sh.b0:sh.b1, sh.h0:sh.h1], k[sh.b0:sh.b1, sh.g0:sh.g1],
                              v[sh.b0:sh.b1, sh.g0:sh.g1], sl, True)
        units = [torch.zeros(B * Hkv, dtype=torch.int64) for _ in range(world)]
        mine = torch.zeros(B * Hkv, dtype=torch.int64)
        for (b, gg) in sh.units():
            mine[b * Hkv + gg] = 1
        dist.all_gather(units, mine)
        full_o = torch.zeros(B, Hq, S, D, dtype=torch.float64)
        full_o[sh.b0:sh.b1, sh.h0:sh.h1] = o
        dist.all_reduce(full_o)
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            out["coverage"] = torch.stack(units).sum(0).tolist()
            out["o"] = full_o
            out["tmax"] = t.item()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B,Hq,Hkv", [(2, 4, 4), (1, 8, 2), (4, 6, 3)])
def test_two_rank_sharding(B, Hq, Hkv):
    from oracle import coalibi_oracle as orc
    S, D, world = 24, 8, 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, B, Hq, Hkv, S, D, out), nprocs=world, join=True,
                       start_method="spawn")
    assert out["coverage"] == [1] * (B * Hkv)
    g = torch.Generator().manual_seed(0)
    q = torch.randn(B, Hq, S, D, generator=g, dtype=torch.float64)
    k = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64)
    v = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64)
    o_ref, _, _ = orc.forward(q, k, v, orc.api_slopes(Hq, 8.0, torch.float64), True)
    assert torch.allclose(out["o"], o_ref, atol=1e-12)
    assert out["tmax"] == 2.0


def test_plan_errors():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "co-alibi_b200"))
    from co_alibi_attn.sharding import shard_plan
    with pytest.raises(ValueError):
        shard_plan(3, 6, 3, 2, 0)
    sh = shard_plan(8, 16, 16, 8, 3)
    assert (sh.b0, sh.b1, sh.g0, sh.g1) == (3, 4, 0, 16)
    sh = shard_plan(4, 32, 8, 8, 5)
    assert (sh.b0, sh.b1, sh.g0, sh.g1, sh.h0, sh.h1) == (0, 4, 5, 6, 20, 24)
