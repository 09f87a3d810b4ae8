"""(b, h)-sharded attention on several GPUs (needs two or more; skipped otherwise).

One process per GPU: each rank runs ``sharded_attention`` forward and backward on
its own contiguous block of (batch element, kv head) units -- no collective on
the data path -- and NCCL gathers the shards' o / dq / dk / dv for verification,
the way bench.py verifies its multi-GPU runs.  The gathered batch must be
bit-identical to one GPU running the whole batch through ``co_alibi_attention``
(each unit's kernels do the same arithmetic wherever it runs) and match the CPU
oracle."""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests._common import make_inputs, oracle_fwd_pv, oracle_bwd, check_o, rel_err, GRAD_REL

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHAPE = (2, 8, 4, 640, 128)  # B, Hq, Hkv, S, D: 8 (b, kv head) units


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import sys
    for p in (ROOT, os.path.join(ROOT, "co-alibi_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    from co_alibi_attn.sharding import shard_plan, sharded_attention
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        B, Hq, Hkv, S, D = SHAPE
        q, k, v, do = make_inputs(B, Hq, Hkv, S, S, D, torch.float16, seed=51)
        sh = shard_plan(B, Hq, Hkv, world, rank)
        ql, kl, vl = (t[sh.b0:sh.b1, a:b].to(dev).requires_grad_(True)
                      for t, (a, b) in ((q, (sh.h0, sh.h1)), (k, (sh.g0, sh.g1)), (v, (sh.g0, sh.g1))))
        o = sharded_attention(ql, kl, vl, sh, Hq, causal=True)
        o.backward(do[sh.b0:sh.b1, sh.h0:sh.h1].to(dev))
        torch.cuda.synchronize()
        gathered = []
        for t in (o.detach(), ql.grad, kl.grad, vl.grad):
            buf = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=dev)
            dist.all_gather_into_tensor(buf, t.contiguous())
            gathered.append(buf)
        torch.cuda.synchronize()
        if rank == 0:
            out.put((0, [g.cpu() for g in gathered]))
        else:
            out.put((rank, None))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_sharded_nccl_gather_matches_single_gpu_and_oracle():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 4 if n >= 4 else 2
    from tests.test_context_parallel import _collect
    from co_alibi_attn.sharding import shard_plan
    import co_alibi_attn
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, qu)) for r in range(world)]
    for p in procs:
        p.start()
    got = _collect(procs, qu, world, 600)
    B, Hq, Hkv, S, D = SHAPE
    G = Hq // Hkv
    q, k, v, do = make_inputs(B, Hq, Hkv, S, S, D, torch.float16, seed=51)
    full = [torch.empty_like(q), torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)]
    for r in range(world):
        sh = shard_plan(B, Hq, Hkv, world, r)
        for i, x in enumerate(got[0]):
            per = G if i < 2 else 1
            full[i][sh.b0:sh.b1, sh.g0 * per:sh.g1 * per] = x[r]
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o1 = co_alibi_attn.co_alibi_attention(qc, kc, vc, causal=True)
    o1.backward(do.cuda())
    torch.cuda.synchronize()
    for name, a, b in zip(("o", "dq", "dk", "dv"), full, (o1.detach(), qc.grad, kc.grad, vc.grad)):
        assert torch.equal(a, b.cpu()), f"{name}: gathered shards differ from the single-GPU run"
    scale = 1.0 / math.sqrt(D)
    o_ref, _, _, pav = oracle_fwd_pv(q, k, v, True, scale)
    ok, err = check_o(full[0], o_ref, torch.float16, pav)
    assert ok, f"O max-abs {err:.3e}"
    for name, x, r in zip(("dq", "dk", "dv"), full[1:], oracle_bwd(q, k, v, do, True, scale)):
        assert rel_err(x, r) <= GRAD_REL, name
