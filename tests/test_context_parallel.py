"""Sequence-sharded (context-parallel) Co-ALiBi.

CPU: the shard merge and the backward carries with float64 oracle stand-ins for
the per-shard kernels, in one process and as a gloo ring of three ranks, against
the oracle on the whole sequence (tight: the algebra is exact; what remains is the
oracle's 1e-9 guard on each softmax denominator, which sharding repeats per shard).
GPU: the same with the sm_100a kernels (coalibi_fwd / coalibi_bwd_carry) against
the float64 oracle at the usual tolerances, and against the unsharded kernels."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests._common import make_inputs, oracle_fwd_pv, oracle_bwd, check_o, rel_err, GRAD_REL

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# --- float64 stand-ins for the per-shard kernels (test only) -----------------
def _expand(x, hq):
    return x if x.shape[1] == hq else x.repeat_interleave(hq // x.shape[1], dim=1)


def _group(dx, hkv):
    b, hq, s, d = dx.shape
    return dx if hq == hkv else dx.view(b, hkv, hq // hkv, s, d).sum(2)


def oracle_shard_fwd(q, k, v, slopes, causal, sm_scale):
    """(o, lse, rowsig) of one key shard: what coalibi_fwd returns for it."""
    from oracle import coalibi_oracle as orc
    return orc.forward(q, k, v, slopes, causal, sm_scale, torch.float64)


def oracle_shard_bwd(q, k, v, o, do, lse, rowsig, slopes, causal, sm_scale, carry):
    """(dq, dk, dv) of one key shard given the whole row's o / lse / do, rowsig of
    the shard and the keys right of it, and the dA prefix carried in from the left:
    the contract of coalibi_bwd_carry, written out densely in float64."""
    from oracle import coalibi_oracle as orc
    Hq, Hkv, Sq, Skv = q.shape[1], k.shape[1], q.shape[2], k.shape[2]
    kf, vf = _expand(k.double(), Hq), _expand(v.double(), Hq)
    sl = slopes.double().view(1, Hq, 1, 1)
    mask = orc.causal_mask(Sq, Skv, causal).view(1, 1, Sq, Skv)
    p = q.double() @ kf.transpose(-1, -2) * sm_scale
    sig = torch.sigmoid(p).masked_fill(mask, 0.0)
    z = rowsig.double().unsqueeze(-1) - (torch.cumsum(sig, -1) - sig)   # global suffix sum
    P = torch.exp(p - sl * z - lse.double().unsqueeze(-1)).masked_fill(mask, 0.0)
    dP = do.double() @ vf.transpose(-1, -2)
    delta = (do.double() * o.double()).sum(-1, keepdim=True)
    dA = (P * (dP - delta)).masked_fill(mask, 0.0)
    c = carry.double().unsqueeze(-1) + torch.cumsum(dA, -1)
    dS = (dA - sl * sig * (1 - sig) * c).masked_fill(mask, 0.0)
    dq = dS @ kf * sm_scale
    dk = dS.transpose(-1, -2) @ q.double() * sm_scale
    dv = P.transpose(-1, -2) @ do.double()
    return dq, _group(dk, Hkv), _group(dv, Hkv)


STAND_INS = (oracle_shard_fwd, oracle_shard_bwd)


def _whole(q, k, v, do, causal, scale):
    from oracle import coalibi_oracle as orc
    sl = orc.api_slopes(q.shape[1], 8.0, q.dtype)
    return orc.forward_backward(q, k, v, do, sl, causal, scale, torch.float64)


@pytest.mark.parametrize("shape", [
    # B, Hq, Hkv, S, D, n_shards, causal
    (1, 2, 2, 48, 16, 4, True),
    (2, 4, 2, 37, 8, 3, True),      # GQA, ragged last shard
    (1, 3, 3, 50, 16, 4, False),
    (1, 4, 1, 20, 8, 7, False),     # more shards than fit evenly
])
def test_sharded_merge_is_exact_with_oracle_shards(shape):
    from co_alibi_attn.context_parallel import sequence_sharded_attention
    B, Hq, Hkv, S, D, n, causal = shape
    q, k, v, do = (t.double() for t in make_inputs(B, Hq, Hkv, S, S, D, torch.float32, seed=S + n))
    scale = 1.0 / math.sqrt(D)
    q, k, v = (t.requires_grad_(True) for t in (q, k, v))
    o = sequence_sharded_attention(q, k, v, n, causal=causal, sm_scale=scale, _shard_fns=STAND_INS)
    o.backward(do)
    o_r, _, _, dq_r, dk_r, dv_r = _whole(q.detach(), k.detach(), v.detach(), do, causal, scale)
    assert (o.detach() - o_r).abs().max().item() < 1e-8
    for name, x, r in (("dq", q.grad, dq_r), ("dk", k.grad, dk_r), ("dv", v.grad, dv_r)):
        assert rel_err(x, r) < 1e-8, name


def test_sharded_non_causal_different_query_and_key_lengths():
    """Non-causal rows need no shared boundaries: 30 query rows in 3 shards against
    70 keys in 3 shards of 24, 24 and 22."""
    from co_alibi_attn.context_parallel import sequence_sharded_attention
    q, k, v, do = (t.double() for t in make_inputs(2, 4, 2, 30, 70, 8, torch.float32, seed=12))
    q, k, v = (t.requires_grad_(True) for t in (q, k, v))
    o = sequence_sharded_attention(q, k, v, 3, causal=False, sm_scale=0.4, _shard_fns=STAND_INS)
    o.backward(do)
    o_r, _, _, dq_r, dk_r, dv_r = _whole(q.detach(), k.detach(), v.detach(), do, False, 0.4)
    assert (o.detach() - o_r).abs().max().item() < 1e-8
    for name, x, r in (("dq", q.grad, dq_r), ("dk", k.grad, dk_r), ("dv", v.grad, dv_r)):
        assert rel_err(x, r) < 1e-8, name


def test_sharded_causal_needs_matching_boundaries():
    from co_alibi_attn.context_parallel import sequence_sharded_attention
    q, k, v, _ = (t.double() for t in make_inputs(1, 2, 2, 20, 30, 8, torch.float32))
    with pytest.raises(ValueError):
        sequence_sharded_attention(q, k, v, 3, causal=True, _shard_fns=STAND_INS)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _collect(procs, qu, n, limit):
    """n results from the workers' queue; fails fast when a worker has died."""
    import queue
    import time
    got, t0 = {}, time.time()
    while len(got) < n:
        try:
            r, val = qu.get(timeout=2)
            got[r] = val
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead, f"worker exited with {dead}"
            assert time.time() - t0 < limit, "workers timed out"
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return got


def _local(x, layout, world, rank):
    """This rank's chunks of x (sequence axis 2), in chunk_layout order."""
    from co_alibi_attn.context_parallel import chunk_layout
    own = chunk_layout(layout, world, rank)
    n = world * len(own)
    L = x.shape[2] // n
    return torch.cat([x[:, :, i * L:(i + 1) * L] for i in own], dim=2)


def _global(parts, layout, world):
    """Inverse of _local over all ranks: the whole sequence from every rank's chunks."""
    from co_alibi_attn.context_parallel import chunk_layout
    chunks = {}
    for r in range(world):
        own = chunk_layout(layout, world, r)
        L = parts[r].shape[2] // len(own)
        for j, i in enumerate(own):
            chunks[i] = parts[r][:, :, j * L:(j + 1) * L]
    return torch.cat([chunks[i] for i in sorted(chunks)], dim=2)


def _ring_worker(rank, world, port, causal, layout, out):
    import sys
    for p in (ROOT, os.path.join(ROOT, "co-alibi_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    from co_alibi_attn.context_parallel import ring_attention
    from tests.test_context_parallel import STAND_INS, _local
    from tests._common import make_inputs
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v, do = (t.double() for t in make_inputs(1, 4, 2, 12 * world, 12 * world, 8, torch.float32, seed=5))
        ql, kl, vl = (_local(t, layout, world, rank).requires_grad_(True) for t in (q, k, v))
        o = ring_attention(ql, kl, vl, causal=causal, sm_scale=0.3, layout=layout, _shard_fns=STAND_INS)
        o.backward(_local(do, layout, world, rank))
        out.put((rank, [t.detach().numpy().copy() for t in (o, ql.grad, kl.grad, vl.grad)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
@pytest.mark.parametrize("causal", [True, False])
def test_ring_gloo_three_ranks_with_oracle_shards(causal, layout):
    """Three gloo ranks, each with its chunks of the sequence, key / value shards and
    dk / dv accumulators passed around the ring (sends overlapped with the pairs):
    the reassembled outputs and gradients equal the oracle on the whole sequence."""
    world = 3
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, causal, layout, qu)) for r in range(world)]
    for p in procs:
        p.start()
    got = _collect(procs, qu, world, 300)
    q, k, v, do = (t.double() for t in make_inputs(1, 4, 2, 12 * world, 12 * world, 8, torch.float32, seed=5))
    ref = _whole(q, k, v, do, causal, 0.3)
    # worker order (o, dq, dk, dv); forward_backward order (o, lse, rowsig, dq, dk, dv)
    for j, (i, name) in enumerate(((0, "o"), (3, "dq"), (4, "dk"), (5, "dv"))):
        x = _global([torch.from_numpy(got[r][j]) for r in range(world)], layout, world)
        assert (x - ref[i]).abs().max().item() < 1e-8, name


def test_chunk_layouts():
    from co_alibi_attn.context_parallel import chunk_layout
    assert [chunk_layout("contiguous", 4, r) for r in range(4)] == [[0], [1], [2], [3]]
    zz = [chunk_layout("zigzag", 4, r) for r in range(4)]
    assert zz == [[0, 7], [1, 6], [2, 5], [3, 4]]
    # causal work per rank (visible chunk pairs, diagonal counted as 1/2) is equal under zig-zag
    assert len({sum(i + 0.5 for i in own) for own in zz}) == 1
    with pytest.raises(ValueError):
        chunk_layout("striped", 4, 0)


def test_ring_without_process_group_is_one_rank():
    """No process group: one rank holding the whole sequence (zig-zag: its two halves)."""
    from co_alibi_attn.context_parallel import ring_attention
    q, k, v, do = (t.double() for t in make_inputs(2, 4, 2, 40, 40, 8, torch.float32, seed=8))
    q, k, v = (t.requires_grad_(True) for t in (q, k, v))
    o = ring_attention(q, k, v, causal=True, sm_scale=0.3, layout="zigzag", _shard_fns=STAND_INS)
    o.backward(do)
    ref = _whole(q.detach(), k.detach(), v.detach(), do, True, 0.3)
    for x, i in ((o.detach(), 0), (q.grad, 3), (k.grad, 4), (v.grad, 5)):
        assert (x - ref[i]).abs().max().item() < 1e-8
    with pytest.raises(ValueError):
        ring_attention(q[:, :, :39], k[:, :, :39], v[:, :, :39], layout="zigzag", _shard_fns=STAND_INS)


# --- GPU: the sm_100a shard kernels ------------------------------------------
GPU_CASES = [
    # B, Hq, Hkv, S, D, n_shards, causal, dtype
    (1, 4, 4, 1024, 128, 4, True, torch.float16),
    (2, 8, 2, 700, 64, 3, False, torch.bfloat16),     # GQA, ragged shards
    (1, 8, 2, 1000, 128, 2, True, torch.bfloat16),
    (1, 2, 2, 64, 128, 5, True, torch.float16),       # 13-row shards: the decode forward per shard
    (1, 6, 3, 777, 64, 3, True, torch.float16),       # D = 64 pass B with a carry, causal, GQA, 259-row shards
]


@pytest.mark.gpu
def test_sharded_kernels_non_causal_rectangular():
    """Non-causal, 300 query rows against 1000 keys, 4 shards each side (GQA, bf16)."""
    import co_alibi_attn
    from co_alibi_attn.context_parallel import sequence_sharded_attention
    q, k, v, do = make_inputs(1, 8, 2, 300, 1000, 128, torch.bfloat16, seed=77)
    scale = 1.0 / math.sqrt(128)
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = sequence_sharded_attention(qc, kc, vc, 4, causal=False, sm_scale=scale)
    o.backward(do.cuda())
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0
    o_ref, _, _, pav = oracle_fwd_pv(q, k, v, False, scale)
    ok, err = check_o(o.detach().cpu(), o_ref, torch.bfloat16, pav)
    assert ok, f"O max-abs {err:.3e}"
    for name, x, r in zip(("dq", "dk", "dv"), (qc.grad, kc.grad, vc.grad), oracle_bwd(q, k, v, do, False, scale)):
        assert rel_err(x.cpu(), r) <= GRAD_REL, name


@pytest.mark.gpu
@pytest.mark.parametrize("case", GPU_CASES,
                         ids=[f"B{c[0]}H{c[1]}-{c[2]}S{c[3]}D{c[4]}n{c[5]}{'c' if c[6] else 'nc'}" for c in GPU_CASES])
def test_sharded_kernels_match_oracle(case):
    import co_alibi_attn
    from co_alibi_attn.context_parallel import sequence_sharded_attention
    B, Hq, Hkv, S, D, n, causal, dt = case
    q, k, v, do = make_inputs(B, Hq, Hkv, S, S, D, dt, seed=S + 3 * n)
    scale = 1.0 / math.sqrt(D)
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = sequence_sharded_attention(qc, kc, vc, n, causal=causal, sm_scale=scale)
    o.backward(do.cuda())
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0
    o_ref, _, _, pav = oracle_fwd_pv(q, k, v, causal, scale)
    ok, err = check_o(o.detach().cpu(), o_ref, dt, pav)
    assert ok, f"O max-abs {err:.3e}"
    dq_r, dk_r, dv_r = oracle_bwd(q, k, v, do, causal, scale)
    for name, x, r in (("dq", qc.grad, dq_r), ("dk", kc.grad, dk_r), ("dv", vc.grad, dv_r)):
        e = rel_err(x.cpu(), r)
        assert e <= GRAD_REL, f"{name} relative error {e:.3e}"
    # and close to the unsharded kernels
    qu, ku, vu = (t.cuda().requires_grad_(True) for t in (q, k, v))
    ou = co_alibi_attn.co_alibi_attention(qu, ku, vu, causal=causal, sm_scale=scale)
    ou.backward(do.cuda())
    # (bf16 outputs differ by an ulp or two where the merge rounds differently)
    assert rel_err(o.detach().cpu(), ou.detach().cpu()) < 5e-3
    assert rel_err(qc.grad.cpu(), qu.grad.cpu()) < GRAD_REL


@pytest.mark.gpu
def test_ring_one_rank_zigzag_kernels_match_oracle():
    """ring_attention without a process group (one rank, two zig-zag halves) on the
    kernels: the code path of bench.py --config cp at N=1."""
    import co_alibi_attn
    from co_alibi_attn.context_parallel import ring_attention
    q, k, v, do = make_inputs(1, 8, 2, 1024, 1024, 128, torch.bfloat16, seed=41)
    scale = 1.0 / math.sqrt(128)
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = ring_attention(qc, kc, vc, causal=True, layout="zigzag")
    o.backward(do.cuda())
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0
    o_ref, _, _, pav = oracle_fwd_pv(q, k, v, True, scale)
    ok, err = check_o(o.detach().cpu(), o_ref, torch.bfloat16, pav)
    assert ok, f"O max-abs {err:.3e}"
    for name, x, r in zip(("dq", "dk", "dv"), (qc.grad, kc.grad, vc.grad), oracle_bwd(q, k, v, do, True, scale)):
        assert rel_err(x.cpu(), r) <= GRAD_REL, name


def _nccl_ring_worker(rank, world, port, out):
    import sys
    for p in (ROOT, os.path.join(ROOT, "co-alibi_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    from co_alibi_attn.context_parallel import ring_attention
    from tests._common import make_inputs
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from tests.test_context_parallel import _local
        S = 512 * world
        q, k, v, do = make_inputs(1, 8, 2, S, S, 128, torch.bfloat16, seed=31)
        ql, kl, vl = (_local(t, "zigzag", world, rank).cuda().requires_grad_(True) for t in (q, k, v))
        o = ring_attention(ql, kl, vl, causal=True, layout="zigzag")
        o.backward(_local(do, "zigzag", world, rank).cuda())
        torch.cuda.synchronize()
        out.put((rank, [t.detach().float().cpu().numpy().copy() for t in (o, ql.grad, kl.grad, vl.grad)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_ring_nccl_matches_oracle():
    """Zig-zag chunks on every GPU, the ring over NCCL (needs 2 or more GPUs)."""
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two GPUs")
    world = min(world, 4)
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_ring_worker, args=(r, world, port, qu)) for r in range(world)]
    for p in procs:
        p.start()
    got = _collect(procs, qu, world, 600)
    S = 512 * world
    q, k, v, do = make_inputs(1, 8, 2, S, S, 128, torch.bfloat16, seed=31)
    scale = 1.0 / math.sqrt(128)
    cat = lambda i: _global([torch.from_numpy(got[r][i]) for r in range(world)], "zigzag", world)  # noqa: E731
    o_ref, _, _, pav = oracle_fwd_pv(q, k, v, True, scale)
    ok, err = check_o(cat(0).to(torch.bfloat16), o_ref, torch.bfloat16, pav)
    assert ok, f"O max-abs {err:.3e}"
    for i, r in zip((1, 2, 3), oracle_bwd(q, k, v, do, True, scale)):
        assert rel_err(cat(i), r) <= GRAD_REL
