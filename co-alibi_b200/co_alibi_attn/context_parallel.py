"""Sequence (context) parallel Co-ALiBi: rows whose keys are split into shards.

The reference has no sequence parallelism (its backward keeps O(S^2) partials,
``co_alibi_attn/co_alibi_attn.py:91-96``); this module evaluates attention over
key shards with the sm_100a kernels and merges the pieces exactly.

Forward.  For a query row and key shard c, the kernels compute the shard's
output o_c, log-sum-exp lse_c and sigmoid total T_c with the sigmoid suffix sum z
restarted at the shard's right end.  The keys right of shard c add
R_c = sum_{c' > c} T_c' to every z in it, i.e. shift its logits by -slope * R_c,
so lse'_c = lse_c - slope * R_c, and the whole row is the log-sum-exp merge:
LSE = logsumexp_c lse'_c, O = sum_c exp(lse'_c - LSE) o_c, rowsig = sum_c T_c.

Backward.  Per key shard the backward kernels take the whole row's O, LSE and dO,
rowsig = T_c + R_c (so z is the global suffix) and the dA prefix carried in from
the shards to the left, C_c = sum_{c' < c} w_c' (dO . o_c' - delta) with
w_c = exp(lse'_c - LSE) and delta = dO . O (coalibi_bwd_carry); dq sums over the
shards, dk / dv of a shard over the query shards that see it.

With causal masking the query and key shards share boundaries: query shard r sees
key shards c < r unmasked and shard r with the top-left mask.

``sequence_sharded_attention`` runs the shards one after another on one device
(the building block, and its check); ``ring_attention`` gives every rank of a
process group chunks of the sequence (one contiguous shard, or two zig-zag
chunks that balance the causal work) and passes key / value shards (and, in the
backward, dk / dv accumulators) around the ring.
"""
import torch
import torch.distributed as dist

from .co_alibi_attn import _api_slopes, _bwd, _check_inputs, _fwd

__all__ = ["sequence_sharded_attention", "ring_attention", "chunk_layout"]


def _kernel_fwd(q, k, v, slopes, causal, sm_scale):
    return _fwd(q.contiguous(), k.contiguous(), v.contiguous(), slopes, causal, sm_scale)


def _kernel_bwd(q, k, v, o, do, lse, rowsig, slopes, causal, sm_scale, carry_in):
    return _bwd(q.contiguous(), k.contiguous(), v.contiguous(), o, do, lse.contiguous(), rowsig.contiguous(),
                slopes, causal, sm_scale, dA_carry_in=carry_in.contiguous())


def _acc(dtype):
    """float32 for the merge arithmetic and accumulators (float64 kept, for float64 stand-ins)."""
    return torch.promote_types(dtype, torch.float32)


def _f(x):
    return x if x.dtype == _acc(x.dtype) else x.float()


def _dot(a, b):
    """Row dot products over D in the accumulator precision (one converted copy)."""
    return a.to(_acc(a.dtype), copy=True).mul_(b).sum(-1)


class _RowMerge:
    """Right-to-left merge of one query shard's key-shard partials."""

    def __init__(self, slopes):
        self.sl = _f(slopes).view(1, -1, 1)
        self.parts = {}  # c -> (o_c, lse_c, T_c)

    def add(self, c, o_c, lse_c, t_c):
        self.parts[c] = (o_c, _f(lse_c), _f(t_c))

    def finish(self, dtype):
        """Merged (O, LSE, rowsig) and, per shard, (o_c, shifted lse'_c, T_c, R_c)."""
        R = None
        lse_all = o_all = None
        self.shifted = {}
        for c in sorted(self.parts, reverse=True):  # right to left
            o_c, lse_c, t_c = self.parts[c]
            if R is None:
                R = torch.zeros_like(t_c)
            lse_p = lse_c - self.sl.to(lse_c.dtype) * R
            self.shifted[c] = (o_c, lse_p, t_c, R)
            if lse_all is None:
                lse_all, o_all = lse_p, o_c.to(_acc(o_c.dtype), copy=True)
            else:
                new = torch.logaddexp(lse_all, lse_p)
                o_all.mul_(torch.exp(lse_all - new).unsqueeze(-1)).addcmul_(o_c, torch.exp(lse_p - new).unsqueeze(-1))
                lse_all = new
            R = R + t_c
        self.lse, self.rowsig = lse_all, R
        return o_all.to(dtype), lse_all, R

    def carries(self, o, do):
        """dA carry-in C_c of every shard (left to right) for the row's O and dO."""
        delta = _dot(do, o)
        C, out = torch.zeros_like(delta), {}
        for c in sorted(self.shifted):
            o_c, lse_p, t_c, R = self.shifted[c]
            out[c] = C
            w = torch.exp(lse_p - self.lse)
            C = C + w * (_dot(do, o_c) - delta)
        return out


def _split(x, n):
    S = x.shape[2]
    step = -(-S // n)
    return [x[:, :, i:i + step] for i in range(0, S, step)]


class _SequenceSharded(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, slopes, n_shards, causal, sm_scale, fwd_fn, bwd_fn):
        qs, ks, vs = _split(q, n_shards), _split(k, n_shards), _split(v, n_shards)
        if causal and [t.shape[2] for t in qs] != [t.shape[2] for t in ks]:
            raise ValueError("causal sequence sharding needs Sq == Skv (shared shard boundaries)")
        outs, merges = [], []
        for r, q_r in enumerate(qs):
            m = _RowMerge(slopes)
            for c in range(len(ks)):
                if causal and c > r:
                    continue
                m.add(c, *fwd_fn(q_r, ks[c], vs[c], slopes, causal and c == r, sm_scale))
            o_r, _, _ = m.finish(q.dtype)
            outs.append(o_r)
            merges.append(m)
        o = torch.cat(outs, dim=2)
        ctx.save_for_backward(q, k, v, o, slopes)
        ctx.merges, ctx.n_shards, ctx.causal, ctx.sm_scale = merges, n_shards, causal, sm_scale
        ctx.bwd_fn = bwd_fn
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, slopes = ctx.saved_tensors
        n, causal, scale = ctx.n_shards, ctx.causal, ctx.sm_scale
        qs, ks, vs = _split(q, n), _split(k, n), _split(v, n)
        os_, dos = _split(o, n), _split(do.to(q.dtype).contiguous(), n)
        acc = torch.promote_types(q.dtype, torch.float32)
        dq = [torch.zeros(t.shape, dtype=acc, device=q.device) for t in qs]
        dk = [torch.zeros(t.shape, dtype=acc, device=q.device) for t in ks]
        dv = [torch.zeros(t.shape, dtype=acc, device=q.device) for t in vs]
        for r, m in enumerate(ctx.merges):
            o_r, do_r = os_[r].contiguous(), dos[r].contiguous()
            carry = m.carries(o_r, do_r)
            for c, (o_c, lse_p, t_c, R) in m.shifted.items():
                g = ctx.bwd_fn(qs[r], ks[c], vs[c], o_r, do_r, m.lse, t_c + R, slopes, causal and c == r, scale,
                               carry[c])
                dq[r].add_(g[0])
                dk[c].add_(g[1])
                dv[c].add_(g[2])
        cat = lambda xs, t: torch.cat(xs, dim=2).to(t.dtype)  # noqa: E731
        return cat(dq, q), cat(dk, k), cat(dv, v), None, None, None, None, None, None


def sequence_sharded_attention(q, k, v, n_shards, causal=True, sm_scale=None, bias_max=8.0, _shard_fns=None):
    """``co_alibi_attention`` evaluated over ``n_shards`` sequence shards on one
    device and merged exactly (forward and backward); the single-device form of
    ``ring_attention``.  ``_shard_fns`` as in ``ring_attention``."""
    if sm_scale is None:
        sm_scale = 1.0 / (q.shape[-1] ** 0.5)
    fwd_fn, bwd_fn = _shard_fns or (_kernel_fwd, _kernel_bwd)
    slopes = _api_slopes(q.shape[1], bias_max, q.dtype, q.device)
    if _shard_fns is None:
        _check_inputs(q, k, v, slopes)
    return _SequenceSharded.apply(q.contiguous(), k.contiguous(), v.contiguous(), slopes, n_shards, causal, sm_scale,
                                  fwd_fn, bwd_fn)


# ---------------------------------------------------------------------------
# ring over a process group: every rank holds equal-length chunks of the sequence
# ---------------------------------------------------------------------------
def chunk_layout(layout, world, rank):
    """Global chunk indices (in order) that ``rank`` holds.  "contiguous": the
    sequence in ``world`` chunks, chunk r on rank r.  "zigzag": ``2 * world``
    chunks, rank r holding chunks r and 2 * world - 1 - r, so that with causal
    masking every rank has the same number of visible scores."""
    if layout == "contiguous":
        return [rank]
    if layout == "zigzag":
        return [rank, 2 * world - 1 - rank]
    raise ValueError(f"unknown layout {layout!r} (contiguous or zigzag)")


def _world_rank(group):
    if group is None and not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _ring_start(tensors, group):
    """Start sending ``tensors`` to the next rank and receiving the previous
    rank's; returns (receive buffers, requests)."""
    world, rank = _world_rank(group)
    glob = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
    nxt, prv = glob((rank + 1) % world), glob((rank - 1) % world)
    recv = [torch.empty_like(t) for t in tensors]
    ops = [dist.P2POp(dist.isend, t, nxt, group) for t in tensors] + \
          [dist.P2POp(dist.irecv, t, prv, group) for t in recv]
    return recv, dist.batch_isend_irecv(ops)


def _finish(recv, reqs):
    for r in reqs:
        r.wait()
    return recv


def _pieces(x, n):
    L = x.shape[2] // n
    return [x[:, :, i * L:(i + 1) * L] for i in range(n)]


class _Ring(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, slopes, causal, sm_scale, group, layout, fwd_fn, bwd_fn):
        world, rank = _world_rank(group)
        own = chunk_layout(layout, world, rank)
        qc = dict(zip(own, _pieces(q, len(own))))
        merges = {i: _RowMerge(slopes) for i in own}
        kv = [k, v]
        for s in range(world):
            src = (rank - s) % world
            pending = _ring_start(kv, group) if s + 1 < world else None   # next shard, overlapped
            for j, kj, vj in zip(chunk_layout(layout, world, src), _pieces(kv[0], len(own)), _pieces(kv[1], len(own))):
                for i in own:
                    if not (causal and j > i):
                        merges[i].add(j, *fwd_fn(qc[i], kj, vj, slopes, causal and i == j, sm_scale))
            if pending is not None:
                kv = _finish(*pending)
        o = torch.cat([merges[i].finish(q.dtype)[0] for i in own], dim=2)
        ctx.save_for_backward(q, k, v, o, slopes)
        ctx.merges, ctx.causal, ctx.sm_scale, ctx.group, ctx.layout, ctx.bwd_fn = \
            merges, causal, sm_scale, group, layout, bwd_fn
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, slopes = ctx.saved_tensors
        group, merges, causal, scale, layout = ctx.group, ctx.merges, ctx.causal, ctx.sm_scale, ctx.layout
        world, rank = _world_rank(group)
        own = chunk_layout(layout, world, rank)
        n = len(own)
        do = do.to(q.dtype).contiguous()
        acc_t = torch.promote_types(q.dtype, torch.float32)
        qc, oc, doc = (dict(zip(own, [t.contiguous() for t in _pieces(x, n)])) for x in (q, o, do))
        carries = {i: merges[i].carries(oc[i], doc[i]) for i in own}
        dq = {i: torch.zeros(qc[i].shape, dtype=acc_t, device=q.device) for i in own}
        kv, acc, acc_pending = [k, v], None, None
        for s in range(world):
            src = (rank - s) % world
            kv_pending = _ring_start(kv, group) if s + 1 < world else None
            gk = torch.zeros(k.shape, dtype=acc_t, device=k.device)
            gv = torch.zeros(v.shape, dtype=acc_t, device=v.device)
            for jj, (j, kj, vj) in enumerate(zip(chunk_layout(layout, world, src), _pieces(kv[0], n),
                                                 _pieces(kv[1], n))):
                L = kj.shape[2]
                for i in own:
                    if j not in merges[i].shifted:
                        continue
                    o_c, lse_p, t_c, R = merges[i].shifted[j]
                    g = ctx.bwd_fn(qc[i], kj, vj, oc[i], doc[i], merges[i].lse, t_c + R, slopes,
                                   causal and i == j, scale, carries[i][j])
                    dq[i].add_(g[0])
                    gk[:, :, jj * L:(jj + 1) * L].add_(g[1])
                    gv[:, :, jj * L:(jj + 1) * L].add_(g[2])
            # the visiting shard's dk / dv accumulators arrive while its pairs computed
            if acc_pending is not None:
                acc = _finish(*acc_pending)
                gk.add_(acc[0])
                gv.add_(acc[1])
            acc_pending = _ring_start([gk, gv], group) if world > 1 else ([gk, gv], [])
            if kv_pending is not None:
                kv = _finish(*kv_pending)
        # after `world` passes the accumulators of this rank's own chunks are back here
        dk, dv = _finish(*acc_pending)
        dq = torch.cat([dq[i] for i in own], dim=2)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None, None, None, None, None, None


def ring_attention(q, k, v, causal=True, sm_scale=None, bias_max=8.0, group=None, layout="contiguous",
                   _shard_fns=None):
    """Co-ALiBi attention over a sequence split across the ranks of ``group``.
    Rank r passes its chunks of q [B, Hq, S_r, D] and k, v [B, Hkv, S_r, D] (all
    heads; every rank the same S_r), concatenated in the order ``chunk_layout``
    gives -- one contiguous shard, or with ``layout="zigzag"`` chunks r and
    2 * world - 1 - r of a sequence cut into 2 * world -- and gets its rows of the
    output, with gradients for its chunks.  Key / value shards travel around the
    ring, each send overlapped with the pairs computed on the shard before it; no
    rank holds the whole sequence.  ``_shard_fns`` (tests only) replaces the
    per-shard kernels with a (forward, backward) pair of the same signature."""
    if sm_scale is None:
        sm_scale = 1.0 / (q.shape[-1] ** 0.5)
    fwd_fn, bwd_fn = _shard_fns or (_kernel_fwd, _kernel_bwd)
    slopes = _api_slopes(q.shape[1], bias_max, q.dtype, q.device)
    if _shard_fns is None:
        _check_inputs(q, k, v, slopes)
    n = len(chunk_layout(layout, 1, 0))
    if q.shape[2] % n or k.shape[2] != q.shape[2]:
        raise ValueError(f"ring_attention: q and k / v need the same sequence length, a multiple of {n}")
    return _Ring.apply(q.contiguous(), k.contiguous(), v.contiguous(), slopes, causal, sm_scale, group, layout,
                       fwd_fn, bwd_fn)
