"""Host-resident batches: Co-ALiBi attention on pinned CPU tensors with the
host<->device copies overlapped with the kernels.

Every (batch, head) slice of the problem is independent (the reference kernels
launch one program per (batch*head, block): ``co_alibi_attn/co_alibi_attn.py:40``
and ``:83``), so the batch is cut into chunks -- one batch element and a range
of kv heads (with their query heads) each, contiguous in host memory -- and
pipelined over three CUDA streams: the copy-in of chunk c+1, the forward (and
backward) of chunk c and the copy-out of chunk c-1 run at the same time, and the
copies in the two PCIe directions overlap each other.  Every chunk runs with the
slopes of its global head indices, so results are identical to
``co_alibi_attention`` on the whole batch on the device.
"""
import torch

from .co_alibi_attn import _api_slopes, _bwd, _check_inputs, _fwd

__all__ = ["co_alibi_attention_from_host", "chunk_plan"]

# One (copy-in, compute, copy-out) stream triple per device, reused by every call:
# the caching allocator keeps freed blocks per stream, so fresh streams on each
# call would make every call allocate new device memory.
_streams = {}


def _stream_triple(dev):
    t = _streams.get(dev.index)
    if t is None:
        with torch.cuda.device(dev):
            t = (torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream())
        _streams[dev.index] = t
    return t


def _check_host(name, t, dtype):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cpu":
        raise ValueError(f"{name} must be a CPU (host) tensor, got {t.device}")
    if t.dtype != dtype:
        raise ValueError(f"{name} has dtype {t.dtype}, expected {dtype}")
    if t.dim() != 4:
        raise ValueError(f"{name} must be [B, H, S, D], got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def chunk_plan(B, Hkv, chunks):
    """The pieces a host batch goes through the device in: (batch element, kv heads
    [g0, g1)) triples covering every (b, kv head) unit once, in memory order.
    Pieces hold about m = B * Hkv / chunks kv heads (at most one batch element);
    from 4 chunks up the first batch element starts with pieces of 1, 2, 4, ...
    heads and the last one ends with them, so that the pipeline fills after a small copy-in and drains
    after a small kernel and copy-out.  A piece never crosses a batch element."""
    m = max(1, min(Hkv, -(-(B * Hkv) // chunks)))
    ramp = []
    while chunks >= 4 and (2 * ramp[-1] if ramp else 1) < m:
        ramp.append(2 * ramp[-1] if ramp else 1)

    def split(n):  # n heads in about n / m near-equal pieces
        k = max(1, round(n / m))
        return [n // k + (1 if i < n % k else 0) for i in range(k)] if n else []

    units = []
    for b in range(B):
        pre = ramp if b == 0 else []
        post = ramp[::-1] if b == B - 1 else []
        if sum(pre) + sum(post) > Hkv:
            pre, post = ([], []) if B > 1 or sum(ramp) > Hkv else (ramp, [])
        g = 0
        for sz in pre + split(Hkv - sum(pre) - sum(post)) + post:
            units.append((b, g, g + sz))
            g += sz
    return units


def co_alibi_attention_from_host(q, k, v, do=None, causal=True, sm_scale=None, bias_max=8.0, out=None,
                                 device=None, slopes=None, chunks=16):
    """Co-ALiBi attention of host tensors, streamed through one GPU.

    q: [B, Hq, Sq, D]; k, v: [B, Hkv, Skv, D]; ``do`` (optional): [B, Hq, Sq, D],
    the gradient of the output.  All contiguous CPU tensors of one dtype, ideally
    in pinned memory (pageable memory works but its copies do not overlap).
    Returns host tensors ``(o,)`` or, with ``do``, ``(o, dq, dk, dv)``; when
    ``out`` is given (a tuple of the same shapes, CPU tensors) the results are
    written there.  ``slopes`` (optional, [Hq]) replaces the slope table of
    ``co_alibi_attention`` (for instance the global-head slopes of a head shard).
    The batch goes through the device in about ``chunks`` pieces of (batch
    element, kv-head range), smaller at the start and the end (``chunk_plan``).
    The call returns once the results are in host memory.
    """
    _check_host("q", q, q.dtype)
    _check_host("k", k, q.dtype)
    _check_host("v", v, q.dtype)
    if do is not None:
        _check_host("do", do, q.dtype)
        if do.shape != q.shape:
            raise ValueError(f"do has shape {tuple(do.shape)}, expected {tuple(q.shape)}")
    B, Hq = q.shape[0], q.shape[1]
    Hkv = k.shape[1]
    if k.shape[0] != B or v.shape != k.shape or k.shape[-1] != q.shape[-1] or Hq % Hkv != 0:
        raise ValueError(f"inconsistent shapes q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}")
    if chunks < 1:
        raise ValueError("chunks must be >= 1")
    if slopes is not None and tuple(slopes.shape) != (Hq,):
        raise ValueError(f"slopes must have shape ({Hq},)")
    shapes = [q.shape] if do is None else [q.shape, q.shape, k.shape, v.shape]
    if out is None:
        pin = q.is_pinned()
        out = tuple(torch.empty(s, dtype=q.dtype, pin_memory=pin) for s in shapes)
    else:
        out = tuple(out)
        if len(out) != len(shapes) or any(o.shape != s or o.dtype != q.dtype or o.device.type != "cpu"
                                          or not o.is_contiguous() for o, s in zip(out, shapes)):
            raise ValueError("out must hold contiguous CPU tensors of the result shapes and dtype")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if sm_scale is None:
        sm_scale = 1.0 / (q.shape[-1] ** 0.5)
    G = Hq // Hkv
    units = chunk_plan(B, Hkv, chunks)
    gstep = max(g1 - g0 for _, g0, g1 in units)
    n = len(units)
    ins = [q, k, v] + ([] if do is None else [do])
    with torch.cuda.device(dev):
        sl = (_api_slopes(Hq, bias_max, q.dtype, dev) if slopes is None
              else slopes.to(device=dev).contiguous())
        caller = torch.cuda.current_stream()
        s_in, s_comp, s_out = _stream_triple(dev)
        for s in (s_in, s_comp, s_out):
            s.wait_stream(caller)
        # two device slots per input: chunk c+2 overwrites chunk c's inputs once its compute finished
        sizes = [(1, gstep * G) + tuple(q.shape[2:]), (1, gstep) + tuple(k.shape[2:]),
                 (1, gstep) + tuple(v.shape[2:]), (1, gstep * G) + tuple(q.shape[2:])]
        slots = [[torch.empty(sz, dtype=q.dtype, device=dev) for sz in sizes[:len(ins)]] for _ in range(min(2, n))]
        comp_done = []
        keep = []
        for c, (b, g0, g1) in enumerate(units):
            h0, h1 = g0 * G, g1 * G
            hosts = [q[b:b + 1, h0:h1], k[b:b + 1, g0:g1], v[b:b + 1, g0:g1]]
            if do is not None:
                hosts.append(do[b:b + 1, h0:h1])
            buf = [t[:, : h.shape[1]] for t, h in zip(slots[c % 2], hosts)]
            with torch.cuda.stream(s_in):
                if c >= 2:
                    s_in.wait_event(comp_done[c - 2])
                for d, h in zip(buf, hosts):
                    d.copy_(h, non_blocking=True)
                h2d = torch.cuda.Event()
                h2d.record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(h2d)
                # the kernels the autograd Function runs, called directly (no graph per chunk)
                slc = sl[h0:h1]
                if c == 0:
                    _check_inputs(buf[0], buf[1], buf[2], slc)
                o, lse, rowsig = _fwd(buf[0], buf[1], buf[2], slc, causal, sm_scale)
                if do is None:
                    res = (o,)
                else:
                    res = (o,) + tuple(_bwd(buf[0], buf[1], buf[2], o, buf[3], lse, rowsig, slc, causal, sm_scale))
                ev = torch.cuda.Event()
                ev.record(s_comp)
                comp_done.append(ev)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                dsts = [out[0][b:b + 1, h0:h1]]
                if do is not None:
                    dsts += [out[1][b:b + 1, h0:h1], out[2][b:b + 1, g0:g1], out[3][b:b + 1, g0:g1]]
                for h, d in zip(dsts, res):
                    d.record_stream(s_out)
                    h.copy_(d, non_blocking=True)
            keep.append(res)
        for s in (s_in, s_comp, s_out):
            caller.wait_stream(s)
        s_out.synchronize()
    return out
