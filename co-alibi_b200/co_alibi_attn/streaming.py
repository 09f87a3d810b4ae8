"""Host-resident batches: Co-ALiBi attention on pinned CPU tensors with the
host<->device copies overlapped with the kernels.

Every (batch, head) slice of the problem is independent (the reference kernels
launch one program per (batch*head, block): ``co_alibi_attn/co_alibi_attn.py:40``
and ``:83``), so the batch is cut into chunks of batch elements and pipelined
over three CUDA streams: the copy-in of chunk c+1, the forward (and backward)
of chunk c and the copy-out of chunk c-1 run at the same time, and the copies
in the two PCIe directions overlap each other.  Results are identical to
``co_alibi_attention`` on the whole batch on the device.
"""
import torch

from .co_alibi_attn import co_alibi_attention

__all__ = ["co_alibi_attention_from_host"]

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


def co_alibi_attention_from_host(q, k, v, do=None, causal=True, sm_scale=None, bias_max=8.0, out=None,
                                 device=None, chunk=1, fn=None):
    """Co-ALiBi attention of host tensors, streamed through one GPU.

    q: [B, Hq, Sq, D]; k, v: [B, Hkv, Skv, D]; ``do`` (optional): [B, Hq, Sq, D],
    the gradient of the output.  All CPU tensors of one dtype, ideally in pinned
    memory (pageable memory works but its copies do not overlap).  Returns host
    tensors ``(o,)`` or, with ``do``, ``(o, dq, dk, dv)``; when ``out`` is given
    (a tuple of the same shapes, pinned CPU tensors) the results are written
    there.  ``chunk`` batch elements go through the device at a time.  ``fn``
    (optional) replaces the per-chunk attention call: ``fn(q, k, v) -> o`` on
    device tensors (for instance a head shard with global-head slopes).  The
    call returns once the results are in host memory.
    """
    _check_host("q", q, q.dtype)
    _check_host("k", k, q.dtype)
    _check_host("v", v, q.dtype)
    if do is not None:
        _check_host("do", do, q.dtype)
        if do.shape != q.shape:
            raise ValueError(f"do has shape {tuple(do.shape)}, expected {tuple(q.shape)}")
    B = q.shape[0]
    if k.shape[0] != B or v.shape != k.shape or k.shape[-1] != q.shape[-1]:
        raise ValueError(f"inconsistent shapes q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}")
    if chunk < 1:
        raise ValueError("chunk must be >= 1")
    shapes = [q.shape] if do is None else [q.shape, q.shape, k.shape, v.shape]
    if out is None:
        pin = q.is_pinned()
        out = tuple(torch.empty(s, dtype=q.dtype, pin_memory=pin) for s in shapes)
    else:
        out = tuple(out)
        if len(out) != len(shapes) or any(o.shape != s or o.dtype != q.dtype or o.device.type != "cpu"
                                          for o, s in zip(out, shapes)):
            raise ValueError("out must hold CPU tensors of the result shapes and dtype")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if fn is None:
        def fn(q_, k_, v_):
            return co_alibi_attention(q_, k_, v_, causal, sm_scale, bias_max)
    ins = [q, k, v] + ([] if do is None else [do])
    n = (B + chunk - 1) // chunk
    with torch.cuda.device(dev):
        caller = torch.cuda.current_stream()
        s_in, s_comp, s_out = _stream_triple(dev)
        for s in (s_in, s_comp, s_out):
            s.wait_stream(caller)
        # two device slots per input: chunk c+2 overwrites chunk c's inputs once its compute finished
        slots = [[torch.empty((min(chunk, B),) + tuple(t.shape[1:]), dtype=t.dtype, device=dev) for t in ins]
                 for _ in range(min(2, n))]
        comp_done = []
        keep = []
        for c in range(n):
            b0, b1 = c * chunk, min(B, (c + 1) * chunk)
            buf = [t[: b1 - b0] for t in slots[c % 2]]
            with torch.cuda.stream(s_in):
                if c >= 2:
                    s_in.wait_event(comp_done[c - 2])
                for d, h in zip(buf, ins):
                    d.copy_(h[b0:b1], non_blocking=True)
                h2d = torch.cuda.Event()
                h2d.record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(h2d)
                if do is None:
                    with torch.no_grad():
                        res = (fn(buf[0], buf[1], buf[2]),)
                else:
                    qq, kk, vv = (t.detach().requires_grad_(True) for t in buf[:3])
                    o = fn(qq, kk, vv)
                    o.backward(buf[3])
                    res = (o.detach(), qq.grad, kk.grad, vv.grad)
                ev = torch.cuda.Event()
                ev.record(s_comp)
                comp_done.append(ev)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                for h, d in zip(out, res):
                    d.record_stream(s_out)
                    h[b0:b1].copy_(d, non_blocking=True)
            keep.append(res)
        caller.wait_stream(s_out)
        for s in (s_in, s_comp):
            caller.wait_stream(s)
        s_out.synchronize()
    return out
