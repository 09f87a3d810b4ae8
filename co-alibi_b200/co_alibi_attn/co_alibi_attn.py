"""Host side of the Co-ALiBi hot path: the reference's public API and autograd
contract (``co_alibi_attn/co_alibi_attn.py:11-148``) over the sm_100a kernels of
``libcoalibi_sm100.so``.

Differences from the reference, all invisible to callers:
* GQA/MQA: K/V keep their Hkv heads; the kernels map q head h to kv head
  h // (Hq/Hkv) and sum dK/dV over each group in-kernel, replacing
  ``repeat_interleave`` (reference :143-146) and its autograd group sum.
* The backward needs no O(S^2) dk/dv partial buffers (reference :89-99, :132-133).
* The slope tensor is built once per (Hq, bias_max, dtype, device) and reused
  instead of being copied host-to-device on every call (reference :147).
"""
import math
import os
import threading

import torch

from . import _lib

_DTYPES = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}
_SLOPE_DTYPES = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


def _get_coalibi_slopes(n_heads: int, bias_max: float = 8.0) -> torch.Tensor:
    """ALiBi slope table, restating ``co_alibi_attn/co_alibi_attn.py:11-22``:
    n = 2**floor(log2 H) geometric slopes (2**(-bias_max/n))**(h+1), then for a
    non-power-of-two H the odd powers of 2**(-(bias_max/2)/n); absolute value."""
    def get_slopes(n_heads):
        n = 2 ** math.floor(math.log2(n_heads))
        m_0 = 2.0 ** (-bias_max / n)
        m = torch.pow(m_0, torch.arange(1, 1 + n))
        if n < n_heads:
            m_hat_0 = 2.0 ** (-(bias_max / 2) / n)
            m_hat = torch.pow(m_hat_0, torch.arange(1, 1 + 2 * (n_heads - n), 2))
            m = torch.cat([m, m_hat])
        return m
    return torch.abs(get_slopes(n_heads))


_slope_cache = {}
_status_cache = {}
_cache_lock = threading.Lock()

# Optional per-kernel timing hook used by bench.py: when set to a dict, every
# forward / backward launch records CUDA events around each of its kernels on
# the launching stream, appending (start, end) pairs under the kernel's name
# ("fwd", "bwd_delta", "bwd_a", "bwd_b").  The backward then launches its three
# kernels through coalibi_bwd_phases instead of one coalibi_bwd call.
kernel_events = None


def _ev():
    return torch.cuda.Event(enable_timing=True)


def _api_slopes(n_heads, bias_max, dtype, device):
    key = (n_heads, float(bias_max), dtype, device)
    t = _slope_cache.get(key)
    if t is None:
        t = (2.0 * _get_coalibi_slopes(n_heads, bias_max)).to(device, dtype=dtype)
        with _cache_lock:
            _slope_cache[key] = t
    return t


def device_status(device=None, reset=False) -> int:
    """Kernel-side error code recorded on ``device`` (0 = none; 10 = a bounded
    in-kernel wait timed out).  Reading it synchronises with the device."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    t = _status_word(dev)
    code = int(t.item())
    if reset:
        t.zero_()
    return code


def _status_word(device):
    t = _status_cache.get(device)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        with _cache_lock:
            _status_cache[device] = t
    return t


def _check_inputs(q, k, v, slopes):
    batch_size, num_heads, seq_len_q, head_dim = q.shape
    _, num_kv_heads, seq_len_kv, _ = k.shape
    assert k.shape == (batch_size, num_kv_heads, seq_len_kv, head_dim)
    assert v.shape == (batch_size, num_kv_heads, seq_len_kv, head_dim)
    assert num_heads % num_kv_heads == 0, "num_heads must be a multiple of num_kv_heads"
    assert q.is_cuda and k.is_cuda and v.is_cuda, "Inputs must be CUDA tensors"
    assert slopes.shape == (num_heads,), f"Slopes shape {slopes.shape} doesn't match num_heads {num_heads}"
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"co_alibi_attn: q/k/v must all be float16 or bfloat16, got "
                        f"{q.dtype}/{k.dtype}/{v.dtype}")
    if head_dim not in (64, 128):
        raise ValueError(f"co_alibi_attn: head_dim must be 64 or 128, got {head_dim}")
    if slopes.dtype not in _SLOPE_DTYPES:
        raise TypeError(f"co_alibi_attn: slopes must be float16/bfloat16/float32, got {slopes.dtype}")


def _verbose(which, B, Hq, Hkv, Sq, Skv, D, causal, device):
    """With COALIBI_VERBOSE=1, print the launch configuration of each call, as the
    reference prints its autotuned configs (co_alibi_attn/co_alibi_attn.py:58-63,
    :125-130)."""
    if os.getenv("COALIBI_VERBOSE", "0") == "1":
        print(f"[Co-ALIBI] {_lib.describe_launch(which, B, Hq, Hkv, Sq, Skv, D, causal, device.index)}")


# Sq limit of coalibi_fwd_decode (COALIBI_DECODE_MAX_SQ in coalibi.h)
DECODE_MAX_SQ = 16


def _fwd(q, k, v, slopes, causal, sm_scale, decode=None):
    """Forward kernels: the split-over-keys coalibi_fwd_decode for few query rows
    (Sq <= DECODE_MAX_SQ; 2.3-4x faster there), else coalibi_fwd.  ``decode``
    forces one or the other."""
    if decode is None:
        decode = q.shape[2] <= DECODE_MAX_SQ
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, Sq), device=q.device, dtype=torch.float32)
    rowsig = torch.empty((B, Hq, Sq), device=q.device, dtype=torch.float32)
    a = _lib.CoalibiFwdArgs(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), slopes=slopes.data_ptr(),
        o=o.data_ptr(), lse=lse.data_ptr(), rowsig=rowsig.data_ptr(),
        B=B, Hq=Hq, Hkv=Hkv, Sq=Sq, Skv=Skv, D=D, dtype=_DTYPES[q.dtype],
        slopes_dtype=_SLOPE_DTYPES[slopes.dtype], causal=1 if causal else 0, sm_scale=float(sm_scale),
        status=_status_word(q.device).data_ptr(), timeout_ms=0)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rec = kernel_events
    if rec is not None:
        e0, e1 = _ev(), _ev()
        e0.record()
    lib = _lib.load()
    if decode:
        if Sq > DECODE_MAX_SQ:
            raise ValueError(f"co_alibi_attn: the decode forward takes Sq <= {DECODE_MAX_SQ}, got {Sq}")
        nbytes = lib.coalibi_fwd_decode_workspace_bytes(B, Hq, Hkv, Sq, Skv, D)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        _lib.check(lib.coalibi_fwd_decode(a, ws.data_ptr(), nbytes, stream), "coalibi_fwd_decode")
    else:
        _lib.check(lib.coalibi_fwd(a, stream), "coalibi_fwd")
    if rec is not None:
        e1.record()
        rec.setdefault("fwd", []).append((e0, e1))
    _verbose(_lib.DECODE if decode else _lib.FWD, B, Hq, Hkv, Sq, Skv, D, causal, q.device)
    return o, lse, rowsig


def _bwd(q, k, v, o, do, lse, rowsig, slopes, causal, sm_scale, dA_carry_in=None, min_workspace=False):
    """Backward kernels.  ``dA_carry_in`` (float32 [B, Hq, Sq]) marks k / v as one
    key shard of longer rows (coalibi_bwd_carry): the sum of P (dP - delta) over the
    keys left of the shard; o, lse and do are then the whole row's, rowsig the
    sigmoid total of the shard and of every key right of it.  The workspace is the
    library's preferred size for the problem (coalibi_bwd_workspace_size: P / dS
    stored by the first kernel while that stays below 24 GiB); ``min_workspace``
    (or COALIBI_BWD_WORKSPACE=min in the environment, for memory-tight callers) gives
    it the smallest size instead, which makes the backward recompute P / dS in a
    scratch of 8 bytes per row per 32 keys."""
    if os.getenv("COALIBI_BWD_WORKSPACE", "") == "min":
        min_workspace = True
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    lib = _lib.load()
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    a = _lib.CoalibiBwdArgs(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), dout=do.data_ptr(),
        lse=lse.data_ptr(), rowsig=rowsig.data_ptr(), slopes=slopes.data_ptr(),
        dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(), workspace=None, workspace_bytes=0,
        B=B, Hq=Hq, Hkv=Hkv, Sq=Sq, Skv=Skv, D=D, dtype=_DTYPES[q.dtype],
        slopes_dtype=_SLOPE_DTYPES[slopes.dtype], causal=1 if causal else 0, sm_scale=float(sm_scale),
        status=_status_word(q.device).data_ptr(), timeout_ms=0)
    nbytes = (lib.coalibi_bwd_workspace_min_bytes(B, Hq, Hkv, Sq, Skv, D) if min_workspace
              else lib.coalibi_bwd_workspace_size(a))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rec = kernel_events
    if dA_carry_in is not None:
        if rec is not None:
            e0, e1 = _ev(), _ev()
            e0.record()
        _lib.check(lib.coalibi_bwd_carry(a, dA_carry_in.data_ptr(), stream), "coalibi_bwd_carry")
        if rec is not None:
            e1.record()
            rec.setdefault("bwd_carry", []).append((e0, e1))
    elif rec is None:
        _lib.check(lib.coalibi_bwd(a, stream), "coalibi_bwd")
    else:
        for bit, name in ((1, "bwd_delta"), (2, "bwd_a"), (4, "bwd_b")):
            e0, e1 = _ev(), _ev()
            e0.record()
            _lib.check(lib.coalibi_bwd_phases(a, bit, stream), "coalibi_bwd_phases")
            e1.record()
            rec.setdefault(name, []).append((e0, e1))
    _verbose(_lib.BWD, B, Hq, Hkv, Sq, Skv, D, causal, q.device)
    return dq, dk, dv


class CoALIBIAttention(torch.autograd.Function):
    """Autograd contract of ``co_alibi_attn/co_alibi_attn.py:24-135``:
    ``apply(q, k, v, slopes, causal, sm_scale)``; saves q, k, v, o, lse,
    row_sig_total and slopes; backward returns (dq, dk, dv, None, None, None) in
    the input dtypes.  K/V may carry fewer heads than Q (Hq % Hkv == 0)."""

    @staticmethod
    def forward(ctx, q, k, v, slopes, causal, sm_scale):
        _check_inputs(q, k, v, slopes)
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        slopes = slopes.contiguous()
        with torch.cuda.device(q.device):
            o, lse, row_sig_total = _fwd(q, k, v, slopes, causal, sm_scale)
        ctx.save_for_backward(q, k, v, o, lse, row_sig_total, slopes)
        ctx.sm_scale = sm_scale
        ctx.causal = causal
        ctx.head_dim = q.shape[-1]
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, row_sig_total, slopes = ctx.saved_tensors
        do = do.to(q.dtype).contiguous()
        with torch.cuda.device(q.device):
            dq, dk, dv = _bwd(q, k, v, o, do, lse, row_sig_total, slopes, ctx.causal, ctx.sm_scale)
        return dq, dk, dv, None, None, None


def co_alibi_attention(q, k, v, causal=True, sm_scale=None, bias_max=8.0):
    """Co-ALiBi attention, same signature and results as the reference
    ``co_alibi_attention`` (``co_alibi_attn/co_alibi_attn.py:137-148``).

    q: [B, Hq, Sq, D]; k, v: [B, Hkv, Skv, D] with Hq % Hkv == 0; float16 or
    bfloat16 CUDA tensors; D in {64, 128}.  Returns o: [B, Hq, Sq, D]."""
    if sm_scale is None:
        sm_scale = 1.0 / (q.shape[-1] ** 0.5)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    num_q_heads = q.shape[1]
    slopes = _api_slopes(num_q_heads, bias_max, q.dtype, q.device)
    return CoALIBIAttention.apply(q, k, v, slopes, causal, sm_scale)
