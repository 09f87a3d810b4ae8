"""Shared helpers for the parity tests: seeded inputs (CPU generator, so the CPU
oracle and the GPU see identical bits), oracle evaluation and error metrics."""
import math

import numpy as np
import torch

from oracle import coalibi_oracle as orc


def make_inputs(B, Hq, Hkv, Sq, Skv, D, dtype, seed=0, std=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, Hq, Sq, D, generator=g) * std).to(dtype)
    k = (torch.randn(B, Hkv, Skv, D, generator=g) * std).to(dtype)
    v = (torch.randn(B, Hkv, Skv, D, generator=g) * std).to(dtype)
    do = torch.randn(B, Hq, Sq, D, generator=g).to(dtype)
    return q, k, v, do


def oracle_fwd(q, k, v, causal, sm_scale, bias_max=8.0, compute_dtype=torch.float64):
    slopes = orc.api_slopes(q.shape[1], bias_max, q.dtype)
    return orc.forward(q, k, v, slopes, causal, sm_scale, compute_dtype)


def oracle_bwd(q, k, v, do, causal, sm_scale, bias_max=8.0, compute_dtype=torch.float64):
    slopes = orc.api_slopes(q.shape[1], bias_max, q.dtype)
    return orc.backward(q, k, v, do, slopes, causal, sm_scale, compute_dtype)


def calc_sim(x, y):
    """The reference's similarity metric (``model.py:83-90``)."""
    x, y = x.double(), y.double()
    den = (x * x + y * y).sum()
    if den == 0:
        return 1.0
    return (2 * (x * y).sum() / den).item()


def rel_err(x, ref):
    x, ref = x.double(), ref.double()
    return ((x - ref).norm() / ref.norm().clamp_min(1e-30)).item()


def half_ulp_bf16(x):
    """Half a bfloat16 ulp at |x| (8 significant bits)."""
    ax = x.double().abs().clamp_min(2.0 ** -126)
    e = torch.floor(torch.log2(ax))
    return 0.5 * torch.pow(2.0, e - 7)


O_ATOL = 2e-3      # O max-abs gate for float16 outputs (north_star tolerance)
GRAD_REL = 1e-2    # dQ/dK/dV relative (Frobenius) error gate


def check_o(o, o_ref, dtype, p_abs_v=None):
    """float16: |O - O_ref| <= 2e-3.

    bfloat16: two roundings the reference algorithm itself performs exceed 2e-3 --
    the output cast (half a bf16 ulp of O) and the cast of the softmax weights P to
    V's dtype before the PV product (co_alibi_attn/co_alibi_fwd_kernel.py:113), whose
    effect on O_i is at most u * sum_j P_ij |v_j| with u = 2^-8 the bf16 unit
    roundoff.  The gate is 2e-3 + half_ulp(O_ref) + u * (P @ |V|)_ref, where
    ``p_abs_v`` is (P @ |V|) from the oracle."""
    err = (o.double() - o_ref.double()).abs()
    if dtype == torch.float16:
        bound = torch.full_like(err, O_ATOL)
    else:
        bound = O_ATOL + half_ulp_bf16(o_ref)
        if p_abs_v is not None:
            bound = bound + 2.0 ** -8 * p_abs_v.double()
    worst = (err - bound).max().item()
    return worst <= 0, err.max().item()


def oracle_fwd_pv(q, k, v, causal, sm_scale, bias_max=8.0, compute_dtype=torch.float64):
    """(o, lse, rowsig, P @ |V|) -- the last term bounds the effect of rounding P."""
    slopes = orc.api_slopes(q.shape[1], bias_max, q.dtype)
    o, lse, rs, it = orc.forward(q, k, v, slopes, causal, sm_scale, compute_dtype,
                                 return_intermediates=True)
    hq, hkv = q.shape[1], k.shape[1]
    va = v.to(compute_dtype).abs().repeat_interleave(hq // hkv, dim=1)
    return o, lse, rs, it["s"] @ va


def oracle_slice(q, k, v, do, slopes, b, h, causal, sm_scale=None, rows_per_chunk=2048,
                 compute_dtype=torch.float32):
    """The oracle on one (b, h) slice, evaluated in blocks of query rows so that
    long sequences (S = 8192) stay within a few GB of host memory.  Rows are
    independent in the forward and in dQ; dK / dV are sums over rows, so the blocks'
    contributions are added.  Returns (o, lse, rowsig, P@|V|) and, when ``do`` is
    given, (dq, dk, dv) of this query head (dK / dV before any GQA group sum)."""
    Hq, Hkv = q.shape[1], k.shape[1]
    g = h // (Hq // Hkv)
    ks, vs = k[b:b + 1, g:g + 1], v[b:b + 1, g:g + 1]
    sl = slopes[h:h + 1]
    Sq = q.shape[2]
    outs = {n: [] for n in ("o", "lse", "rs", "pv", "dq")}
    dk = dv = None
    va = vs.to(compute_dtype).abs()
    for r0 in range(0, Sq, rows_per_chunk):
        r1 = min(Sq, r0 + rows_per_chunk)
        qs = q[b:b + 1, h:h + 1, r0:r1]
        o, lse, rs, it = orc.forward(qs, ks, vs, sl, causal, sm_scale, compute_dtype,
                                     return_intermediates=True, q_offset=r0)
        outs["o"].append(o[0, 0])
        outs["lse"].append(lse[0, 0])
        outs["rs"].append(rs[0, 0])
        outs["pv"].append((it["s"] @ va)[0, 0])
        if do is not None:
            dq_c, dk_c, dv_c = orc.backward(qs, ks, vs, do[b:b + 1, h:h + 1, r0:r1], sl, causal, sm_scale,
                                            compute_dtype, q_offset=r0, intermediates=it)
            outs["dq"].append(dq_c[0, 0])
            dk = dk_c[0, 0] if dk is None else dk + dk_c[0, 0]
            dv = dv_c[0, 0] if dv is None else dv + dv_c[0, 0]
        del it
    fwd = tuple(torch.cat(outs[n]) for n in ("o", "lse", "rs", "pv"))
    if do is None:
        return fwd
    return fwd + (torch.cat(outs["dq"]), dk, dv)
