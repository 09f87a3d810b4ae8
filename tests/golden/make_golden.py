"""Generate the golden vectors in this folder from the reference's own Python code.

Run once, in a container where a checkout of the reference is available, with
``COALIBI_REFERENCE`` naming the checkout's root directory (the one holding
``model.py`` and ``co_alibi_attn/``)::

    COALIBI_REFERENCE=<path to the reference checkout> python tests/golden/make_golden.py

What is recorded (all float64 unless noted), each from the reference code path
named beside it:

* ``slopes.npz`` -- ``_get_coalibi_slopes(H, bias_max)`` (float32) for H = 1..64 and
  bias_max in {2.5, 4, 8, 16} (``co_alibi_attn/co_alibi_attn.py:11-22``).
* ``model_py.npz`` -- ``model.CoALIBI.apply`` forward and its hand-written backward
  at the self-test shape B=2, H=3, N=5, D=4 (``model.py:5-78``, ``model.py:100-157``;
  slope 1, causal).
* ``case_<name>.npz`` -- forward outputs (o, lse, rowsig) from
  ``benchmark_fwd_pass.ref_forward(..., return_intermediates=True)`` and gradients
  (dq, dk, dv) from autograd through ``benchmark_bwd_pass.ref_forward``, both
  carrying the per-head slope ``2 * _get_coalibi_slopes(H, bias_max)``.  GQA cases
  expand K/V with ``repeat_interleave`` exactly as ``co_alibi_attn.py:143-146`` does,
  so autograd returns the group-summed dK/dV.  Non-causal cases are obtained from
  the same causal reference code by prepending Skv-1 zero-gradient query rows: with
  the top-left causal mask every appended row i >= Skv-1 sees all keys, and the
  padding rows receive dO = 0 so they add nothing to dK/dV.

Inputs come from a CPU ``torch.Generator`` seeded per case.
"""
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
def _load_reference():
    ref = os.environ.get("COALIBI_REFERENCE")
    if not ref or not os.path.isdir(os.path.join(ref, "co_alibi_attn")):
        raise SystemExit("set COALIBI_REFERENCE to the reference checkout's root directory "
                         "(the one holding model.py and co_alibi_attn/)")
    sys.path.insert(0, ref)
    import model  # noqa: E402
    from co_alibi_attn.co_alibi_attn import _get_coalibi_slopes  # noqa: E402
    import co_alibi_attn.benchmark_fwd_pass as bfp  # noqa: E402
    import co_alibi_attn.benchmark_bwd_pass as bbp  # noqa: E402
    return model, _get_coalibi_slopes, bfp, bbp


CASES = [
    # name, B, Hq, Hkv, Sq, Skv, D, causal, bias_max
    ("ragged37", 1, 4, 4, 37, 37, 16, True, 8.0),
    ("h3_s20", 2, 3, 3, 20, 20, 8, True, 8.0),
    ("h12_s33", 1, 12, 12, 33, 33, 8, True, 8.0),
    ("noncausal24", 1, 4, 4, 24, 24, 16, False, 8.0),
    ("gqa_8_2", 1, 8, 2, 29, 29, 16, True, 8.0),
    ("mqa_4_1", 1, 4, 1, 19, 19, 8, True, 8.0),
    ("rect_q16_k40", 1, 4, 4, 16, 40, 16, True, 8.0),
    ("rect_q40_k16", 1, 2, 2, 40, 16, 8, True, 8.0),
    ("bias4", 1, 8, 8, 27, 27, 8, True, 4.0),
    ("noncausal_gqa", 1, 6, 3, 13, 21, 8, False, 8.0),
]


def run_case(name, B, Hq, Hkv, Sq, Skv, D, causal, bias_max, seed, ref):
    model, get_slopes, bfp, bbp = ref
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Sq, D, generator=g, dtype=torch.float64)
    k = torch.randn(B, Hkv, Skv, D, generator=g, dtype=torch.float64)
    v = torch.randn(B, Hkv, Skv, D, generator=g, dtype=torch.float64)
    do = torch.randn(B, Hq, Sq, D, generator=g, dtype=torch.float64)
    scale = 1.0 / math.sqrt(D)

    pad = 0 if causal else Skv - 1
    qp = torch.cat([torch.zeros(B, Hq, pad, D, dtype=torch.float64), q], dim=2)
    dop = torch.cat([torch.zeros(B, Hq, pad, D, dtype=torch.float64), do], dim=2)

    grp = Hq // Hkv
    ke = k.repeat_interleave(grp, dim=1)
    ve = v.repeat_interleave(grp, dim=1)
    o, _p, _sig, z, lse = bfp.ref_forward(qp, ke, ve, scale, bias_max=bias_max,
                                          return_intermediates=True)
    rowsig = z[..., 0]

    qr = qp.clone().requires_grad_(True)
    kr = k.clone().requires_grad_(True)
    vr = v.clone().requires_grad_(True)
    out, _ = bbp.ref_forward(qr, kr.repeat_interleave(grp, dim=1),
                             vr.repeat_interleave(grp, dim=1), scale, bias_max=bias_max)
    out.backward(dop)
    sl = (2.0 * get_slopes(Hq, bias_max)).to(torch.float64)
    return dict(
        q=q.numpy(), k=k.numpy(), v=v.numpy(), do=do.numpy(),
        slopes=sl.numpy(), causal=np.array(causal), sm_scale=np.array(scale),
        bias_max=np.array(bias_max),
        o=o[:, :, pad:].numpy(), lse=lse[:, :, pad:].numpy(), rowsig=rowsig[:, :, pad:].numpy(),
        dq=qr.grad[:, :, pad:].numpy(), dk=kr.grad.numpy(), dv=vr.grad.numpy(),
        fwd_bwd_out_maxdiff=np.array((out.detach() - o).abs().max().item()),
    )


def main():
    ref = _load_reference()
    model, get_slopes, bfp, bbp = ref

    tables = {}
    for bm in (2.5, 4.0, 8.0, 16.0):
        for h in range(1, 65):
            tables[f"bm{bm}_h{h}"] = get_slopes(h, bm).numpy()
    np.savez_compressed(os.path.join(HERE, "slopes.npz"), **tables)

    g = torch.Generator().manual_seed(1234)
    B, H, N, D = 2, 3, 5, 4
    q = torch.randn(B, H, N, D, generator=g, dtype=torch.float64, requires_grad=True)
    k = torch.randn(B, H, N, D, generator=g, dtype=torch.float64, requires_grad=True)
    v = torch.randn(B, H, N, D, generator=g, dtype=torch.float64, requires_grad=True)
    do = torch.randn(B, H, N, D, generator=g, dtype=torch.float64)
    scale = 1.0 / math.sqrt(D)
    o = model.CoALIBI.apply(q, k, v, scale)
    o.backward(do)
    np.savez_compressed(os.path.join(HERE, "model_py.npz"),
                        q=q.detach().numpy(), k=k.detach().numpy(), v=v.detach().numpy(),
                        do=do.numpy(), sm_scale=np.array(scale), o=o.detach().numpy(),
                        dq=q.grad.numpy(), dk=k.grad.numpy(), dv=v.grad.numpy())

    for i, case in enumerate(CASES):
        res = run_case(*case, seed=100 + i, ref=ref)
        np.savez_compressed(os.path.join(HERE, f"case_{case[0]}.npz"), **res)
        print(case[0], "ok", float(res["fwd_bwd_out_maxdiff"]))


if __name__ == "__main__":
    main()
