"""cfg3 at its stated shape: GQA B=4, Hq=32, Hkv=8, S=8192, D=128, bfloat16,
causal, forward and backward through ``co_alibi_attention``.  The reference serves
this configuration by expanding K/V with ``repeat_interleave``
(co_alibi_attn/co_alibi_attn.py:143-146) and summing dK/dV over each group of four
query heads through autograd; this build keeps K/V at Hkv heads and sums the group
in-kernel.  The float32 oracle checks whole (b, h) slices on the CPU (in blocks of
query rows): all four query heads of the last kv head of the last batch element --
the last CTAs of every grid, every query tile including the last -- with their
dK/dV group sum, and two slices elsewhere."""
import math

import pytest
import torch

from tests._common import make_inputs, check_o, rel_err, calc_sim, oracle_slice, GRAD_REL

pytestmark = pytest.mark.gpu


def test_cfg3_gqa_s8192_forward_backward():
    import co_alibi_attn
    from oracle import coalibi_oracle as orc
    B, Hq, Hkv, S, D, dt = 4, 32, 8, 8192, 128, torch.bfloat16
    G = Hq // Hkv
    q, k, v, do = make_inputs(B, Hq, Hkv, S, S, D, dt, seed=8)
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = co_alibi_attn.co_alibi_attention(qc, kc, vc, causal=True)
    o.backward(do.cuda())
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0
    o, dq, dk, dv = o.detach().cpu(), qc.grad.cpu(), kc.grad.cpu(), vc.grad.cpu()
    del qc, kc, vc
    torch.cuda.empty_cache()
    assert dk.shape == (B, Hkv, S, D) and dv.shape == (B, Hkv, S, D)
    sl = orc.api_slopes(Hq, 8.0, dt)
    b, g = B - 1, Hkv - 1
    group = [(b, h) for h in range(g * G, (g + 1) * G)]
    dk_ref = dv_ref = None
    for (bb, h) in group + [(0, 0), (1, 17)]:
        o_ref, _, _, p_abs_v, dq_ref, dk_h, dv_h = oracle_slice(q, k, v, do, sl, bb, h, True)
        ok, err = check_o(o[bb, h], o_ref, dt, p_abs_v)
        assert ok, f"(b={bb}, h={h}) O max-abs {err:.3e}"
        e = rel_err(dq[bb, h], dq_ref)
        assert e <= GRAD_REL, f"(b={bb}, h={h}) dq relative error {e:.3e}"
        if (bb, h) in group:
            dk_ref = dk_h if dk_ref is None else dk_ref + dk_h
            dv_ref = dv_h if dv_ref is None else dv_ref + dv_h
    for name, x, r in (("dk", dk[b, g], dk_ref), ("dv", dv[b, g], dv_ref)):
        e = rel_err(x, r)
        assert e <= GRAD_REL, f"(b={b}, g={g}) {name} (group of {G} heads) relative error {e:.3e}"
        assert 1 - calc_sim(x, r) <= 1e-4, f"{name} 1-sim {1 - calc_sim(x, r):.3e}"
