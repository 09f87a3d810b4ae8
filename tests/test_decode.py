"""Decode forward (few query rows against a long key/value sequence): the
split-over-keys kernels (coalibi_fwd_decode) against the oracle -- o, lse and the
row sigmoid totals -- plus the C-ABI's argument checks on the CPU."""
import ctypes
import math

import pytest
import torch

from tests._common import make_inputs, check_o, oracle_fwd_pv, oracle_bwd, rel_err, GRAD_REL


def test_decode_workspace_and_validation_on_cpu():
    from co_alibi_attn import _lib
    lib = _lib.load()
    assert lib.coalibi_fwd_decode_workspace_bytes(1, 8, 2, 1, 4096, 128) > 0
    assert lib.coalibi_fwd_decode_workspace_bytes(1, 8, 2, 17, 4096, 128) == 0   # Sq above the limit
    assert lib.coalibi_fwd_decode_workspace_bytes(1, 8, 3, 1, 4096, 128) == 0    # Hq % Hkv
    base = dict(q=16, k=16, v=16, slopes=16, o=16, lse=16, rowsig=16, B=1, Hq=2, Hkv=2, Sq=1, Skv=300, D=128,
                dtype=0, slopes_dtype=0, causal=0, sm_scale=0.1, status=None, timeout_ms=0)
    a = _lib.CoalibiFwdArgs(**base)
    assert lib.coalibi_fwd_decode(ctypes.byref(a), None, 0, None) == 8          # no workspace
    need = lib.coalibi_fwd_decode_workspace_bytes(1, 2, 2, 1, 300, 128)
    assert lib.coalibi_fwd_decode(ctypes.byref(a), 16 + 256, need - 4, None) == 8  # too small
    assert lib.coalibi_fwd_decode(ctypes.byref(a), 16 + 8, need, None) == 8     # not 16-byte aligned
    a.Sq = 17
    assert lib.coalibi_fwd_decode(ctypes.byref(a), 16 + 256, 1 << 20, None) == 4  # Sq above the limit
    a.Sq, a.D = 1, 96
    assert lib.coalibi_fwd_decode(ctypes.byref(a), 16 + 256, 1 << 20, None) == 2


CASES = [
    # B, Hq, Hkv, Sq, Skv, D, causal, dtype
    (2, 8, 2, 1, 1000, 128, False, torch.bfloat16),     # GQA, one new token
    (1, 4, 4, 1, 5000, 64, False, torch.float16),
    (2, 4, 1, 3, 777, 128, True, torch.float16),        # top-left causal: rows see keys <= i
    (1, 32, 8, 16, 2048, 128, False, torch.bfloat16),   # 64 rows per kv head: four row groups
    (1, 6, 3, 5, 333, 64, False, torch.bfloat16),
    (1, 8, 8, 1, 65536, 128, False, torch.float16),     # long key/value sequence
    (3, 2, 2, 16, 129, 128, True, torch.float16),
]


def _ids(c):
    B, Hq, Hkv, Sq, Skv, D, causal, dt = c
    return f"B{B}H{Hq}-{Hkv}Sq{Sq}Skv{Skv}D{D}{'c' if causal else 'nc'}{'bf16' if dt == torch.bfloat16 else 'f16'}"


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[_ids(c) for c in CASES])
def test_decode_matches_oracle(case):
    import co_alibi_attn
    import co_alibi_attn.co_alibi_attn as impl
    B, Hq, Hkv, Sq, Skv, D, causal, dt = case
    assert Sq <= impl.DECODE_MAX_SQ
    q, k, v, _ = make_inputs(B, Hq, Hkv, Sq, Skv, D, dt, seed=17)
    scale = 1.0 / math.sqrt(D)
    with torch.no_grad():
        qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
        slopes = impl._api_slopes(Hq, 8.0, dt, qc.device)
        o, lse, rowsig = impl._fwd(qc, kc, vc, slopes, causal, scale, decode=True)
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0
    o_ref, lse_ref, rs_ref, pav = oracle_fwd_pv(q, k, v, causal, scale)
    ok, err = check_o(o.cpu(), o_ref, dt, pav)
    assert ok, f"O max-abs {err:.3e}"
    assert (lse.cpu().double() - lse_ref).abs().max().item() < 2e-3 * max(1.0, lse_ref.abs().max().item())
    assert ((rowsig.cpu().double() - rs_ref).abs() / rs_ref.abs().clamp_min(1.0)).max().item() < 2e-3


@pytest.mark.gpu
def test_decode_side_outputs_drive_the_backward():
    """The decode forward's o / lse / rowsig fed to the backward kernels give the
    oracle's gradients (the backward consumes exactly those side outputs)."""
    import co_alibi_attn
    import co_alibi_attn.co_alibi_attn as impl
    B, Hq, Hkv, Sq, Skv, D = 2, 4, 2, 8, 300, 128
    q, k, v, do = make_inputs(B, Hq, Hkv, Sq, Skv, D, torch.float16, seed=23)
    scale = 1.0 / math.sqrt(D)
    qc, kc, vc, doc = q.cuda(), k.cuda(), v.cuda(), do.cuda()
    slopes = impl._api_slopes(Hq, 8.0, torch.float16, qc.device)
    o, lse, rowsig = impl._fwd(qc, kc, vc, slopes, False, scale, decode=True)
    dq, dk, dv = impl._bwd(qc, kc, vc, o, doc, lse, rowsig, slopes, False, scale)
    torch.cuda.synchronize()
    assert co_alibi_attn.device_status(reset=True) == 0
    dq_r, dk_r, dv_r = oracle_bwd(q, k, v, do, False, scale)
    for name, x, r in (("dq", dq, dq_r), ("dk", dk, dk_r), ("dv", dv, dv_r)):
        assert rel_err(x.cpu(), r) <= GRAD_REL, name
