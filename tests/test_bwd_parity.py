"""Backward parity: autograd through the public API (sm_100a kernels) against the
CPU oracle's gradients on identical seeded inputs."""
import glob
import math
import os

import numpy as np
import pytest
import torch

from tests._common import make_inputs, oracle_bwd, rel_err, calc_sim, GRAD_REL

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

CASES = [
    # B, Hq, Hkv, Sq, Skv, D, causal, dtype
    (1, 2, 2, 128, 128, 128, True, torch.float16),
    (1, 2, 2, 256, 256, 128, True, torch.float16),
    (1, 4, 4, 37, 37, 128, True, torch.float16),
    (2, 3, 3, 255, 255, 64, True, torch.float16),
    (1, 2, 2, 129, 129, 128, False, torch.bfloat16),
    (1, 8, 2, 300, 300, 128, True, torch.bfloat16),
    (1, 4, 1, 200, 200, 64, True, torch.float16),
    (1, 2, 2, 16, 300, 128, True, torch.float16),
    (1, 2, 2, 300, 16, 64, True, torch.float16),
    (1, 3, 3, 384, 384, 64, False, torch.float16),
    (1, 4, 4, 1024, 1024, 128, True, torch.float16),
    (1, 12, 12, 513, 513, 64, True, torch.bfloat16),
    (1, 6, 3, 257, 190, 128, False, torch.float16),
    (1, 8, 2, 333, 333, 64, False, torch.bfloat16),
]


def _ids(c):
    B, Hq, Hkv, Sq, Skv, D, causal, dt = c
    return f"B{B}H{Hq}-{Hkv}S{Sq}x{Skv}D{D}{'c' if causal else 'nc'}{'bf16' if dt == torch.bfloat16 else 'f16'}"


@pytest.fixture(scope="module")
def api():
    import co_alibi_attn
    return co_alibi_attn


def _run(api, q, k, v, do, causal, scale, bias_max=8.0):
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = api.co_alibi_attention(qc, kc, vc, causal=causal, sm_scale=scale, bias_max=bias_max)
    o.backward(do.cuda())
    torch.cuda.synchronize()
    assert api.device_status(reset=True) == 0
    return o.detach().cpu(), qc.grad.cpu(), kc.grad.cpu(), vc.grad.cpu()


@pytest.mark.parametrize("case", CASES, ids=[_ids(c) for c in CASES])
def test_backward_matches_oracle(api, case):
    B, Hq, Hkv, Sq, Skv, D, causal, dtype = case
    q, k, v, do = make_inputs(B, Hq, Hkv, Sq, Skv, D, dtype, seed=Sq * 13 + D)
    scale = 1.0 / math.sqrt(D)
    _, dq, dk, dv = _run(api, q, k, v, do, causal, scale)
    assert dq.dtype == dtype and dk.shape == k.shape and dv.shape == v.shape
    dq_r, dk_r, dv_r = oracle_bwd(q, k, v, do, causal, scale)
    for name, x, r in (("dq", dq, dq_r), ("dk", dk, dk_r), ("dv", dv, dv_r)):
        e = rel_err(x, r)
        assert e <= GRAD_REL, f"{name} relative error {e:.3e}"
        assert 1 - calc_sim(x, r) <= 1e-4, f"{name} 1-sim {1 - calc_sim(x, r):.3e}"


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "case_*.npz"))),
                         ids=lambda p: os.path.basename(p)[5:-4])
def test_backward_golden_fixtures(api, path):
    """Reference-generated gradients (small D) through the kernels by zero-padding D
    to 64; padded gradient columns must come back exactly zero."""
    g = np.load(path)
    q, k, v, do = (torch.from_numpy(g[n]) for n in ("q", "k", "v", "do"))
    D0 = q.shape[-1]
    pad = lambda t: torch.nn.functional.pad(t, (0, 64 - D0)).to(torch.float16)
    causal, scale, bm = bool(g["causal"]), float(g["sm_scale"]), float(g["bias_max"])
    _, dq, dk, dv = _run(api, pad(q), pad(k), pad(v), pad(do), causal, scale, bm)
    for name, x in (("dq", dq), ("dk", dk), ("dv", dv)):
        assert x[..., D0:].abs().max().item() == 0.0, name
        e = rel_err(x[..., :D0], torch.from_numpy(g[name]))
        assert e <= 2 * GRAD_REL, f"{name} vs reference fixture: relative error {e:.3e}"
    dq_r, dk_r, dv_r = oracle_bwd(pad(q)[..., :D0], pad(k)[..., :D0], pad(v)[..., :D0], pad(do)[..., :D0],
                                  causal, scale, bm)
    for name, x, r in (("dq", dq, dq_r), ("dk", dk, dk_r), ("dv", dv, dv_r)):
        assert rel_err(x[..., :D0], r) <= GRAD_REL, name


def test_backward_bench_shape_sampled(api):
    """README bench shape (B8 H16 S4096 D128 fp16 causal); the oracle checks eight
    (b, h) slices in float32 on the CPU, from the first and the last CTAs of the
    pass A grid (query-major) and the pass B grid (key-major) and between them."""
    from oracle import coalibi_oracle as orc
    from tests._common import oracle_slice
    from tests.test_fwd_parity import BENCH_SLICES
    B, H, S, D = 8, 16, 4096, 128
    q, k, v, do = make_inputs(B, H, H, S, S, D, torch.float16, seed=0)
    _, dq, dk, dv = _run(api, q, k, v, do, True, 1.0 / math.sqrt(D))
    sl = orc.api_slopes(H, 8.0, torch.float16)
    for (b, h) in BENCH_SLICES:
        t = oracle_slice(q, k, v, do, sl, b, h, True)
        for name, x, r in (("dq", dq[b, h], t[4]), ("dk", dk[b, h], t[5]), ("dv", dv[b, h], t[6])):
            e = rel_err(x, r)
            assert e <= GRAD_REL, f"(b={b}, h={h}) {name} relative error {e:.3e}"


def test_backward_gqa_ragged_long_sampled(api):
    """GQA (4 query heads per kv head), bf16, S = 4000 (ragged last tile): dQ of two
    query heads and dK/dV of one kv head (its four query heads' contributions summed)
    against the float32 oracle."""
    from oracle import coalibi_oracle as orc
    B, Hq, Hkv, S, D = 2, 32, 8, 4000, 128
    q, k, v, do = make_inputs(B, Hq, Hkv, S, S, D, torch.bfloat16, seed=4)
    _, dq, dk, dv = _run(api, q, k, v, do, True, 1.0 / math.sqrt(D))
    sl = orc.api_slopes(Hq, 8.0, torch.bfloat16)
    b, g = 1, 5
    units = [(b, h) for h in range(4 * g, 4 * g + 4)]
    res = orc.forward_sliced(q, k, v, sl, True, None, torch.float32, units=units, with_backward=True, do=do)
    for h in (4 * g, 4 * g + 3):
        e = rel_err(dq[b, h], res[(b, h)][3])
        assert e <= GRAD_REL, f"(b={b}, h={h}) dq relative error {e:.3e}"
    dk_ref = sum(res[u][4] for u in units)
    dv_ref = sum(res[u][5] for u in units)
    for name, x, r in (("dk", dk[b, g], dk_ref), ("dv", dv[b, g], dv_ref)):
        e = rel_err(x, r)
        assert e <= GRAD_REL, f"(b={b}, g={g}) {name} relative error {e:.3e}"


RECOMPUTE_CASES = [c for i, c in enumerate(CASES) if i in (1, 3, 4, 5, 7, 8, 12)]


@pytest.mark.parametrize("case", RECOMPUTE_CASES, ids=[_ids(c) for c in RECOMPUTE_CASES])
def test_backward_recompute_path_matches_oracle(api, case):
    """The backward given only its smallest workspace (coalibi_bwd_workspace_min_bytes),
    where pass B recomputes P and dS from pass A's running sums instead of reading
    them: the path problems whose P / dS scratch would pass the cap take."""
    from co_alibi_attn.co_alibi_attn import _fwd, _bwd, _api_slopes
    B, Hq, Hkv, Sq, Skv, D, causal, dtype = case
    q, k, v, do = make_inputs(B, Hq, Hkv, Sq, Skv, D, dtype, seed=Sq * 13 + D)
    scale = 1.0 / math.sqrt(D)
    qc, kc, vc, doc = (t.cuda() for t in (q, k, v, do))
    sl = _api_slopes(Hq, 8.0, dtype, qc.device)
    o, lse, rs = _fwd(qc, kc, vc, sl, causal, scale)
    dq, dk, dv = _bwd(qc, kc, vc, o, doc, lse, rs, sl, causal, scale, min_workspace=True)
    torch.cuda.synchronize()
    assert api.device_status(reset=True) == 0
    for name, x, r in zip(("dq", "dk", "dv"), (dq, dk, dv), oracle_bwd(q, k, v, do, causal, scale)):
        e = rel_err(x.cpu(), r)
        assert e <= GRAD_REL, f"{name} relative error {e:.3e}"


def test_backward_deterministic(api):
    q, k, v, do = make_inputs(1, 4, 2, 700, 700, 128, torch.float16, seed=9)
    r1 = _run(api, q, k, v, do, True, 1 / math.sqrt(128))
    r2 = _run(api, q, k, v, do, True, 1 / math.sqrt(128))
    for a, b in zip(r1, r2):
        assert torch.equal(a, b)
