"""The CPU oracle against golden vectors produced by the reference's own code.

Fixtures come from ``tests/golden/make_golden.py`` (reference ``model.py``,
``benchmark_fwd_pass.ref_forward``, ``benchmark_bwd_pass.ref_forward`` and
``_get_coalibi_slopes``).
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import coalibi_oracle as orc

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(glob.glob(os.path.join(GOLD, "case_*.npz")))


def test_slope_tables_bit_exact():
    tabs = np.load(os.path.join(GOLD, "slopes.npz"))
    assert len(tabs.files) == 4 * 64
    for key in tabs.files:
        bm, h = key[2:].split("_h")
        got = orc.coalibi_slopes(int(h), float(bm)).numpy()
        np.testing.assert_array_equal(got, tabs[key], err_msg=key)


def test_model_py_selftest_vectors():
    g = np.load(os.path.join(GOLD, "model_py.npz"))
    q, k, v, do = (torch.from_numpy(g[n]) for n in ("q", "k", "v", "do"))
    slopes = torch.ones(q.shape[1], dtype=torch.float64)
    o, _, _ = orc.forward(q, k, v, slopes, True, float(g["sm_scale"]))
    dq, dk, dv = orc.backward(q, k, v, do, slopes, True, float(g["sm_scale"]))
    for name, t in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        np.testing.assert_allclose(t.numpy(), g[name], rtol=1e-10, atol=1e-12, err_msg=name)


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(c)[5:-4] for c in CASES])
def test_reference_cases(path):
    g = np.load(path)
    q, k, v, do = (torch.from_numpy(g[n]) for n in ("q", "k", "v", "do"))
    slopes = torch.from_numpy(g["slopes"])
    causal = bool(g["causal"])
    scale = float(g["sm_scale"])
    # the oracle's own slope table must equal the one the reference passed
    np.testing.assert_array_equal(
        (2.0 * orc.coalibi_slopes(q.shape[1], float(g["bias_max"]))).double().numpy(), g["slopes"])
    o, lse, rowsig = orc.forward(q, k, v, slopes, causal, scale)
    dq, dk, dv = orc.backward(q, k, v, do, slopes, causal, scale)
    np.testing.assert_allclose(o.numpy(), g["o"], rtol=0, atol=1e-12)
    np.testing.assert_allclose(lse.numpy(), g["lse"], rtol=0, atol=1e-12)
    np.testing.assert_allclose(rowsig.numpy(), g["rowsig"], rtol=0, atol=1e-12)
    # the gradient fixtures come from torch.softmax without the 1e-9 epsilon
    for name, t in (("dq", dq), ("dk", dk), ("dv", dv)):
        np.testing.assert_allclose(t.numpy(), g[name], rtol=1e-7, atol=1e-8, err_msg=name)


def test_row_dA_sums_to_zero():
    """sum_j dA_ij = 0 per row (up to the 1e-9 softmax epsilon), so the final
    inclusive prefix carry vanishes."""
    gen = torch.Generator().manual_seed(7)
    q, k, v, do = (torch.randn(1, 2, 33, 8, generator=gen, dtype=torch.float64) for _ in range(4))
    sl = orc.api_slopes(2, 8.0, torch.float64)
    _, _, _, it = orc.forward(q, k, v, sl, True, None, return_intermediates=True)
    s = it["s"]
    ds = do @ v.transpose(-1, -2)
    da = s * (ds - (ds * s).sum(-1, keepdim=True))
    assert da.sum(-1).abs().max().item() < 1e-7


def test_flop_counts():
    f, b = orc.algorithmic_flops(8, 16, 4096, 4096, 128, True)
    assert f == 4 * 128 * 8 * 16 * (4096 * 4097 // 2)
    assert f + b == pytest.approx(1.9246e12, rel=1e-4)
    f, _ = orc.algorithmic_flops(16, 12, 2048, 2048, 64, False)
    assert f == pytest.approx(2.0616e11, rel=1e-4)


def test_sliced_matches_dense():
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(2, 4, 17, 8, generator=gen, dtype=torch.float64)
    k = torch.randn(2, 2, 17, 8, generator=gen, dtype=torch.float64)
    v = torch.randn(2, 2, 17, 8, generator=gen, dtype=torch.float64)
    do = torch.randn(2, 4, 17, 8, generator=gen, dtype=torch.float64)
    sl = orc.api_slopes(4, 8.0, torch.float64)
    o, lse, rs = orc.forward(q, k, v, sl, True)
    dq, _, _ = orc.backward(q, k, v, do, sl, True)
    res = orc.forward_sliced(q, k, v, sl, True, compute_dtype=torch.float64,
                             with_backward=True, do=do)
    for (b, h), t in res.items():
        assert torch.allclose(t[0], o[b, h]) and torch.allclose(t[1], lse[b, h])
        assert torch.allclose(t[3], dq[b, h])
