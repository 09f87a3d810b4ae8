"""coalibi_bwd_noalloc through the C ABI: the backward for callers that cannot
allocate device memory at the call (plugin/FFI hosts that own only the tensors
they pass, or code that must avoid a device-synchronising cudaMalloc).  Its
scratch is a fixed 64 MiB device array inside the library, so its results must
equal those of coalibi_bwd with a caller-allocated workspace -- checked on two
calls in a row, the second running over what the first left in the array.

This file is named so that pytest collects it last."""
import ctypes
import math

import pytest
import torch

from tests._common import make_inputs, rel_err, GRAD_REL

pytestmark = pytest.mark.gpu


def _args(lib_mod, q, k, v, o, do, lse, rowsig, slopes, dq, dk, dv, causal, ws=None):
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    return lib_mod.CoalibiBwdArgs(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), dout=do.data_ptr(),
        lse=lse.data_ptr(), rowsig=rowsig.data_ptr(), slopes=slopes.data_ptr(),
        dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(),
        workspace=ws.data_ptr() if ws is not None else None,
        workspace_bytes=ws.numel() if ws is not None else 0,
        B=B, Hq=Hq, Hkv=Hkv, Sq=Sq, Skv=Skv, D=D,
        dtype=lib_mod.F16 if q.dtype == torch.float16 else lib_mod.BF16,
        slopes_dtype=lib_mod.F32, causal=1 if causal else 0, sm_scale=1.0 / math.sqrt(D),
        status=None, timeout_ms=0)


@pytest.mark.parametrize("shape", [
    # B, Hq, Hkv, S, D, causal, dtype
    (1, 4, 4, 1000, 128, True, torch.float16),
    (2, 8, 2, 777, 64, False, torch.bfloat16),
])
def test_noalloc_matches_workspace_backward(shape):
    from co_alibi_attn import _lib
    from co_alibi_attn.co_alibi_attn import _fwd
    lib = _lib.load()
    B, Hq, Hkv, S, D, causal, dtype = shape
    q, k, v, do = (t.cuda() for t in make_inputs(B, Hq, Hkv, S, S, D, dtype, seed=21))
    slopes = (2.0 * torch.tensor([2.0 ** (-8.0 * (h + 1) / Hq) for h in range(Hq)])).float().cuda()
    o, lse, rowsig = _fwd(q, k, v, slopes, causal, 1.0 / math.sqrt(D))
    stream = torch.cuda.current_stream().cuda_stream

    ref = [torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)]
    a = _args(_lib, q, k, v, o, do, lse, rowsig, slopes, *ref, causal)
    nbytes = lib.coalibi_bwd_workspace_size(ctypes.byref(a))
    # the static array holds this problem's preferred (stored P / dS) layout, so both
    # calls run the same kernels
    assert nbytes <= _lib.NOALLOC_SCRATCH_BYTES
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    a = _args(_lib, q, k, v, o, do, lse, rowsig, slopes, *ref, causal, ws)
    assert lib.coalibi_bwd(ctypes.byref(a), stream) == 0

    for call in range(2):
        got = [torch.full_like(q, float("nan")), torch.full_like(k, float("nan")), torch.full_like(v, float("nan"))]
        a = _args(_lib, q, k, v, o, do, lse, rowsig, slopes, *got, causal)
        rc = lib.coalibi_bwd_noalloc(ctypes.byref(a), stream)
        assert rc == 0, lib.coalibi_last_error().decode()
        torch.cuda.synchronize()
        for name, x, r in zip(("dq", "dk", "dv"), got, ref):
            assert torch.isfinite(x).all(), f"call {call}: {name} not fully written"
            e = rel_err(x.cpu(), r.cpu())
            assert e <= GRAD_REL, f"call {call}: {name} differs from coalibi_bwd: relative error {e:.3e}"
            # the backward is deterministic, so with the same inputs the results are
            # bit-identical: nothing the previous call left in the shared array leaks in
            assert torch.equal(x, r), f"call {call}: {name} not bit-identical to coalibi_bwd"


def test_noalloc_rejects_oversized_problem():
    """A problem whose scratch exceeds the static array is refused before launch."""
    from co_alibi_attn import _lib
    lib = _lib.load()
    t = torch.zeros(16, device="cuda", dtype=torch.float16)
    B, H, S, D = 8, 16, 4096, 128
    assert lib.coalibi_bwd_workspace_min_bytes(B, H, H, S, S, D) > _lib.NOALLOC_SCRATCH_BYTES
    a = _lib.CoalibiBwdArgs(q=t.data_ptr(), k=t.data_ptr(), v=t.data_ptr(), o=t.data_ptr(),
                            dout=t.data_ptr(), lse=t.data_ptr(), rowsig=t.data_ptr(), slopes=t.data_ptr(),
                            dq=t.data_ptr(), dk=t.data_ptr(), dv=t.data_ptr(), workspace=None,
                            workspace_bytes=0, B=B, Hq=H, Hkv=H, Sq=S, Skv=S, D=D, dtype=_lib.F16,
                            slopes_dtype=_lib.F16, causal=1, sm_scale=0.1, status=None, timeout_ms=0)
    rc = lib.coalibi_bwd_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == 8  # COALIBI_ERR_WORKSPACE
    assert "static scratch" in lib.coalibi_last_error().decode()
