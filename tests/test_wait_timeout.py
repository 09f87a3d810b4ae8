"""Bounded waits end with an error status instead of hanging the GPU.

Every in-kernel wait of the library gives up after its timeout, raises the CTA's
abort flag and records COALIBI_ERR_TIMEOUT in the caller's status word.  The
self-test entry point exercises exactly that path with barriers nothing ever
arrives on (no fault, trap or endless loop is involved); afterwards the CUDA
context must still run the attention kernels correctly.
"""
import ctypes
import time

import pytest
import torch

from co_alibi_attn import _lib

pytestmark = pytest.mark.gpu

TIMEOUT = 10  # COALIBI_ERR_TIMEOUT


def test_wait_times_out_and_context_survives():
    from _common import make_inputs, oracle_fwd, check_o
    from co_alibi_attn import co_alibi_attention

    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    t0 = time.monotonic()
    rc = lib.coalibi_selftest_wait_timeout(20, ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(stream))
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    assert rc == 0, _lib.strerror(rc)
    assert int(status.item()) == TIMEOUT
    assert elapsed < 5.0, f"a 20 ms bounded wait took {elapsed:.2f} s"

    # a second run keeps the first recorded code (compare-and-swap from 0)
    rc = lib.coalibi_selftest_wait_timeout(20, ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(stream))
    torch.cuda.synchronize()
    assert rc == 0 and int(status.item()) == TIMEOUT

    # the context is intact: a normal forward still matches the oracle
    q, k, v, _ = make_inputs(1, 2, 2, 256, 256, 128, torch.float16, seed=5)
    scale = 128 ** -0.5
    o = co_alibi_attention(q.cuda(), k.cuda(), v.cuda(), causal=True, sm_scale=scale)
    torch.cuda.synchronize()
    o_ref = oracle_fwd(q, k, v, True, scale)[0]
    ok, maxerr = check_o(o.cpu(), o_ref, torch.float16)
    assert ok, f"O max-abs error {maxerr:.3e}"


def test_selftest_rejects_null_status():
    lib = _lib.load()
    rc = lib.coalibi_selftest_wait_timeout(20, None, None)
    assert rc != 0
