"""C ABI and host logic without a GPU: the library loads on a CPU-only host,
exports every function include/coalibi.h declares, validates arguments before
touching a device, and the Python layer keeps the reference's error behaviour."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    txt = open(os.path.join(ROOT, "include", "coalibi.h")).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_]+\**\s+\**(coalibi_[a-z_0-9]+)\s*\(", txt, re.M)))


def test_library_exports_every_header_function():
    from co_alibi_attn import _lib
    lib = _lib.load()
    names = _header_functions()
    assert "coalibi_fwd" in names and "coalibi_bwd_noalloc" in names
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(_lib.EXPORTS) == names
    assert lib.coalibi_abi_version() == 1


def test_strerror_and_workspace_size():
    from co_alibi_attn import _lib
    lib = _lib.load()
    for code in range(0, 11):
        assert _lib.strerror(code)
    assert "head dim" in _lib.strerror(2)
    # recompute layout: delta float per (b, h, padded row), carries float2 per (b, h, 32-key block, padded row)
    sq_pad, nkb = 4096, 4096 // 32
    want_min = 8 * 16 * sq_pad * 4 + 8 * 16 * nkb * sq_pad * 8
    assert lib.coalibi_bwd_workspace_min_bytes(8, 16, 16, 4096, 4096, 128) == want_min
    assert lib.coalibi_bwd_workspace_min_bytes(1, 4, 4, 37, 37, 64) == 256 * ((4 * 128 * 4 + 255) // 256) + \
        256 * ((4 * 2 * 128 * 8 + 255) // 256)
    # stored layout: delta, then P and dS as 32 KB tiles, one per visible (query tile, key tile) pair
    a = _lib.CoalibiBwdArgs(B=8, Hq=16, Hkv=16, Sq=4096, Skv=4096, D=128, causal=1)
    tiles = 32 * 33 // 2
    want_stored = 8 * 16 * sq_pad * 4 + 2 * 8 * 16 * tiles * 32768
    assert lib.coalibi_bwd_workspace_size(ctypes.byref(a)) == want_stored
    a.causal = 0
    assert lib.coalibi_bwd_workspace_size(ctypes.byref(a)) == 8 * 16 * sq_pad * 4 + 2 * 8 * 16 * 32 * 32 * 32768
    assert lib.coalibi_bwd_workspace_bytes(8, 16, 16, 4096, 4096, 128) == lib.coalibi_bwd_workspace_size(
        ctypes.byref(a))
    # rectangular causal (top-left): query tile q sees key tiles 0..min(q, n_kv - 1)
    a = _lib.CoalibiBwdArgs(B=1, Hq=2, Hkv=1, Sq=40 * 128, Skv=10 * 128, D=64, causal=1)
    tiles = 10 * 11 // 2 + 30 * 10
    assert lib.coalibi_bwd_workspace_size(ctypes.byref(a)) == 2 * 40 * 128 * 4 + 2 * 2 * tiles * 32768
    # past the 24 GiB cap of the stored P / dS scratch: the recompute layout
    a = _lib.CoalibiBwdArgs(B=1, Hq=32, Hkv=8, Sq=32768, Skv=32768, D=128, causal=1)
    assert lib.coalibi_bwd_workspace_size(ctypes.byref(a)) == lib.coalibi_bwd_workspace_min_bytes(
        1, 32, 8, 32768, 32768, 128)
    assert lib.coalibi_bwd_workspace_bytes(0, 4, 4, 37, 37, 64) == 0


def _fwd_args(_lib, **kw):
    base = dict(q=16, k=16, v=16, slopes=16, o=16, lse=16, rowsig=16, B=1, Hq=2, Hkv=2, Sq=8, Skv=8, D=128,
                dtype=0, slopes_dtype=0, causal=1, sm_scale=0.1, status=None, timeout_ms=0)
    base.update(kw)
    return _lib.CoalibiFwdArgs(**base)


@pytest.mark.parametrize("kw,code", [
    (dict(D=96), 2), (dict(dtype=2), 3), (dict(slopes_dtype=7), 3), (dict(Hkv=3, Hq=4), 4),
    (dict(B=0), 4), (dict(q=None), 1), (dict(q=24), 5),
])
def test_fwd_argument_validation_happens_before_device_use(kw, code):
    from co_alibi_attn import _lib
    lib = _lib.load()
    assert lib.coalibi_fwd(ctypes.byref(_fwd_args(_lib, **kw)), None) == code
    assert lib.coalibi_fwd(None, None) == 1


def test_bwd_validation_and_phase_mask():
    from co_alibi_attn import _lib
    lib = _lib.load()
    a = _lib.CoalibiBwdArgs(q=16, k=16, v=16, o=16, dout=16, lse=16, rowsig=16, slopes=16, dq=16, dk=16,
                            dv=16, workspace=None, workspace_bytes=0, B=1, Hq=2, Hkv=2, Sq=8, Skv=8, D=64,
                            dtype=0, slopes_dtype=0, causal=1, sm_scale=0.1, status=None, timeout_ms=0)
    assert lib.coalibi_bwd(ctypes.byref(a), None) == 8          # no workspace
    assert lib.coalibi_bwd_phases(ctypes.byref(a), 8, None) == 4  # bad phase mask
    a.workspace, a.workspace_bytes = 256 + 16, 1 << 20
    assert lib.coalibi_bwd(ctypes.byref(a), None) == 5          # workspace not 256-aligned
    assert lib.coalibi_bwd_carry(ctypes.byref(a), None, None) == 1  # no dA carry
    assert lib.coalibi_bwd_carry(ctypes.byref(a), 16, None) == 5    # (then the same checks as coalibi_bwd)
    big = _lib.CoalibiBwdArgs(**{f: getattr(a, f) for f, _ in _lib.CoalibiBwdArgs._fields_})
    big.B, big.Hq, big.Hkv, big.Sq, big.Skv, big.D = 8, 16, 16, 4096, 4096, 128
    assert lib.coalibi_bwd_noalloc(ctypes.byref(big), None) == 8  # exceeds the static scratch
    big.workspace, big.workspace_bytes = 256, lib.coalibi_bwd_workspace_min_bytes(8, 16, 16, 4096, 4096, 128) - 1
    assert lib.coalibi_bwd(ctypes.byref(big), None) == 8          # below the smallest (recompute) layout
    assert "static scratch" in lib.coalibi_last_error().decode()
    # invalid shapes get the same status as from coalibi_bwd, before the size check
    bad = _lib.CoalibiBwdArgs(**{f: getattr(big, f) for f, _ in _lib.CoalibiBwdArgs._fields_})
    bad.Hq, bad.Hkv = 6, 4
    assert lib.coalibi_bwd_noalloc(ctypes.byref(bad), None) == 4
    bad.Hq, bad.Hkv, bad.B, bad.Sq = 16, 16, 1 << 20, 1 << 20  # B * Hq * query tiles overflows int32
    assert lib.coalibi_bwd_noalloc(ctypes.byref(bad), None) == 4
    bad.B, bad.Sq, bad.D = 1, 128, 96
    assert lib.coalibi_bwd_noalloc(ctypes.byref(bad), None) == 2


def test_describe_launch_validates_before_device_use():
    from co_alibi_attn import _lib
    lib = _lib.load()
    buf = ctypes.create_string_buffer(256)
    assert lib.coalibi_describe_launch(0, 1, 2, 2, 128, 128, 96, 1, 0, buf, len(buf)) == 2
    assert lib.coalibi_describe_launch(0, 1, 6, 4, 128, 128, 128, 1, 0, buf, len(buf)) == 4
    assert lib.coalibi_describe_launch(0, 1, 2, 2, 128, 128, 128, 1, 0, None, 0) == 1


def test_slope_table_matches_reference_fixture():
    import numpy as np
    from co_alibi_attn.co_alibi_attn import _get_coalibi_slopes
    tabs = np.load(os.path.join(ROOT, "tests", "golden", "slopes.npz"))
    for h in (1, 3, 4, 12, 16, 32, 48, 64):
        for bm in (2.5, 4.0, 8.0, 16.0):
            assert np.array_equal(_get_coalibi_slopes(h, bm).float().numpy(), tabs[f"bm{bm}_h{h}"])


def test_python_layer_rejects_cpu_tensors_like_the_reference():
    from co_alibi_attn import co_alibi_attention
    q = torch.randn(1, 2, 8, 64, dtype=torch.float16)
    with pytest.raises(AssertionError):
        co_alibi_attention(q, q, q)


def test_sharded_api_slopes_are_global():
    from co_alibi_attn.sharding import shard_plan, shard_slopes
    from co_alibi_attn.co_alibi_attn import _get_coalibi_slopes
    sh = shard_plan(4, 32, 8, 8, 5)
    s = shard_slopes(32, sh, 8.0, torch.float32, "cpu")
    assert torch.equal(s, (2.0 * _get_coalibi_slopes(32, 8.0))[20:24].float())


def test_sharded_slopes_are_views_of_the_cached_table():
    # no per-call host-to-device copy: every call returns a view into one cached table
    from co_alibi_attn.sharding import shard_plan, shard_slopes
    sh = shard_plan(4, 32, 8, 8, 5)
    a = shard_slopes(32, sh, 8.0, torch.float32, "cpu")
    b = shard_slopes(32, sh, 8.0, torch.float32, "cpu")
    assert a.is_contiguous() and a.shape == (4,)
    assert a.data_ptr() == b.data_ptr()
    assert a.untyped_storage().data_ptr() == b.untyped_storage().data_ptr()
