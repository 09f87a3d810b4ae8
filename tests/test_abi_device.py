"""The C ABI leaves the calling thread's CUDA state as it found it.

Every entry point makes the device that owns its tensors current while it runs
(the tensor-map encoder and the launches need that context) and puts the
caller's previous context back before it returns -- including "no context" on a
thread that never touched CUDA, and another device's context when the tensors
live elsewhere.  A stream that belongs to another device than the tensors is
refused with COALIBI_ERR_DEVICE."""
import ctypes
import math
import threading

import pytest
import torch

from tests._common import make_inputs

pytestmark = pytest.mark.gpu


def _cuda_driver():
    drv = ctypes.CDLL("libcuda.so.1")
    drv.cuCtxGetCurrent.argtypes = [ctypes.POINTER(ctypes.c_void_p)]
    drv.cuCtxGetCurrent.restype = ctypes.c_int
    return drv


def _current_ctx(drv):
    c = ctypes.c_void_p()
    assert drv.cuCtxGetCurrent(ctypes.byref(c)) == 0
    return c.value


def _problem(dev, B=1, Hq=4, Hkv=2, S=300, D=128):
    from co_alibi_attn import _lib
    q, k, v, do = (t.to(dev) for t in make_inputs(B, Hq, Hkv, S, S, D, torch.float16, seed=41))
    slopes = torch.tensor([2.0 ** (-(h + 1)) for h in range(Hq)], dtype=torch.float32, device=dev)
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, S, dtype=torch.float32, device=dev)
    rs = torch.empty_like(lse)
    fa = _lib.CoalibiFwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), slopes=slopes.data_ptr(),
                             o=o.data_ptr(), lse=lse.data_ptr(), rowsig=rs.data_ptr(), B=B, Hq=Hq, Hkv=Hkv,
                             Sq=S, Skv=S, D=D, dtype=_lib.F16, slopes_dtype=_lib.F32, causal=1,
                             sm_scale=1.0 / math.sqrt(D), status=None, timeout_ms=0)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    lib = _lib.load()
    nbytes = lib.coalibi_bwd_workspace_bytes(B, Hq, Hkv, S, S, D)  # enough for either mask
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    ba = _lib.CoalibiBwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), dout=do.data_ptr(),
                             lse=lse.data_ptr(), rowsig=rs.data_ptr(), slopes=slopes.data_ptr(),
                             dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(), workspace=ws.data_ptr(),
                             workspace_bytes=nbytes, B=B, Hq=Hq, Hkv=Hkv, Sq=S, Skv=S, D=D, dtype=_lib.F16,
                             slopes_dtype=_lib.F32, causal=1, sm_scale=1.0 / math.sqrt(D), status=None,
                             timeout_ms=0)
    keep = (q, k, v, do, slopes, o, lse, rs, dq, dk, dv, ws)
    return fa, ba, keep


def _calls(lib, fa, ba, stream):
    """(name, thunk) for every entry point that launches work."""
    return [
        ("coalibi_fwd", lambda: lib.coalibi_fwd(ctypes.byref(fa), stream)),
        ("coalibi_bwd", lambda: lib.coalibi_bwd(ctypes.byref(ba), stream)),
        ("coalibi_bwd_phases", lambda: lib.coalibi_bwd_phases(ctypes.byref(ba), 7, stream)),
        ("coalibi_bwd_noalloc", lambda: lib.coalibi_bwd_noalloc(ctypes.byref(ba), stream)),
    ]


def test_fresh_thread_keeps_no_context():
    """A thread with no CUDA context current calls every entry point; afterwards it
    still has none, and the results equal those of calls made from the main thread."""
    from co_alibi_attn import _lib
    lib = _lib.load()
    drv = _cuda_driver()
    fa, ba, keep = _problem("cuda:0")
    o, dq = keep[5], keep[8]
    for _, call in _calls(lib, fa, ba, None):
        assert call() == 0
    torch.cuda.synchronize()
    o_ref, dq_ref = o.clone(), dq.clone()
    o.zero_()
    dq.zero_()
    torch.cuda.synchronize()
    seen = {}

    def worker():
        seen["before"] = _current_ctx(drv)
        for name, call in _calls(lib, fa, ba, None):
            seen[name] = call()
            seen[name + ":ctx"] = _current_ctx(drv)
        buf = ctypes.create_string_buffer(256)
        seen["describe"] = lib.coalibi_describe_launch(0, 1, 4, 2, 300, 300, 128, 1, 0, buf, len(buf))
        seen["describe:ctx"] = _current_ctx(drv)

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert seen["before"] is None
    for name, _ in _calls(lib, fa, ba, None):
        assert seen[name] == 0, f"{name}: {lib.coalibi_last_error().decode()}"
        assert seen[name + ":ctx"] is None, f"{name} left a context current on the calling thread"
    assert seen["describe"] == 0 and seen["describe:ctx"] is None
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref) and torch.equal(dq, dq_ref)


def test_main_thread_device_unchanged():
    from co_alibi_attn import _lib
    lib = _lib.load()
    torch.cuda.set_device(0)
    fa, ba, _ = _problem("cuda:0")
    stream = torch.cuda.current_stream(0).cuda_stream
    for name, call in _calls(lib, fa, ba, stream):
        assert call() == 0, name
        assert torch.cuda.current_device() == 0
    torch.cuda.synchronize()


@pytest.mark.multigpu
def test_other_device_tensors_leave_current_device():
    """Tensors on cuda:1 with cuda:0 current: the call runs on device 1 and device 0 is
    current again afterwards; a device-0 stream for device-1 tensors is refused."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from co_alibi_attn import _lib
    lib = _lib.load()
    drv = _cuda_driver()
    torch.cuda.set_device(0)
    torch.zeros(1, device="cuda:0")
    ctx0 = _current_ctx(drv)
    fa, ba, keep = _problem("cuda:1")
    s1 = torch.cuda.current_stream(1).cuda_stream
    for name, call in _calls(lib, fa, ba, s1):
        assert call() == 0, f"{name}: {lib.coalibi_last_error().decode()}"
        assert torch.cuda.current_device() == 0 and _current_ctx(drv) == ctx0, name
    torch.cuda.synchronize(1)
    # a thread with no context current: afterwards still none, and the runtime's
    # device selection of that thread is still its default (device 0)
    seen = {}

    def worker():
        seen["rc"] = lib.coalibi_fwd(ctypes.byref(fa), s1)
        seen["ctx"] = _current_ctx(drv)
        seen["dev"] = torch.cuda.current_device()

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert seen == {"rc": 0, "ctx": None, "dev": 0}, seen
    torch.cuda.synchronize(1)
    # a stream created on device 0 (the legacy default stream, handle 0, would mean
    # "the default stream of the device being used" and is always accepted)
    s0 = torch.cuda.Stream(device=0)
    assert lib.coalibi_fwd(ctypes.byref(fa), s0.cuda_stream) == 9  # COALIBI_ERR_DEVICE
    assert "belongs to device 0" in lib.coalibi_last_error().decode()
    assert torch.cuda.current_device() == 0 and _current_ctx(drv) == ctx0
