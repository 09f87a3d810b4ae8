"""ctypes binding of libcoalibi_sm100.so (the C ABI in include/coalibi.h).

The library is built in-tree (``python co-alibi_b200/build.py``).  There is no
fallback: if it cannot be loaded, every call raises.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcoalibi_sm100.so")

F16, BF16, F32 = 0, 1, 2
ERR_TIMEOUT = 10

c_int, c_uint, c_float, c_void_p, c_size_t = (ctypes.c_int, ctypes.c_uint, ctypes.c_float,
                                              ctypes.c_void_p, ctypes.c_size_t)


class CoalibiFwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("slopes", c_void_p),
        ("o", c_void_p), ("lse", c_void_p), ("rowsig", c_void_p),
        ("B", c_int), ("Hq", c_int), ("Hkv", c_int), ("Sq", c_int), ("Skv", c_int), ("D", c_int),
        ("dtype", c_int), ("slopes_dtype", c_int), ("causal", c_int), ("sm_scale", c_float),
        ("status", c_void_p), ("timeout_ms", c_uint),
    ]


class CoalibiBwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("o", c_void_p), ("dout", c_void_p),
        ("lse", c_void_p), ("rowsig", c_void_p), ("slopes", c_void_p),
        ("dq", c_void_p), ("dk", c_void_p), ("dv", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("B", c_int), ("Hq", c_int), ("Hkv", c_int), ("Sq", c_int), ("Skv", c_int), ("D", c_int),
        ("dtype", c_int), ("slopes_dtype", c_int), ("causal", c_int), ("sm_scale", c_float),
        ("status", c_void_p), ("timeout_ms", c_uint),
    ]


EXPORTS = ("coalibi_fwd", "coalibi_fwd_decode", "coalibi_fwd_decode_workspace_bytes", "coalibi_bwd",
           "coalibi_bwd_carry", "coalibi_bwd_phases", "coalibi_bwd_noalloc", "coalibi_bwd_workspace_size",
           "coalibi_bwd_workspace_bytes", "coalibi_bwd_workspace_min_bytes", "coalibi_selftest_wait_timeout",
           "coalibi_strerror",
           "coalibi_abi_version", "coalibi_last_error", "coalibi_describe_launch")

NOALLOC_SCRATCH_BYTES = 64 << 20  # COALIBI_NOALLOC_SCRATCH_BYTES

_lock = threading.Lock()
_lib = None


def load():
    """Load (once) and return the CDLL; raises RuntimeError when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"co_alibi_attn: CUDA library {LIB_PATH} not found; build it with "
                    "`python co-alibi_b200/build.py` (no CPU fallback exists)")
            lib = ctypes.CDLL(LIB_PATH)
            lib.coalibi_fwd.argtypes = [ctypes.POINTER(CoalibiFwdArgs), c_void_p]
            lib.coalibi_fwd.restype = c_int
            lib.coalibi_fwd_decode.argtypes = [ctypes.POINTER(CoalibiFwdArgs), c_void_p, c_size_t, c_void_p]
            lib.coalibi_fwd_decode.restype = c_int
            lib.coalibi_fwd_decode_workspace_bytes.argtypes = [c_int] * 6
            lib.coalibi_fwd_decode_workspace_bytes.restype = c_size_t
            lib.coalibi_bwd.argtypes = [ctypes.POINTER(CoalibiBwdArgs), c_void_p]
            lib.coalibi_bwd.restype = c_int
            lib.coalibi_bwd_carry.argtypes = [ctypes.POINTER(CoalibiBwdArgs), c_void_p, c_void_p]
            lib.coalibi_bwd_carry.restype = c_int
            lib.coalibi_bwd_phases.argtypes = [ctypes.POINTER(CoalibiBwdArgs), c_int, c_void_p]
            lib.coalibi_bwd_phases.restype = c_int
            lib.coalibi_bwd_noalloc.argtypes = [ctypes.POINTER(CoalibiBwdArgs), c_void_p]
            lib.coalibi_bwd_noalloc.restype = c_int
            lib.coalibi_bwd_workspace_bytes.argtypes = [c_int] * 6
            lib.coalibi_bwd_workspace_bytes.restype = c_size_t
            lib.coalibi_bwd_workspace_min_bytes.argtypes = [c_int] * 6
            lib.coalibi_bwd_workspace_min_bytes.restype = c_size_t
            lib.coalibi_bwd_workspace_size.argtypes = [ctypes.POINTER(CoalibiBwdArgs)]
            lib.coalibi_bwd_workspace_size.restype = c_size_t
            lib.coalibi_selftest_wait_timeout.argtypes = [ctypes.c_uint, c_void_p, c_void_p]
            lib.coalibi_selftest_wait_timeout.restype = c_int
            lib.coalibi_strerror.argtypes = [c_int]
            lib.coalibi_strerror.restype = ctypes.c_char_p
            lib.coalibi_last_error.argtypes = []
            lib.coalibi_last_error.restype = ctypes.c_char_p
            lib.coalibi_describe_launch.argtypes = [c_int] * 9 + [ctypes.c_char_p, c_size_t]
            lib.coalibi_describe_launch.restype = c_int
            lib.coalibi_abi_version.argtypes = []
            lib.coalibi_abi_version.restype = c_int
            _lib = lib
    return _lib


FWD, DECODE, BWD = 0, 1, 2  # `which` of coalibi_describe_launch


def describe_launch(which: int, B: int, Hq: int, Hkv: int, Sq: int, Skv: int, D: int, causal: bool,
                    device: int) -> str:
    """The library's launch configuration for a problem, as text (coalibi_describe_launch)."""
    buf = ctypes.create_string_buffer(768)
    check(load().coalibi_describe_launch(which, B, Hq, Hkv, Sq, Skv, D, 1 if causal else 0, device, buf, len(buf)),
          "coalibi_describe_launch")
    return buf.value.decode()


def strerror(code: int) -> str:
    return load().coalibi_strerror(code).decode()


def check(code: int, what: str):
    if code != 0:
        detail = load().coalibi_last_error().decode()
        raise RuntimeError(f"co_alibi_attn: {what} failed: {strerror(code)} (code {code})"
                           + (f": {detail}" if detail else ""))
