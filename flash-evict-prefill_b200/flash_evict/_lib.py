"""ctypes binding of the C ABI in include/flash_evict.h.

The shared library `libflash_evict_b200.so` sits next to this file and is
built by `flash-evict-prefill_b200/build.py` (or `__graft_entry__.build()`).
There is no fallback: if the library is missing or fails to load, every
compute call raises.
"""
import ctypes
import os
import threading

LIB_NAME = "libflash_evict_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

STATUS_OK = 0
STATUS_INVALID = 1
STATUS_UNSUPPORTED = 2
STATUS_CUDA = 3
STATUS_TIMEOUT = 4
STATUS_BAD_INDEX = 5
DTYPE_F16 = 0
DTYPE_BF16 = 1
QUERY_BLOCK = 256

_STATUS_NAMES = {
    STATUS_INVALID: "invalid argument",
    STATUS_UNSUPPORTED: "unsupported",
    STATUS_CUDA: "CUDA error",
    STATUS_TIMEOUT: "device watchdog timeout",
    STATUS_BAD_INDEX: "gather index out of range",
}

_I64P = ctypes.POINTER(ctypes.c_int64)
_VP = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_F32 = ctypes.c_float

# name -> (restype, argtypes); mirrors include/flash_evict.h
SIGNATURES = {
    "fe_attention_fwd": (_INT, [_VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _VP, _I64, _I64, _I64, _I64, _I64,
                                _INT, _INT, _F32, _VP, _I64, _VP]),
    "fe_replay_scores": (_INT, [_VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _VP, _I64, _I64, _I64, _I64, _I64,
                                _INT, _INT, _F32, _F32, _I64, _INT, _VP, _I64, _VP]),
    "fe_replay_first_scored_row": (_I64, [_I64, _F32, _I64]),
    "fe_replay_scores_range": (_INT, [_VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _VP, _I64, _I64, _I64, _I64, _I64,
                                      _INT, _INT, _F32, _F32, _I64, _INT, _VP, _I64, _I64, _I64, _VP]),
    "fe_select_tokens": (_INT, [_VP, _I64, _I64, _I64, _I64, _I64, _VP, _VP, _INT, _VP]),
    "fe_evict": (_INT, [_VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I64,
                        _I64, _INT, _INT, _F32, _F32, _I64, _INT, _I64, _I64, _I64, _VP]),
    "fe_gather_tokens": (_INT, [_VP, _I64P, _VP, _I64P, _VP, _VP, _VP, _I64, _I64, _I64, _I64, _I64, _I64, _VP]),
    "fe_select_gather": (_INT, [_VP, _I64, _I64, _I64, _I64, _I64, _I64, _VP, _VP, _INT, _VP, _I64P, _VP, _I64P,
                                _VP, _VP, _I64, _I64, _VP]),
    "fe_select_multi": (_INT, [_VP, _I64, _I64, _I64, _INT, _VP, _VP, _VP, _VP, _VP, _INT, _VP, _I64P, _VP, _I64P,
                               _VP, _VP, _I64, _I64, _VP]),
    "fe_evict_compact": (_INT, [_VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I64, _I64,
                                _I64, _I64, _I64, _INT, _INT, _F32, _F32, _I64, _INT, _I64, _I64, _I64, _VP]),
    "fe_snap_workspace_floats": (_I64, [_I64, _I64, _I64, _I64, _I64]),
    "fe_snap_scores": (_INT, [_VP, _I64P, _VP, _I64P, _VP, _VP, _I64, _I64, _I64, _I64, _I64, _I64, _INT, _F32,
                              _I64, _VP]),
    "fe_evict_noalloc": (_INT, [_VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _VP, _VP, _VP, _I64, _I64, _I64,
                                _I64, _I64, _INT, _INT, _F32, _F32, _I64, _INT, _I64, _I64, _I64, _VP]),
    "fe_device_status": (_INT, [_INT, _INT, ctypes.POINTER(_INT)]),
    "fe_set_watchdog_ns": (None, [_I64]),
    "fe_watchdog_selftest": (_INT, [_I64, _VP]),
    "fe_selftest_exp2": (_INT, [_VP, _VP, _VP, _I64, _VP]),
    "fe_last_error": (ctypes.c_char_p, []),
    "fe_abi_version": (_INT, []),
}

_lock = threading.Lock()
_lib = None


def load():
    """Load the native library (once). Raises RuntimeError if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"flash_evict native library not found at {LIB_PATH}; build it with "
                    "`python flash-evict-prefill_b200/build.py` (sm_100a, nvcc)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def strides(t):
    """int64[4] array of a 4-D tensor's element strides."""
    return (ctypes.c_int64 * 4)(*t.stride())


def status_name(code):
    return _STATUS_NAMES.get(code, f"status {code}")


def check(rc):
    if rc != STATUS_OK:
        msg = load().fe_last_error().decode(errors="replace")
        raise RuntimeError(f"flash_evict native call failed ({_STATUS_NAMES.get(rc, rc)}): {msg}")


def device_status(device, clear=True):
    """Largest status code any kernel raised on `device` since the last clear."""
    out = ctypes.c_int(0)
    check(load().fe_device_status(int(device), 1 if clear else 0, ctypes.byref(out)))
    return out.value
