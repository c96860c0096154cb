"""ctypes binding of libspilltune_b200.so (the C ABI in include/spilltune_b200.h).

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises.  The library is built in-tree by ``spilltune_b200.build``.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libspilltune_b200.so")

FL_OK = 0
FL_ERR_ARG = 1
FL_ERR_UNSUPPORTED = 2
FL_ERR_CUDA = 3
FL_ERR_DEVICE = 4

_lock = threading.Lock()
_lib = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t

SIGNATURES = {
    "fl_version": ([], _INT),
    "fl_last_error": ([], ctypes.c_char_p),
    "fl_status": ([_INT, _P], _INT),
    "fl_wait_selftest": ([ctypes.c_uint64, _P], _INT),
    "fl_dequant": ([_P, _P, _P, _I64, _P, _P], _INT),
    "fl_fwd_workspace_bytes": ([_I64, _I64, _INT], _SZ),
    "fl_fwd": ([_P, _I64, _I64, _P, _P, _P, _I64, _P, _P, _INT, _F, _P, _P, _SZ, _P], _INT),
    "fl_bwd_workspace_bytes": ([_I64, _I64, _I64, _INT], _SZ),
    "fl_fwd_workspace_bytes_split": ([_I64, _I64, _I64, _INT], _SZ),
    "fl_bwd_workspace_bytes_split": ([_I64, _I64, _I64, _INT], _SZ),
    "fl_bwd": ([_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _INT, _F, _P, _P, _P, _INT, _P, _SZ, _P], _INT),
    "fl_bwd_ts": ([_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _INT, _F, _P, _P, _P, _P, _INT, _P, _SZ, _P], _INT),
    "fl_fwd_noalloc": ([_P, _I64, _I64, _P, _P, _P, _I64, _P, _P, _INT, _F, _P, _P], _INT),
    "fl_nf4dq_scales": ([_P, _P, _P, _F, _I64, _P, _P], _INT),
    "fl_dequant_nf4dq": ([_P, _P, _P, _I64, _P, _P], _INT),
    "fl_fwd_nf4dq": ([_P, _I64, _I64, _P, _P, _P, _I64, _P, _P, _INT, _F, _P, _P, _SZ, _P], _INT),
    "fl_bwd_nf4dq": ([_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _INT, _F, _P, _P, _P, _INT, _P, _SZ, _P],
                     _INT),
    "fl_bwd_nf4dq_ts": ([_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _INT, _F, _P, _P, _P, _P, _INT, _P, _SZ,
                         _P], _INT),
    "fl_ce_workspace_bytes": ([_I64, _I64], _SZ),
    "fl_ce_chunk": ([_P, _I64, _I64, _P, _I64, _P, _F, _P, _P, _P, _SZ, _P], _INT),
    "fl_grouped_workspace_bytes": ([_I64, _INT, _I64, _I64, _INT], _SZ),
    "fl_grouped_fwd": ([_P, _P, _I64, _I64, _INT, _P, _P, _P, _I64, _P, _P, _INT, _F, _P, _P, _SZ, _P], _INT),
    "fl_grouped_bwd": ([_P, _P, _P, _I64, _I64, _I64, _INT, _P, _P, _P, _P, _P, _INT, _F, _P, _P, _P, _INT, _P,
                        _SZ, _P], _INT),
}


class FLError(RuntimeError):
    """A libspilltune_b200 entry point returned a nonzero status."""

    def __init__(self, code, message):
        super().__init__(f"{message} (code {code})")
        self.code = code


def load(path=None):
    """Load (once) and return the ctypes handle; raises if the library is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"unsupported_capability: {p} is not built; run `python -m spilltune_b200.build` "
                "(the frozen-linear path has no CPU fallback)")
        lib = ctypes.CDLL(p)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def check(code, what=""):
    if code != FL_OK:
        msg = load().fl_last_error().decode(errors="replace")
        if code == FL_ERR_ARG:
            raise ValueError(f"{what}: {msg}")
        raise FLError(code, f"{what}: {msg}")


def status(reset=False):
    """The current device's status word (FL_STATUS_* bits of kernels that gave
    up a bounded wait or saw bad input); synchronises the device."""
    v = ctypes.c_uint32(0)
    check(load().fl_status(int(bool(reset)), ctypes.byref(v)), "fl_status")
    return v.value


def call(name, *args):
    rc = getattr(load(), name)(*args)
    check(rc, name)
    return rc
