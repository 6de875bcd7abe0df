"""ctypes binding of the C ABI in ``include/nslg_b200.h``.

The shared library is built in-tree by ``python -m nanoslg_b200.build`` and loaded
from ``nanoslg_b200/lib/libnslg_b200.so``.  There is no fallback: when the library is
missing every op raises.  Loading needs no GPU; calling a kernel does.
"""
import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libnslg_b200.so")

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

OK = 0
ERR_ARG = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_WORKSPACE = 4

DEV_BAD_PAGE = 1
DEV_BAD_SLOT = 2
DEV_BAD_POSITION = 4
DEV_WAIT_TIMEOUT = 8
DEV_BAD_PLAN = 16

_i32, _i64, _f32, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p

# name -> (restype, argtypes); the order of argtypes is the header's.
SIGNATURES = {
    "nslg_version": (ctypes.c_char_p, []),
    "nslg_last_error": (ctypes.c_char_p, []),
    "nslg_rope_kv_append": (_i32, [_i32, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _i64,
                                   _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp]),
    "nslg_decode_workspace_bytes": (_i64, [_i32, _i32, _i32]),
    "nslg_paged_decode_split_heads": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp,
                                             _vp, _i64, _vp, _vp, _vp, _f32, _vp, _i64, _vp,
                                             _vp]),
    "nslg_split_heads_plan": (_i32, [_i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp,
                                     _vp]),
    "nslg_paged_decode": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp,
                                 _vp, _i64, _vp, _vp, _vp, _f32, _vp, _i64, _vp, _vp]),
    "nslg_paged_decode_noalloc": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _i64, _vp,
                                         _i64, _vp, _vp, _i64, _vp, _vp, _vp, _f32, _vp, _vp]),
    "nslg_paged_prefill": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _i64, _i64, _vp, _i64,
                                  _vp, _vp, _i32, _vp, _vp, _i64, _vp, _vp, _vp, _f32, _i32, _vp,
                                  _vp]),
    "nslg_silu_mul": (_i32, [_i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp]),
    "nslg_linear": (_i32, [_i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp]),
    "nslg_linear_swiglu": (_i32, [_i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _vp,
                                  _vp]),
    "nslg_linear_rope_append": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64,
                                       _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp]),
    "nslg_rmsnorm_residual": (_i32, [_i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _vp, _i64,
                                     _f32, _vp]),
    "nslg_plan_decode": (_i32, [_i32, _i32, _vp, _vp, _i32, _vp, _vp, _i64, _i64, _vp, _vp, _vp,
                                _vp, _vp, _vp, _vp, _i64, _vp, _vp]),
    "nslg_zero_pages": (_i32, [_vp, _i32, _vp, _i64, _i64, _i64, _vp, _vp]),
    "nslg_append_paged_decode": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64,
                                        _vp, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _vp, _vp,
                                        _vp, _f32, _vp, _i64, _vp, _vp]),
    "nslg_argmax_rows": (_i32, [_i32, _i32, _i32, _vp, _i64, _i64, _vp, _vp, _vp]),
    "nslg_plan_decode_host": (_i32, [_i32, _i32, _vp, _vp, _i32, _vp, _i32, _vp, _vp, _vp, _i64,
                                     _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "nslg_ipc_alloc": (_i32, [_i64, ctypes.POINTER(_vp), _vp]),
    "nslg_ipc_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "nslg_ipc_close": (_i32, [_vp]),
    "nslg_ipc_free": (_i32, [_vp]),
    "nslg_tp_allreduce_rmsnorm": (_i32, [_i32, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp,
                                         _vp, _i64, _vp, _vp, _i64, _f32, _i64, _vp, _vp]),
    "nslg_tp_reduce_pushed_rmsnorm": (_i32, [_i32, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64,
                                             _vp, _vp, _i64, _vp, _vp, _i64, _f32, _i64, _vp,
                                             _vp]),
    "nslg_tp_allreduce_rmsnorm_emulated": (_i32, [_i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64,
                                                  _vp, _vp, _i64, _vp, _vp, _i64, _f32, _i64,
                                                  _vp, _vp]),
    "nslg_linear_tp_push": (_i32, [_i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _i32,
                                   _i32, _vp, _i64, _vp, _vp, _vp]),
}

IPC_HANDLE_BYTES = 64
TP_MAX_WORLD = 8
TP_COUNTER_BYTES = 1024

_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
    """A non-zero status from the native library."""

    def __init__(self, fn, code, msg):
        super().__init__(f"{fn} failed (status {code}): {msg}")
        self.code = code


def lib():
    """Loads the shared library once and declares every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"nanoslg_b200 native library not found at {LIB_PATH}; "
                    "build it with `python -m nanoslg_b200.build`")
            h = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


def call(name, *args):
    """Calls entry point ``name`` and raises NativeError on a non-zero status."""
    fn = getattr(lib(), name)
    rc = fn(*args)
    if rc != OK:
        msg = lib().nslg_last_error().decode(errors="replace")
        raise NativeError(name, rc, msg)
    return rc


def version():
    return lib().nslg_version().decode()
