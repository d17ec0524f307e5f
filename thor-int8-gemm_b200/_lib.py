"""ctypes binding of the C ABI (include/thor_int8_gemm_b200.h).

Loading the library needs no GPU; calling a compute entry point does.  There is
no CPU fallback: if the shared library is missing, `load()` raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libthor_int8_gemm_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

T8G_OK = 0
T8G_ERR_INVALID_ARGUMENT = 1
T8G_ERR_UNSUPPORTED = 2
T8G_ERR_CUDA = 3

OUT_BF16, OUT_F16, OUT_F32 = 0, 1, 2
QUANT_INT8, QUANT_FP8_E4M3 = 0, 1

_vp, _i64, _i32, _u64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64
_f32 = ctypes.c_float

# name -> (restype, argtypes); the order follows the header.
SIGNATURES = {
    "t8g_version": (ctypes.c_char_p, []),
    "t8g_last_error": (ctypes.c_char_p, []),
    "t8g_device_status": (_i32, [_vp, ctypes.POINTER(_i32)]),
    "t8g_status_mirror": (_i32, [ctypes.POINTER(ctypes.POINTER(_i32))]),
    "t8g_get_device": (_i32, [ctypes.POINTER(_i32)]),
    "t8g_set_device": (_i32, [_i32]),
    "t8g_gemm_i8_dequant": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i32,
                                   _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "t8g_gemm_fp8_dequant": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i32,
                                    _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "t8g_gemm_i8_swiglu": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "t8g_gemm_fp8_swiglu": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "t8g_gemm_i8_swiglu_quant": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp,
                                        _i64, _i64, _i64, _i64, _i64, _i32, _vp]),
    "t8g_gemm_fp8_swiglu_quant": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp,
                                         _i64, _i64, _i64, _i64, _i64, _i32, _vp]),
    "t8g_gemm_i8_gated": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp,
                                 _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "t8g_gemm_fp8_gated": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp,
                                  _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "t8g_quant_rows": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i32, _vp]),
    "t8g_rms_mod_quant": (_i32, [_vp, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _i32, _f32,
                                 _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i32, _vp]),
    "t8g_rms_mod_quant_tensorwise": (_i32, [_vp, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _i32, _f32,
                                            _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i32, _vp]),
    "t8g_swiglu_quant": (_i32, [_vp, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "t8g_swiglu_quant_tensorwise": (_i32, [_vp, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i32, _vp]),
    "t8g_rms_mod_quant_tensorwise_noalloc": (_i32, [_vp, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _i32, _f32,
                                                    _vp, _i64, _vp, _i64, _vp, _i64, _i64, _i32, _vp]),
    "t8g_wait_selftest": (_i32, [_u64, _vp, _vp]),
}


class T8GError(RuntimeError):
    """A C-ABI call returned a nonzero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"thor_int8_gemm_b200 error {code}: {message}")
        self.code = code
        self.message = message


_lock = threading.Lock()
_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the shared library once and attach the signatures."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(f"{p} is missing; build it with `python thor-int8-gemm_b200/build.py`")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(rc: int) -> None:
    if rc != T8G_OK:
        raise T8GError(rc, load().t8g_last_error().decode(errors="replace"))


def version() -> str:
    return load().t8g_version().decode()
