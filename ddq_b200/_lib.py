"""ctypes binding of the C ABI in ``include/ddq_b200.h``.

The product path calls the CUDA library only through these functions.  If the
library is missing the first call raises; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

_c_int64 = ctypes.c_int64
_vp = ctypes.c_void_p

# name -> (restype, argtypes)
_SIGNATURES = {
    "ddq_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ddq_version": (ctypes.c_int, []),
    "ddq_quantize_e4m3": (ctypes.c_int, [_vp, ctypes.c_int, _c_int64, _c_int64, _vp, _vp, _vp]),
    "ddq_w8a16_gemm_workspace_size": (ctypes.c_size_t, [_c_int64, _c_int64, _c_int64]),
    "ddq_w8a16_gemm_kernel_count": (ctypes.c_int, [_c_int64, _c_int64, _c_int64]),
    "ddq_w8a16_gemm": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, _vp, _c_int64, _c_int64,
                                      _c_int64, _vp, ctypes.c_size_t, _vp]),
    "ddq_w8a16_gemm_noalloc": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, _vp, _c_int64,
                                              _c_int64, _c_int64, _vp]),
    "ddq_w8a16_gemm_swiglu_workspace_size": (ctypes.c_size_t, [_c_int64, _c_int64, _c_int64]),
    "ddq_w8a16_gemm_swiglu": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, _vp, _c_int64,
                                             _c_int64, _c_int64, _vp, ctypes.c_size_t, _vp]),
    "ddq_decode_attention_split": (ctypes.c_int, [_vp, _c_int64, _vp, _vp, _c_int64, _c_int64,
                                                  _vp, _vp, _vp, _vp, _c_int64, _vp, _vp,
                                                  _c_int64, _c_int64, _c_int64, _c_int64,
                                                  ctypes.c_float, ctypes.c_int, _vp]),
    "ddq_prefill_rope_kv": (ctypes.c_int, [_vp, _c_int64, _vp, _vp, _c_int64, _c_int64, _vp, _vp,
                                           _c_int64, _vp, _vp, _vp, _c_int64, _c_int64, _c_int64,
                                           _c_int64, _c_int64, _vp]),
    "ddq_w8a16_gemm_qkv_rope_kv": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, _c_int64,
                                                  _c_int64, _c_int64, _c_int64, _c_int64, _c_int64,
                                                  _vp, _vp, _c_int64, _c_int64, _vp, _vp, _c_int64,
                                                  _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "ddq_decode_attention": (ctypes.c_int, [_vp, _c_int64, _vp, _vp, _c_int64, _c_int64, _vp, _vp,
                                            _vp, _vp, _c_int64, _c_int64, _c_int64, _c_int64,
                                            _c_int64, ctypes.c_float, _vp]),
    "ddq_add_rmsnorm": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_float, _vp, _vp, _c_int64,
                                       _c_int64, _vp]),
    "ddq_add_rmsnorm_split": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp, _vp,
                                             _c_int64, _c_int64, _vp]),
    "ddq_w8a16_gemm_planes": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, _vp,
                                             _c_int64, _c_int64, _c_int64, ctypes.c_int, _vp]),
    "ddq_argmax_f16": (ctypes.c_int, [_vp, _c_int64, _c_int64, _vp, _vp]),
    "ddq_lm_head_argmax_workspace_size": (ctypes.c_size_t, [_c_int64, _c_int64, _c_int64]),
    "ddq_lm_head_argmax": (ctypes.c_int, [_vp, _vp, _vp, _c_int64, _c_int64, _c_int64, _c_int64,
                                          _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "ddq_unpack_argmax": (ctypes.c_int, [_vp, _c_int64, _vp, _vp]),
    "ddq_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), _vp]),
    "ddq_set_debug": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint64]),
    "ddq_read_trace": (ctypes.c_int, [_vp, ctypes.c_int, _vp]),
}

EXPORTED = tuple(_SIGNATURES)

DTYPE_NONE, DTYPE_F16, DTYPE_F32 = 0, 1, 2
ERR_SHAPE = 2  # DDQ_ERR_SHAPE: the entry does not take this shape

_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    return os.environ.get("DDQ_B200_LIB", LIB_PATH)


def load() -> ctypes.CDLL:
    """Load the native library once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"ddq_b200: native CUDA library not found at {path}; "
                    "build it with `python -m ddq_b200.build` (there is no CPU fallback)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().ddq_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"{what}: {status_string(status)} (ddq status {status})")
