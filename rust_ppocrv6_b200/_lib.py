"""ctypes bindings for librechead.so (declarations in include/rechead.h).

The library is the only compute path: importing a compute function without the built
library, or calling it without an sm_100 device, raises — there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "librechead.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "rechead.h")

RH_OK = 0
RH_ERR_INVALID_ARG = 1
RH_ERR_CUDA = 2
RH_ERR_TIMEOUT = 3
RH_ERR_UNSUPPORTED = 4
RH_ERR_NO_DEVICE = 5
RH_ERR_DEVICE_FAULT = 6

_c_int, _c_i64, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p
_i64p = ctypes.POINTER(ctypes.c_int64)
_u32 = ctypes.c_uint32

# name -> (restype, argtypes)
SIGNATURES = {
    "rh_version": (_c_int, []),
    "rh_device_count": (_c_int, [ctypes.POINTER(_c_int)]),
    "rh_last_error": (ctypes.c_char_p, []),
    "rh_ctx_create": (_c_int, [_vp, _c_int, ctypes.POINTER(_vp)]),
    "rh_ctx_destroy": (None, [_vp]),
    "rh_ctx_num_devices": (_c_int, [_vp]),
    "rh_ctx_set_timeout_ms": (_c_int, [_vp, _c_int]),
    "rh_weight_pack": (_c_int, [_vp, _vp, _c_i64, _c_i64, _vp, _c_i64, ctypes.POINTER(_vp)]),
    "rh_weight_pack_f32": (_c_int, [_vp, _vp, _c_i64, _c_i64, _vp, _c_i64, ctypes.POINTER(_vp)]),
    "rh_weight_pack_compact": (_c_int, [_vp, _vp, _c_i64, _c_i64, _vp, _c_i64, ctypes.POINTER(_vp)]),
    "rh_weight_tile_bytes": (_c_i64, [_vp]),
    "rh_weight_set_bias": (_c_int, [_vp, _vp, _vp, _c_i64]),
    "rh_weight_export": (_c_int, [_vp, _vp, _vp, _vp]),
    "rh_weight_export_image": (_c_int, [_vp, _vp, _vp, _vp]),
    "rh_weight_dims": (_c_int, [_vp, _i64p, _i64p]),
    "rh_weight_device_bytes": (_c_i64, [_vp]),
    "rh_weight_free": (None, [_vp]),
    "rh_matmul_quantized_b": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _vp]),
    "rh_matmul_transposed_b": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _vp]),
    "rh_head_decode": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _vp, _vp]),
    "rh_head_decode_lines": (_c_int, [_vp, _vp, _vp, _vp, _c_i64, _c_i64, _vp, _vp]),
    "rh_head_decode_device": (_c_int, [_vp, _vp, _c_int, _vp, _c_i64, _vp, _vp, _vp]),
    "rh_head_decode_kt": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _vp]),
    "rh_head_decode_kt_device": (_c_int, [_vp, _vp, _c_int, _vp, _c_i64, _c_i64, _vp, _vp, _vp]),
    "rh_matmul_quantized_b_device": (_c_int, [_vp, _vp, _c_int, _vp, _c_i64, _vp, _vp]),
    "rh_head_decode_device_noalloc": (_c_int, [_vp, _vp, _c_int, _vp, _c_i64, _vp, _vp, _vp]),
    "rh_sync": (_c_int, [_vp, _c_int]),
    "rh_launch_count": (_c_i64, [_vp, _c_int]),
    "rh_ctc_collapse": (_c_i64, [_vp, _vp, _vp, _c_i64, _vp, _vp, _vp]),
    "rh_ctc_collapse_device": (_c_int, [_vp, _c_int, _vp, _vp, _vp, _c_i64, _vp, _vp, _vp, _vp]),
    "rh_head_decode_ctc": (_c_int, [_vp, _vp, _vp, _vp, _c_i64, _c_i64, _vp, _vp, _vp]),
    "rh_head_decode_kt_ctc": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, _vp]),
    "rh_rec_resized_width": (_u32, [_u32, _u32, _u32, _u32]),
    "rh_rec_batch_shape": (_c_int, [_vp, _vp, _c_i64, _u32, _u32, _vp, _vp, _vp]),
    "rh_rec_preprocess": (_c_int, [_vp, _vp, _c_i64, _vp, _vp, _vp, _c_i64, _u32, _u32, _vp, _c_i64, _vp, _vp]),
    "rh_rec_preprocess_device": (_c_int, [_vp, _c_int, _vp, _c_i64, _vp, _vp, _vp, _c_i64, _u32, _u32, _vp, _c_i64,
                                          _vp, _vp, _vp]),
}

_lib = None


def header_symbols() -> list[str]:
    """Every function name declared in include/rechead.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(rh_[a-z0-9_]+)\s*\(", text)))


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        if not build_if_missing:
            raise ImportError(f"{LIB_PATH} is not built; run `python -m rust_ppocrv6_b200.build`")
        from . import build

        build.build()
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class RecHeadError(RuntimeError):
    """A failed rh_* call. `code` is the RH_ERR_* value; INVALID_ARG corresponds to the
    reference's OcrError::OperatorError."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[rh error {code}] {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != RH_OK:
        raise RecHeadError(rc, load().rh_last_error().decode("utf-8", "replace"))
