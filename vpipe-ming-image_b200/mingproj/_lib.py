"""ctypes bindings of libmingproj.so (the C-ABI declared in include/mingproj.h).

The library is loaded from this directory only. Loading it needs no GPU; every
compute entry point reports MP_ECUDA when no device is usable. There is no CPU
fallback behind these bindings: if the library is missing, importing the
projection API raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmingproj.so"

MP_OK, MP_EINVAL, MP_ENOMEM, MP_ECUDA, MP_ETIMEOUT = 0, 1, 2, 3, 4
MP_QUANT_AFFINE, MP_QUANT_SYMMETRIC = 0, 1
MP_MAX_SLOTS = 8
MP_MAX_SEGMENTS = 16
MP_GROUP = 64

# Every function include/mingproj.h declares, with its ctypes signature.
_vp = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64


class WeightDesc(C.Structure):
    _fields_ = [("n", _i32), ("k", _i32), ("bits", _i32), ("group", _i32), ("mode", _i32)]


class Engagement(C.Structure):
    _fields_ = [
        ("linear_calls", _i64), ("lora_proj", _i64), ("gemm_w8", _i64), ("gemm_w4", _i64),
        ("gemm_dense", _i64), ("lora_down", _i64), ("modulation", _i64), ("kernels", _i64),
        ("flops", C.c_double), ("bytes", C.c_double),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class TensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_char_p), ("ndim", _i32),
                ("shape", _i64 * 8), ("data", C.c_void_p), ("bytes", C.c_size_t)]


SIGNATURES = {
    "mp_create": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "mp_destroy": (C.c_int, [_vp]),
    "mp_last_error": (C.c_char_p, [_vp]),
    "mp_status_string": (C.c_char_p, [C.c_int]),
    "mp_sync_check": (C.c_int, [_vp, _vp]),
    "mp_set_wait_limit": (C.c_int, [_vp, C.c_uint64]),
    "mp_selftest_wait": (C.c_int, [_vp, C.c_uint64, _vp]),
    "mp_linear_swiglu": (C.c_int, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _i32, _vp]),
    "mp_linear_heads": (C.c_int, [_vp, C.POINTER(_vp), C.POINTER(_vp), C.c_int, _vp, _i64, _i32,
                                  C.POINTER(_vp), C.c_float, _vp, _vp, _vp]),
    "mp_rms_residual": (C.c_int, [_vp, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _vp, C.c_int,
                                  C.c_int, C.c_float, _vp]),
    "mp_attention": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int, C.c_int, _i64, C.c_float, _vp, _i64,
                               _vp]),
    "mp_weight_upload": (C.c_int, [_vp, C.POINTER(WeightDesc), _vp, _vp, _vp, C.POINTER(_vp)]),
    "mp_weight_free": (C.c_int, [_vp, _vp]),
    "mp_weight_read_codes": (C.c_int, [_vp, _vp, _vp, C.c_size_t]),
    "mp_lora_bind": (C.c_int, [_vp, _vp, C.c_int, _vp, _vp, C.c_int]),
    "mp_lora_unbind": (C.c_int, [_vp, _vp, C.c_int]),
    "mp_set_strength": (C.c_int, [_vp, C.c_int, C.c_float]),
    "mp_get_strength": (C.c_int, [_vp, C.c_int, C.POINTER(C.c_float)]),
    "mp_set_strengths_rows": (C.c_int, [_vp, C.POINTER(C.c_float), C.POINTER(_i32), C.c_int]),
    "mp_set_image_rows": (C.c_int, [_vp, C.c_int]),
    "mp_state_version": (C.c_int, [_vp, C.POINTER(C.c_uint64)]),
    "mp_linear": (C.c_int, [_vp, _vp, _vp, _i64, _vp, _i64, C.c_int, _vp]),
    "mp_linear_shared": (C.c_int, [_vp, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_i64), C.c_int,
                                   _vp, _i64, C.c_int, _vp]),
    "mp_modulation_create": (C.c_int, [_vp, C.c_int, C.POINTER(_vp), C.POINTER(_vp),
                                       C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp)]),
    "mp_modulation_free": (C.c_int, [_vp, _vp]),
    "mp_modulation_all": (C.c_int, [_vp, _vp, _vp, C.c_int, _vp, _vp, _vp, _vp]),
    "mp_linear_lora_static": (C.c_int, [_vp, _vp, _vp, _i64, _vp, _vp, C.c_int, C.c_float, _vp,
                                        _i64, C.c_int, _vp]),
    "mp_pack_open": (C.c_int, [C.c_char_p, C.POINTER(_vp)]),
    "mp_pack_last_error": (C.c_char_p, []),
    "mp_pack_close": (C.c_int, [_vp]),
    "mp_pack_count": (C.c_int, [_vp]),
    "mp_pack_tensor_at": (C.c_int, [_vp, C.c_int, C.POINTER(TensorInfo)]),
    "mp_pack_find": (C.c_int, [_vp, C.c_char_p, C.POINTER(TensorInfo)]),
    "mp_pack_metadata": (C.c_char_p, [_vp, C.c_char_p]),
    "mp_pack_error": (C.c_char_p, [_vp]),
    "mp_pack_upload": (C.c_int, [_vp, _vp, C.c_char_p, C.POINTER(_vp)]),
    "mp_pack_quantize": (C.c_int, [C.c_char_p, C.c_char_p, C.c_int, C.POINTER(C.c_int),
                                   C.POINTER(C.c_int)]),
    "mp_engagement_get": (C.c_int, [_vp, C.POINTER(Engagement)]),
    "mp_engagement_reset": (C.c_int, [_vp]),
}

_lib = None


def load() -> C.CDLL:
    """Loads libmingproj.so (once) and declares every signature. Raises when
    the library has not been built — the product path never runs without it."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python vpipe-ming-image_b200/build.py` "
                "(there is no CPU fallback for the projection path)")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class MPError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def status_name(status: int) -> str:
    return load().mp_status_string(status).decode()
