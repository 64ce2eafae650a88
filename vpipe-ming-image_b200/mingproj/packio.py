"""Pack I/O through the C-ABI (mp_pack_*): safetensors checkpoints and packs
read by the library's own reader (memory-mapped, shards of a directory
merged), projections uploaded straight from an open pack as the reference's
load_qw_ detects them, and the w8 / w4 pack writer with the reference's
selection (src/ming-quant-family.cc:31-59). Host only, except Pack.upload.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import MP_OK, MPError

_NP = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32, "F64": np.float64,
       "U32": np.uint32, "I32": np.int32, "U8": np.uint8, "I8": np.int8, "I64": np.int64,
       "U16": np.uint16, "I16": np.int16, "U64": np.uint64}


def _raise(rc: int, msg: str) -> None:
    raise MPError(rc, f"{_lib.status_name(rc)}: {msg}")


class Pack:
    """An open checkpoint / pack (one .safetensors file or a directory of shards)."""

    def __init__(self, path):
        self.lib = _lib.load()
        h = C.c_void_p()
        rc = self.lib.mp_pack_open(str(path).encode(), C.byref(h))
        if rc != MP_OK:
            _raise(rc, self.lib.mp_pack_last_error().decode())
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.mp_pack_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        self.close()

    def __len__(self) -> int:
        return self.lib.mp_pack_count(self.h)

    def _info(self, i: int | None = None, name: str | None = None) -> _lib.TensorInfo:
        info = _lib.TensorInfo()
        if name is not None:
            rc = self.lib.mp_pack_find(self.h, name.encode(), C.byref(info))
        else:
            rc = self.lib.mp_pack_tensor_at(self.h, i, C.byref(info))
        if rc != MP_OK:
            raise KeyError(name if name is not None else i)
        return info

    def names(self) -> list[str]:
        return [self._info(i).name.decode() for i in range(len(self))]

    def dtype(self, name: str) -> str:
        return self._info(name=name).dtype.decode()

    def shape(self, name: str) -> tuple[int, ...]:
        info = self._info(name=name)
        return tuple(int(info.shape[d]) for d in range(info.ndim))

    def array(self, name: str) -> np.ndarray:
        """A copy of the tensor (bf16 as uint16 bit patterns)."""
        info = self._info(name=name)
        dt = _NP[info.dtype.decode()]
        raw = C.string_at(info.data, info.bytes)
        return np.frombuffer(raw, dtype=dt).reshape([int(info.shape[d]) for d in range(info.ndim)]).copy()

    def metadata(self, key: str) -> str | None:
        v = self.lib.mp_pack_metadata(self.h, key.encode())
        return v.decode() if v is not None else None

    def upload(self, ctx, base: str):
        """The projection `base` uploaded as load_qw_ would read it; returns a
        mingproj.proj.Weight."""
        from .proj import Weight, WeightInfo
        h = C.c_void_p()
        ctx._check(self.lib.mp_pack_upload(ctx.h, self.h, base.encode(), C.byref(h)))
        codes = self._info(name=base + ".weight")
        if self._has(base + ".scales"):
            sc = self._info(name=base + ".scales")
            k = int(sc.shape[1]) * 64
            bits = int(codes.shape[1]) * 32 // k
            mode = 0 if self._has(base + ".biases") else 1
        else:
            k, bits, mode = int(codes.shape[1]), 0, 0
        return Weight(ctx, h, WeightInfo(int(codes.shape[0]), k, bits, mode))

    def _has(self, name: str) -> bool:
        info = _lib.TensorInfo()
        return self.lib.mp_pack_find(self.h, name.encode(), C.byref(info)) == MP_OK


def quantize_pack(src, dst, bits: int) -> tuple[int, int]:
    """Writes the w8 / w4 pack of `src` to `dst`; returns (quantized, copied)."""
    lib = _lib.load()
    nq, nk = C.c_int(), C.c_int()
    rc = lib.mp_pack_quantize(str(src).encode(), str(dst).encode(), int(bits), C.byref(nq),
                              C.byref(nk))
    if rc != MP_OK:
        _raise(rc, lib.mp_pack_last_error().decode())
    return int(nq.value), int(nk.value)


__all__ = ["Pack", "quantize_pack"]
