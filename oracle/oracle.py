"""TEST INFRASTRUCTURE — the CPU oracle of the projection hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product path (vpipe-ming-image_b200/mingproj) never does.

Two restatements of the same arithmetic, which check each other:
  * `projection_np` — numpy, fp64, direct from the definitions (small sizes);
  * `projection` — the plain-C fp64 oracle (oracle/mp_oracle.c), OpenMP.
Both follow the reference's `lin` (src/ming-dit.cc:1763-1771): base GEMM of
the dequantized pack weight, plus every live LoRA slot's s * B (A x), with
alpha already folded into A. See mp_oracle.c for the (partly unpinned) dequant
rule and its citations.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "mp_oracle.c"
BUILD = HERE / "_build"
LIB = BUILD / "libmporacle.so"


def build() -> Path:
    """Compiles the C oracle (gcc, -O3, OpenMP) into oracle/_build/."""
    BUILD.mkdir(exist_ok=True)
    if not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        subprocess.run(["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared",
                        "-o", str(LIB), str(SRC), "-lm"], check=True)
    return LIB


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        vp = C.c_void_p
        L.mpo_unpack_codes.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int, vp]
        L.mpo_pack_codes.argtypes = [vp, C.c_int, C.c_int, C.c_int, vp]
        L.mpo_dequant.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp]
        L.mpo_projection.argtypes = [vp, C.c_int64, C.c_int, vp, vp, vp, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_int, vp, vp, vp, vp, vp]
        L.mpo_modulation.argtypes = [vp, C.c_int, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int,
                                     C.c_int, vp]
        L.mpo_f32_to_bf16.argtypes = [C.c_float]
        L.mpo_f32_to_bf16.restype = C.c_uint16
        L.mpo_threads.restype = C.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---- bf16 helpers (numpy) ---------------------------------------------------

def bf16_to_f64(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bits (uint16)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


# ---- codes ------------------------------------------------------------------

def unpack_codes_np(codes: np.ndarray, k: int, bits: int, symmetric: bool = False) -> np.ndarray:
    """U32 codes [n, k*bits/32] -> int32 [n, k]; code j of a word at bits
    [j*bits, (j+1)*bits)."""
    per = 32 // bits
    n = codes.shape[0]
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    v = (codes.astype(np.uint32)[:, :, None] >> shifts) & np.uint32((1 << bits) - 1)
    q = v.reshape(n, k).astype(np.int32)
    if symmetric:
        q = q.astype(np.uint8).view(np.int8).astype(np.int32)
    return q


def pack_codes_np(q: np.ndarray, bits: int) -> np.ndarray:
    """int [n, k] (values < 2^bits, or int8 for symmetric) -> U32 [n, k*bits/32]."""
    per = 32 // bits
    n, k = q.shape
    v = (q.astype(np.int64) & ((1 << bits) - 1)).astype(np.uint32).reshape(n, k // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    return np.bitwise_or.reduce(v << shifts, axis=2).astype(np.uint32)


def unpack_codes(codes: np.ndarray, k: int, bits: int, symmetric: bool = False) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    q = np.empty((codes.shape[0], k), dtype=np.int32)
    lib().mpo_unpack_codes(_p(codes), codes.shape[0], k, bits, int(symmetric), _p(q))
    return q


def pack_codes(q: np.ndarray, bits: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.int32)
    n, k = q.shape
    codes = np.empty((n, k * bits // 32), dtype=np.uint32)
    lib().mpo_pack_codes(_p(q), n, k, bits, _p(codes))
    return codes


# ---- dequant / projection -----------------------------------------------------

def dequant_np(data, scales, biases, n, k, bits, symmetric=False) -> np.ndarray:
    if bits == 0:
        return bf16_to_f64(np.asarray(data, dtype=np.uint16).reshape(n, k))
    q = unpack_codes_np(np.asarray(data, dtype=np.uint32), k, bits, symmetric).astype(np.float64)
    s = np.repeat(bf16_to_f64(np.asarray(scales, dtype=np.uint16)), 64, axis=1)
    b = 0.0 if biases is None else np.repeat(bf16_to_f64(np.asarray(biases, dtype=np.uint16)),
                                             64, axis=1)
    return s * q + b


def dequant(data, scales, biases, n, k, bits, symmetric=False) -> np.ndarray:
    w = np.empty((n, k), dtype=np.float64)
    data = np.ascontiguousarray(data)
    sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.uint16)
    bi = None if biases is None else np.ascontiguousarray(biases, dtype=np.uint16)
    lib().mpo_dequant(_p(data), _p(sc), _p(bi), n, k, bits, int(symmetric), _p(w))
    return w


def projection_np(x_bf16, data, scales, biases, n, k, bits, symmetric=False, slots=()) -> np.ndarray:
    """numpy fp64 restatement. slots: iterable of (A bf16 [r,k], B bf16 [n,r], s)."""
    x = bf16_to_f64(np.asarray(x_bf16, dtype=np.uint16))
    w = dequant_np(data, scales, biases, n, k, bits, symmetric)
    y = x @ w.T
    for a, b, s in slots:
        if s == 0.0:
            continue
        t = (x @ bf16_to_f64(a).T) * s
        y = y + t @ bf16_to_f64(b).T
    return y


def projection(x_bf16, data, scales, biases, n, k, bits, symmetric=False, slots=()) -> np.ndarray:
    """The C fp64 oracle. x_bf16: uint16 [m, >=k] (row-major; leading dim = shape[1])."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    m, ldx = x.shape
    y = np.empty((m, n), dtype=np.float64)
    slots = list(slots)
    ns = len(slots)
    a_arr = [np.ascontiguousarray(a, dtype=np.uint16) for a, _, _ in slots]
    b_arr = [np.ascontiguousarray(b, dtype=np.uint16) for _, b, _ in slots]
    A = (C.c_void_p * max(ns, 1))(*[a.ctypes.data for a in a_arr])
    B = (C.c_void_p * max(ns, 1))(*[b.ctypes.data for b in b_arr])
    R = np.array([a.shape[0] for a in a_arr] or [0], dtype=np.int32)
    S = np.array([float(s) for _, _, s in slots] or [0.0], dtype=np.float64)
    data = np.ascontiguousarray(data)
    sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.uint16)
    bi = None if biases is None else np.ascontiguousarray(biases, dtype=np.uint16)
    lib().mpo_projection(_p(x), ldx, m, _p(data), _p(sc), _p(bi), n, k, bits, int(symmetric), ns,
                         C.cast(A, C.c_void_p), C.cast(B, C.c_void_p), _p(R), _p(S), _p(y))
    return y


def projection_two_rounding(x_bf16, data, scales, biases, n, k, bits, symmetric=False,
                            slots=(), round_t: bool = False) -> np.ndarray:
    """The reference's ORDER of the LoRA addition (src/ming-dit.cc:1763-1771):
    `lin_base` writes the base output y, rounded to bf16, then
    `lora::Applier::apply` adds every live slot's s * B (A x) onto it and the
    sum is rounded to bf16 again (the fused kernel rounds once). With
    `round_t` the rank-space intermediate s * (A x) is rounded to bf16 too
    (the applier's intermediate dtype is not pinned by the reference tree).
    fp64 arithmetic between the roundings; returns the bf16 values as fp64."""
    x = bf16_to_f64(np.asarray(x_bf16, dtype=np.uint16))
    w = dequant_np(data, scales, biases, n, k, bits, symmetric)
    y = bf16_to_f64(f32_to_bf16((x @ w.T).astype(np.float32)))
    delta = np.zeros_like(y)
    for a, b, s in slots:
        if s == 0.0:
            continue
        t = (x @ bf16_to_f64(a).T) * s
        if round_t:
            t = bf16_to_f64(f32_to_bf16(t.astype(np.float32)))
        delta = delta + t @ bf16_to_f64(b).T
    return bf16_to_f64(f32_to_bf16((y + delta).astype(np.float32)))


def modulation(temb_bf16, data, scales, biases, bias, n, k, bits, symmetric=False) -> np.ndarray:
    t = np.ascontiguousarray(temb_bf16, dtype=np.uint16)
    m = t.shape[0]
    out = np.empty((m, n), dtype=np.float64)
    data = np.ascontiguousarray(data)
    sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.uint16)
    bi = None if biases is None else np.ascontiguousarray(biases, dtype=np.uint16)
    lib().mpo_modulation(_p(t), m, _p(data), _p(sc), _p(bi),
                         _p(np.ascontiguousarray(bias, dtype=np.uint16)), n, k, bits,
                         int(symmetric), _p(out))
    return out


# ---- the sandwich-norm residual step ------------------------------------------

def _bf16_round32(f: np.ndarray) -> np.ndarray:
    """float32 values rounded to bf16 (ties to even), back as float32."""
    return (f32_to_bf16(f).astype(np.uint32) << 16).view(np.float32)


def rms_residual(x_bf16, o_bf16, o_gain_bf16, gate_bf16, nrm_gain_bf16, eps: float):
    """The block's norm + residual sequence after to_out / w2, in float32 with
    bf16 storage between the steps, as the reference chains them
    (src/ming-dit.cc:2096-2101, :2256-2261): rms of the sub-layer output with
    its gain (the rms kernel, :1780-1787), the tanh-gated residual into the
    joint stream (gated_residual_tanh, src/metal/ming_ops.metal:55-93) or the
    plain residual, then rms of the joint stream with the next gain (:2104).
    mean = sum * (1/h); products and sums rounded one at a time. Inputs are
    bf16 bit arrays ([m, h] rows, [h] vectors; o / gate / nrm gain may be
    None). Returns (x', nrm) as bf16 bit arrays (nrm None without a gain)."""
    def f(b):
        return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)

    def rms(v, g):
        inv_h = np.float32(1.0) / np.float32(v.shape[1])
        ss = np.sum(v.astype(np.float64) * v.astype(np.float64), axis=1).astype(np.float32)
        r = (np.float32(1.0) / np.sqrt((ss * inv_h + np.float32(eps)).astype(np.float64)))
        return _bf16_round32((v * r.astype(np.float32)[:, None]) * f(g)[None, :])

    x = f(x_bf16)
    if o_bf16 is not None:
        s = rms(f(o_bf16), o_gain_bf16)
        if gate_bf16 is not None:
            s = np.tanh(f(gate_bf16).astype(np.float64)).astype(np.float32)[None, :] * s
        x = _bf16_round32(x + s)
    nrm = f32_to_bf16(rms(x, nrm_gain_bf16)) if nrm_gain_bf16 is not None else None
    return f32_to_bf16(x), nrm


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    """Relative L2 of `a` against `b` — the measure of every numerical bar in the
    reference (tests/ming-test.h:54-67)."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    if a.size != b.size or a.size == 0:
        return 1.0
    num = float(np.sum((a - b) ** 2))
    den = float(np.sum(b * b))
    return float(np.sqrt(num / den)) if den > 0 else float(np.sqrt(num))
