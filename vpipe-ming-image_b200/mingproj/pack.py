"""The w8 / w4 group-64 pack format of the DiT's block projections, and the
seeded synthetic weights the benchmark configurations are defined on.

Pack format (reference: load_qw_, src/ming-dit.cc:802-831; quant detection
:1115-1135; shapes pinned by tests/ming-quant-test.cc:526-530):
  <name>.weight  U32  [N, K*bits/32]  codes, code j of a word at bits
                                      [j*bits, (j+1)*bits)
  <name>.scales  BF16 [N, K/64]
  <name>.biases  BF16 [N, K/64]
  w[n, k] = scales[n, k/64] * q[n, k] + biases[n, k/64]
Detection: a pack carries `.scales` beside a block's codes;
group = hidden / scales.shape[1]; bits = codes.shape[1] * 32 / K, which must
be 4 or 8, else the checkpoint is read as dense.

What is quantized (src/ming-quant-family.h:31-47, .cc:31-59): every 2-D
matrix of the three block stacks — attention.to_q/to_k/to_v/to_out.0,
feed_forward.w1/w3/w2 and the per-block adaLN_modulation.0 — and nothing at
the model level (all_x_embedder, cap_embedder, t_embedder., all_final_layer).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

GROUP = 64
PROJ_NAMES = ("attention.to_q", "attention.to_k", "attention.to_v", "attention.to_out.0",
              "feed_forward.w1", "feed_forward.w3", "feed_forward.w2")
MODEL_LEVEL_EXCLUDE = ("all_x_embedder", "cap_embedder", "t_embedder.", "all_final_layer")


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def pack_codes(q: np.ndarray, bits: int) -> np.ndarray:
    """int codes [n, k] -> U32 [n, k*bits/32], LSB first (signed 8-bit codes are
    stored as their two's-complement byte)."""
    per = 32 // bits
    n, k = q.shape
    if k % per:
        raise ValueError(f"k={k} is not a multiple of {per}")
    if bits == 8:
        return np.ascontiguousarray(q.astype(np.int64) & 0xFF, dtype=np.uint8).view("<u4").reshape(n, k // 4)
    lo = (q[:, 0::2].astype(np.uint8) & 0xF)
    hi = (q[:, 1::2].astype(np.uint8) & 0xF)
    byte = (lo | (hi << 4)).astype(np.uint8)
    return np.ascontiguousarray(byte).view("<u4").reshape(n, k // 8)


def detect_bits(codes_shape, scales_shape, hidden: int) -> tuple[int, int]:
    """The reference's detection rule (src/ming-dit.cc:1115-1135): returns
    (bits, group); bits 0 means "read as dense"."""
    if len(scales_shape) != 2 or len(codes_shape) != 2 or scales_shape[1] <= 0:
        return 0, GROUP
    group = hidden // scales_shape[1]
    if group <= 0:
        group = GROUP
    K = scales_shape[1] * group
    bits = codes_shape[1] * 32 // K if K > 0 else 0
    return (bits if bits in (4, 8) else 0), group


def tensor_bits(codes_shape, scales_shape, group: int) -> int:
    """Per-tensor bits once the checkpoint's group is known (load_qw_,
    src/ming-dit.cc:811-815): K = scales.shape[1] * group,
    bits = codes.shape[1] * 32 / K, read as 8 when 8 and 4 otherwise."""
    K = scales_shape[1] * group
    bits = codes_shape[1] * 32 // K if K > 0 else 0
    return 8 if bits == 8 else 4


@dataclass
class PackedWeight:
    """One projection weight in pack form (host numpy arrays)."""
    n: int
    k: int
    bits: int                 # 0 dense, 4, 8
    mode: int                 # 0 affine, 1 symmetric (8-bit only)
    data: np.ndarray          # U32 codes [n, k*bits/32] or bf16 bits [n, k]
    scales: np.ndarray | None = None   # bf16 bits [n, k/64]
    biases: np.ndarray | None = None   # bf16 bits [n, k/64] (None for symmetric)

    @property
    def nbytes(self) -> int:
        b = self.data.nbytes
        if self.scales is not None:
            b += self.scales.nbytes
        if self.biases is not None:
            b += self.biases.nbytes
        return b


def quantize_affine(w: np.ndarray, bits: int) -> PackedWeight:
    """Min/max affine quantization per 64-wide K group (this build's quantizer
    for fixtures; the host's model-quantize is not in the reference tree)."""
    n, k = w.shape
    g = w.reshape(n, k // GROUP, GROUP).astype(np.float32)
    lo, hi = g.min(axis=2), g.max(axis=2)
    qmax = (1 << bits) - 1
    scale = np.maximum((hi - lo) / qmax, 1e-8).astype(np.float32)
    sb = f32_to_bf16_bits(scale)
    bb = f32_to_bf16_bits(lo)
    s32 = bf16_bits_to_f32(sb)[:, :, None]
    b32 = bf16_bits_to_f32(bb)[:, :, None]
    q = np.clip(np.rint((g - b32) / s32), 0, qmax).astype(np.int32).reshape(n, k)
    return PackedWeight(n, k, bits, 0, pack_codes(q, bits), sb, bb)


def synthetic_affine(rng: np.random.Generator, n: int, k: int, bits: int) -> PackedWeight:
    """BASELINE configs 2/3/5: codes uniform over the full range, bf16 scales
    ~U(0.002, 0.02); w8 biases = -128*scale, w4 biases = -8*scale + N(0, scale)."""
    qmax = (1 << bits) - 1
    q = rng.integers(0, qmax + 1, size=(n, k), dtype=np.int32)
    scale = rng.uniform(0.002, 0.02, size=(n, k // GROUP)).astype(np.float32)
    if bits == 8:
        bias = -128.0 * scale
    else:
        bias = -8.0 * scale + rng.normal(0.0, 1.0, size=scale.shape).astype(np.float32) * scale
    return PackedWeight(n, k, bits, 0, pack_codes(q, bits), f32_to_bf16_bits(scale),
                        f32_to_bf16_bits(bias.astype(np.float32)))


def synthetic_symmetric_w8(rng: np.random.Generator, n: int, k: int) -> PackedWeight:
    """signed codes uniform in [-127, 127], one bf16 scale per
    64-wide K group ~U(0.002, 0.02), no bias."""
    q = rng.integers(-127, 128, size=(n, k), dtype=np.int32)
    scale = rng.uniform(0.002, 0.02, size=(n, k // GROUP)).astype(np.float32)
    return PackedWeight(n, k, 8, 1, pack_codes(q, 8), f32_to_bf16_bits(scale), None)


def synthetic_dense(rng: np.random.Generator, n: int, k: int, std: float = 0.02) -> PackedWeight:
    """dense bf16 weights ~N(0, std)."""
    w = rng.normal(0.0, std, size=(n, k)).astype(np.float32)
    return PackedWeight(n, k, 0, 0, f32_to_bf16_bits(w), None, None)


def synthetic_lora(rng: np.random.Generator, n: int, k: int, rank: int,
                   b_std: float = 0.01) -> tuple[np.ndarray, np.ndarray]:
    """A ~N(0, 1/r) [r, k], B ~N(0, b_std) [n, r], as bf16 bits."""
    a = rng.normal(0.0, 1.0 / np.sqrt(rank), size=(rank, k)).astype(np.float32)
    b = rng.normal(0.0, b_std, size=(n, rank)).astype(np.float32)
    return f32_to_bf16_bits(a), f32_to_bf16_bits(b)


def to_torch_u32(codes: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(codes.view(np.int32))


def selection_counts(names, hidden_layers: int = 30, refiners: int = 2) -> dict:
    """Counts what a pack of the given tensor names quantizes, in the terms of
    tests/ming-quant-test.cc:507-549: block matrices with scales vs model-level
    dense weights."""
    quant = dense_model = 0
    names = set(names)
    for nm in names:
        if not nm.endswith(".weight"):
            continue
        base = nm[: -len(".weight")]
        block = nm.startswith(("layers.", "noise_refiner.", "context_refiner."))
        if block and "norm" not in base and (base + ".scales") in names:
            quant += 1
        elif not block:
            dense_model += 1
    return {"quantized": quant, "dense_model": dense_model}
