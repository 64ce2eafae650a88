"""Seeded random weights of the reference's small test DiT (dim 1024, 8 heads
x 128, one context and one noise refiner, 2 layers, cap_feat_dim 256;
tests/ming-dit-test.cc:5-12 of the reference) and its three cases (256 image
rows + 64 + 37 caption rows; 256 + 64 + 70; 240 + 64 + 37; t = 0.3). The
reference's goldens are not available, so the weights are synthetic."""
from __future__ import annotations

import numpy as np

from mingproj.pack import PROJ_NAMES, bf16_bits_to_f32, f32_to_bf16_bits

DIM, HEADS, NREF, NLAY, CAPF, PATCH = 1024, 8, 1, 2, 256, 64
FFN = int(DIM / 3 * 8)
ADALN, TMID = 256, 1024
CASES = {"case_a": (16, 16, 64, 37), "case_b": (16, 16, 64, 70), "case_c": (16, 15, 64, 37)}
SIGMA = 0.7


def block_prefixes():
    return ([f"context_refiner.{i}." for i in range(NREF)] +
            [f"noise_refiner.{i}." for i in range(NREF)] +
            [f"layers.{i}." for i in range(NLAY)])


def make_weights(seed: int = 0) -> dict:
    """name -> bf16 bits (uint16)."""
    rng = np.random.default_rng(seed)

    def lin(n, k, gain=1.0):
        return f32_to_bf16_bits(rng.normal(0, gain / np.sqrt(k), size=(n, k)).astype(np.float32))

    def vec(n, mean=0.0, std=0.02):
        return f32_to_bf16_bits((mean + rng.normal(0, std, size=n)).astype(np.float32))

    w = {}
    w["all_x_embedder.2-1.weight"] = lin(DIM, PATCH)
    w["all_x_embedder.2-1.bias"] = vec(DIM)
    w["cap_embedder.0.weight"] = vec(CAPF, 1.0, 0.1)
    w["cap_embedder.1.weight"] = lin(DIM, CAPF)
    w["cap_embedder.1.bias"] = vec(DIM)
    w["t_embedder.mlp.0.weight"] = lin(TMID, ADALN)
    w["t_embedder.mlp.0.bias"] = vec(TMID)
    w["t_embedder.mlp.2.weight"] = lin(ADALN, TMID)
    w["t_embedder.mlp.2.bias"] = vec(ADALN)
    for pre in block_prefixes():
        for name in PROJ_NAMES:
            if name in ("feed_forward.w1", "feed_forward.w3"):
                w[pre + name + ".weight"] = lin(FFN, DIM)
            elif name == "feed_forward.w2":
                w[pre + name + ".weight"] = lin(DIM, FFN)
            else:
                w[pre + name + ".weight"] = lin(DIM, DIM)
        w[pre + "attention.norm_q.weight"] = vec(DIM // HEADS, 1.0, 0.1)
        w[pre + "attention.norm_k.weight"] = vec(DIM // HEADS, 1.0, 0.1)
        for nm in ("attention_norm1", "attention_norm2", "ffn_norm1", "ffn_norm2"):
            w[pre + nm + ".weight"] = vec(DIM, 1.0, 0.1)
        if not pre.startswith("context_refiner"):
            w[pre + "adaLN_modulation.0.weight"] = lin(4 * DIM, ADALN, 0.5)
            w[pre + "adaLN_modulation.0.bias"] = vec(4 * DIM)
    w["all_final_layer.2-1.adaLN_modulation.1.weight"] = lin(DIM, ADALN, 0.5)
    w["all_final_layer.2-1.adaLN_modulation.1.bias"] = vec(DIM)
    w["all_final_layer.2-1.linear.weight"] = lin(PATCH, DIM)
    w["all_final_layer.2-1.linear.bias"] = vec(PATCH)
    return w


def make_inputs(case: str, seed: int = 1):
    gh, gw, qrows, brows = CASES[case]
    rng = np.random.default_rng(seed + 101 * sorted(CASES).index(case))
    lat = f32_to_bf16_bits(rng.normal(size=(gh * gw, PATCH)).astype(np.float32))
    cap = np.zeros((qrows + brows, DIM), dtype=np.float32)
    cap[:qrows, :CAPF] = rng.normal(size=(qrows, CAPF))
    cap[qrows:, :] = rng.normal(size=(brows, DIM))
    return lat, f32_to_bf16_bits(cap), qrows, gh, gw


def as_f32(w: dict) -> dict:
    return {k: bf16_bits_to_f32(v) for k, v in w.items()}
