"""Adapter key parsing and the slot-binding rules of the reference's
bind_loras_ (src/ming-dit.cc:2893-3005), restated as the reference's own test
cases (tests/ming-dit-test.cc:1165-1168, :1196-1225, :1342-1386)."""
import json
from pathlib import Path

import numpy as np
import pytest

from mingproj import lora as L
from mingproj.pack import f32_to_bf16_bits

# the small DiT of the reference's goldens: dim 1024, 1 refiner each, 2 layers
DIM, FFN, NREF, NLAY = 128, int(128 / 3 * 8), 1, 2


def _factors(rng, rank, out, inp):
    a = rng.normal(0, 1.0, size=(rank, inp)).astype(np.float32)
    b = rng.normal(0, 0.01, size=(out, rank)).astype(np.float32)
    return a, b


def _adapter(rng, rank=8):
    mods = {}
    for name in L.module_names(NREF, NLAY):
        out, inp = L.module_shape(name, DIM, FFN)
        mods[name] = _factors(rng, rank, out, inp)
    return mods


def _write(path, mods, spelling, alpha=16.0):
    t, meta = {}, None
    for name, (a, b) in mods.items():
        if spelling == "diffusers":
            t[f"transformer.{name}.lora_A.weight"] = f32_to_bf16_bits(a * (alpha / a.shape[0]))
            t[f"transformer.{name}.lora_B.weight"] = f32_to_bf16_bits(b)
        elif spelling == "peft":
            t[f"base_model.model.{name}.lora_A.default.weight"] = f32_to_bf16_bits(a)
            t[f"base_model.model.{name}.lora_B.default.weight"] = f32_to_bf16_bits(b)
            meta = {"lora_alpha": str(alpha)}
        elif spelling == "kohya":
            flat = name.replace(".", "_")
            t[f"lora_unet_{flat}.lora_down.weight"] = f32_to_bf16_bits(a)
            t[f"lora_unet_{flat}.lora_up.weight"] = f32_to_bf16_bits(b)
            t[f"lora_unet_{flat}.alpha"] = np.array(alpha, dtype=np.float32)
    L.write_safetensors(path, t, metadata=meta)


def test_module_capacity():
    # tests/ming-dit-test.cc:1165-1168 (small: 28) and :2026 (real: 238)
    pins = json.loads((Path(__file__).resolve().parent / "golden" /
                       "reference_pins.json").read_text())
    rule = pins["lora_capacity_rule"]
    assert L.module_capacity(1, 2) == rule["per_block"] * (rule["refiner_stacks"] * 1 + 2) == 28
    assert L.module_capacity(1, 2) == len(L.module_names(1, 2))
    assert L.module_capacity(2, 30) == pins["lora_capacity_real_model"]["value"] == 238
    assert L.module_capacity(2, 30) == len(L.module_names(2, 30))


def test_three_spellings_bind_identically(tmp_path):
    rng = np.random.default_rng(0)
    mods = _adapter(rng)
    bound = {}
    for sp in ("diffusers", "peft", "kohya"):
        p = tmp_path / f"adapter_{sp}.safetensors"
        _write(p, mods, sp)
        sb = L.bind_adapter(p, DIM, FFN, NREF, NLAY)
        assert sb.modules == 28 and sb.skipped == 0, sb.message
        bound[sp] = sb
    for name in L.module_names(NREF, NLAY):
        d = bound["diffusers"].bound[name]
        for sp in ("peft", "kohya"):
            f = bound[sp].bound[name]
            # alpha folding (16 / 8 = 2, a power of two) is exact in bf16
            assert np.array_equal(f.a, d.a), (sp, name)
            assert np.array_equal(f.b, d.b), (sp, name)


def test_alpha_folded_into_a(tmp_path):
    rng = np.random.default_rng(1)
    a, b = _factors(rng, 4, DIM, DIM)
    p = tmp_path / "k.safetensors"
    L.write_safetensors(p, {"lora_unet_layers_0_attention_to_q.lora_down.weight": f32_to_bf16_bits(a),
                            "lora_unet_layers_0_attention_to_q.lora_up.weight": f32_to_bf16_bits(b),
                            "lora_unet_layers_0_attention_to_q.alpha": np.array(3.0, np.float32)})
    sb = L.bind_adapter(p, DIM, FFN, NREF, NLAY)
    f = sb.bound["layers.0.attention.to_q"]
    want = f32_to_bf16_bits(L.bf16_bits_to_f32(f32_to_bf16_bits(a)) * np.float32(3.0 / 4))
    assert np.array_equal(f.a, want)


def test_foreign_adapter_binds_nothing_and_says_so(tmp_path):
    p = tmp_path / "foreign.safetensors"
    L.write_safetensors(p, {"transformer_blocks.0.attn.to_q.lora_A.weight":
                            f32_to_bf16_bits(np.ones((4, DIM), np.float32)),
                            "transformer_blocks.0.attn.to_q.lora_B.weight":
                            f32_to_bf16_bits(np.ones((DIM, 4), np.float32))})
    sb = L.bind_adapter(p, DIM, FFN, NREF, NLAY)
    assert sb.modules == 0 and sb.skipped == 0
    assert "bound NO modules" in sb.message


def test_wrong_shape_refuses_whole_slot(tmp_path):
    p = tmp_path / "wrong.safetensors"
    L.write_safetensors(p, {
        "layers.0.attention.to_q.lora_A.weight": f32_to_bf16_bits(np.ones((4, DIM // 2), np.float32)),
        "layers.0.attention.to_q.lora_B.weight": f32_to_bf16_bits(np.ones((DIM // 2, 4), np.float32)),
        "layers.1.attention.to_q.lora_A.weight": f32_to_bf16_bits(np.ones((4, DIM), np.float32)),
        "layers.1.attention.to_q.lora_B.weight": f32_to_bf16_bits(np.ones((DIM, 4), np.float32)),
    })
    sb = L.bind_adapter(p, DIM, FFN, NREF, NLAY)
    assert sb.modules == 0 and sb.skipped == 1
    assert "is NOT applied" in sb.message and "wrong shape (1 fit)" in sb.message


def test_adaln_is_never_adapted(tmp_path):
    p = tmp_path / "ada.safetensors"
    L.write_safetensors(p, {
        "layers.0.adaLN_modulation.0.lora_A.weight": f32_to_bf16_bits(np.ones((4, 256), np.float32)),
        "layers.0.adaLN_modulation.0.lora_B.weight": f32_to_bf16_bits(np.ones((4 * DIM, 4), np.float32)),
    })
    sb = L.bind_adapter(p, DIM, FFN, NREF, NLAY)
    assert sb.modules == 0


def test_safetensors_round_trip(tmp_path):
    rng = np.random.default_rng(3)
    t = {"a": f32_to_bf16_bits(rng.normal(size=(3, 5)).astype(np.float32)),
         "b": rng.normal(size=(7,)).astype(np.float32)}
    p = tmp_path / "x.safetensors"
    L.write_safetensors(p, t, metadata={"k": "v"})
    back, dtypes, meta = L.read_safetensors(p)
    assert dtypes == {"a": "BF16", "b": "F32"} and meta == {"k": "v"}
    assert np.array_equal(back["a"], t["a"]) and np.array_equal(back["b"], t["b"])
    # the same bytes through the `safetensors` package's own reader
    st = pytest.importorskip("safetensors.torch")
    tt = st.load_file(str(p))
    assert tt["a"].shape == (3, 5)
