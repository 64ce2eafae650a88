"""Pack I/O of the C-ABI library, on the CPU (no device needed):
  * the C++ safetensors reader (mp_pack_*) against this repo's Python writer:
    names, dtypes, shapes, bytes and metadata, one file or a directory of
    shards;
  * the C++ pack writer (mp_pack_quantize) against the reference's selection
    rule and counts (src/ming-quant-family.cc:31-59; tests/ming-quant-test.cc:
    507-549: every block-stack matrix quantized with codes + scales + biases,
    the 7 model-level weights dense, norms untouched) and, value by value,
    against the Python quantizer (mingproj.pack.quantize_affine): identical
    codes, scales and biases;
  * config.json gains the quantization block; refusals on bad input.
"""
import json

import numpy as np
import pytest

from mingproj import pack as P
from mingproj.lora import read_safetensors, write_safetensors
from mingproj.packio import Pack, quantize_pack
from mingproj._lib import MPError, MP_EINVAL

DIM, FFN, ADA, PATCH, CAPF, TMID = 128, 384, 64, 64, 64, 128
NREF, NLAY = 2, 3
PROJ = ["attention.to_q", "attention.to_k", "attention.to_v", "attention.to_out.0",
        "feed_forward.w1", "feed_forward.w2", "feed_forward.w3"]


def _checkpoint(seed=0):
    """A small DiT checkpoint with the real model's names (bf16 unless noted)."""
    rng = np.random.default_rng(seed)
    lin = lambda n, k: P.f32_to_bf16_bits(rng.normal(0, 1 / np.sqrt(k), (n, k)).astype(np.float32))  # noqa: E731
    vec = lambda n: P.f32_to_bf16_bits((1 + 0.1 * rng.normal(size=n)).astype(np.float32))  # noqa: E731
    w = {"all_x_embedder.2-1.weight": lin(DIM, PATCH), "all_x_embedder.2-1.bias": vec(DIM),
         "cap_embedder.0.weight": vec(CAPF), "cap_embedder.1.weight": lin(DIM, CAPF),
         "t_embedder.mlp.0.weight": lin(TMID, ADA), "t_embedder.mlp.2.weight": lin(ADA, TMID),
         "all_final_layer.2-1.adaLN_modulation.1.weight": lin(DIM, ADA),
         "all_final_layer.2-1.linear.weight": lin(PATCH, DIM)}
    pres = ([f"context_refiner.{i}." for i in range(NREF)] +
            [f"noise_refiner.{i}." for i in range(NREF)] + [f"layers.{i}." for i in range(NLAY)])
    for pre in pres:
        for nm in PROJ:
            shape = (FFN, DIM) if nm in ("feed_forward.w1", "feed_forward.w3") else \
                (DIM, FFN) if nm == "feed_forward.w2" else (DIM, DIM)
            w[pre + nm + ".weight"] = lin(*shape)
        for nm in ("attention.norm_q", "attention.norm_k", "attention_norm1", "attention_norm2",
                   "ffn_norm1", "ffn_norm2"):
            w[pre + nm + ".weight"] = vec(DIM if "norm_" not in nm or "attention_" in nm
                                          or "ffn_" in nm else DIM)
        if not pre.startswith("context_refiner"):
            w[pre + "adaLN_modulation.0.weight"] = lin(4 * DIM, ADA)
            w[pre + "adaLN_modulation.0.bias"] = vec(4 * DIM)
    return w


def _is_block(name):
    return name.startswith(("layers.", "noise_refiner.", "context_refiner."))


def test_reader_matches_python_writer(tmp_path):
    rng = np.random.default_rng(1)
    t = {"a.weight": P.f32_to_bf16_bits(rng.normal(size=(5, 8)).astype(np.float32)),
         "b.f32": rng.normal(size=(3, 4, 2)).astype(np.float32),
         "c.f16": rng.normal(size=(7,)).astype(np.float16),
         "d.codes": rng.integers(0, 2**32, size=(4, 2), dtype=np.uint64).astype(np.uint32),
         "e.empty": np.zeros((0, 3), dtype=np.float32)}
    path = tmp_path / "x.safetensors"
    write_safetensors(path, t, dtypes={"d.codes": "U32"}, metadata={"format": "pt", "note": 'q"\\'})
    with Pack(path) as pk:
        assert sorted(pk.names()) == sorted(t)
        assert pk.dtype("a.weight") == "BF16" and pk.dtype("b.f32") == "F32"
        assert pk.dtype("c.f16") == "F16" and pk.dtype("d.codes") == "U32"
        for k, v in t.items():
            assert pk.shape(k) == v.shape
            got = pk.array(k)
            assert got.dtype == v.dtype and np.array_equal(got, v), k
        assert pk.metadata("format") == "pt" and pk.metadata("note") == 'q"\\'
        assert pk.metadata("absent") is None
        with pytest.raises(KeyError):
            pk.shape("nope")


def test_reader_merges_shards(tmp_path):
    w = _checkpoint()
    names = sorted(w)
    d = tmp_path / "transformer"
    d.mkdir()
    write_safetensors(d / "model-00001-of-00002.safetensors", {k: w[k] for k in names[::2]})
    write_safetensors(d / "model-00002-of-00002.safetensors", {k: w[k] for k in names[1::2]})
    with Pack(d) as pk:
        assert sorted(pk.names()) == names
        for k in names[:5] + names[-5:]:
            assert np.array_equal(pk.array(k), w[k])


def test_reader_refuses_bad_files(tmp_path):
    with pytest.raises(MPError) as e:
        Pack(tmp_path / "missing.safetensors")
    assert e.value.status == MP_EINVAL
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(b"\xff" * 16)  # header length past the end
    with pytest.raises(MPError):
        Pack(bad)
    trunc = tmp_path / "trunc.safetensors"
    write_safetensors(trunc, {"a": np.zeros((100,), np.float32)})
    trunc.write_bytes(trunc.read_bytes()[:-40])  # data shorter than the header says
    with pytest.raises(MPError) as e:
        Pack(trunc)
    assert "out of range" in str(e.value)
    dup = tmp_path / "dup"
    dup.mkdir()
    write_safetensors(dup / "a.safetensors", {"x": np.zeros(2, np.float32)})
    write_safetensors(dup / "b.safetensors", {"x": np.zeros(2, np.float32)})
    with pytest.raises(MPError):
        Pack(dup)


@pytest.mark.parametrize("bits", [8, 4])
def test_writer_selection_and_values(tmp_path, bits):
    w = _checkpoint(bits)
    src, dst = tmp_path / "dense.safetensors", tmp_path / f"w{bits}.safetensors"
    write_safetensors(src, w, metadata={"format": "pt"})
    nq, nk = quantize_pack(src, dst, bits)
    # the reference's counts for this layout: 7 per context-refiner block,
    # 8 (the 7 projections + adaLN) per modulated block
    assert nq == NREF * 7 + (NREF + NLAY) * 8
    out, dtypes, meta = read_safetensors(dst)
    assert meta.get("format") == "pt"
    quant = dense_model = 0
    for name in w:
        if not name.endswith(".weight"):
            assert np.array_equal(out[name], w[name])
            continue
        base = name[:-7]
        if _is_block(name) and "norm" not in base:
            assert dtypes[name] == "U32" and dtypes[base + ".scales"] == "BF16"
            assert out[name].shape == (w[name].shape[0], w[name].shape[1] * bits // 32)
            ref = P.quantize_affine(P.bf16_bits_to_f32(w[name]), bits)
            assert np.array_equal(out[name], ref.data), name
            assert np.array_equal(out[base + ".scales"], ref.scales), name
            assert np.array_equal(out[base + ".biases"], ref.biases), name
            quant += 1
        else:
            assert base + ".scales" not in out and np.array_equal(out[name], w[name]), name
            if not _is_block(name):
                dense_model += 1
    assert quant == nq
    assert dense_model == 7   # tests/ming-quant-test.cc:547-551
    # the pack reads back through the reader with the pack's detection shapes
    with Pack(dst) as pk:
        nm = "layers.1.feed_forward.w2"
        codes, sc = pk.shape(nm + ".weight"), pk.shape(nm + ".scales")
        assert P.detect_bits(codes, sc, DIM)[0] in (0, bits)  # hidden = the block width
        assert codes[1] * 32 == sc[1] * 64 * bits             # tests/ming-quant-test.cc:526-530


def test_writer_directory_and_config(tmp_path):
    w = _checkpoint(3)
    src = tmp_path / "transformer"
    src.mkdir()
    names = sorted(w)
    write_safetensors(src / "m-1.safetensors", {k: w[k] for k in names[:40]})
    write_safetensors(src / "m-2.safetensors", {k: w[k] for k in names[40:]})
    (src / "config.json").write_text(json.dumps({"_class_name": "DiffusionTransformer",
                                                 "dim": DIM, "n_layers": NLAY}))
    dst = tmp_path / "pack"
    nq, nk = quantize_pack(src, dst, 8)
    assert nq == NREF * 7 + (NREF + NLAY) * 8
    cfg = json.loads((dst / "config.json").read_text())
    assert cfg["quantization"] == {"bits": 8, "group_size": 64}
    assert cfg["_class_name"] == "DiffusionTransformer" and cfg["dim"] == DIM
    with Pack(dst) as pk:
        assert pk.dtype("layers.0.attention.to_q.weight") == "U32"
        assert pk.dtype("layers.0.attention_norm1.weight") == "BF16"
        assert pk.dtype("cap_embedder.1.weight") == "BF16"


def test_writer_refuses(tmp_path):
    with pytest.raises(MPError):
        quantize_pack(tmp_path / "none.safetensors", tmp_path / "o.safetensors", 8)
    src = tmp_path / "s.safetensors"
    write_safetensors(src, {"a.weight": np.zeros((2, 64), np.float32)})
    with pytest.raises(MPError) as e:
        quantize_pack(src, tmp_path / "o.safetensors", 3)
    assert e.value.status == MP_EINVAL
