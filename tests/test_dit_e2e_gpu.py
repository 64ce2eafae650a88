"""End-to-end DiT forward on the GPU (every block projection and the batched
modulation through the kernels) against the fp32 CPU forward: rel-L2 <= 0.0158,
the plugin's own bar for bf16 against fp32 (README.md:123-125 of the
reference). Also the pack path, runtime LoRA against fused weights (the
reference's bars, tests/ming-dit-test.cc:1241-1246) and strength-0 bit
identity (:1249-1273)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import dit_fixtures as fx
from oracle import oracle as O
from oracle.dit_ref import DitRef
from mingproj import pack as P
from mingproj.dit_forward import DitForward, DitModelConfig
from mingproj.lora import Factors, SlotBinding

pytestmark = pytest.mark.gpu

# bf16 forward vs fp32 forward: the reference's own bar (README.md:124, recorded in
# tests/golden/reference_pins.json)
BAR = json.loads((Path(__file__).resolve().parent / "golden" /
                  "reference_pins.json").read_text())["bf16_forward_rel_l2_bar"]["value"]
K_SMALL_TOL = 0.035  # runtime LoRA vs the fused reference (tests/ming-dit-test.cc:810-815)

CFG = DitModelConfig(dim=fx.DIM, n_heads=fx.HEADS, n_refiner=fx.NREF, n_layers=fx.NLAY,
                     cap_feat_dim=fx.CAPF, patch_dim=fx.PATCH)


def _dev(bits):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).cuda()


def _gpu(fwd, case):
    lat, cap, q, gh, gw = fx.make_inputs(case)
    y = fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)
    return y


def _ref(wf32, case):
    lat, cap, q, gh, gw = fx.make_inputs(case)
    ref = DitRef(wf32, fx.DIM, fx.HEADS, fx.NREF, fx.NLAY, fx.CAPF)
    return ref.forward(P.bf16_bits_to_f32(lat), P.bf16_bits_to_f32(cap), q, gh, gw,
                       fx.SIGMA).numpy()


@pytest.fixture(scope="module")
def dense(ctx):
    w = fx.make_weights(0)
    fwd = DitForward(ctx, CFG, w, torch.device("cuda", 0))
    yield fwd, w
    fwd.free()


N_PROJ = 7 * (2 * fx.NREF + fx.NLAY)  # projection modules of the small DiT (28)


@pytest.mark.parametrize("case", sorted(fx.CASES))
def test_forward_matches_fp32(ctx, dense, case):
    fwd, w = dense
    fwd._cap_cache.clear()
    ctx.reset_engagement()
    y = _gpu(fwd, case).float().cpu().numpy()
    ctx.sync_check()
    e = ctx.engagement()
    # engagement first (tests/ming-dit-test.cc:638-676): every projection of
    # every block ran through the kernels once, dense, no adapter engaged, and
    # all modulated blocks in one modulation call -- only then accuracy
    assert e["linear_calls"] == N_PROJ and e["gemm_dense"] == N_PROJ
    assert e["lora_proj"] == 0 and e["lora_down"] == 0 and e["modulation"] == 1
    ref = _ref(fx.as_f32(w), case)
    err = O.rel_l2(y, ref)
    assert err <= BAR, f"{case}: rel-L2 {err:.4f} > {BAR}"


def _packed(w: dict, bits: int = 8):
    """Every block matrix whose width the group divides, quantized (w2's K =
    2730 stays dense, as the reference's selection rule does), and the same
    weights dequantized for the fp32 oracle."""
    packed, deq = dict(w), fx.as_f32(w)
    for k, v in w.items():
        base = k[:-len(".weight")] if k.endswith(".weight") else None
        if base is None or not any(base.endswith(n) for n in P.PROJ_NAMES + ("adaLN_modulation.0",)):
            continue
        if v.shape[1] % 64:
            continue
        pw = P.quantize_affine(P.bf16_bits_to_f32(v), bits)
        packed[k] = pw
        deq[k] = O.dequant(pw.data, pw.scales, pw.biases, pw.n, pw.k, bits).astype(np.float32)
    return packed, deq


def test_pack_forward(ctx):
    """w8 pack (see _packed); the oracle runs the same dequantized weights in
    fp32."""
    w = fx.make_weights(0)
    packed, deq = _packed(w)
    fwd = DitForward(ctx, CFG, packed, torch.device("cuda", 0))
    ctx.reset_engagement()
    y = _gpu(fwd, "case_a").float().cpu().numpy()
    e = ctx.engagement()
    fwd.free()
    err = O.rel_l2(y, _ref(deq, "case_a"))
    assert e["gemm_w8"] == 6 * (2 * fx.NREF + fx.NLAY) and e["gemm_dense"] == 2 * fx.NREF + fx.NLAY
    assert err <= BAR, f"pack rel-L2 {err:.4f}"


def test_pack_file_forward(ctx, tmp_path):
    """The same w8 pack written by the library's C++ pack writer to a
    .safetensors file and read back by its reader (projections uploaded by
    mp_pack_upload's load_qw_-style detection): the forward is bit-identical to
    the one built from the Python-quantized arrays, and within the bar of the
    fp32 oracle on the dequantized weights."""
    from mingproj.lora import write_safetensors
    from mingproj.packio import Pack, quantize_pack
    w = fx.make_weights(0)
    src, dst = tmp_path / "dense.safetensors", tmp_path / "w8.safetensors"
    write_safetensors(src, w)
    nq, _ = quantize_pack(src, dst, 8)
    assert nq == 6 * (2 * fx.NREF + fx.NLAY) + (fx.NREF + fx.NLAY)  # w2 (K 2730) stays dense
    packed, deq = dict(w), fx.as_f32(w)
    for k, v in w.items():
        base = k[:-len(".weight")] if k.endswith(".weight") else None
        if base is None or not any(base.endswith(n) for n in P.PROJ_NAMES + ("adaLN_modulation.0",)):
            continue
        if v.shape[1] % 64:
            continue
        pw = P.quantize_affine(P.bf16_bits_to_f32(v), 8)
        packed[k] = pw
        deq[k] = O.dequant(pw.data, pw.scales, pw.biases, pw.n, pw.k, 8).astype(np.float32)
    with Pack(dst) as pk:
        fwd = DitForward(ctx, CFG, pk, torch.device("cuda", 0))
    y_file = _gpu(fwd, "case_b")
    fwd.free()
    fwd = DitForward(ctx, CFG, packed, torch.device("cuda", 0))
    y_dict = _gpu(fwd, "case_b")
    fwd.free()
    ctx.sync_check()
    assert torch.equal(y_file.view(torch.int16), y_dict.view(torch.int16))
    err = O.rel_l2(y_file.float().cpu().numpy(), _ref(deq, "case_b"))
    assert err <= BAR, f"pack-file rel-L2 {err:.4f}"


def test_caption_cache(ctx, dense):
    """The caption cache (src/ming-dit.cc:1543-1577): the same caption bytes
    hit (also for another image size) and give the bits a cold forward gives;
    another caption, a strength change or a new adapter binding misses."""
    fwd, w = dense
    fwd._cap_cache.clear()
    lat, cap, q, gh, gw = fx.make_inputs("case_a")
    y0 = fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)
    assert not fwd.last_cap_cache_hit
    y1 = fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)
    assert fwd.last_cap_cache_hit and torch.equal(y0.view(torch.int16), y1.view(torch.int16))
    # another image size (case_c: 16 x 15) with the same caption: a hit, and
    # the bits of a forward with the cache off
    lat_c, _, _, gh_c, gw_c = fx.make_inputs("case_c")
    y2 = fwd.forward(_dev(lat_c), _dev(cap), q, gh_c, gw_c, 0.3)
    assert fwd.last_cap_cache_hit
    fwd.cap_cache_entries = 0
    fwd._cap_cache.clear()
    y2_cold = fwd.forward(_dev(lat_c), _dev(cap), q, gh_c, gw_c, 0.3)
    assert torch.equal(y2.view(torch.int16), y2_cold.view(torch.int16))
    fwd.cap_cache_entries = 4
    fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)  # refills the entry
    assert not fwd.last_cap_cache_hit
    # a different caption misses; both entries then serve
    _, cap_b, q_b, _, _ = fx.make_inputs("case_b")
    fwd.forward(_dev(lat), _dev(cap_b), q_b, gh, gw, fx.SIGMA)
    assert not fwd.last_cap_cache_hit
    fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)
    assert fwd.last_cap_cache_hit
    fwd.forward(_dev(lat), _dev(cap_b), q_b, gh, gw, fx.SIGMA)
    assert fwd.last_cap_cache_hit
    # a strength change drops every entry
    ctx.set_strength(3, 0.5)
    fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)
    assert not fwd.last_cap_cache_hit
    ctx.set_strength(3, 1.0)
    fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)
    assert not fwd.last_cap_cache_hit
    # a new binding drops them too (its strength was already 1.0)
    binding, _ = _adapter(seed=9)
    fwd.proj.bind_slot(1, binding)
    ya = fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)
    assert not fwd.last_cap_cache_hit
    fwd.proj.unbind_slot(1)
    yb = fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)
    assert not fwd.last_cap_cache_hit and torch.equal(yb.view(torch.int16), y1.view(torch.int16))
    assert not torch.equal(ya.view(torch.int16), y1.view(torch.int16))


def _adapter(seed=5, rank=8, alpha=16.0):
    rng = np.random.default_rng(seed)
    bound, fused_delta = {}, {}
    for pre in fx.block_prefixes():
        for name in P.PROJ_NAMES:
            out, inp = ((fx.FFN, fx.DIM) if name in ("feed_forward.w1", "feed_forward.w3") else
                        (fx.DIM, fx.FFN) if name == "feed_forward.w2" else (fx.DIM, fx.DIM))
            a = rng.normal(0, 1 / np.sqrt(inp), size=(rank, inp)).astype(np.float32)
            b = rng.normal(0, 0.5 / np.sqrt(rank), size=(out, rank)).astype(np.float32)
            a_fold = P.f32_to_bf16_bits(a * np.float32(alpha / rank))
            b_bits = P.f32_to_bf16_bits(b)
            bound[pre + name] = Factors(a_fold, b_bits)
            fused_delta[pre + name + ".weight"] = (P.bf16_bits_to_f32(b_bits).astype(np.float64) @
                                                   P.bf16_bits_to_f32(a_fold).astype(np.float64))
    return SlotBinding("synthetic", bound), fused_delta


def test_runtime_lora_matches_fused_and_strength_zero_is_base(ctx, dense):
    fwd, w = dense
    base = _gpu(fwd, "case_a")
    binding, delta = _adapter()
    assert fwd.proj.bind_slot(0, binding) == 7 * (2 * fx.NREF + fx.NLAY)
    ctx.set_strength(0, 1.0)
    ctx.reset_engagement()
    adapted = _gpu(fwd, "case_a")
    lora_proj = ctx.engagement()["lora_proj"]
    ctx.set_strength(0, 0.0)
    off = _gpu(fwd, "case_a")
    ctx.set_strength(0, 1.0)
    again = _gpu(fwd, "case_a")
    fwd.proj.unbind_slot(0)
    fused = fx.as_f32(w)
    for k, d in delta.items():
        fused[k] = (fused[k].astype(np.float64) + d).astype(np.float32)
    ref = _ref(fused, "case_a")
    a_np = adapted.float().cpu().numpy()
    vs_fused = O.rel_l2(a_np, ref)
    moved = O.rel_l2(base.float().cpu().numpy(), a_np)
    assert lora_proj == 7 * (2 * fx.NREF + fx.NLAY)
    assert vs_fused < K_SMALL_TOL, f"vs fused {vs_fused:.4f}"
    assert moved > 0.1 and moved > 10 * vs_fused, f"moved {moved:.4f}, err {vs_fused:.4f}"
    assert torch.equal(off.view(torch.int16), base.view(torch.int16)), "strength 0 != base"
    assert torch.equal(again.view(torch.int16), adapted.view(torch.int16)), "not repeatable"


def test_cfg_batch_matches_separate_forwards(ctx, dense):
    """Classifier-free guidance as one batched pass (the conditional and the
    negative caption over the same latents): every
    projection runs once over both images' rows, and each image's output has
    the bits of its own forward, with per-image timesteps too."""
    fwd, w = dense
    lat, cap, q, gh, gw = fx.make_inputs("case_a")
    neg = np.zeros_like(cap)
    lat2 = fx.make_inputs("case_b")[0]
    lat_d = torch.stack([_dev(lat), _dev(lat2)])
    fwd._cap_cache.clear()
    yb = fwd.forward_batch(lat_d, [_dev(cap), _dev(neg)], q, gh, gw, [fx.SIGMA, 0.3])
    fwd._cap_cache.clear()
    y0 = fwd.forward(_dev(lat), _dev(cap), q, gh, gw, fx.SIGMA)
    y1 = fwd.forward(_dev(lat2), _dev(neg), q, gh, gw, 0.3)
    assert yb.shape == (2,) + tuple(y0.shape)
    assert torch.equal(yb[0].view(torch.int16), y0.view(torch.int16)), "image 0 differs"
    assert torch.equal(yb[1].view(torch.int16), y1.view(torch.int16)), "image 1 differs"
    # and against the fp32 restatement, image by image
    ref0 = _ref(fx.as_f32(w), "case_a")
    assert O.rel_l2(yb[0].float().cpu().numpy(), ref0) <= BAR


def test_graph_replay_matches_eager(ctx, dense):
    """The per-step forward as one CUDA-graph replay: the bits of the eager
    batched forward on the same inputs, step after step with new latents and
    timesteps (one capture); a LoRA strength or binding change captures again
    and the replay follows the new state."""
    fwd, w = dense
    lat, cap, q, gh, gw = fx.make_inputs("case_a")
    lat2 = fx.make_inputs("case_b")[0]
    caps = [_dev(cap), _dev(np.zeros_like(cap))]
    runner = fwd.graph(2, q, gh, gw, cap.shape[0])
    steps = [(torch.stack([_dev(lat), _dev(lat2)]), [0.9, 0.9]),
             (torch.stack([_dev(lat2), _dev(lat)]), [0.5, 0.3]),
             (torch.stack([_dev(lat), _dev(lat)]), [0.1, 0.7])]
    outs = [runner(l, caps, s) for l, s in steps]
    assert runner.captures == 1 and runner.replays == 3
    for (l, s), y in zip(steps, outs):
        ye = fwd.forward_batch(l, caps, q, gh, gw, s)
        assert torch.equal(y.view(torch.int16), ye.view(torch.int16)), s
    # an adapter bound and engaged: captured again, close to the eager path
    # (which may take the fused LoRA prologue, with its own summation order)
    binding, _ = _adapter(seed=11)
    fwd.proj.bind_slot(2, binding)
    ctx.set_strength(2, 0.8)
    ya = runner(*steps[1][:1], caps, steps[1][1])
    assert runner.captures == 2
    ye = fwd.forward_batch(steps[1][0], caps, q, gh, gw, steps[1][1])
    moved = O.rel_l2(outs[1].float().cpu().numpy(), ya.float().cpu().numpy())
    err = O.rel_l2(ye.float().cpu().numpy(), ya.float().cpu().numpy())
    assert moved > 0.05 and err < 5e-3, (moved, err)
    # strength 0: captured again, and the base bits come back
    ctx.set_strength(2, 0.0)
    y0 = runner(*steps[1][:1], caps, steps[1][1])
    assert runner.captures == 3
    assert torch.equal(y0.view(torch.int16), outs[1].view(torch.int16))
    fwd.proj.unbind_slot(2)
    ctx.set_strength(2, 1.0)
    runner.release()
    ctx.sync_check()


def test_lora_pack_moves_like_bf16(ctx, dense):
    """The same adapter on a w8 pack of the same model moves the pack's
    output as it moves the bf16 model's: the reference's test_lora_pack
    (tests/ming-dit-test.cc:2056-2102), restated on the synthetic small DiT.
    Engagement is checked first: packed GEMMs ran and every projection took
    the adapter; strength 0 gives the pack's base bits."""
    fwd_bf, w = dense
    binding, _ = _adapter(seed=21)
    fwd_bf._cap_cache.clear()
    bf_base = _gpu(fwd_bf, "case_b").float().cpu().numpy()
    assert fwd_bf.proj.bind_slot(0, binding) == N_PROJ
    ctx.set_strength(0, 1.0)
    bf_lora = _gpu(fwd_bf, "case_b").float().cpu().numpy()
    fwd_bf.proj.unbind_slot(0)

    packed, _ = _packed(w)
    fwd = DitForward(ctx, CFG, packed, torch.device("cuda", 0))
    try:
        base = _gpu(fwd, "case_b")
        assert fwd.proj.bind_slot(0, binding) == N_PROJ
        ctx.reset_engagement()
        r = _gpu(fwd, "case_b")
        ctx.sync_check()
        e = ctx.engagement()
        assert e["gemm_w8"] > 0 and e["lora_proj"] == N_PROJ
        ctx.set_strength(0, 0.0)
        z = _gpu(fwd, "case_b")
        ctx.set_strength(0, 1.0)
    finally:
        fwd.free()
    rn, bn = r.float().cpu().numpy(), base.float().cpu().numpy()
    moved = O.rel_l2(rn, bn)
    bf_moved = O.rel_l2(bf_lora, bf_base)
    d_base = O.rel_l2(bn, bf_base)
    d_lora = O.rel_l2(rn, bf_lora)
    assert 0.5 * bf_moved < moved < 2.0 * bf_moved, (moved, bf_moved)
    assert d_lora < 1.5 * d_base + 0.01, (d_lora, d_base)
    assert torch.equal(z.view(torch.int16), base.view(torch.int16)), "strength 0 != pack base"


def test_config_keys_drive_the_slots(ctx, tmp_path):
    """The caller-side keys (mingproj.lora_config) on a real forward, as the
    reference's generator test drives them (tests/ming-lora-test.cc:268-337):
    `lora2` alone binds slot 1 at `lora2_scale`; its strength is live per
    request (0 gives the base bits, back to 0.5 gives the adapted bits
    again); a later beat naming another `lora2` path is ignored and said."""
    from mingproj import lora as L
    from mingproj import lora_config as LC

    rng = np.random.default_rng(3)
    t = {}
    for pre in fx.block_prefixes():
        for name in P.PROJ_NAMES:
            out, inp = ((fx.FFN, fx.DIM) if name in ("feed_forward.w1", "feed_forward.w3") else
                        (fx.DIM, fx.FFN) if name == "feed_forward.w2" else (fx.DIM, fx.DIM))
            t[f"transformer.{pre}{name}.lora_A.weight"] = P.f32_to_bf16_bits(
                rng.normal(0, 1 / np.sqrt(inp), size=(8, inp)).astype(np.float32))
            t[f"transformer.{pre}{name}.lora_B.weight"] = P.f32_to_bf16_bits(
                rng.normal(0, 0.2, size=(out, 8)).astype(np.float32))
    adir = tmp_path / "style"
    adir.mkdir()
    L.write_safetensors(adir / "style.safetensors", t)

    def resolve(ref):  # a directory holding one .safetensors, or a file
        pth = Path(ref)
        if pth.is_dir():
            files = sorted(pth.glob("*.safetensors"))
            return str(files[0]) if len(files) == 1 else None
        return str(pth) if pth.is_file() else None

    fwd = DitForward(ctx, CFG, fx.make_weights(0), torch.device("cuda", 0))
    try:
        base = _gpu(fwd, "case_a")
        cfg = {"lora2": str(adir), "lora2_scale": 0.5}
        st = LC.bind_from_config(fwd.proj, LC.forwarded_config(cfg), resolve, fx.DIM, fx.FFN)
        assert fwd.proj.lora_modules(1) == N_PROJ and fwd.proj.lora_modules(0) == 0
        assert f"runtime LoRA modules bound: lora2 {N_PROJ}" in st.infos
        assert ctx.strength(1) == 0.5 and ctx.strength(0) == 1.0
        ctx.reset_engagement()
        h = _gpu(fwd, "case_a")
        assert ctx.engagement()["lora_proj"] == N_PROJ
        v0 = ctx.state_version()
        assert LC.apply_keys({"lora2_scale": 0.0}, st, ctx.set_strength) == 1
        assert ctx.state_version() != v0
        z = _gpu(fwd, "case_a")
        assert LC.apply_keys({"lora2_scale": 0.5, "shift": 3.0}, st, ctx.set_strength) == 1
        h2 = _gpu(fwd, "case_a")
        assert LC.apply_keys({"lora2": "/nonexistent/x.safetensors", "lora2_scale": 0.5}, st,
                             ctx.set_strength, fwd.proj.lora_modules) == 0
        h3 = _gpu(fwd, "case_a")
        ctx.sync_check()
    finally:
        for i in range(8):
            ctx.set_strength(i, 1.0)
        fwd.free()
    assert any("is IGNORED" in m for m in st.warnings)
    assert O.rel_l2(h.float().cpu().numpy(), base.float().cpu().numpy()) > 0.005
    assert torch.equal(z.view(torch.int16), base.view(torch.int16)), "lora2_scale 0 != base"
    assert torch.equal(h2.view(torch.int16), h.view(torch.int16)), "back to 0.5 != first"
    assert torch.equal(h3.view(torch.int16), h.view(torch.int16)), "ignored path changed it"


def test_stage_trace_matches_oracle(ctx, dense, tmp_path, monkeypatch):
    """VPIPE_MING_DIT_TRACE (the reference's per-stage trace,
    src/ming-dit.cc:1658-1687): the forward writes the reference's stages
    (embed, ctx, blk<L>) as raw float32 rows, and each is within the forward's
    bar of the fp32 restatement's same stage."""
    fwd, w = dense
    gd, rd = tmp_path / "gpu", tmp_path / "ref"
    monkeypatch.setenv("VPIPE_MING_DIT_TRACE", str(gd))
    _gpu(fwd, "case_a")
    ctx.sync_check()
    monkeypatch.delenv("VPIPE_MING_DIT_TRACE")
    lat, cap, q, gh, gw = fx.make_inputs("case_a")
    DitRef(fx.as_f32(w), fx.DIM, fx.HEADS, fx.NREF, fx.NLAY, fx.CAPF).forward(
        P.bf16_bits_to_f32(lat), P.bf16_bits_to_f32(cap), q, gh, gw, fx.SIGMA, trace_dir=str(rd))
    tags = ["embed", "ctx"] + [f"blk{i}" for i in range(fx.NREF + fx.NLAY)]
    assert sorted(p.stem for p in gd.glob("*.f32")) == sorted(tags)
    for tag in tags:
        a = np.fromfile(gd / f"{tag}.f32", np.float32)
        b = np.fromfile(rd / f"{tag}.f32", np.float32)
        assert a.shape == b.shape and a.size > 0, tag
        err = O.rel_l2(a, b)
        assert err <= BAR, f"{tag}: rel-L2 {err:.4f} > {BAR}"
