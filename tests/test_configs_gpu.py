"""The BASELINE configurations 3-5 at their own sizes, through the C-ABI,
checked against the fp64 oracle on sampled rows (every tile class covered:
first rows, interior, the ragged tail) and through size-independent
properties: live strengths re-set between forwards give back the same bits,
slots at strength 0 reproduce the fewer-slot run bit for bit, and each image of
a batch follows its own strength vector (tests/ming-dit-test.cc:1249-1339 for
the strength semantics)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from mingproj import pack as P

pytestmark = pytest.mark.gpu

TOL = 5e-3  # per-projection rel-L2 vs the fp64 oracle


def _x_dev(seed: int, m: int, k: int) -> torch.Tensor:
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)


def _rows_host(x: torch.Tensor, rows: np.ndarray) -> np.ndarray:
    idx = torch.from_numpy(rows).to(x.device)
    return x.index_select(0, idx).view(torch.int16).cpu().numpy().view(np.uint16)


def _host(y: torch.Tensor, rows: np.ndarray) -> np.ndarray:
    idx = torch.from_numpy(rows).to(y.device)
    return y.index_select(0, idx).float().cpu().numpy().astype(np.float64)


def _bits(y: torch.Tensor) -> np.ndarray:
    return y.view(torch.int16).cpu().numpy()


def _sample_rows(rng, m: int, n_inner: int = 40) -> np.ndarray:
    tail = np.arange(max(0, m - 24), m)
    head = np.arange(0, 8)
    inner = rng.choice(m, size=n_inner, replace=False)
    return np.unique(np.concatenate([head, inner, tail]))


def _upload(ctx, pw):
    return ctx.upload(pw.n, pw.k, pw.bits, pw.data, pw.scales, pw.biases, mode=pw.mode)


def test_config3_w4_2048_strengths_reset_between_forwards(ctx):
    """Config 3: x [16896, 3840] (16384 image + 512 text tokens), w4 affine
    group 64, eight rank-32 slots; 11 forwards with the strengths re-set
    before each. Forwards with the same strengths are bit-identical; three
    of them are checked against the oracle."""
    rng = np.random.default_rng(3)
    m, n, k = 16896, 3840, 3840
    pw = P.synthetic_affine(rng, n, k, 4)
    w = _upload(ctx, pw)
    facs = []
    for i in range(8):
        a, b = P.synthetic_lora(rng, n, k, 32)
        w.bind(i, a, b)
        facs.append((a, b))
    x = _x_dev(30, m, k)
    sets = [rng.uniform(-1.0, 1.5, size=8) for _ in range(3)]
    outs = {}
    for step in range(11):
        which = step % 3
        for i in range(8):
            ctx.set_strength(i, float(sets[which][i]))
        y = ctx.linear(w, x)
        ctx.sync_check()
        if which not in outs:
            outs[which] = (y, _bits(y))
        else:
            assert np.array_equal(_bits(y), outs[which][1]), f"forward {step} differs"
    rows = _sample_rows(rng, m)
    xr = _rows_host(x, rows)
    for which in range(3):
        slots = [(facs[i][0], facs[i][1], float(sets[which][i])) for i in range(8)]
        ref = O.projection(xr, pw.data, pw.scales, pw.biases, n, k, 4, False, slots)
        err = O.rel_l2(_host(outs[which][0], rows), ref)
        assert err <= TOL, f"strength set {which}: rel-L2 {err:.3e}"
    for i in range(8):
        ctx.set_strength(i, 1.0)
    w.free()


def test_config4_dense_cfg_zero_strength_slots_bit_identical(ctx):
    """Config 4: dense bf16 base ~N(0, 0.02), CFG batch 2 (M = 2 x 4352),
    eight slots bound; slots 3-8 at strength 0 reproduce, bit for bit, the
    run of the same weight with only slots 1-2 bound; oracle parity on rows
    of both CFG halves."""
    rng = np.random.default_rng(4)
    m, n, k = 2 * 4352, 3840, 3840
    pw = P.synthetic_dense(rng, n, k, std=0.02)
    w8 = _upload(ctx, pw)
    w2 = _upload(ctx, pw)
    ranks = [4, 8, 8, 16, 16, 32, 32, 64]
    facs = [P.synthetic_lora(rng, n, k, r) for r in ranks]
    for i, f in enumerate(facs):
        w8.bind(i, *f)
        if i < 2:
            w2.bind(i, *f)
    ctx.set_strength(0, 0.7)
    ctx.set_strength(1, -0.4)
    for i in range(2, 8):
        ctx.set_strength(i, 0.0)
    x = _x_dev(40, m, k)
    y8 = ctx.linear(w8, x)
    y2 = ctx.linear(w2, x)
    ctx.sync_check()
    assert np.array_equal(_bits(y8), _bits(y2)), "zero-strength slots must not change a bit"
    rows = _sample_rows(rng, m)
    ref = O.projection(_rows_host(x, rows), pw.data, None, None, n, k, 0, False,
                       [(facs[0][0], facs[0][1], 0.7), (facs[1][0], facs[1][1], -0.4)])
    err = O.rel_l2(_host(y8, rows), ref)
    for i in range(8):
        ctx.set_strength(i, 1.0)
    w8.free()
    w2.free()
    assert err <= TOL, f"rel-L2 {err:.3e}"


def test_config4_quantized_modulation_m2(ctx):
    """Config 4's quantized adaLN modulation Linear [3840 -> 4 x 3840] at
    M = 2 (the CFG pair), two blocks in one launch, against the oracle."""
    rng = np.random.default_rng(41)
    H, K, m = 3840, 3840, 2
    pws, ws, biases = [], [], []
    for _ in range(2):
        pw = P.synthetic_affine(rng, 4 * H, K, 8)
        pws.append(pw)
        ws.append(_upload(ctx, pw))
        biases.append(P.f32_to_bf16_bits(rng.normal(0, 0.02, 4 * H).astype(np.float32)))
    mset = ctx.modulation_set(ws, biases)
    temb = P.f32_to_bf16_bits(rng.normal(size=(m, K)).astype(np.float32))
    tdev = torch.from_numpy(temb.view(np.int16).copy()).view(torch.bfloat16).cuda()
    mods, _, _ = ctx.modulation(mset, tdev, fold=False)
    ctx.sync_check()
    mods = mods.float().cpu().numpy()
    mset.free()
    for w in ws:
        w.free()
    for b in range(2):
        ref = O.modulation(temb, pws[b].data, pws[b].scales, pws[b].biases, biases[b], 4 * H, K,
                           8)
        assert O.rel_l2(mods[b], ref) <= TOL


def test_config5_batch8_per_image_strengths(ctx):
    """Config 5: a batch of 8 images (8 x 4352 rows) through one launch, w8,
    mixed ranks 8..64, each image with its own strength vector over the
    shared slots (per-row-segment strengths)."""
    rng = np.random.default_rng(5)
    per, n, k = 4352, 3840, 3840
    m = 8 * per
    pw = P.synthetic_affine(rng, n, k, 8)
    w = _upload(ctx, pw)
    ranks = [8, 16, 24, 32, 40, 48, 56, 64]
    facs = [P.synthetic_lora(rng, n, k, r, b_std=0.02) for r in ranks]
    for i, f in enumerate(facs):
        w.bind(i, *f)
    S = rng.uniform(-1.0, 1.5, size=(8, 8)).astype(np.float32)
    S[2, :] = 0.0   # an image with every adapter off
    S[5, 3] = 0.0   # one slot off for one image
    starts = (np.arange(9) * per).astype(np.int32)
    ctx.set_strengths_rows(S, starts)
    x = _x_dev(50, m, k)
    y = ctx.linear(w, x)
    ctx.sync_check()
    ctx.clear_strengths_rows()
    try:
        for g in range(8):
            rows = g * per + _sample_rows(rng, per, n_inner=6)
            slots = [(facs[i][0], facs[i][1], float(S[g, i])) for i in range(8)]
            ref = O.projection(_rows_host(x, rows), pw.data, pw.scales, pw.biases, n, k, 8, False,
                               slots)
            err = O.rel_l2(_host(y, rows), ref)
            assert err <= TOL, f"image {g}: rel-L2 {err:.3e}"
    finally:
        w.free()
