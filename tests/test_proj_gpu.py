"""Parity of the sm_100a projection kernel (through the C-ABI) against the fp64
CPU oracle: per-projection rel-L2 <= 5e-3, bit-exact
strength-0 and slot-position properties (reference tests
tests/ming-dit-test.cc:1249-1339, tests/ming-lora-test.cc:283-312)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from mingproj import pack as P
from mingproj.proj import MP_QUANT_SYMMETRIC

pytestmark = pytest.mark.gpu

TOL = 5e-3  # per-projection rel-L2 vs the fp64 dequant+LoRA host reference


def _x(rng, m, k, ld=None):
    ld = ld or k
    x = rng.normal(0.0, 1.0, size=(m, ld)).astype(np.float32)
    return P.f32_to_bf16_bits(x)


def _upload(ctx, pw: P.PackedWeight):
    return ctx.upload(pw.n, pw.k, pw.bits, pw.data, pw.scales, pw.biases, mode=pw.mode)


def _to_dev(bits16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits16.view(np.int16)).view(torch.bfloat16).cuda()


def _host(y: torch.Tensor) -> np.ndarray:
    return y.float().cpu().numpy().astype(np.float64)


def _bits(y: torch.Tensor) -> np.ndarray:
    return y.view(torch.int16).cpu().numpy()


def _weight(rng, n, k, bits, mode=0):
    if bits == 0:
        return P.synthetic_dense(rng, n, k)
    if mode == MP_QUANT_SYMMETRIC:
        return P.synthetic_symmetric_w8(rng, n, k)
    return P.synthetic_affine(rng, n, k, bits)


@pytest.mark.parametrize("bits,mode", [(0, 0), (8, 0), (4, 0), (8, 1)])
@pytest.mark.parametrize("m,n,k", [(256, 128, 64), (300, 256, 256), (64, 384, 128),
                                   (130, 128, 192), (1, 128, 64), (517, 640, 640)])
def test_base_matches_oracle(ctx, bits, mode, m, n, k):
    rng = np.random.default_rng(1000 + m + n + k + bits)
    pw = _weight(rng, n, k, bits, mode)
    w = _upload(ctx, pw)
    x = _x(rng, m, k)
    y = ctx.linear(w, _to_dev(x))
    ctx.sync_check()
    ref = O.projection(x, pw.data, pw.scales, pw.biases, n, k, bits, mode == 1)
    err = O.rel_l2(_host(y), ref)
    w.free()
    assert err <= TOL, f"rel-L2 {err:.3e} (bits {bits} mode {mode} m {m} n {n} k {k})"


def test_codes_round_trip(ctx):
    rng = np.random.default_rng(7)
    for bits in (8, 4):
        pw = P.synthetic_affine(rng, 256, 512, bits)
        w = _upload(ctx, pw)
        assert np.array_equal(w.read_codes(), pw.data.view(np.uint8).ravel())
        w.free()


@pytest.mark.parametrize("bits", [8, 4, 0])
def test_lora_slots_match_oracle(ctx, bits):
    rng = np.random.default_rng(11 + bits)
    m, n, k = 384, 256, 512
    pw = _weight(rng, n, k, bits)
    w = _upload(ctx, pw)
    ranks = [4, 8, 8, 16, 16, 32, 32, 64]
    strengths = rng.uniform(-1.0, 1.5, size=8)
    slots = []
    for i, r in enumerate(ranks):
        a, b = P.synthetic_lora(rng, n, k, r, b_std=0.05)
        w.bind(i, a, b)
        ctx.set_strength(i, float(strengths[i]))
        slots.append((a, b, float(strengths[i])))
    x = _x(rng, m, k)
    y = ctx.linear(w, _to_dev(x))
    ctx.sync_check()
    ref = O.projection(x, pw.data, pw.scales, pw.biases, n, k, bits, False, slots)
    base = O.projection(x, pw.data, pw.scales, pw.biases, n, k, bits, False)
    err = O.rel_l2(_host(y), ref)
    moved = O.rel_l2(base, ref)
    for i in range(8):
        ctx.set_strength(i, 1.0)
    w.free()
    assert moved > 10 * TOL, f"adapters barely move the output ({moved:.3e})"
    assert err <= TOL, f"rel-L2 {err:.3e} with 8 slots (moved {moved:.3e})"


def test_strength_zero_is_base_bit_exact(ctx):
    rng = np.random.default_rng(21)
    m, n, k = 300, 256, 256
    pw = P.synthetic_affine(rng, n, k, 8)
    w = _upload(ctx, pw)
    xd = _to_dev(_x(rng, m, k))
    base = _bits(ctx.linear(w, xd))
    a, b = P.synthetic_lora(rng, n, k, 16)
    w.bind(0, a, b)
    ctx.set_strength(0, 0.8)
    adapted = _bits(ctx.linear(w, xd))
    ctx.set_strength(0, 0.0)
    off = _bits(ctx.linear(w, xd))
    ctx.set_strength(0, 0.8)
    back = _bits(ctx.linear(w, xd))
    ctx.set_strength(0, 1.0)
    w.free()
    assert not np.array_equal(adapted, base)
    assert np.array_equal(off, base), "strength 0 must reproduce the base bit for bit"
    assert np.array_equal(back, adapted), "the strength is live and repeatable"


def test_slot_position_is_bit_exact(ctx):
    """The same adapter in slot 0, 1 or 7 gives the same bits
    (tests/ming-dit-test.cc:1294-1339)."""
    rng = np.random.default_rng(31)
    m, n, k = 256, 256, 256
    pw = P.synthetic_affine(rng, n, k, 4)
    w = _upload(ctx, pw)
    xd = _to_dev(_x(rng, m, k))
    a, b = P.synthetic_lora(rng, n, k, 8)
    outs = []
    for slot in (0, 1, 7):
        w.bind(slot, a, b)
        outs.append(_bits(ctx.linear(w, xd)))
        w.unbind(slot)
    w.free()
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


def test_zero_strength_slots_equal_fewer_slot_run(ctx):
    """8 slots bound with slots 3-8 at strength 0 must be
    bit-identical to the 2-slot run."""
    rng = np.random.default_rng(41)
    m, n, k = 320, 384, 384
    pw = P.synthetic_dense(rng, n, k)
    ranks = [4, 8, 8, 16, 16, 32, 32, 64]
    facs = [P.synthetic_lora(rng, n, k, r) for r in ranks]
    xd = _to_dev(_x(rng, m, k))
    w2 = _upload(ctx, pw)
    for i in range(2):
        w2.bind(i, *facs[i])
    ctx.set_strength(0, 0.7)
    ctx.set_strength(1, -0.4)
    two = _bits(ctx.linear(w2, xd))
    w8 = _upload(ctx, pw)
    for i in range(8):
        w8.bind(i, *facs[i])
    for i in range(2, 8):
        ctx.set_strength(i, 0.0)
    eight = _bits(ctx.linear(w8, xd))
    for i in range(8):
        ctx.set_strength(i, 1.0)
    w2.free()
    w8.free()
    assert np.array_equal(two, eight)


def test_per_row_strengths(ctx):
    """Config 5: each image (row segment) has its own strength vector."""
    rng = np.random.default_rng(51)
    n, k = 256, 256
    rows = [128, 200, 72]
    m = sum(rows)
    pw = P.synthetic_affine(rng, n, k, 8)
    w = _upload(ctx, pw)
    ranks = [8, 16, 32]
    facs = [P.synthetic_lora(rng, n, k, r, b_std=0.05) for r in ranks]
    for i, f in enumerate(facs):
        w.bind(i, *f)
    S = np.zeros((3, 8), dtype=np.float32)
    S[:, :3] = rng.uniform(-1.0, 1.5, size=(3, 3))
    S[1, 2] = 0.0
    starts = np.cumsum([0] + rows).astype(np.int32)
    ctx.set_strengths_rows(S, starts)
    x = _x(rng, m, k)
    y = _host(ctx.linear(w, _to_dev(x)))
    ctx.clear_strengths_rows()
    ctx.sync_check()
    w.free()
    for g in range(3):
        r0, r1 = starts[g], starts[g + 1]
        slots = [(facs[i][0], facs[i][1], float(S[g, i])) for i in range(3)]
        ref = O.projection(x[r0:r1], pw.data, pw.scales, pw.biases, n, k, 8, False, slots)
        err = O.rel_l2(y[r0:r1], ref)
        assert err <= TOL, f"segment {g}: rel-L2 {err:.3e}"


def test_linear_shared_equals_separate(ctx):
    """One shared call equals separate calls. The rank-space pre-GEMM may split
    K differently for the stacked and the single-weight rank widths, which
    changes only fp32 summation order: outputs agree to within one bf16 ulp."""
    rng = np.random.default_rng(61)
    m, n, k = 260, 256, 384
    pws = [P.synthetic_affine(rng, n, k, 8) for _ in range(3)]
    ws = [_upload(ctx, p) for p in pws]
    for j, w in enumerate(ws):
        for i, r in enumerate([4, 16, 32][: j + 1]):
            w.bind(i, *P.synthetic_lora(rng, n, k, r))
    ctx.set_strength(0, 0.5)
    ctx.set_strength(1, -1.0)
    ctx.set_strength(2, 1.25)
    xd = _to_dev(_x(rng, m, k))
    sep = [_bits(ctx.linear(w, xd)) for w in ws]
    sh = [_bits(y) for y in ctx.linear_shared(ws, xd)]
    for i in range(3):
        ctx.set_strength(i, 1.0)
    for w in ws:
        w.free()
    for a, b in zip(sep, sh):
        fa, fb = P.bf16_bits_to_f32(a), P.bf16_bits_to_f32(b)
        # one bf16 ulp of the larger magnitude (8 significant bits)
        assert np.all(np.abs(fa - fb) <= np.maximum(np.abs(fa), np.abs(fb)) * 2.0**-7 + 1e-30)
        assert np.mean(a != b) < 0.01


@pytest.mark.parametrize("m,k", [(1024, 3840), (256, 10240), (4352, 640)])
def test_split_k_pre_gemm_matches_oracle_and_repeats(ctx, m, k):
    """Rank-space pre-GEMMs with few token tiles split K across CTAs and add
    the fp32 partials in split order in a second pass: parity with the oracle
    and bit-identical repeats."""
    rng = np.random.default_rng(m + k)
    n = 256
    pw = P.synthetic_affine(rng, n, k, 8)
    w = _upload(ctx, pw)
    slots = []
    for i, r in enumerate([4, 8, 8, 16, 16, 32, 32, 64]):
        a, b = P.synthetic_lora(rng, n, k, r, b_std=0.05)
        w.bind(i, a, b)
        s = float(rng.uniform(-1.0, 1.5))
        ctx.set_strength(i, s)
        slots.append((a, b, s))
    x = _x(rng, m, k)
    xd = _to_dev(x)
    y1 = ctx.linear(w, xd)
    y2 = ctx.linear(w, xd)
    ctx.sync_check()
    rows = np.sort(rng.choice(m, size=min(m, 96), replace=False))
    ref = O.projection(x[rows], pw.data, pw.scales, pw.biases, n, k, 8, False, slots)
    base = O.projection(x[rows], pw.data, pw.scales, pw.biases, n, k, 8, False)
    for i in range(8):
        ctx.set_strength(i, 1.0)
    w.free()
    assert np.array_equal(_bits(y1), _bits(y2)), "split-K result must not vary between runs"
    assert O.rel_l2(base, ref) > 10 * TOL
    err = O.rel_l2(_host(y1)[rows], ref)
    assert err <= TOL, f"rel-L2 {err:.3e}"


def test_engagement_counts(ctx):
    rng = np.random.default_rng(71)
    m, n, k = 128, 128, 128
    w = _upload(ctx, P.synthetic_affine(rng, n, k, 8))
    ctx.reset_engagement()
    xd = _to_dev(_x(rng, m, k))
    ctx.linear(w, xd)
    a, b = P.synthetic_lora(rng, n, k, 8)
    w.bind(3, a, b)
    ctx.linear(w, xd)
    e = ctx.engagement()
    w.free()
    assert e["linear_calls"] == 2 and e["lora_proj"] == 1 and e["gemm_w8"] == 2
    assert e["lora_down"] == 1 and e["kernels"] == 3
    want = 2 * (2.0 * m * n * k) + 2.0 * m * 8 * (k + n)
    assert abs(e["flops"] - want) < 1e-6 * want


def test_config1_full_size_sampled_rows(ctx):
    """BASELINE config 1 at full size (x [4096, 3840], symmetric w8, one rank-16
    slot at 0.8, seed 0), checked against the fp64 oracle on a row sample."""
    rng = np.random.default_rng(0)
    m, n, k = 4096, 3840, 3840
    x = P.f32_to_bf16_bits(rng.normal(0.0, 1.0, size=(m, k)).astype(np.float32))
    pw = P.synthetic_symmetric_w8(rng, n, k)
    a = P.f32_to_bf16_bits(rng.normal(0.0, 1.0 / 4.0, size=(16, k)).astype(np.float32))
    b = P.f32_to_bf16_bits(rng.normal(0.0, 0.01, size=(n, 16)).astype(np.float32))
    w = _upload(ctx, pw)
    w.bind(0, a, b)
    ctx.set_strength(0, 0.8)
    y = ctx.linear(w, _to_dev(x))
    ctx.sync_check()
    rows = np.sort(rng.choice(m, size=48, replace=False))
    ref = O.projection(x[rows], pw.data, pw.scales, None, n, k, 8, True, [(a, b, 0.8)])
    got = _host(y)[rows]
    ctx.set_strength(0, 1.0)
    w.free()
    err = O.rel_l2(got, ref)
    assert err <= TOL, f"config 1 sampled rel-L2 {err:.3e}"


@pytest.mark.parametrize("m,n,k", [(357, 1024, 2730), (100, 2730, 1024)])
def test_dense_ragged_k_with_lora(ctx, m, n, k):
    """Dense weights of any width (the small DiT's FFN is 2730 wide): rows are
    stored at a padded pitch and the last K tile reads zeros."""
    rng = np.random.default_rng(m + n + k)
    pw = P.synthetic_dense(rng, n, k)
    w = _upload(ctx, pw)
    a, b = P.synthetic_lora(rng, n, k, 8, b_std=0.05)
    w.bind(2, a, b)
    ctx.set_strength(2, 0.6)
    ld = (k + 7) // 8 * 8
    x = _x(rng, m, k, ld)
    xd = _to_dev(x)[:, :k]
    y = ctx.linear(w, xd)
    ctx.sync_check()
    ctx.set_strength(2, 1.0)
    ref = O.projection(np.ascontiguousarray(x[:, :k]), pw.data, None, None, n, k, 0, False,
                       [(a, b, 0.6)])
    assert np.array_equal(w.read_codes().view(np.uint16).reshape(n, k), pw.data)
    w.free()
    assert O.rel_l2(_host(y), ref) <= TOL


@pytest.mark.parametrize("bits", [8, 4, 0])
@pytest.mark.parametrize("m", [4400, 4352, 4200, 2176, 700])
def test_512_token_tiles_ragged_tail(ctx, bits, m):
    """Wide launches take 512-token pair tiles (two accumulators per dequantized
    stage): the last tile's second half is partly past M (4400), absent
    (4352: dropped accumulator) or both halves ragged (4200); narrower ones
    (2176, 700 rows) take 256- or 128-token tiles with their own stage
    layouts and a separate rank-space pre-GEMM. Rows sampled from every tile,
    the tail tile in full, against the oracle; LoRA slots live."""
    rng = np.random.default_rng(m + bits)
    n, k = 3840, 640
    pw = _weight(rng, n, k, bits)
    w = _upload(ctx, pw)
    slots = []
    for i, r in enumerate([8, 16, 32]):
        a, b = P.synthetic_lora(rng, n, k, r, b_std=0.05)
        w.bind(i, a, b)
        s = float(rng.uniform(-1.0, 1.5))
        ctx.set_strength(i, s)
        slots.append((a, b, s))
    x = _x(rng, m, k)
    y = ctx.linear(w, _to_dev(x))
    ctx.sync_check()
    tail0 = (m - 1) // 512 * 512
    rows = np.unique(np.concatenate([rng.choice(tail0, size=64, replace=False),
                                     np.arange(tail0, m)]))
    ref = O.projection(x[rows], pw.data, pw.scales, pw.biases, n, k, bits, False, slots)
    for i in range(3):
        ctx.set_strength(i, 1.0)
    w.free()
    got = _host(y)[rows]
    assert np.all(np.isfinite(got))
    err = O.rel_l2(got, ref)
    assert err <= TOL, f"rel-L2 {err:.3e} (bits {bits}, m {m})"


def test_shared_stack_cache_follows_reuploaded_weights(ctx):
    """Weights freed and uploaded again (possibly at the same host addresses)
    with other adapters never reuse the stacked factors cached for the first
    ones: each shared call matches the oracle."""
    rng = np.random.default_rng(91)
    m, n, k = 260, 256, 256
    x = _x(rng, m, k)
    xd = _to_dev(x)
    for rep in range(4):
        pws = [P.synthetic_dense(rng, n, k, std=0.05) for _ in range(2)]
        ws = [_upload(ctx, p) for p in pws]
        slots = []
        for j, w in enumerate(ws):
            a, b = P.synthetic_lora(rng, n, k, 16, b_std=0.05)
            w.bind(j, a, b)
            slots.append([(a, b, 1.0)])
        ys = ctx.linear_shared(ws, xd)
        ctx.sync_check()
        for j in range(2):
            ref = O.projection(x, pws[j].data, None, None, n, k, 0, False, slots[j])
            err = O.rel_l2(_host(ys[j]), ref)
            assert err <= TOL, f"re-upload {rep}, weight {j}: rel-L2 {err:.3e}"
        for w in ws:
            w.free()


@pytest.mark.parametrize("bits", [8, 4])
def test_reference_rounding_order_within_the_bar(ctx, bits):
    """The fused kernel rounds base + adapters once; the reference rounds the
    base output to bf16 and the sum again (src/ming-dit.cc:1763-1771). At
    config-2/3 magnitudes (4352-row text-plus-image shape cut to 640 rows,
    K 3840, eight slots of ranks {4..64}, B ~N(0, 0.01), strengths
    ~U(-1, 1.5)) the kernel's output sits within the per-projection bar of
    the reference-order result, as it does of the exact fp64 value."""
    rng = np.random.default_rng(31 + bits)
    m, n, k = 640, 768, 3840
    pw = P.synthetic_affine(rng, n, k, bits)
    w = _upload(ctx, pw)
    slots = []
    for i, r in enumerate((4, 8, 8, 16, 16, 32, 32, 64)):
        a, b = P.synthetic_lora(rng, n, k, r, b_std=0.01)
        s = float(rng.uniform(-1.0, 1.5))
        w.bind(i, a, b)
        ctx.set_strength(i, s)
        slots.append((a, b, s))
    x = _x(rng, m, k)
    try:
        y = _host(ctx.linear(w, _to_dev(x)))
        ctx.sync_check()
    finally:
        for i in range(8):
            ctx.set_strength(i, 1.0)
        w.free()
    two = O.projection_two_rounding(x, pw.data, pw.scales, pw.biases, n, k, bits, False, slots,
                                    round_t=True)
    exact = O.projection(x, pw.data, pw.scales, pw.biases, n, k, bits, False, slots)
    assert O.rel_l2(y, two) <= TOL, f"vs reference order {O.rel_l2(y, two):.3e}"
    assert O.rel_l2(y, exact) <= TOL, f"vs exact {O.rel_l2(y, exact):.3e}"


@pytest.mark.parametrize("bits,m,k,ranks", [
    (8, 256, 3840, [4, 8, 8, 16, 16, 32, 32, 64]),   # config-2 context refiner, to_out
    (8, 256, 10240, [4, 8, 8, 16, 16, 32, 32, 64]),  # config-2 context refiner, w2
    (4, 512, 3840, [32] * 8),                        # config-3 context refiner, to_out
])
def test_small_m_split_k_matches_oracle_and_batches(ctx, bits, m, k, ranks):
    """Few rows per image (the context refiner over a caption,
    src/ming-dit.cc:2388-2420): the projection splits K across CTA pairs and
    adds the fp32 partial sums in split order. Parity with the oracle on
    sampled rows, and a batch of two images (row segments with their own
    strengths) has each image's bits of its own call, because the token tile
    and the split counts are chosen from one image's rows."""
    rng = np.random.default_rng(bits * 1000 + m + k)
    n = 3840
    pw = P.synthetic_affine(rng, n, k, bits)
    w = _upload(ctx, pw)
    facs = []
    for i, r in enumerate(ranks):
        a, b = P.synthetic_lora(rng, n, k, r, b_std=0.05)
        w.bind(i, a, b)
        facs.append((a, b))
    S = rng.uniform(-1.0, 1.5, size=(2, 8)).astype(np.float32)
    x = _x(rng, 2 * m, k)
    singles = []
    try:
        for g in range(2):
            for i in range(8):
                ctx.set_strength(i, float(S[g, i]))
            ctx.reset_engagement()
            singles.append(_bits(ctx.linear(w, _to_dev(x[g * m:(g + 1) * m]))))
            launched = ctx.engagement()["kernels"]
        ctx.set_strengths_rows(S, np.array([0, m, 2 * m], dtype=np.int32))
        yb = ctx.linear(w, _to_dev(x))
        ctx.clear_strengths_rows()
        ctx.sync_check()
    finally:
        for i in range(8):
            ctx.set_strength(i, 1.0)
        w.free()
    # pre-GEMM (with or without its reduce), split projection and its reduce
    assert launched >= 3, f"{launched} kernels: the projection did not split K"
    yb_bits = _bits(yb)
    for g in range(2):
        assert np.array_equal(yb_bits[g * m:(g + 1) * m], singles[g]), \
            f"image {g} of the batch differs from its own call"
    rows = np.sort(rng.choice(m, size=48, replace=False))
    for g in range(2):
        slots = [(facs[i][0], facs[i][1], float(S[g, i])) for i in range(8)]
        xr = x[g * m + rows]
        ref = O.projection(xr, pw.data, pw.scales, pw.biases, n, k, bits, False, slots)
        err = O.rel_l2(P.bf16_bits_to_f32(singles[g][rows]).astype(np.float64), ref)
        assert err <= TOL, f"image {g}: rel-L2 {err:.3e}"
