"""q/k/v with the attention-head epilogue (mp_linear_heads): one launch writes
the three projections head-major [heads][m][128], q and k after the per-head
RMSNorm and the interleaved-pair rotary embedding, as the reference's block
runs them (src/ming-dit.cc:2078-2088: lin q/k/v, rms over each 128-wide head
row, tr_rope, v transposed). Checked against
  * the fp64 oracle projection followed by the same chain with the bf16
    roundings of the unfused sequence (rel-L2 <= 5e-3, the per-projection bar);
  * this library's own unfused sequence (linear_shared, then the head norm and
    rotary embedding in torch fp32, then the transpose): v bit-identical,
    q/k within a bf16 rounding (the sum of squares is added in another order).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from mingproj import pack as P

pytestmark = pytest.mark.gpu

TOL = 5e-3
EPS = 1e-5
HD = 128


def _bf16(a) -> np.ndarray:
    return O.bf16_to_f64(P.f32_to_bf16_bits(np.asarray(a, dtype=np.float32)))


def _head_chain_ref(y64: np.ndarray, gain: np.ndarray, cos: np.ndarray, sin: np.ndarray):
    """[rows, n] fp64 projection -> [heads, rows, 128]: bf16 output, per-head
    RMSNorm (rounded), rotary pairs (rounded)."""
    rows, n = y64.shape
    y = _bf16(y64).reshape(rows, n // HD, HD)
    r = 1.0 / np.sqrt((y * y).mean(-1, keepdims=True) + EPS)
    z = _bf16(y * r * gain[None, None, :])
    z0, z1 = z[..., 0::2], z[..., 1::2]
    c, s = cos[:, None, :], sin[:, None, :]
    out = np.empty_like(z)
    out[..., 0::2] = z0 * c - z1 * s
    out[..., 1::2] = z0 * s + z1 * c
    return _bf16(out).transpose(1, 0, 2)


def _torch_chain(y: torch.Tensor, gain: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """The unfused sequence in torch (fp32 math, bf16 between the steps)."""
    m, n = y.shape
    xf = y.reshape(m, n // HD, HD).float()
    z = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS) * gain.float()).to(torch.bfloat16)
    zf = z.float()
    x0, x1 = zf[..., 0::2], zf[..., 1::2]
    c, s = cos[:, None, :], sin[:, None, :]
    out = torch.empty_like(zf)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out.to(torch.bfloat16).transpose(0, 1).contiguous()


def _weight(rng, n, k, bits):
    if bits == 0:
        return P.synthetic_dense(rng, n, k, std=0.05)
    return P.synthetic_affine(rng, n, k, bits)


def _tables(rng, m):
    ang = rng.uniform(-60.0, 60.0, size=(m, HD // 2))
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def _sample(rng, m, n_inner=40):
    if m <= 600:
        return np.arange(m)
    return np.unique(np.concatenate([np.arange(8), rng.choice(m, n_inner, replace=False),
                                     np.arange(m - 24, m)]))


@pytest.mark.parametrize("bits", [8, 4, 0])
@pytest.mark.parametrize("m,n,k,lora", [(300, 384, 256, False), (1100, 640, 384, True),
                                         (4352, 3840, 3840, True), (517, 256, 512, False)])
def test_heads_match_oracle_and_unfused(ctx, bits, m, n, k, lora):
    rng = np.random.default_rng(10 * m + n + k + bits)
    pws = [_weight(rng, n, k, bits) for _ in range(3)]
    ws = [ctx.upload(p.n, p.k, p.bits, p.data, p.scales, p.biases) for p in pws]
    slots = [[], [], []]
    if lora:
        st = rng.uniform(-1.0, 1.5, size=4)
        for i, w in enumerate(ws):
            for j, r in enumerate([8, 16, 32][: 3 - i]):
                a, b = P.synthetic_lora(rng, n, k, r, b_std=0.05)
                w.bind(i + j, a, b)
                slots[i].append((a, b, float(st[i + j])))
        for i in range(4):
            ctx.set_strength(i, float(st[i]))
    gains = [rng.uniform(0.5, 1.5, size=HD).astype(np.float32) for _ in range(2)]
    gbits = [P.f32_to_bf16_bits(g) for g in gains]
    gdev = [torch.from_numpy(g.view(np.int16).copy()).view(torch.bfloat16).cuda() for g in gbits]
    cos, sin = _tables(rng, m)
    cd, sd = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    x = P.f32_to_bf16_bits(rng.normal(size=(m, k)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    try:
        q, kk, v = ctx.linear_heads(ws, xd, norm_w=[gdev[0], gdev[1], None], eps=EPS,
                                    rope_cos=cd, rope_sin=sd)
        ys = ctx.linear_shared(ws, xd)
        ctx.sync_check()
        assert q.shape == (n // HD, m, HD) and v.shape == (n // HD, m, HD)
        # v: the projection, transposed, bit for bit (no adapters: same K order)
        v_ref = ys[2].reshape(m, n // HD, HD).transpose(0, 1).contiguous()
        if not lora:
            assert torch.equal(v.view(torch.int16), v_ref.view(torch.int16)), "v differs"
        else:
            assert O.rel_l2(v.float().cpu().numpy(), v_ref.float().cpu().numpy()) <= 1e-3
        # q, k: against the unfused torch sequence on the same projections
        for got, y, g in ((q, ys[0], gdev[0]), (kk, ys[1], gdev[1])):
            ref = _torch_chain(y, g, cd, sd)
            err = O.rel_l2(got.float().cpu().numpy().astype(np.float64),
                           ref.float().cpu().numpy().astype(np.float64))
            diff = (got.view(torch.int16) != ref.view(torch.int16)).float().mean().item()
            assert err <= 2e-3, f"vs unfused: rel-L2 {err:.2e}"
            assert diff <= 0.02, f"vs unfused: {diff:.3%} of the values differ"
        # all three against the fp64 oracle chain on sampled rows
        rows = _sample(rng, m)
        for i, got in enumerate((q, kk, v)):
            y64 = O.projection(x[rows], pws[i].data, pws[i].scales, pws[i].biases, n, k,
                               pws[i].bits, False, slots[i])
            if i < 2:
                ref = _head_chain_ref(y64, O.bf16_to_f64(gbits[i]), cos[rows].astype(np.float64),
                                      sin[rows].astype(np.float64))
            else:
                ref = _bf16(y64).reshape(len(rows), n // HD, HD).transpose(1, 0, 2)
            g = got[:, torch.from_numpy(rows).cuda(), :].float().cpu().numpy().astype(np.float64)
            err = O.rel_l2(g, ref)
            assert err <= TOL, f"member {i}: rel-L2 {err:.3e} vs the oracle"
    finally:
        for i in range(8):
            ctx.set_strength(i, 1.0)
        for w in ws:
            w.free()


def test_heads_two_members_no_norm(ctx):
    """q and k alone, neither normed (norm_w None): plain head-major stores."""
    rng = np.random.default_rng(91)
    m, n, k = 700, 512, 256
    pws = [_weight(rng, n, k, 8) for _ in range(2)]
    ws = [ctx.upload(p.n, p.k, p.bits, p.data, p.scales, p.biases) for p in pws]
    x = P.f32_to_bf16_bits(rng.normal(size=(m, k)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    try:
        outs = ctx.linear_heads(ws, xd)
        ys = ctx.linear_shared(ws, xd)
        ctx.sync_check()
        for o, y in zip(outs, ys):
            ref = y.reshape(m, n // HD, HD).transpose(0, 1).contiguous()
            assert torch.equal(o.view(torch.int16), ref.view(torch.int16))
    finally:
        for w in ws:
            w.free()


def test_heads_argument_errors(ctx):
    from mingproj._lib import MPError, MP_EINVAL
    rng = np.random.default_rng(5)
    p = _weight(rng, 200, 256, 8)  # 200 is not a whole number of heads
    w = ctx.upload(p.n, p.k, p.bits, p.data, p.scales, p.biases)
    xd = torch.zeros((64, 256), dtype=torch.bfloat16, device="cuda")
    try:
        with pytest.raises(MPError) as e:
            ctx.linear_heads([w], xd, outs=[torch.empty((2, 64, 128), dtype=torch.bfloat16,
                                                        device="cuda")])
        assert e.value.status == MP_EINVAL
    finally:
        w.free()
    p = _weight(rng, 256, 256, 8)
    w = ctx.upload(p.n, p.k, p.bits, p.data, p.scales, p.biases)
    g = torch.ones(128, dtype=torch.bfloat16, device="cuda")
    try:
        with pytest.raises(MPError) as e:  # a normed member without rotary tables
            ctx.linear_heads([w], xd, norm_w=[g])
        assert e.value.status == MP_EINVAL
    finally:
        w.free()
