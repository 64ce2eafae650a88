"""The FFN gate/up pair with its SwiGLU fused into the projection epilogue
(mp_linear_swiglu) against the fp64 oracle: h = bf16(silu(g) * u) with g and u
the bf16 outputs of the two projections, as the reference's gpu_ff computes
them (src/ming-dit.cc:2155-2157, swiglu at src/metal/ming_ops.metal:95-112),
with and without live adapters; and against this library's own separate w1 /
w3 launches followed by the same SwiGLU."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from mingproj import pack as P

pytestmark = pytest.mark.gpu

TOL = 5e-3


def _bf16(a: np.ndarray) -> np.ndarray:
    return O.bf16_to_f64(P.f32_to_bf16_bits(np.asarray(a, dtype=np.float32)))


def _swiglu_ref(g64: np.ndarray, u64: np.ndarray) -> np.ndarray:
    g = _bf16(g64)
    u = _bf16(u64)
    return _bf16(g / (1.0 + np.exp(-g)) * u)


def _weight(rng, n, k, bits):
    if bits == 0:
        return P.synthetic_dense(rng, n, k, std=0.05)
    return P.synthetic_affine(rng, n, k, bits)


@pytest.mark.parametrize("bits", [8, 4, 0])
@pytest.mark.parametrize("m,n,k,lora", [(300, 384, 256, False), (517, 640, 512, True),
                                         (4352, 10240, 256, True), (1100, 2730, 384, True)])
def test_swiglu_matches_oracle(ctx, bits, m, n, k, lora):
    rng = np.random.default_rng(m + n + k + bits)
    p1, p3 = _weight(rng, n, k, bits), _weight(rng, n, k, bits)
    w1 = ctx.upload(p1.n, p1.k, p1.bits, p1.data, p1.scales, p1.biases)
    w3 = ctx.upload(p3.n, p3.k, p3.bits, p3.data, p3.scales, p3.biases)
    s1, s3 = [], []
    if lora:
        # W1 in slots 0-2, W3 in slots 1-3 (ranks twice W1's): different stacks
        st = rng.uniform(-1.0, 1.5, size=4)
        for i, r in enumerate([8, 16, 32]):
            a1, b1 = P.synthetic_lora(rng, n, k, r, b_std=0.05)
            a3, b3 = P.synthetic_lora(rng, n, k, 2 * r, b_std=0.05)
            w1.bind(i, a1, b1)
            w3.bind(i + 1, a3, b3)
            s1.append((a1, b1, float(st[i])))
            s3.append((a3, b3, float(st[i + 1])))
        for i in range(4):
            ctx.set_strength(i, float(st[i]))
    x = P.f32_to_bf16_bits(rng.normal(size=(m, k)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    h = ctx.linear_swiglu(w1, w3, xd)
    sep1 = ctx.linear(w1, xd)
    sep3 = ctx.linear(w3, xd)
    ctx.sync_check()
    rows = np.unique(np.concatenate([np.arange(min(m, 40)), np.arange(max(0, m - 40), m),
                                     rng.choice(m, size=min(m, 40), replace=False)]))
    g = O.projection(x[rows], p1.data, p1.scales, p1.biases, n, k, bits, False, s1)
    u = O.projection(x[rows], p3.data, p3.scales, p3.biases, n, k, bits, False, s3)
    ref = _swiglu_ref(g, u)
    got = h.float().cpu().numpy().astype(np.float64)
    # the same SwiGLU over this library's separate gate and up outputs
    gs = sep1.float()
    us = sep3.float()
    via_sep = (gs / (1.0 + torch.exp(-gs)) * us).to(torch.bfloat16).float().cpu().numpy()
    for i in range(4):
        ctx.set_strength(i, 1.0)
    w1.free()
    w3.free()
    err = O.rel_l2(got[rows], ref)
    assert err <= TOL, f"rel-L2 {err:.3e} vs oracle (bits {bits}, m {m}, n {n}, lora {lora})"
    assert O.rel_l2(got, via_sep.astype(np.float64)) <= 2e-3
