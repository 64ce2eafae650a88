"""Batched adaLN modulation (mp_modulation_all) against the fp64 oracle: the
reference's fill_mod (src/ming-dit.cc:2266-2273) for several blocks at once,
mods = W temb + b, nw1 = an1 (1 + mods[0:H]), nw3 = fn1 (1 + mods[2H:3H])."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from mingproj import pack as P

pytestmark = pytest.mark.gpu

TOL = 5e-3


def _dev(bits):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("bits", [8, 4, 0])
@pytest.mark.parametrize("m", [1, 2, 4, 8])
@pytest.mark.parametrize("H,K", [(256, 256), (384, 3840), (256, 192)])
def test_modulation_matches_oracle(ctx, bits, m, H, K):
    """K 256 and 3840 take the lane-per-row path (up to 8 tokens per launch,
    4 at K 3840), K 192 the generic one (4 tokens per launch: 8 tokens are two
    launches)."""
    rng = np.random.default_rng(bits * 100 + m * 10 + H)
    nb = 3
    ws, pws, biases, an1, fn1 = [], [], [], [], []
    for _ in range(nb):
        pw = (P.synthetic_affine(rng, 4 * H, K, bits) if bits else
              P.synthetic_dense(rng, 4 * H, K, std=0.05))
        pws.append(pw)
        ws.append(ctx.upload(pw.n, pw.k, pw.bits, pw.data, pw.scales, pw.biases))
        biases.append(P.f32_to_bf16_bits(rng.normal(0, 0.02, 4 * H).astype(np.float32)))
        an1.append(P.f32_to_bf16_bits((1 + 0.1 * rng.normal(size=H)).astype(np.float32)))
        fn1.append(P.f32_to_bf16_bits((1 + 0.1 * rng.normal(size=H)).astype(np.float32)))
    mset = ctx.modulation_set(ws, biases, an1, fn1)
    temb = P.f32_to_bf16_bits(rng.normal(size=(m, K)).astype(np.float32))
    mods, nw1, nw3 = ctx.modulation(mset, _dev(temb))
    ctx.sync_check()
    mods = mods.float().cpu().numpy()
    nw1 = nw1.float().cpu().numpy()
    nw3 = nw3.float().cpu().numpy()
    mset.free()
    for w in ws:
        w.free()
    for b in range(nb):
        ref = O.modulation(temb, pws[b].data, pws[b].scales, pws[b].biases, biases[b], 4 * H, K,
                           bits)
        assert O.rel_l2(mods[b], ref) <= TOL
        # the fold reads the bf16-rounded mods, as the reference's modulate does
        mb = O.bf16_to_f64(P.f32_to_bf16_bits(mods[b].astype(np.float32)))
        want1 = O.bf16_to_f64(an1[b])[None, :] * (1.0 + mb[:, :H])
        want3 = O.bf16_to_f64(fn1[b])[None, :] * (1.0 + mb[:, 2 * H:3 * H])
        assert O.rel_l2(nw1[b], want1) <= 4e-3 and O.rel_l2(nw3[b], want3) <= 4e-3


@pytest.mark.parametrize("bits", [8, 4, 0])
@pytest.mark.parametrize("H,K", [(256, 256), (256, 3840), (256, 192)])
def test_modulation_rows_independent_of_batch(ctx, bits, H, K):
    """A token's modulation row has the same bits whether it is computed alone
    (M = 1, one image) or inside a batch (M = 2, 4 or 8: one launch on the
    lane-per-row path, where each token runs its own FMA chains; two launches
    of 4 on the generic path): the batched DiT forward relies on it for image
    i to equal its own forward."""
    rng = np.random.default_rng(7 + bits + K)
    nb = 2
    ws, biases, an1, fn1 = [], [], [], []
    for _ in range(nb):
        pw = (P.synthetic_affine(rng, 4 * H, K, bits) if bits else
              P.synthetic_dense(rng, 4 * H, K, std=0.05))
        ws.append(ctx.upload(pw.n, pw.k, pw.bits, pw.data, pw.scales, pw.biases))
        biases.append(P.f32_to_bf16_bits(rng.normal(0, 0.02, 4 * H).astype(np.float32)))
        an1.append(P.f32_to_bf16_bits((1 + 0.1 * rng.normal(size=H)).astype(np.float32)))
        fn1.append(P.f32_to_bf16_bits((1 + 0.1 * rng.normal(size=H)).astype(np.float32)))
    mset = ctx.modulation_set(ws, biases, an1, fn1)
    temb = _dev(P.f32_to_bf16_bits(rng.normal(size=(8, K)).astype(np.float32)))
    try:
        batched = {mm: ctx.modulation(mset, temb[:mm]) for mm in (2, 4, 8)}
        single = [ctx.modulation(mset, temb[i:i + 1]) for i in range(8)]
        ctx.sync_check()
        for mm, outs in batched.items():
            for i in range(mm):
                for got, want in zip(outs, single[i]):
                    assert torch.equal(got[:, i].view(torch.int16), want[:, 0].view(torch.int16)), \
                        f"M={mm} row {i} differs from its M=1 launch"
    finally:
        mset.free()
        for w in ws:
            w.free()
