"""Non-causal attention over head-major q, k, v (mp_attention, the tcgen05
kernel) against the plain PyTorch fp32 reference of the same op, the
reference's run_attn (src/ming-dit.cc:1905-2039): softmax(scale q K^T) V per
head, written token-major. Covers sequence lengths around the 128-key tile
(1, 127, 128, 129, ragged), many heads at the DiT's joint length, peaked
logits and a key order whose running maximum rises tile after tile (the
online rescaling), and run-to-run bit identity. Bar: rel-L2 <= 5e-3 against
fp32 (P and the output are rounded to bf16)."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 5e-3


def _ref(q, k, v, scale):
    qf, kf, vf = q.float(), k.float(), v.float()
    att = torch.softmax((qf @ kf.transpose(1, 2)) * scale, dim=-1) @ vf  # [nh, s, 128]
    return att.transpose(0, 1).reshape(q.shape[1], -1)


def _inputs(nh, s, std, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda sd: (torch.randn((nh, s, 128), device="cuda", generator=g) * sd).to(torch.bfloat16)  # noqa: E731
    return mk(std), mk(std), mk(1.0)


@pytest.mark.parametrize("nh,s,std", [(1, 1, 1.0), (2, 127, 1.0), (1, 128, 1.0), (3, 129, 1.0),
                                      (2, 300, 1.0), (4, 1000, 2.0), (30, 4352, 1.0),
                                      (2, 517, 3.0)])
def test_attention_matches_fp32(ctx, nh, s, std):
    q, k, v = _inputs(nh, s, std, 10 * nh + s)
    scale = 1.0 / math.sqrt(128)
    o = ctx.attention(q, k, v)
    ctx.sync_check()
    ref = _ref(q, k, v, scale)
    err = O.rel_l2(o.float().cpu().numpy(), ref.cpu().numpy())
    assert err <= TOL, f"rel-L2 {err:.2e}"
    o2 = ctx.attention(q, k, v)
    ctx.sync_check()
    assert torch.equal(o.view(torch.int16), o2.view(torch.int16)), "not bit-identical run to run"


def _ref_rows(q, k, v, scale, rows):
    """fp32 reference for the query rows `rows` only (every key), head by head."""
    outs = []
    for h in range(q.shape[0]):
        lg = (q[h, rows].float() @ k[h].float().T) * scale
        outs.append(torch.softmax(lg, dim=-1) @ v[h].float())
    return torch.stack(outs, 0).transpose(0, 1).reshape(len(rows), -1)


@pytest.mark.parametrize("nh,s", [(30, 16896), (30, 8448), (8, 16384), (4, 357), (4, 390)])
def test_attention_long_and_caption_lengths(ctx, nh, s):
    """The config-3 joint length (16384 image + 512 caption rows), the
    noise-refiner length at 2048^2, half the joint length, and caption-like
    256 + N lengths whose last key tile is ragged; the fp32 reference is
    taken on a sample of query rows (first, last, the ragged tail and random
    rows) against all keys."""
    q, k, v = _inputs(nh, s, 1.0, 7 * nh + s)
    scale = 1.0 / math.sqrt(128)
    o = ctx.attention(q, k, v)
    ctx.sync_check()
    g = torch.Generator().manual_seed(s)
    rows = sorted(set([0, 1, s - 1] + list(range(max(0, s - 130), s, 7)) +
                      torch.randint(0, s, (min(s, 384),), generator=g).tolist()))
    ref = _ref_rows(q, k, v, scale, torch.tensor(rows, device="cuda"))
    err = O.rel_l2(o[rows].float().cpu().numpy(), ref.cpu().numpy())
    assert err <= TOL, f"rel-L2 {err:.2e}"


def test_attention_rising_maximum(ctx):
    """Keys ordered so each 128-key tile holds larger logits than the last:
    every tile raises the running maximum and rescales the partial output."""
    nh, s = 2, 1024
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.ones((nh, s, 128), device="cuda")
    ramp = torch.linspace(-4.0, 4.0, s, device="cuda")[None, :, None]
    k = (ramp * torch.ones((nh, s, 128), device="cuda")
         + 0.05 * torch.randn((nh, s, 128), device="cuda", generator=g))
    v = torch.randn((nh, s, 128), device="cuda", generator=g)
    q, k, v = q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)
    scale = 0.05
    o = ctx.attention(q, k, v, scale=scale)
    ctx.sync_check()
    err = O.rel_l2(o.float().cpu().numpy(), _ref(q, k, v, scale).cpu().numpy())
    assert err <= TOL, f"rel-L2 {err:.2e}"


def test_attention_fp64_pin_small():
    """The fp32 torch reference itself against an fp64 numpy restatement on a
    small case (CPU only: pins the reference the GPU cases use)."""
    rng = np.random.default_rng(0)
    nh, s = 2, 37
    q, k, v = (torch.from_numpy(rng.normal(size=(nh, s, 128)).astype(np.float32)) for _ in range(3))
    scale = 1.0 / math.sqrt(128)
    lg = np.einsum("hid,hjd->hij", q.double().numpy(), k.double().numpy()) * scale
    p = np.exp(lg - lg.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ref64 = np.einsum("hij,hjd->hid", p, v.double().numpy()).transpose(1, 0, 2).reshape(s, -1)
    assert O.rel_l2(_ref(q, k, v, scale).numpy(), ref64) < 1e-5


def test_attention_argument_errors(ctx):
    from mingproj._lib import MPError, MP_EINVAL
    q = torch.zeros((2, 64, 128), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((64, 200), dtype=torch.bfloat16, device="cuda")  # ldo < 128 * nh
    with pytest.raises(MPError) as e:
        ctx.attention(q, q, q, out=out)
    assert e.value.status == MP_EINVAL
    with pytest.raises(ValueError):
        ctx.attention(q[:, :, :64].contiguous(), q, q)
