"""The sandwich-norm residual step (mp_rms_residual) against the oracle's
float32 restatement of the reference's rms -> gated residual -> rms chain
(src/ming-dit.cc:2096-2104, :2256-2261; src/metal/ming_ops.metal:55-93) and
against the unfused torch sequence the GPU DiT forward ran before: within a
bf16 rounding (sums of squares and tanh are evaluated in another order /
library), bit-identical between runs."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from mingproj import pack as P

pytestmark = pytest.mark.gpu

EPS = 1e-5


def _dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _close(got: np.ndarray, ref: np.ndarray, what: str):
    err = O.rel_l2(O.bf16_to_f64(got), O.bf16_to_f64(ref))
    diff = float(np.mean(got != ref))
    assert err <= 2e-3, f"{what}: rel-L2 {err:.2e}"
    assert diff <= 0.02, f"{what}: {diff:.3%} of the values differ"


def _torch_chain(x, o, og, gate, ng, eps):
    """The unfused torch sequence (fp32 math, bf16 between steps)."""
    def rms(v, w):
        vf = v.float()
        return (vf * torch.rsqrt(vf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(torch.bfloat16)
    x = x.clone()
    if o is not None:
        s = rms(o, og).float()
        if gate is not None:
            x = (x.float() + torch.tanh(gate.float()) * s).to(torch.bfloat16)
        else:
            x = (x.float() + s).to(torch.bfloat16)
    return x, (rms(x, ng) if ng is not None else None)


@pytest.mark.parametrize("m,h", [(4352, 3840), (301, 1024), (7, 512), (3, 8192)])
@pytest.mark.parametrize("mode", ["gated+nrm", "resid+nrm", "gated", "nrm-only"])
def test_rms_residual_matches_oracle_and_unfused(ctx, m, h, mode):
    rng = np.random.default_rng(m + h + len(mode))
    xb = P.f32_to_bf16_bits(rng.normal(size=(m, h)).astype(np.float32))
    ob = P.f32_to_bf16_bits((rng.normal(size=(m, h)) * 3.0).astype(np.float32))
    og = P.f32_to_bf16_bits(rng.uniform(0.5, 1.5, size=h).astype(np.float32))
    gate = P.f32_to_bf16_bits(rng.normal(size=h).astype(np.float32))
    ng = P.f32_to_bf16_bits(rng.uniform(0.5, 1.5, size=h).astype(np.float32))
    use_o = mode != "nrm-only"
    use_gate = mode.startswith("gated")
    use_n = mode.endswith("nrm") or mode == "nrm-only"
    x = _dev(xb)
    o, ogd, gd, ngd = _dev(ob), _dev(og), _dev(gate), _dev(ng)
    nrm = ctx.rms_residual(x, o if use_o else None, ogd if use_o else None,
                           gd if use_gate else None, ngd if use_n else None, eps=EPS)
    ctx.sync_check()
    xr, nr = O.rms_residual(xb, ob if use_o else None, og, gate if use_gate else None,
                            ng if use_n else None, EPS)
    _close(_bits(x), xr, "x vs oracle")
    tx, tn = _torch_chain(_dev(xb), o if use_o else None, ogd, gd if use_gate else None,
                          ngd if use_n else None, EPS)
    _close(_bits(x), _bits(tx), "x vs unfused")
    if use_n:
        _close(_bits(nrm), nr, "nrm vs oracle")
        _close(_bits(nrm), _bits(tn), "nrm vs unfused")
    else:
        assert nrm is None
    # the same inputs give the same bits
    x2 = _dev(xb)
    nrm2 = ctx.rms_residual(x2, o if use_o else None, ogd if use_o else None,
                            gd if use_gate else None, ngd if use_n else None, eps=EPS)
    ctx.sync_check()
    assert np.array_equal(_bits(x2), _bits(x))
    if use_n:
        assert np.array_equal(_bits(nrm2), _bits(nrm))


def test_rms_residual_strided_rows(ctx):
    """Row strides wider than h (views into wider buffers), in and out."""
    rng = np.random.default_rng(3)
    m, h, ld = 100, 768, 1024
    xb = P.f32_to_bf16_bits(rng.normal(size=(m, ld)).astype(np.float32))
    ob = P.f32_to_bf16_bits(rng.normal(size=(m, ld)).astype(np.float32))
    g = P.f32_to_bf16_bits(rng.uniform(0.5, 1.5, size=h).astype(np.float32))
    x = _dev(xb)
    nrm_buf = torch.zeros((m, ld), dtype=torch.bfloat16, device="cuda")
    ctx.rms_residual(x[:, :h], _dev(ob)[:, :h], _dev(g), None, _dev(g), eps=EPS,
                     nrm=nrm_buf[:, :h])
    ctx.sync_check()
    xr, nr = O.rms_residual(xb[:, :h], ob[:, :h], g, None, g, EPS)
    _close(_bits(x)[:, :h], xr, "x")
    _close(_bits(nrm_buf)[:, :h], nr, "nrm")
    assert np.array_equal(_bits(x)[:, h:], xb[:, h:]), "columns past h were touched"
    assert not _bits(nrm_buf)[:, h:].any(), "nrm columns past h were touched"


def test_rms_residual_argument_errors(ctx):
    from mingproj._lib import MPError, MP_EINVAL
    x = torch.zeros((4, 12), dtype=torch.bfloat16, device="cuda")  # h not a multiple of 8
    g = torch.ones(12, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(MPError) as e:
        ctx.rms_residual(x, None, None, None, g)
    assert e.value.status == MP_EINVAL
    x = torch.zeros((4, 8200), dtype=torch.bfloat16, device="cuda")  # past the row limit
    g = torch.ones(8200, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(MPError) as e:
        ctx.rms_residual(x, None, None, None, g)
    assert e.value.status == MP_EINVAL
