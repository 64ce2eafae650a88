"""The allocation-free projection entry point (mp_linear_lora_static), for
callers that cannot call cudaMalloc (a host memory planner that owns every
device allocation, or a serving loop where allocating could synchronize the
device). It must give the same result as the allocating entry point with the
same adapter bound in a slot, on two calls in a row that reuse the library's
fixed rank-space array. This file is collected last on purpose."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from mingproj import pack as P
from mingproj.proj import Context

pytestmark = pytest.mark.gpu

TOL = 5e-3  # the per-projection rel-L2 bar every projection test uses


def _dev(bits16):
    return torch.from_numpy(bits16.view(np.int16)).view(torch.bfloat16).cuda()


def test_static_scratch_matches_allocating_entry_point():
    ctx = Context(0)
    rng = np.random.default_rng(2024)
    n, k = 384, 512
    pw = P.synthetic_affine(rng, n, k, 8)
    cases = [(520, 16, 0.7), (300, 40, -1.2)]  # (m, rank, strength) of two calls in a row
    ref_w = ctx.upload(n, k, 8, pw.data, pw.scales, pw.biases)
    static_w = ctx.upload(n, k, 8, pw.data, pw.scales, pw.biases)
    prepared = []
    for m, rank, s in cases:
        x = P.f32_to_bf16_bits(rng.normal(size=(m, k)).astype(np.float32))
        a, b = P.synthetic_lora(rng, n, k, rank, b_std=0.05)
        ref_w.bind(0, a, b)
        ctx.set_strength(0, s)
        want = ctx.linear(ref_w, _dev(x)).float().cpu().numpy()
        ref_w.unbind(0)
        prepared.append((x, a, b, s, want))
    ctx.set_strength(0, 1.0)
    got = []
    for x, a, b, s, _ in prepared:
        y = ctx.linear_lora_static(static_w, _dev(x), _dev(a), _dev(b), s)
        got.append(y.float().cpu().numpy())
    ctx.sync_check()
    for (x, a, b, s, want), g in zip(prepared, got):
        assert O.rel_l2(g, want) <= TOL
        ref = O.projection(x, pw.data, pw.scales, pw.biases, n, k, 8, False, [(a, b, s)])
        assert O.rel_l2(g, ref) <= TOL
    ref_w.free()
    static_w.free()
    ctx.close()


def test_static_scratch_rejects_oversize():
    ctx = Context(0)
    rng = np.random.default_rng(7)
    n, k = 128, 64
    pw = P.synthetic_affine(rng, n, k, 8)
    w = ctx.upload(n, k, 8, pw.data, pw.scales, pw.biases)
    a = torch.zeros((64, k), dtype=torch.bfloat16, device="cuda")
    b = torch.zeros((n, 64), dtype=torch.bfloat16, device="cuda")
    x = torch.zeros((40000, k), dtype=torch.bfloat16, device="cuda")  # 40000 * 64 > 2 Mi
    with pytest.raises(Exception, match="exceeds the static scratch"):
        ctx.linear_lora_static(w, x, a, b, 1.0)
    w.free()
    ctx.close()
