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


def test_static_scratch_allocates_nothing_and_ignores_bound_slots():
    """Device memory is unchanged across static calls (after a first call
    that loads the kernels), strength 0 gives the bits of the plain base
    projection, and a slot bound to the weight with mp_lora_bind is not
    applied: the result still matches the single-adapter oracle."""
    ctx = Context(0)
    rng = np.random.default_rng(99)
    m, n, k, rank = 260, 256, 384, 24
    pw = P.synthetic_affine(rng, n, k, 4)
    w = ctx.upload(n, k, 4, pw.data, pw.scales, pw.biases)
    x = P.f32_to_bf16_bits(rng.normal(size=(m, k)).astype(np.float32))
    a, b = P.synthetic_lora(rng, n, k, rank, b_std=0.05)
    xd, ad, bd = _dev(x), _dev(a), _dev(b)
    outs = [torch.empty((m, n), dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    base = ctx.linear(w, xd)  # no slot bound: the plain base projection
    ctx.linear_lora_static(w, xd, ad, bd, 0.5, out=outs[0])  # loads the kernels
    other_a, other_b = P.synthetic_lora(rng, n, k, 16, b_std=0.5)
    w.bind(0, other_a, other_b)  # bound and live, but not this entry point's business
    ctx.set_strength(0, 1.0)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    ctx.linear_lora_static(w, xd, ad, bd, 0.0, out=outs[1])
    ctx.linear_lora_static(w, xd, ad, bd, 0.5, out=outs[2])
    ctx.sync_check()
    free1 = torch.cuda.mem_get_info()[0]
    ref = O.projection(x, pw.data, pw.scales, pw.biases, n, k, 4, False, [(a, b, 0.5)])
    try:
        assert free1 == free0, f"device memory moved by {free0 - free1} bytes"
        assert torch.equal(outs[1].view(torch.int16), base.view(torch.int16)), \
            "strength 0 != the base projection"
        assert torch.equal(outs[2].view(torch.int16), outs[0].view(torch.int16)), \
            "a bound slot changed the static result"
        assert O.rel_l2(outs[2].float().cpu().numpy(), ref) <= TOL
    finally:
        w.unbind(0)
        w.free()
        ctx.close()
