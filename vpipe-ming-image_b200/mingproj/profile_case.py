"""One kernel of the path on synthetic inputs, for profiling and timing.

    python -m mingproj.profile_case --m 4352 --n 10240 --k 3840 --bits 8 \
        --ranks 4,8,8,16,16,32,32,64 --reps 20
    python -m mingproj.profile_case --op attention --m 4352 --heads 30 --reps 20
    python -m mingproj.profile_case --op rms_residual --m 4352 --k 3840 --reps 20

Prints the CUDA-event time per call and the algorithmic rate: TFLOP/s for a
projection (mp_linear: rank-space pre-GEMM + fused projection) or the
attention (mp_attention over head-major q / k / v of m rows), GB/s for the
gated sandwich-norm residual step (mp_rms_residual over m rows of width k).
Holds only that call's tensors on the device, so it is a small case for
`ncu`.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .dit import _device_affine, _device_dense
from .proj import Context


def _timed(fn, reps: int, warmup: int, ctx) -> float:
    """Microseconds per call, CUDA events on the current stream."""
    for _ in range(warmup):
        fn()
    ctx.sync_check()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ctx.sync_check()
    return e0.elapsed_time(e1) * 1e3 / reps


def _attention(a, ctx, dev, gen) -> None:
    q, k, v = [torch.randn((a.heads, a.m, 128), device=dev, generator=gen).to(torch.bfloat16)
               for _ in range(3)]
    us = _timed(lambda: ctx.attention(q, k, v), a.reps, a.warmup, ctx)
    flops = 4.0 * a.m * a.m * 128 * a.heads
    print(json.dumps({"op": "attention", "s": a.m, "heads": a.heads, "us_per_call": us,
                      "tflops": flops / (us * 1e-6) / 1e12}))


def _rms_residual(a, ctx, dev, gen) -> None:
    mk = lambda *shape: torch.randn(shape, device=dev, generator=gen).to(torch.bfloat16)  # noqa: E731
    x, o, nrm = mk(a.m, a.k), mk(a.m, a.k), mk(a.m, a.k)
    o_gain, gate, nrm_gain = mk(a.k), mk(a.k), mk(a.k)
    us = _timed(lambda: ctx.rms_residual(x, o, o_gain, gate, nrm_gain, nrm=nrm), a.reps, a.warmup,
                ctx)
    nbytes = 4.0 * a.m * a.k * 2  # read o and x, write x and nrm
    print(json.dumps({"op": "rms_residual", "m": a.m, "h": a.k, "us_per_call": us,
                      "gbs": nbytes / (us * 1e-6) / 1e9}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["linear", "attention", "rms_residual"], default="linear")
    ap.add_argument("--heads", type=int, default=30)
    ap.add_argument("--m", type=int, default=4352)
    ap.add_argument("--n", type=int, default=10240)
    ap.add_argument("--k", type=int, default=3840)
    ap.add_argument("--bits", type=int, default=8)
    ap.add_argument("--ranks", type=str, default="4,8,8,16,16,32,32,64")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    ctx = Context(0)
    gen = torch.Generator(device=dev).manual_seed(0)
    if a.op != "linear":
        (_attention if a.op == "attention" else _rms_residual)(a, ctx, dev, gen)
        ctx.close()
        return
    if a.bits == 0:
        w = ctx.upload(a.n, a.k, 0, _device_dense(gen, a.n, a.k, dev))
    else:
        w = ctx.upload(a.n, a.k, a.bits, *_device_affine(gen, a.n, a.k, a.bits, dev))
    ranks = [int(r) for r in a.ranks.split(",") if r.strip()] if a.ranks else []
    for i, r in enumerate(ranks):
        A = (torch.randn((r, a.k), device=dev, generator=gen) / np.sqrt(r)).to(torch.bfloat16)
        B = (torch.randn((a.n, r), device=dev, generator=gen) * 0.01).to(torch.bfloat16)
        w.bind(i, A, B)
        ctx.set_strength(i, 0.5)
    x = torch.randn((a.m, a.k), device=dev, generator=gen).to(torch.bfloat16)
    y = torch.empty((a.m, a.n), device=dev, dtype=torch.bfloat16)
    for _ in range(a.warmup):
        ctx.linear(w, x, y)
    ctx.sync_check()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        ctx.linear(w, x, y)
    e1.record()
    torch.cuda.synchronize()
    ctx.sync_check()
    us = e0.elapsed_time(e1) * 1e3 / a.reps
    flops = 2.0 * a.m * a.n * a.k + sum(2.0 * a.m * r * (a.k + a.n) for r in ranks)
    print(json.dumps({"m": a.m, "n": a.n, "k": a.k, "bits": a.bits, "ranks": ranks,
                      "us_per_call": us, "tflops": flops / (us * 1e-6) / 1e12}))
    w.free()
    ctx.close()


if __name__ == "__main__":
    main()
