"""One fused projection launch on synthetic inputs, for profiling and timing.

    python -m mingproj.profile_case --m 4352 --n 10240 --k 3840 --bits 8 \
        --ranks 4,8,8,16,16,32,32,64 --reps 20

Prints the CUDA-event time per mp_linear call (rank-space pre-GEMM + fused
projection) and the algorithmic TFLOP/s. Holds only this one projection's
tensors on the device, so it is a small case for `ncu`.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .dit import _device_affine, _device_dense
from .proj import Context


def main() -> None:
    ap = argparse.ArgumentParser()
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
