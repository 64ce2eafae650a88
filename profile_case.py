"""One kernel of the path on synthetic inputs, for profiling and timing.

    python profile_case.py --m 16896 --n 10240 --k 3840 --bits 4 \
        --ranks 32,32,32,32,32,32,32,32 --reps 20
    python profile_case.py --op attention --m 4352 --heads 30 --reps 20
    python profile_case.py --op rms_residual --m 4352 --k 3840 --reps 20
    python profile_case.py --op modulation --m 1 --bits 8 --reps 20

Prints the CUDA-event time per call and the algorithmic rate: TFLOP/s for a
projection (mp_linear: rank-space pre-GEMM + fused projection; back to back,
or with --flush each call alone after a 256 MB read, the median) or the
attention (mp_attention over head-major q / k / v of m rows), GB/s for the
gated sandwich-norm residual step (mp_rms_residual over m rows of width k)
and for the batched modulation (mp_modulation_all over 32 blocks' adaLN
weights [4 * 3840, k] for m tokens; every call is preceded by a read of a
256 MB buffer, so the weights come from HBM, not L2, and no dirty line is
written back during the call). Holds only that call's
tensors on the device, so it is a small case for `ncu`.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent / "vpipe-ming-image_b200"))

from mingproj.dit import _device_affine, _device_dense  # noqa: E402
from mingproj.proj import Context  # noqa: E402


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


def _modulation(a, ctx, dev, gen) -> None:
    H, K, nb = 3840, a.k if a.k != 3840 or a.op_k_set else 256, 32
    ws, bias, an1, fn1 = [], [], [], []
    for _ in range(nb):
        if a.bits:
            ws.append(ctx.upload(4 * H, K, a.bits, *_device_affine(gen, 4 * H, K, a.bits, dev)))
        else:
            ws.append(ctx.upload(4 * H, K, 0, _device_dense(gen, 4 * H, K, dev)))
        bias.append((torch.randn(4 * H, device=dev, generator=gen) * 0.02).to(torch.bfloat16))
        an1.append(torch.ones(H, device=dev, dtype=torch.bfloat16))
        fn1.append(torch.ones(H, device=dev, dtype=torch.bfloat16))
    mset = ctx.modulation_set(ws, bias, an1, fn1)
    temb = torch.randn((a.m, K), device=dev, generator=gen).to(torch.bfloat16)
    flush = torch.ones(64 << 20, dtype=torch.int32, device=dev)  # 256 MB, read before each call
    for _ in range(a.warmup):
        ctx.modulation(mset, temb)
    ctx.sync_check()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(a.reps)]
    for e0, e1 in ev:
        # evicts the weights from L2 by reading, so no dirty line of the flush
        # is written back while the timed call runs
        flush.sum()
        e0.record()
        ctx.modulation(mset, temb)
        e1.record()
    torch.cuda.synchronize()
    ctx.sync_check()
    us = float(np.median([e0.elapsed_time(e1) * 1e3 for e0, e1 in ev]))
    wb = (K * a.bits / 8 + 4 * (K // 64)) if a.bits else 2 * K
    nbytes = nb * (4 * H * (wb + 2) + 2 * H * 2 * (1 + a.m) + 4 * H * 2 * a.m)
    print(json.dumps({"op": "modulation", "blocks": nb, "k": K, "bits": a.bits, "m": a.m,
                      "us_per_call": us, "bytes": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9}))
    mset.free()
    for w in ws:
        w.free()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["linear", "attention", "rms_residual", "modulation"],
                    default="linear")
    ap.add_argument("--heads", type=int, default=30)
    ap.add_argument("--m", type=int, default=4352)
    ap.add_argument("--n", type=int, default=10240)
    ap.add_argument("--k", type=int, default=3840)
    ap.add_argument("--bits", type=int, default=8)
    ap.add_argument("--ranks", type=str, default="4,8,8,16,16,32,32,64")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--flush", action="store_true",
                    help="projection: time each call alone after an L2-evicting read (median)")
    a = ap.parse_args()
    a.op_k_set = "--k" in sys.argv
    dev = torch.device("cuda", 0)
    ctx = Context(0)
    gen = torch.Generator(device=dev).manual_seed(0)
    if a.op != "linear":
        {"attention": _attention, "rms_residual": _rms_residual,
         "modulation": _modulation}[a.op](a, ctx, dev, gen)
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
    if a.flush:
        # each call timed alone after a read of a 256 MB buffer: the weights
        # and x come from HBM, as in a forward whose other layers evicted them
        flush = torch.ones(64 << 20, dtype=torch.int32, device=dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(a.reps)]
        for e0, e1 in ev:
            flush.sum()
            e0.record()
            ctx.linear(w, x, y)
            e1.record()
        torch.cuda.synchronize()
        ctx.sync_check()
        us = float(np.median([e0.elapsed_time(e1) * 1e3 for e0, e1 in ev]))
    else:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.reps):
            ctx.linear(w, x, y)
        e1.record()
        torch.cuda.synchronize()
        ctx.sync_check()
        us = e0.elapsed_time(e1) * 1e3 / a.reps
    flops = 2.0 * a.m * a.n * a.k + sum(2.0 * a.m * r * (a.k + a.n) for r in ranks)
    # algorithmic bytes: codes (or bf16 weights), the group scale/bias words,
    # x, y and the LoRA A / B stacks
    wbytes = a.n * a.k * a.bits / 8 + a.n * (a.k // 64) * 4 if a.bits else 2.0 * a.n * a.k
    nbytes = wbytes + 2.0 * a.m * (a.k + a.n) + sum(2.0 * r * (a.k + a.n) for r in ranks)
    print(json.dumps({"m": a.m, "n": a.n, "k": a.k, "bits": a.bits, "ranks": ranks,
                      "flush": a.flush, "us_per_call": us, "tflops": flops / (us * 1e-6) / 1e12,
                      "bytes": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9}))
    w.free()
    ctx.close()


if __name__ == "__main__":
    main()
