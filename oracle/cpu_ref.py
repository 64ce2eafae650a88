"""TEST INFRASTRUCTURE / CPU BASELINE — a torch fp32 CPU restatement of the
projection path, the stand-in for the reference's golden path (its torch
fp32 CPU forward, driven by tools/dump_ming_golden.py, which is not in the
reference tree). Only bench.py's CPU-baseline leg and `--impl reference` use
it, to time the CPU on the same shapes; it is never the product path.

Arithmetic per projection (reference `lin`, src/ming-dit.cc:1763-1771, and
the dequant rule of oracle/mp_oracle.c):
    y = x W^T + sum_i s_i (x A_i^T) B_i^T,  W = scale * q + bias (fp32).
Weights are dequantized once, as a golden forward would hold them; the timed
part is the projections.
"""
from __future__ import annotations

import os
import time

import torch

PROJ = (("attention.to_q", "h", "h"), ("attention.to_k", "h", "h"), ("attention.to_v", "h", "h"),
        ("attention.to_out.0", "h", "h"), ("feed_forward.w1", "ff", "h"),
        ("feed_forward.w3", "ff", "h"), ("feed_forward.w2", "h", "ff"))


def dequant_affine_cpu(codes_u8: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                       bits: int) -> torch.Tensor:
    """codes bytes [n, k*bits/8] (uint8), scales/biases fp32 [n, k/64] -> fp32 [n, k]."""
    if bits == 8:
        q = codes_u8.to(torch.float32)
    else:
        lo = (codes_u8 & 0xF).to(torch.float32)
        hi = (codes_u8 >> 4).to(torch.float32)
        q = torch.stack([lo, hi], dim=-1).reshape(codes_u8.shape[0], -1)
    n, k = q.shape
    q = q.view(n, k // 64, 64)
    return (q * scales[:, :, None] + biases[:, :, None]).reshape(n, k)


class CpuBlock:
    """One block's seven projections in fp32 on the CPU, with LoRA slots."""

    def __init__(self, H: int, FF: int, bits: int, ranks, seed: int):
        g = torch.Generator().manual_seed(seed)
        dims = {"h": H, "ff": FF}
        self.w, self.loras = {}, {}
        for name, no, ki in PROJ:
            n, k = dims[no], dims[ki]
            if bits == 0:
                w = torch.randn((n, k), generator=g) * 0.02
            else:
                codes = torch.randint(0, 256, (n, k * bits // 8), dtype=torch.uint8, generator=g)
                sc = torch.rand((n, k // 64), generator=g) * 0.018 + 0.002
                bi = -128.0 * sc if bits == 8 else -8.0 * sc
                w = dequant_affine_cpu(codes, sc, bi, bits)
            self.w[name] = w.contiguous()
            self.loras[name] = [((torch.randn((r, k), generator=g) / r ** 0.5).contiguous(),
                                 (torch.randn((n, r), generator=g) * 0.01).contiguous())
                                for r in ranks]

    def run(self, x_h: torch.Tensor, x_ff: torch.Tensor, strengths) -> dict:
        out = {}
        for name, no, ki in PROJ:
            x = x_ff if ki == "ff" else x_h
            y = x @ self.w[name].T
            for (a, b), s in zip(self.loras[name], strengths):
                if s != 0.0:
                    y += ((x @ a.T) * s) @ b.T
            out[name] = y
        return out


def block_flops(m: int, H: int, FF: int, ranks) -> float:
    r = float(sum(ranks))
    return 2.0 * m * (4 * H * H + 3 * FF * H) + 2.0 * m * r * (4 * 2 * H + 3 * (H + FF))


def time_block(rows: int, H: int = 3840, FF: int = 10240, bits: int = 8,
               ranks=(4, 8, 8, 16, 16, 32, 32, 64), reps: int = 1, seed: int = 0,
               threads: int | None = None, block: CpuBlock | None = None) -> dict:
    """Times `reps` runs of one block's projections at `rows` rows on all host
    threads (weights made once per call unless `block` is given); returns
    TFLOP/s and what the sample was."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    blk = block if block is not None else CpuBlock(H, FF, bits, ranks, seed)
    g = torch.Generator().manual_seed(seed + 1)
    x_h = torch.randn((rows, H), generator=g)
    x_ff = torch.randn((rows, FF), generator=g)
    strengths = [0.5] * len(ranks)
    blk.run(x_h[: min(rows, 64)], x_ff[: min(rows, 64)], strengths)  # warm-up
    t0 = time.perf_counter()
    for _ in range(reps):
        blk.run(x_h, x_ff, strengths)
    dt = time.perf_counter() - t0
    flops = block_flops(rows, H, FF, ranks) * reps
    return {"tflops": flops / dt / 1e12, "seconds": dt, "flops": flops, "threads": threads,
            "rows": rows, "reps": reps}
