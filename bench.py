"""Benchmark of the fused quant + 8-slot-LoRA DiT projection path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 3|2|5]

One STEP is one forward's worth of the hot path: the full 34-block projection
set of a Ming-Image DiT forward plus the batched adaLN modulation of the 32
modulated blocks. The headline (default) workload is BASELINE config 3, the
north-star target: a 2048x2048 image (16384 image rows + 512 caption rows,
joint 16896), w4 affine group-64 packs, eight LoRA slots all of rank 32, the
strengths re-drawn before every forward as the denoise schedule re-sets them
(11 steps = one 11-forward generation). Inputs are seeded synthetic tensors
of the stated shapes (the reference's checkpoint and prompts are not
available); every forward streams every block's packed weights (3.4 GB at w4),
far more than L2, so no flush is needed between steps.

Under torchrun (N > 1) every rank runs a config-3 forward of its own image
(image sharding, no collective on the data path: weak scaling); the JSON line
reports the whole-job TFLOP/s over the max-over-ranks device time. The same
run also measures BASELINE config 5 (`config5_batch`): a batch of 8 images,
split by image over the N ranks (8 / N per rank, all in one launch per
projection, per-image strength vectors), its device time per step as the max
over ranks (strong scaling; --no-config5 skips it).

`--shard rows` instead splits ONE image's token rows across the N ranks
(equal 32-row-aligned slices, configs 2-4): every rank projects its slice of
every block, and each block's K and V are all-gathered over NCCL on a side
stream while the block's remaining projections run (strong scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "vpipe-ming-image_b200"))

METRIC = "fused quant+8-LoRA DiT-projection TFLOP/s & % TC peak at 1/2/4/8 B200"
RANKS = (4, 8, 8, 16, 16, 32, 32, 64)  # --forward and --shard rows: config 2's slots


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="mp_clocks_", suffix=".csv")[1])

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in self.path.read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 7:
                    rows.append(parts)
        except OSError:
            pass
        finally:
            try:
                self.path.unlink()
            except OSError:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(r[0]) for r in rows if r[0].replace(".", "").isdigit())
        smax = max(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i] == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": smax,
                "reasons": reasons, "samples": len(rows)}


# The benchmark workloads (seeded synthetic tensors of the
# stated shapes and distributions: the reference's checkpoint is not here).
CONFIGS = {
    3: {"img": 16384, "cap": 512, "bits": 4, "ranks": (32,) * 8, "images": 1,
        "workload": ("config3: full 34-block projection set of one 2048x2048 DiT forward "
                     "(IMG 16384 + CAP 512 rows, joint 16896; H 3840, FFN 10240; w4 affine g64; "
                     "8 LoRA slots all r=32; strengths re-drawn ~U(-1,1.5) before every forward "
                     "of the 11-forward denoise schedule) + batched adaLN modulation of 32 "
                     "blocks; one step = one forward")},
    2: {"img": 4096, "cap": 256, "bits": 8, "ranks": (4, 8, 8, 16, 16, 32, 32, 64), "images": 1,
        "workload": ("config2: full 34-block projection set of one 1024x1024 DiT forward "
                     "(IMG 4096 + CAP 256 rows, joint 4352; w8 affine g64; 8 LoRA slots "
                     "r={4,8,8,16,16,32,32,64}, s~U(-1,1.5)) + batched adaLN modulation of 32 "
                     "blocks; one step = one forward")},
    5: {"img": 4096, "cap": 256, "bits": 8, "ranks": (8, 8, 16, 16, 32, 32, 64, 64), "images": 8,
        "workload": ("config5: 34-block projection set of a batch of 8 independent 1024x1024 "
                     "images (each 4096 + 256 rows; w8 affine g64; shared slots "
                     "r={8,8,16,16,32,32,64,64}; per-image strength vectors ~U(-1,1.5) re-drawn "
                     "every step) + batched modulation (one temb row per image); the 8 images "
                     "are split by image over the ranks (8/N each, all of a rank's images in "
                     "one launch per projection); one step = one forward of the whole batch")},
}


def cpu_sample_rows(cfg: dict) -> int:
    """Rows of the bounded CPU sample: one main-layer block at the joint row
    count of one image (the block kind 30 of the 34 blocks run)."""
    return cfg["img"] + cfg["cap"]


def cpu_baseline(cfg: dict) -> dict:
    from oracle import cpu_ref
    rows = cpu_sample_rows(cfg)
    r = cpu_ref.time_block(rows, bits=cfg["bits"], ranks=cfg["ranks"], reps=1)
    return {"value": r["tflops"], "unit": "TFLOP/s", "cores": r["threads"], "kind": "port",
            "sample": (f"one main-layer block's 7 projections (w{cfg['bits']} dequantized once, "
                       f"{len(cfg['ranks'])} LoRA slots) at {r['rows']} rows, torch fp32 CPU "
                       f"restatement, {r['seconds']:.1f} s; TFLOP/s of that sample (a forward "
                       "extrapolates by FLOPs: every block runs the same arithmetic per row)")}


def run_reference(args) -> None:
    """The reference arm: the CPU port of the path (the reference itself is
    Metal-only), one bounded sample per step (the same sample as the main
    arm's cpu_baseline), all host threads, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import cpu_ref
    cfg = CONFIGS[args.config]
    rows = cpu_sample_rows(cfg)
    blk = cpu_ref.CpuBlock(3840, 10240, cfg["bits"], cfg["ranks"], seed=0)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_ref.time_block(rows, bits=cfg["bits"], ranks=cfg["ranks"], reps=1, seed=i,
                               block=blk)
        if i >= args.warmup:
            vals.append(r)
    flops = sum(v["flops"] for v in vals)
    secs = sum(v["seconds"] for v in vals)
    value = flops / secs / 1e12
    sample = (f"one main-layer block's 7 projections at {rows} rows per step (torch fp32 CPU "
              "restatement with the path's dequant and LoRA rule; the reference is Metal-only)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": secs / len(vals) * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg["workload"], "sample": sample},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": vals[0]["threads"],
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_rows(args) -> None:
    """One image's rows sharded over the ranks (strong scaling; configs 2 and
    3): every rank projects its equal, 32-row-aligned slice of every block,
    and each block's K and V are all-gathered over NCCL on side streams that
    overlap the block's to_out, w1/w3 and w2; the timed region ends when every
    gather has landed. Reports the gathers' own device time per block."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from mingproj.dit import (DitDims, DitProjectionSet, Layout, alloc_outputs,
                              modulation_flops, projection_flops)
    from mingproj.parallel import RowGather, row_shards
    from mingproj.proj import Context

    if args.config == 5:
        raise SystemExit("--shard rows splits one image's rows: use --config 2 or 3")
    cfg = CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    peaks = load_peaks()
    dims = DitDims()
    layout = Layout(img=cfg["img"], cap=cfg["cap"])
    ctx = Context(local)
    # one model and one image shared by all ranks: same seeds everywhere
    pset = DitProjectionSet.synthetic(ctx, dims, bits=cfg["bits"], seed=1, device=dev)
    for i, r in enumerate(cfg["ranks"]):
        pset.bind_synthetic(i, r, seed=100 + i, device=dev)
    rng = np.random.default_rng(2)
    gen = torch.Generator(device=dev).manual_seed(3)
    JT = layout.joint
    nrm = torch.randn((JT, dims.dim), device=dev, generator=gen).to(torch.bfloat16)
    ao = torch.randn((JT, dims.dim), device=dev, generator=gen).to(torch.bfloat16)
    ffi = torch.randn((JT, dims.ffn), device=dev, generator=gen).to(torch.bfloat16)
    temb = torch.randn((1, dims.adaln), device=dev, generator=gen).to(torch.bfloat16)
    outs = alloc_outputs(dims, JT, dev)
    stream = torch.cuda.current_stream(dev)
    base_f, lora_f = projection_flops(dims, layout, cfg["ranks"])
    step_flops = base_f + lora_f + modulation_flops(dims, 1)
    # a K and a V gather per block, so every block's collective time is kept
    gathers = ([(RowGather(layout.rows(dims.block_kind(b)), dims.dim, world, rank, dev),
                 RowGather(layout.rows(dims.block_kind(b)), dims.dim, world, rank, dev))
                for b in range(dims.n_blocks)] if world > 1 else None)

    def step():
        for i, s_ in enumerate(rng.uniform(-1.0, 1.5, size=8)):  # re-set every forward
            ctx.set_strength(i, float(s_))
        ctx.modulation(pset.modset, temb)
        for b in range(dims.n_blocks):
            m = layout.rows(dims.block_kind(b))
            sh = row_shards(m, world)[rank]
            gk, gv = gathers[b] if gathers is not None else (None, None)
            if gk is not None and b > 0:
                # the previous block's gathers send its K and V rows as they
                # lie: joined before this block's q/k/v overwrite them (they
                # overlapped the previous block's to_out, w1/w3 and w2)
                for g in gathers[b - 1]:
                    g.wait()

            def around(i, call, rows=sh.rows, gk=gk, gv=gv):
                if rows > 0:
                    call()
                if i == 0 and gk is not None:  # K and V of the block: gather now
                    gk.start(outs["attention.to_k"][:rows])
                    gv.start(outs["attention.to_v"][:rows])
            pset.block_projections(b, nrm[sh.start:sh.stop], ao[sh.start:sh.stop],
                                   ffi[sh.start:sh.stop], outs, around=around)
        if gathers is not None:
            for g in gathers[-1]:
                g.wait()

    for _ in range(args.warmup):
        step()
    ctx.sync_check()
    torch.cuda.synchronize(dev)
    ctx.reset_engagement()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev[0].record(stream)
        for _ in range(args.steps):
            step()
        ev[1].record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
    ctx.sync_check()
    t = torch.tensor([ev[0].elapsed_time(ev[1])], device=dev, dtype=torch.float64)
    nccl = None
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        per_block = [sum(g.last_ms() or 0.0 for g in pair) for pair in gathers]
        nt = torch.tensor([sum(per_block)], device=dev, dtype=torch.float64)
        dist.all_reduce(nt, op=dist.ReduceOp.MAX)
        nccl = {"ms_per_step": float(nt.item()), "ms_per_block_avg": float(nt.item()) / len(per_block),
                "what": "device time of each block's K and V all-gathers on their own streams "
                        "(last step, max over ranks); they overlap the block's remaining "
                        "projections",
                "bytes_received_per_block": 2 * layout.joint * dims.dim * 2 * (world - 1) / world}
    max_ms = float(t.item())
    value = step_flops * args.steps / (max_ms / 1e3) / 1e12
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": cfg["workload"], "l2": "inputs larger than L2",
                       "flops_per_step": step_flops,
                       "parallelism": f"token-rows x{world} (equal 32-row-aligned slices), NCCL "
                                      "all-gather of each block's K and V overlapping the "
                                      "block's remaining projections"},
            "nccl_gather": nccl,
            "roofline": None, "cpu_baseline": None, "e2e": None,
            "gpu_launches": ctx.engagement()["kernels"], "clocks": clk.summary(),
            "peaks": peaks.get("source"),
        }
        print(json.dumps(line), flush=True)
    pset.free()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def run_forward(args) -> None:
    """`--forward`: the whole DiT forward of one 1024x1024 image (64 x 64
    patches + 256 caption rows, the real model's shapes, seeded synthetic w8
    weights and eight LoRA slots as in the default workload) per sampler step,
    eager and as one CUDA-graph replay, for one image and for the CFG batch of
    two (conditional + zero negative caption). The context refiner runs once
    per caption (the caption cache) and is outside the timed steps, as in a
    denoising loop. One GPU; prints one JSON line (not the projection metric)."""
    import numpy as np
    import torch

    from mingproj.dit import Layout, projection_flops
    from mingproj.dit_forward import DitForward, DitModelConfig
    from mingproj.proj import Context

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = DitModelConfig()
    ctx = Context(0)
    fwd = DitForward.synthetic(ctx, cfg, bits=8, seed=1, device=dev)
    for i, r in enumerate(RANKS):
        fwd.proj.bind_synthetic(i, r, seed=100 + i, device=dev)
    for i, sg in enumerate(np.random.default_rng(2).uniform(-1.0, 1.5, size=8)):
        ctx.set_strength(i, float(sg))
    gh = gw = 64
    cap_len = q = 256
    img = gh * gw
    gen = torch.Generator(device=dev).manual_seed(3)
    lat = torch.randn((2, img, cfg.patch_dim), device=dev, generator=gen).to(torch.bfloat16)
    cap = torch.zeros((cap_len, cfg.dim), device=dev, dtype=torch.bfloat16)
    cap[:, :cfg.cap_feat_dim] = torch.randn((cap_len, cfg.cap_feat_dim), device=dev,
                                            generator=gen).to(torch.bfloat16)
    caps = [cap, torch.zeros_like(cap)]
    sigmas = np.linspace(0.95, 0.05, args.warmup + args.steps)
    S = img + cap_len
    layout = Layout(img=img, cap=cap_len)
    base_f, lora_f = projection_flops(fwd.dims, layout, RANKS)
    hd, nh = cfg.head_dim, cfg.n_heads
    # attention: Q K^T and P V, 4 S^2 hd per head; noise refiner over the image
    # rows, main layers over the joint rows (the context refiner is cached)
    attn_f = 4.0 * hd * nh * (cfg.n_refiner * img * img + cfg.n_layers * S * S)
    # projection_flops counts the context refiner's blocks too; they run once
    # per caption, outside the step
    H, FF, rsum = cfg.dim, cfg.ffn, float(sum(RANKS))
    n_ctx = sum(fwd.dims.block_kind(b) == "cap" for b in range(fwd.dims.n_blocks))
    ctx_f = n_ctx * 2.0 * cap_len * ((4 * H * H + 3 * FF * H) +
                                     rsum * (4 * (H + H) + 3 * (H + FF)))
    step_f = base_f + lora_f - ctx_f + attn_f

    res = {}
    with ClockSampler(0) as clk:
        for B in (1, 2):
            lb, cb = lat[:B], caps[:B]
            runner = fwd.graph(B, q, gh, gw, cap_len)
            for mode in ("eager", "graph"):
                call = ((lambda sg: fwd.forward_batch(lb, cb, q, gh, gw, [sg] * B))
                        if mode == "eager" else (lambda sg: runner(lb, cb, [sg] * B)))
                for i in range(args.warmup):
                    call(float(sigmas[i]))
                torch.cuda.synchronize(dev)
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
                t0 = time.perf_counter()
                ev[0].record()
                for i in range(args.steps):
                    call(float(sigmas[args.warmup + i]))
                ev[1].record()
                torch.cuda.synchronize(dev)
                wall = (time.perf_counter() - t0) * 1e3 / args.steps
                ms = ev[0].elapsed_time(ev[1]) / args.steps
                res[f"{mode}_b{B}"] = {"ms_per_step": ms, "host_ms_per_step": wall,
                                       "tflops": B * step_f / (ms / 1e3) / 1e12}
            runner.release()
    ctx.sync_check()
    print(json.dumps({
        "workload": "forward", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "config": {"model": "Ming-Image DiT (H 3840, 30 heads, 2+2 refiner, 30 layers), "
                            "synthetic w8 g64, 8 LoRA slots r={4,..,64}",
                   "image": "1024x1024 (64x64 patches)", "caption_rows": cap_len,
                   "cfg_batch": [1, 2]},
        "flops_per_image_step": step_f, "results": res, "clocks": clk.summary(),
        "data": "synthetic"}))
    fwd.free()
    ctx.close()


def _workload_state(cfg: dict, world: int, rank: int, dev, ctx, seed_base: int):
    """Projection set, slots, inputs and outputs of one rank of a workload.
    Configs 2 and 3: the rank's own image (weak scaling: every rank draws its
    own weights, inputs and strengths). Config 5: the rank's 8 / world images
    of the shared batch (strong scaling: the same model on every rank)."""
    import numpy as np
    import torch

    from mingproj.dit import DitDims, DitProjectionSet, Layout, alloc_outputs

    dims = DitDims()
    layout = Layout(img=cfg["img"], cap=cfg["cap"])
    strong = cfg["images"] > 1
    if strong and cfg["images"] % world != 0:
        raise SystemExit(f"{cfg['images']} images do not split evenly over {world} ranks")
    n_img = cfg["images"] // world if strong else 1
    wseed = seed_base if strong else seed_base + rank
    pset = DitProjectionSet.synthetic(ctx, dims, bits=cfg["bits"], seed=wseed, device=dev)
    for i, r in enumerate(cfg["ranks"]):
        pset.bind_synthetic(i, r, seed=100 * wseed + i, device=dev)
    gen = torch.Generator(device=dev).manual_seed(wseed + 7 + (rank if strong else 0))
    rows = n_img * layout.joint
    st = {
        "dims": dims, "layout": layout, "n_img": n_img, "pset": pset,
        "nrm": torch.randn((rows, dims.dim), device=dev, generator=gen).to(torch.bfloat16),
        "ao": torch.randn((rows, dims.dim), device=dev, generator=gen).to(torch.bfloat16),
        "ffi": torch.randn((rows, dims.ffn), device=dev, generator=gen).to(torch.bfloat16),
        "temb": torch.randn((n_img, dims.adaln), device=dev, generator=gen).to(torch.bfloat16),
        "outs": alloc_outputs(dims, rows, dev),
        "rng": np.random.default_rng(wseed + 11 + (rank if strong else 0)),
    }
    return st


def _step_flops(cfg: dict, st: dict) -> tuple[float, float, float]:
    from mingproj.dit import modulation_flops, projection_flops
    base_f, lora_f = projection_flops(st["dims"], st["layout"], cfg["ranks"])
    n = st["n_img"]
    return n * base_f, n * lora_f, modulation_flops(st["dims"], n)


def _draw(st: dict):
    """This step's strength vectors (one per image), ~U(-1, 1.5)."""
    return st["rng"].uniform(-1.0, 1.5, size=(st["n_img"], 8))


def run_strong_batch(args, world: int, rank: int, dev, ctx) -> dict:
    """Config 5 as a second measurement of the same run: the 8-image batch
    split by image over the ranks, device time per step (max over ranks)."""
    import torch
    import torch.distributed as dist

    cfg = CONFIGS[5]
    st = _workload_state(cfg, world, rank, dev, ctx, seed_base=51)
    base_f, lora_f, mod_f = _step_flops(cfg, st)
    stream = torch.cuda.current_stream(dev)

    def step():
        st["pset"].forward_projections_batch(st["layout"], st["n_img"], _draw(st), st["nrm"],
                                             st["ao"], st["ffi"], st["outs"], temb=st["temb"])
    for _ in range(args.warmup):
        step()
    ctx.sync_check()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev[0].record(stream)
    for _ in range(args.steps):
        step()
    ev[1].record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ctx.sync_check()
    t = torch.tensor([ev[0].elapsed_time(ev[1])], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    ctx.clear_strengths_rows()
    st["pset"].free()
    total_f = world * (base_f + lora_f + mod_f)  # the whole batch's FLOPs per step
    return {"workload": cfg["workload"], "scaling": "strong", "images_per_rank": st["n_img"],
            "ms_per_step": ms, "value": total_f / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "flops_per_step": total_f, "steps": args.steps, "warmup": args.warmup}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=11,
                    help="timed steps (forwards); 11 = one denoise schedule")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=3,
                    help="headline workload (BASELINE config; default 3, the north-star target)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-config5", action="store_true",
                    help="skip the embedded config-5 strong-scaling measurement")
    ap.add_argument("--shard", choices=["images", "rows"], default="images")
    ap.add_argument("--forward", action="store_true",
                    help="time the whole DiT forward (eager and CUDA graph) instead")
    args = ap.parse_args()
    if args.forward:
        run_forward(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    if args.shard == "rows":
        run_rows(args)
        return

    import numpy as np
    import torch
    import torch.distributed as dist

    from mingproj.proj import Context

    cfg = CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    peaks = load_peaks()
    ctx = Context(local)
    st = _workload_state(cfg, world, rank, dev, ctx, seed_base=1)
    dims, layout, pset = st["dims"], st["layout"], st["pset"]
    n_img = st["n_img"]
    base_f, lora_f, mod_f = _step_flops(cfg, st)
    step_flops = base_f + lora_f + mod_f
    stream = torch.cuda.current_stream(dev)

    def step(nrm, ao, ffi, outs, around=None, mod_ev=None):
        s = _draw(st)  # strengths re-set before every forward
        if mod_ev is not None:
            mod_ev[0].record(stream)
            pset.ctx.modulation(pset.modset, st["temb"])
            mod_ev[1].record(stream)
            pset.forward_projections_batch(layout, n_img, s, nrm, ao, ffi, outs, around=around)
        else:
            pset.forward_projections_batch(layout, n_img, s, nrm, ao, ffi, outs,
                                           temb=st["temb"], around=around)

    for _ in range(args.warmup):
        step(st["nrm"], st["ao"], st["ffi"], st["outs"])
    ctx.sync_check()

    # ---- timed region: inputs resident in HBM --------------------------------
    ctx.reset_engagement()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    mod_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    # every projection call (one C-ABI call: its proj_pair_kernel launches, the
    # rank-space pre-GEMM and split-K reduce included) between two events
    n_calls = 4 * dims.n_blocks * args.steps
    call_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(n_calls)]
    call_i = [0]

    def timed(i, call):
        e = call_ev[call_i[0]]
        e[0].record(stream)
        call()
        e[1].record(stream)
        call_i[0] += 1
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev[0].record(stream)
        for i in range(args.steps):
            step(st["nrm"], st["ao"], st["ffi"], st["outs"], around=timed, mod_ev=mod_ev[i])
        ev[1].record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
    ctx.sync_check()
    eng = ctx.engagement()
    t = torch.tensor([ev[0].elapsed_time(ev[1])], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    value = world * step_flops * args.steps / (max_ms / 1e3) / 1e12
    clocks = clk.summary()

    # Roofline of the dominant kernel (proj_pair_kernel): the algorithmic FLOPs of
    # one projection call (base 2*M*N*K of its members + the live slots' LoRA
    # FLOPs) over that call's device time between its two events, averaged.
    proj_launches = eng["kernels"] - args.steps * ((n_img + 3) // 4)  # minus modulation launches
    proj_ms = sum(a.elapsed_time(b) for a, b in call_ev)
    mod_steps_us = [a.elapsed_time(b) * 1e3 for a, b in mod_ev]
    proj_flops = (base_f + lora_f) * args.steps
    achieved = proj_flops / (proj_ms / 1e3) / 1e12
    roofline = {
        "kernel": "proj_pair_kernel", "bound": "tensor", "achieved": achieved,
        "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
        "frac": achieved / peaks["bf16_tflops_sustained"],
        "frac_of_burst": achieved / peaks["bf16_tflops"],
        "peak_kind": f"{peaks['source']} sustained bf16 (kernel timed inside a long step)",
        "unit_of_work": "one projection call: q+k+v, to_out, w1+w3 or w2 of one block",
        "calls_per_step": n_calls / args.steps,
        "launches_per_step": proj_launches / args.steps,
        "launches_of": "proj_pair_kernel (fused projections and any separate pre-GEMMs) + "
                       "lora_reduce_kernel",
        "avg_call_us": proj_ms * 1e3 / n_calls,
        "flops_per_call": proj_flops / n_calls,
        "traffic": None,
    }
    # modulation: minimal bytes per step = 32 packed adaLN weights + group params
    # + bias, and the gains read and written
    H, K = dims.dim, dims.adaln
    wb = K * cfg["bits"] / 8 + 4 * (K // 64) if cfg["bits"] else 2 * K
    mod_bytes = dims.n_modulated * (4 * H * (wb + 2) + 2 * H * 2 * (1 + n_img) +
                                    4 * H * 2 * n_img)
    # the median over the steps: the first step's start event is recorded on
    # an idle GPU (synchronised just before), so its interval also holds the
    # host's launch of the call
    mod_us = float(np.median(mod_steps_us))
    # the same launch timed alone (after the timed region): each call after a
    # 256 MB read that evicts the weights from L2 without leaving dirty lines,
    # at the clock an idle-then-busy GPU gives it; in the step it follows a
    # power-capped projection whose output lines are still dirty in L2
    flush = torch.ones(64 << 20, dtype=torch.int32, device=dev)
    iso_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(10)]
    for e0, e1 in iso_ev:
        flush.sum()
        e0.record(stream)
        pset.ctx.modulation(pset.modset, st["temb"])
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ctx.sync_check()
    iso_us = float(np.median([e0.elapsed_time(e1) * 1e3 for e0, e1 in iso_ev]))
    del flush
    roofline["modulation"] = {
        "kernel": "mod_lane_kernel", "bound": "hbm", "us_per_step": mod_us,
        "us_per_step_of": "median over the timed steps",
        "us_steps": [round(v, 1) for v in mod_steps_us],
        "bytes_per_step": mod_bytes, "achieved_gbs": mod_bytes / (mod_us * 1e-6) / 1e9,
        "peak_gbs": peaks["hbm_gbs"],
        "frac": mod_bytes / (mod_us * 1e-6) / 1e9 / peaks["hbm_gbs"],
        "isolated_us": iso_us,
        "isolated_frac": mod_bytes / (iso_us * 1e-6) / 1e9 / peaks["hbm_gbs"]}
    traffic_file = ROOT / "profiles" / "traffic.json"
    if traffic_file.exists():
        try:
            tr = json.loads(traffic_file.read_text())
            roofline["traffic"] = tr.get(f"config{args.config}", {}).get("bytes_per_launch")
            roofline["traffic_of"] = tr.get(f"config{args.config}", {}).get("launch")
        except (ValueError, OSError, AttributeError):
            pass

    # ---- e2e: through the public API with host buffers ------------------------
    # Every step copies its inputs in from pinned host memory and reads its
    # results (every projection output of the last block) back. The copies run
    # on their own streams, double-buffered, so step i + 1's inputs and step
    # i - 1's results move while step i computes; the timed region spans the
    # first input copy to the last result copy.
    e2e = None
    if not args.no_e2e:
        nrm, ao, ffi, outs = st["nrm"], st["ao"], st["ffi"], st["outs"]
        h_in = [(nrm.cpu().pin_memory(), ao.cpu().pin_memory(), ffi.cpu().pin_memory())
                for _ in range(2)]
        d_in = [(nrm, ao, ffi), (torch.empty_like(nrm), torch.empty_like(ao), torch.empty_like(ffi))]
        d_out = [outs, {k: torch.empty_like(v) for k, v in outs.items()}]
        h_out = [{k: torch.empty_like(v, device="cpu").pin_memory() for k, v in outs.items()}
                 for _ in range(2)]
        h2d = sum(t_.numel() for t_ in h_in[0]) * 2
        d2h = sum(v.numel() for v in outs.values()) * 2
        h2d_s = torch.cuda.Stream(dev)
        d2h_s = torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_done = [torch.cuda.Event() for _ in range(2)]
        ev_read = [torch.cuda.Event() for _ in range(2)]

        def issue_h2d(i):  # inputs of step i into set i % 2
            with torch.cuda.stream(h2d_s):
                if i >= 2:
                    h2d_s.wait_event(ev_done[i % 2])  # step i - 2 has finished reading them
                for d, h in zip(d_in[i % 2], h_in[i % 2]):
                    d.copy_(h, non_blocking=True)
                ev_in[i % 2].record(h2d_s)

        def run_e2e(k):
            h2d_s.wait_stream(stream)
            issue_h2d(0)
            if k > 1:
                issue_h2d(1)
            for i in range(k):
                stream.wait_event(ev_in[i % 2])
                if i >= 2:
                    stream.wait_event(ev_read[i % 2])  # step i - 2's results are read out
                x_n, x_a, x_f = d_in[i % 2]
                step(x_n, x_a, x_f, d_out[i % 2])
                ev_done[i % 2].record(stream)
                with torch.cuda.stream(d2h_s):
                    d2h_s.wait_event(ev_done[i % 2])
                    for name, v in d_out[i % 2].items():
                        h_out[i % 2][name].copy_(v, non_blocking=True)
                    ev_read[i % 2].record(d2h_s)
                if i + 2 < k:
                    issue_h2d(i + 2)
            for j in range(min(k, 2)):
                stream.wait_event(ev_read[(k - 1 - j) % 2])

        run_e2e(2)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev[0].record(stream)
        run_e2e(args.steps)
        ev[1].record(stream)
        torch.cuda.synchronize(dev)
        ctx.sync_check()
        e_ms = torch.tensor([ev[0].elapsed_time(ev[1])], device=dev, dtype=torch.float64)
        if world > 1:
            dist.barrier()
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e2e = {"value": world * step_flops * args.steps / (float(e_ms.item()) / 1e3) / 1e12,
               "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": float(e_ms.item()) / args.steps,
               "what": "C-ABI calls with pinned-host inputs copied in and every projection "
                       "output of the last block copied out each step; copies on their own "
                       "streams, double-buffered, overlapping the neighbouring steps' compute"}
        del h_in, d_in, d_out, h_out
    ctx.clear_strengths_rows()
    pset.free()
    del st
    torch.cuda.empty_cache()

    strong = None
    if args.config != 5 and not args.no_config5:
        strong = run_strong_batch(args, world, rank, dev, ctx)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg)

    if world > 1:
        dist.barrier()
    if rank == 0:
        par = (f"image-sharded x{world}: {n_img} of the batch's {cfg['images']} images per rank, "
               "all in one launch per projection (no data-path collective)"
               if cfg["images"] > 1 else
               f"image-sharded x{world}: one image per rank (no data-path collective)")
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": max_ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if cfg["images"] > 1 else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg["workload"],
                       "l2": "inputs larger than L2: each step streams every block's packed "
                             "weights (w4 3.4 GB / w8 6.4 GB per forward)",
                       "flops_per_step": world * step_flops,
                       "lora_flops_per_step": world * lora_f,
                       "parallelism": par},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(eng["kernels"]),
            "clocks": clocks,
            "engagement": {k: eng[k] for k in ("linear_calls", "lora_proj", "gemm_w8", "gemm_w4",
                                               "lora_down", "modulation", "kernels")},
            "config5_batch": strong,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
