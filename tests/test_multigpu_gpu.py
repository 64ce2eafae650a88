"""Token-row sharding across GPUs (one process per GPU, NCCL): each rank
projects its slice of the rows (equal, 32-row aligned), the row all-gather on its own
stream reassembles the full output on every rank, and that equals the
single-GPU projection of all rows — bit for bit without adapters (rows are
independent and every row's K loop runs in the same order), within the
parity bar with live adapters. Needs 2 GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(ctx, seed, n, k, lora):
    from mingproj import pack as P
    rng = np.random.default_rng(seed)
    pw = P.synthetic_affine(rng, n, k, 8)
    w = ctx.upload(pw.n, pw.k, pw.bits, pw.data, pw.scales, pw.biases)
    if lora:
        for i, r in enumerate([8, 16, 32, 64]):
            w.bind(i, *P.synthetic_lora(rng, n, k, r, b_std=0.02))
            ctx.set_strength(i, 0.25 * (i + 1) - 0.6)
    return w


def _worker(rank, world, port, m, n, k, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from mingproj.parallel import RowGather
        from mingproj.proj import Context
        ctx = Context(rank)
        g = torch.Generator(device="cuda").manual_seed(123)
        x = torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)
        res = {}
        for lora in (False, True):
            w = _weights(ctx, 7, n, k, lora)
            gather = RowGather(m, n, world, rank, f"cuda:{rank}")
            loc = gather.local
            y_loc = ctx.linear(w, x[loc.start:loc.stop])
            gather.start(y_loc)
            y_all = gather.wait()
            ctx.sync_check()
            full = ctx.linear(w, x) if rank == 0 else None
            torch.cuda.synchronize()
            if rank == 0:
                a = y_all.float()
                b = full.float()
                res[lora] = (bool(torch.equal(y_all.view(torch.int16), full.view(torch.int16))),
                             float((a - b).norm() / b.norm()))
            w.free()
        if rank == 0:
            out.update(res)
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_row_sharded_projection_gathers_to_single_gpu_result():
    m, n, k = 4352, 3840, 3840
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker, args=(2, _free_port(), m, n, k, out), nprocs=2, join=True)
    exact_base, err_base = out[False]
    exact_lora, err_lora = out[True]
    assert exact_base, f"base rows differ after the gather (rel-L2 {err_base:.2e})"
    assert err_lora <= 1e-3, f"with adapters: rel-L2 {err_lora:.2e} against one GPU"
