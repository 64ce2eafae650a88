"""Partition and gather order of the multi-GPU path, on CPU ranks (gloo,
world size 2 and 4): shards cover every row exactly once at 32-row-aligned
boundaries, images split evenly, and the row all-gather reassembles the
full sequence in order on every rank."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mingproj.parallel import RowGather, image_shards, padded_rows, row_shards


@pytest.mark.parametrize("m", [1, 127, 128, 256, 4352, 4096, 16896, 4480])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_row_shards_cover_once_aligned(m, world):
    sh = row_shards(m, world)
    assert len(sh) == world
    assert sh[0].start == 0 and sh[-1].stop == m
    for a, b in zip(sh, sh[1:]):
        assert a.stop == b.start
    for s in sh[:-1]:
        assert s.stop % 32 == 0 or s.stop == m
    sizes = [s.rows for s in sh if s.rows > 0]
    assert max(sizes) - min(sizes) <= 32
    assert padded_rows(m, world) >= m


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config_row_counts_split_evenly(world):
    # 4352 = 136 * 32 and 16896 = 528 * 32 rows: equal shards at 2, 4 and 8
    # ranks, so the gather writes the final buffer with no reassembly copy
    for m in (4352, 16896, 16384):
        assert {s.rows for s in row_shards(m, world)} == {m // world}


def test_image_shards():
    assert image_shards(8, 1) == [list(range(8))]
    assert image_shards(8, 4) == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert image_shards(8, 8) == [[i] for i in range(8)]
    assert sum(map(len, image_shards(5, 2))) == 5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = torch.arange(m * n, dtype=torch.float32).view(m, n)
        g = RowGather(m, n, world, rank, "cpu", dtype=torch.float32)
        loc = g.local
        g.start(full[loc.start:loc.stop].clone())
        got = g.wait()
        # even shards: the result is the gather's own buffer, no copy
        out[rank] = (bool(torch.equal(got, full)),
                     (not g.even) or got.data_ptr() == g.recv.data_ptr())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,m", [(2, 4352), (2, 300), (4, 1000), (4, 4352)])
def test_row_gather_order_gloo(world, m):
    n = 8
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker, args=(world, _free_port(), m, n, out), nprocs=world, join=True)
    assert all(out[r][0] and out[r][1] for r in range(world))
