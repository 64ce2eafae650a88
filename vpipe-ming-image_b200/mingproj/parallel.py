"""Multi-GPU partitioning of the projection path: one process per GPU,
torch.distributed for the plumbing.

The projections are row-independent (every token row of y depends only on
the same row of x), and the weights and adapters are replicated on every GPU
(a w8 DiT's 6.2 GB of block codes fits each B200). So the path shards
without any data-path collective:
  * a batch of images is split by IMAGE across ranks (each rank runs whole
    images; the attention consumer only needs its own image);
  * one image's rows are split into contiguous, 128-row-aligned TOKEN-ROW
    shards; a consumer that needs the full sequence (attention needs every
    K and V row) all-gathers the row-sharded outputs — the only collective,
    over NCCL / NVLink, issued on its own stream so it overlaps the next
    projection.
The reference is single-device (no parallelism at all); this module is the
B200 build's own.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

ROW_ALIGN = 128


@dataclass(frozen=True)
class Shard:
    start: int
    stop: int

    @property
    def rows(self) -> int:
        return self.stop - self.start


def row_shards(m: int, world: int, align: int = ROW_ALIGN) -> list[Shard]:
    """Contiguous shards of m rows over `world` ranks, every boundary a
    multiple of `align` (the last shard takes the remainder); ranks past the
    available rows get empty shards. Sizes differ by at most one `align`."""
    if world <= 0:
        raise ValueError("world must be positive")
    units = (m + align - 1) // align
    base, extra = divmod(units, world)
    shards, u = [], 0
    for r in range(world):
        take = base + (1 if r < extra else 0)
        start = min(u * align, m)
        stop = min((u + take) * align, m)
        shards.append(Shard(start, stop))
        u += take
    return shards


def image_shards(n_images: int, world: int) -> list[list[int]]:
    """Images per rank, contiguous and as even as possible."""
    out, i = [], 0
    base, extra = divmod(n_images, world)
    for r in range(world):
        take = base + (1 if r < extra else 0)
        out.append(list(range(i, i + take)))
        i += take
    return out


def padded_rows(m: int, world: int, align: int = ROW_ALIGN) -> int:
    """Rows of the gathered buffer: world equal blocks of the largest shard
    (all_gather_into_tensor wants equal parts)."""
    return world * max(s.rows for s in row_shards(m, world, align))


class RowGather:
    """All-gathers a row-sharded [rows_local, n] output into [m, n] on every
    rank, in rank order. Issues the collective on a dedicated stream (NCCL)
    so the caller can keep launching projections meanwhile; wait() joins it."""

    def __init__(self, m: int, n: int, world: int, rank: int, device, dtype=torch.bfloat16,
                 group=None, align: int = ROW_ALIGN):
        self.m, self.n, self.world, self.rank = m, n, world, rank
        self.shards = row_shards(m, world, align)
        self.block = max(s.rows for s in self.shards)
        self.group = group
        self.device = torch.device(device)
        self.send = torch.zeros((self.block, n), dtype=dtype, device=self.device)
        self.recv = torch.empty((self.block * world, n), dtype=dtype, device=self.device)
        self.stream = (torch.cuda.Stream(device=self.device) if self.device.type == "cuda"
                       else None)
        self._work = None

    @property
    def local(self) -> Shard:
        return self.shards[self.rank]

    @property
    def pending(self) -> bool:
        """A gather has been started and not yet joined."""
        return self._work is not None

    def start(self, y_local: torch.Tensor) -> None:
        """Begin gathering this rank's rows y_local [local.rows, n]."""
        rows = self.local.rows
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.stream):
                self.send[:rows].copy_(y_local[:rows])
                self._work = dist.all_gather_into_tensor(self.recv, self.send, group=self.group,
                                                         async_op=True)
        else:
            self.send[:rows].copy_(y_local[:rows])
            self._work = dist.all_gather_into_tensor(self.recv, self.send, group=self.group,
                                                     async_op=True)

    def wait(self) -> torch.Tensor:
        """Joins the gather and returns the full [m, n] rows in order."""
        if self._work is not None:
            self._work.wait()
            self._work = None
        if self.stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.stream)
        parts = [self.recv[r * self.block: r * self.block + s.rows]
                 for r, s in enumerate(self.shards)]
        return torch.cat(parts, dim=0)
