"""Multi-GPU partitioning of the projection path: one process per GPU,
torch.distributed for the plumbing.

The projections are row-independent (every token row of y depends only on
the same row of x), and the weights and adapters are replicated on every GPU
(a w8 DiT's 6.2 GB of block codes fits each B200). So the path shards
without any data-path collective:
  * a batch of images is split by IMAGE across ranks (each rank runs whole
    images; the attention consumer only needs its own image);
  * one image's rows are split into contiguous TOKEN-ROW shards, equal
    where the row count allows (32-row aligned: 4352 and 16896 rows split
    evenly over 2, 4 and 8 ranks); a consumer that needs the full sequence
    (attention needs every K and V row) all-gathers the row-sharded outputs —
    the only collective, over NCCL / NVLink, issued on its own stream so it
    overlaps the next projection. With equal shards the gather lands
    directly in the final [m, n] buffer (no reassembly copy).
The reference is single-device (no parallelism at all); this module is the
B200 build's own.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

ROW_ALIGN = 32


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
    so the caller can keep launching projections meanwhile; wait() joins it.
    When every shard has the same number of rows, the local rows are sent as
    they are and the gather writes the final [m, n] buffer itself; uneven
    shards go through padded blocks and one reassembly copy. On CUDA the
    collective's device time is recorded (last_ms)."""

    def __init__(self, m: int, n: int, world: int, rank: int, device, dtype=torch.bfloat16,
                 group=None, align: int = ROW_ALIGN):
        self.m, self.n, self.world, self.rank = m, n, world, rank
        self.shards = row_shards(m, world, align)
        self.block = max(s.rows for s in self.shards)
        self.even = all(s.rows == self.block for s in self.shards)
        self.group = group
        self.device = torch.device(device)
        self.send = (None if self.even else
                     torch.zeros((self.block, n), dtype=dtype, device=self.device))
        self.recv = torch.empty((self.block * world, n), dtype=dtype, device=self.device)
        cuda = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(device=self.device) if cuda else None
        self._ev = ([torch.cuda.Event(enable_timing=True) for _ in range(2)] if cuda else None)
        self._timed = False
        self._work = None

    @property
    def local(self) -> Shard:
        return self.shards[self.rank]

    @property
    def pending(self) -> bool:
        """A gather has been started and not yet joined."""
        return self._work is not None

    def _send(self, y_local: torch.Tensor) -> torch.Tensor:
        rows = self.local.rows
        if self.even and y_local.is_contiguous():
            return y_local[:rows]
        buf = self.send if self.send is not None else torch.empty_like(self.recv[:rows])
        buf[:rows].copy_(y_local[:rows])
        return buf

    def start(self, y_local: torch.Tensor) -> None:
        """Begin gathering this rank's rows y_local [local.rows, n] (row-major,
        contiguous rows; not to be written until wait() has joined)."""
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.stream):
                send = self._send(y_local)
                if send.data_ptr() == y_local.data_ptr():
                    y_local.record_stream(self.stream)
                self._ev[0].record(self.stream)
                self._work = dist.all_gather_into_tensor(self.recv, send, group=self.group,
                                                         async_op=True)
                self._ev[1].record(self.stream)
                self._timed = True
        else:
            self._work = dist.all_gather_into_tensor(self.recv, self._send(y_local),
                                                     group=self.group, async_op=True)

    def wait(self) -> torch.Tensor:
        """Joins the gather and returns the full [m, n] rows in order (the
        gather's own buffer when the shards are even)."""
        if self._work is not None:
            self._work.wait()
            self._work = None
        if self.stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.stream)
        if self.even:
            return self.recv[:self.m]
        parts = [self.recv[r * self.block: r * self.block + s.rows]
                 for r, s in enumerate(self.shards)]
        return torch.cat(parts, dim=0)

    def last_ms(self) -> float | None:
        """Device time of the last gather on its stream (after wait() and a
        synchronize), or None."""
        if not self._timed:
            return None
        return self._ev[0].elapsed_time(self._ev[1])
