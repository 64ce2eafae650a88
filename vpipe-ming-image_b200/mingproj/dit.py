"""The DiT's block-linear projection set: every block's seven projections and
the modulated blocks' adaLN Linears, resident on one GPU, with the runtime
LoRA slots bound across all of them.

Reference (vpipe-ming-image):
  Block / BlockLora              src/ming-dit.cc:457-472
  block order: context_refiner x n_refiner (unmodulated, caption rows),
  noise_refiner x n_refiner (modulated, image rows), layers x n_layers
  (modulated, joint rows)        src/ming-dit.cc:2388-2447
  run_block's projections        src/ming-dit.cc:2078-2080, :2094, :2155-2159
  fill_mod                       src/ming-dit.cc:2266-2273
  lora_module_capacity           src/ming-dit.cc:3123-3128
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from .lora import SlotBinding, module_names
from .pack import PROJ_NAMES, PackedWeight
from .proj import Context, ModSet, Weight

QKV = ("attention.to_q", "attention.to_k", "attention.to_v")
FF13 = ("feed_forward.w1", "feed_forward.w3")


@dataclass
class DitDims:
    """ming::DitConfig's fields this path needs (src/ming-config.h:34-56).
    ffn = int(dim / 3 * 8) (the reference's feed-forward width)."""
    dim: int = 3840
    n_heads: int = 30
    n_refiner: int = 2
    n_layers: int = 30
    adaln: int = 256

    @property
    def ffn(self) -> int:
        return int(self.dim / 3 * 8)

    @property
    def n_blocks(self) -> int:
        return 2 * self.n_refiner + self.n_layers

    @property
    def n_modulated(self) -> int:
        return self.n_refiner + self.n_layers

    def block_prefix(self, b: int) -> str:
        if b < self.n_refiner:
            return f"context_refiner.{b}."
        if b < 2 * self.n_refiner:
            return f"noise_refiner.{b - self.n_refiner}."
        return f"layers.{b - 2 * self.n_refiner}."

    def block_kind(self, b: int) -> str:
        """'cap' (context refiner), 'img' (noise refiner) or 'joint' (layers)."""
        if b < self.n_refiner:
            return "cap"
        if b < 2 * self.n_refiner:
            return "img"
        return "joint"


@dataclass
class Layout:
    """Row counts of one forward (ming-layout.h:38-55): the image rows, the
    caption rows (pads dropped) and the joint sequence [image | caption]."""
    img: int
    cap: int

    @property
    def joint(self) -> int:
        return self.img + self.cap

    def rows(self, kind: str) -> int:
        return {"cap": self.cap, "img": self.img, "joint": self.joint}[kind]


def projection_flops(dims: DitDims, layout: Layout, ranks=()) -> tuple[float, float]:
    """Algorithmic FLOPs of one forward's projection set: (base, lora).
    base = sum over blocks of 2 * rows * (4 H^2 + 3 FF H) — the projection part
    of the reference's flops_want (tests/ming-dit-test.cc:507-538); lora = sum
    over blocks, projections and live slots of 2 * rows * r * (K + N)."""
    H, FF = dims.dim, dims.ffn
    rsum = float(sum(ranks))
    base = lora = 0.0
    for b in range(dims.n_blocks):
        m = layout.rows(dims.block_kind(b))
        base += 2.0 * m * (4 * H * H + 3 * FF * H)
        lora += 2.0 * m * rsum * (4 * (H + H) + 3 * (H + FF))
    return base, lora


def modulation_flops(dims: DitDims, m: int = 1, k: int | None = None) -> float:
    k = dims.adaln if k is None else k
    return 2.0 * m * 4 * dims.dim * k * dims.n_modulated


@dataclass
class BlockWeights:
    proj: dict[str, Weight] = field(default_factory=dict)


def _device_affine(gen: torch.Generator, n: int, k: int, bits: int, device) -> tuple:
    """Seeded synthetic affine pack on the device (BASELINE configs 2/3/5):
    codes uniform over the full range, scales ~U(0.002, 0.02), w8 biases
    -128*scale, w4 biases -8*scale + N(0, scale)."""
    nbytes = k * bits // 8
    codes = torch.randint(0, 256, (n, nbytes), dtype=torch.uint8, device=device, generator=gen)
    scale = torch.rand((n, k // 64), device=device, generator=gen) * 0.018 + 0.002
    if bits == 8:
        bias = -128.0 * scale
    else:
        bias = -8.0 * scale + torch.randn((n, k // 64), device=device, generator=gen) * scale
    return (codes.view(torch.int32), scale.to(torch.bfloat16), bias.to(torch.bfloat16))


def _device_dense(gen: torch.Generator, n: int, k: int, device, std: float = 0.02):
    return (torch.randn((n, k), device=device, generator=gen) * std).to(torch.bfloat16)


class DitProjectionSet:
    """All blocks' projection weights (and adaLN Linears) on one device."""

    def __init__(self, ctx: Context, dims: DitDims):
        self.ctx = ctx
        self.dims = dims
        self.blocks: list[BlockWeights] = [BlockWeights() for _ in range(dims.n_blocks)]
        self.modset: ModSet | None = None
        self.ada: list[Weight] = []
        self.slot_ranks: list[dict[str, int]] = [dict() for _ in range(8)]
        self.binding_version = 0  # counts bind / unbind calls (caches keyed on the adapters)

    # ---- construction ------------------------------------------------------
    @classmethod
    def synthetic(cls, ctx: Context, dims: DitDims, bits: int, seed: int,
                  device: torch.device, with_modulation: bool = True) -> "DitProjectionSet":
        s = cls(ctx, dims)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        H, FF = dims.dim, dims.ffn
        shapes = {"attention.to_q": (H, H), "attention.to_k": (H, H), "attention.to_v": (H, H),
                  "attention.to_out.0": (H, H), "feed_forward.w1": (FF, H),
                  "feed_forward.w3": (FF, H), "feed_forward.w2": (H, FF)}
        for b in range(dims.n_blocks):
            for name in PROJ_NAMES:
                n, k = shapes[name]
                if bits == 0:
                    w = ctx.upload(n, k, 0, _device_dense(gen, n, k, device))
                else:
                    c, sc, bi = _device_affine(gen, n, k, bits, device)
                    w = ctx.upload(n, k, bits, c, sc, bi)
                s.blocks[b].proj[name] = w
        torch.cuda.synchronize(device)
        if with_modulation:
            ada, biases, an1, fn1 = [], [], [], []
            for _ in range(dims.n_modulated):
                n, k = 4 * H, dims.adaln
                if bits == 0:
                    ada.append(ctx.upload(n, k, 0, _device_dense(gen, n, k, device)))
                else:
                    c, sc, bi = _device_affine(gen, n, k, bits, device)
                    ada.append(ctx.upload(n, k, bits, c, sc, bi))
                biases.append((torch.randn(n, device=device, generator=gen) * 0.02)
                              .to(torch.bfloat16))
                an1.append((1.0 + 0.1 * torch.randn(H, device=device, generator=gen))
                           .to(torch.bfloat16))
                fn1.append((1.0 + 0.1 * torch.randn(H, device=device, generator=gen))
                           .to(torch.bfloat16))
            s.ada = ada
            s.modset = ctx.modulation_set(ada, biases, an1, fn1)
            s._mod_keep = (biases, an1, fn1)
        return s

    @classmethod
    def from_packed(cls, ctx: Context, dims: DitDims,
                    weights: dict[str, PackedWeight]) -> "DitProjectionSet":
        """Uploads a pack given as module name -> PackedWeight (host arrays)."""
        s = cls(ctx, dims)
        for b in range(dims.n_blocks):
            pre = dims.block_prefix(b)
            for name in PROJ_NAMES:
                pw = weights[pre + name]
                s.blocks[b].proj[name] = ctx.upload(pw.n, pw.k, pw.bits, pw.data, pw.scales,
                                                    pw.biases, mode=pw.mode)
        return s

    # ---- LoRA ----------------------------------------------------------------
    def bind_slot(self, slot: int, binding: SlotBinding) -> int:
        """Binds what `binding` holds into slot `slot` of every module; returns
        the number of modules bound (0 when the slot was refused)."""
        self.unbind_slot(slot)
        self.binding_version += 1
        for b in range(self.dims.n_blocks):
            pre = self.dims.block_prefix(b)
            for name in PROJ_NAMES:
                f = binding.bound.get(pre + name)
                if f is not None:
                    self.blocks[b].proj[name].bind(slot, f.a, f.b)
                    self.slot_ranks[slot][pre + name] = f.rank
        return len(self.slot_ranks[slot])

    def bind_synthetic(self, slot: int, rank: int, seed: int, device, b_std: float = 0.01) -> int:
        """A ~N(0, 1/r), B ~N(0, b_std) on every module."""
        self.unbind_slot(slot)
        self.binding_version += 1
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        for b in range(self.dims.n_blocks):
            pre = self.dims.block_prefix(b)
            for name in PROJ_NAMES:
                w = self.blocks[b].proj[name]
                a = (torch.randn((rank, w.k), device=device, generator=gen) / np.sqrt(rank)
                     ).to(torch.bfloat16)
                bb = (torch.randn((w.n, rank), device=device, generator=gen) * b_std
                      ).to(torch.bfloat16)
                w.bind(slot, a, bb)
                self.slot_ranks[slot][pre + name] = rank
        return len(self.slot_ranks[slot])

    def unbind_slot(self, slot: int) -> None:
        if not self.slot_ranks[slot]:
            return
        self.binding_version += 1
        for b in range(self.dims.n_blocks):
            for name in PROJ_NAMES:
                w = self.blocks[b].proj[name]
                if w.ranks[slot]:
                    w.unbind(slot)
        self.slot_ranks[slot] = {}

    def lora_modules(self, slot: int) -> int:
        return len(self.slot_ranks[slot])

    # ---- the projections of one block ------------------------------------------
    def block_projections(self, b: int, nrm: torch.Tensor, attn_out: torch.Tensor,
                          ffn_in: torch.Tensor, outs: dict[str, torch.Tensor],
                          stream=None, around=None) -> None:
        """The seven projections of block b, in run_block's order: q/k/v on
        `nrm` (one shared rank-space pass), to_out on `attn_out`, w1/w3 on
        `nrm`, w2 on `ffn_in`. `outs` maps projection name -> output tensor
        (rows >= nrm.shape[0]). `around(i, call)` (optional) runs call i (0-3)
        of the block, e.g. between two CUDA events."""
        p = self.blocks[b].proj
        m = nrm.shape[0]
        calls = (
            lambda: self.ctx.linear_shared([p[n] for n in QKV], nrm, [outs[n][:m] for n in QKV],
                                           stream),
            lambda: self.ctx.linear(p["attention.to_out.0"], attn_out,
                                    outs["attention.to_out.0"][:m], stream),
            lambda: self.ctx.linear_shared([p[n] for n in FF13], nrm, [outs[n][:m] for n in FF13],
                                           stream),
            lambda: self.ctx.linear(p["feed_forward.w2"], ffn_in, outs["feed_forward.w2"][:m],
                                    stream),
        )
        for i, call in enumerate(calls):
            if around is None:
                call()
            else:
                around(i, call)

    def forward_projections(self, layout: Layout, nrm: torch.Tensor, attn_out: torch.Tensor,
                            ffn_in: torch.Tensor, outs: dict[str, torch.Tensor],
                            temb: torch.Tensor | None = None, stream=None):
        """Every block's projections over the row counts of `layout` (inputs hold
        at least layout.joint rows), plus the batched modulation when `temb` is
        given. Returns the modulation outputs (or None)."""
        mod = None
        if temb is not None and self.modset is not None:
            mod = self.ctx.modulation(self.modset, temb, stream=stream)
        for b in range(self.dims.n_blocks):
            m = layout.rows(self.dims.block_kind(b))
            self.block_projections(b, nrm[:m], attn_out[:m], ffn_in[:m], outs, stream)
        return mod

    def forward_projections_batch(self, layout: Layout, n_images: int, strengths,
                                  nrm: torch.Tensor, attn_out: torch.Tensor,
                                  ffn_in: torch.Tensor, outs: dict[str, torch.Tensor],
                                  temb: torch.Tensor | None = None, stream=None, around=None):
        """Every block's projections for `n_images` images of the same layout,
        each with its own strength vector over the shared slots (`strengths`
        [n_images, 8]). A block's inputs hold the images one after another
        (image i's rows of a block kind are rows [i R, (i + 1) R), R =
        layout.rows(kind)); every projection runs ONCE over all images' rows
        with per-image row segments, and the modulation takes one temb row per
        image. A single image uses the per-slot strengths."""
        s = np.asarray(strengths, dtype=np.float32).reshape(n_images, -1)
        if n_images == 1:
            self.ctx.clear_strengths_rows()
            for i, v in enumerate(s[0]):
                self.ctx.set_strength(i, float(v))
        mod = None
        if temb is not None and self.modset is not None:
            mod = self.ctx.modulation(self.modset, temb, stream=stream)
        kind_prev = None
        for b in range(self.dims.n_blocks):
            kind = self.dims.block_kind(b)
            R = layout.rows(kind)
            if n_images > 1 and kind != kind_prev:
                self.ctx.set_strengths_rows(s, np.arange(n_images + 1, dtype=np.int32) * R)
            kind_prev = kind
            m = n_images * R
            self.block_projections(b, nrm[:m], attn_out[:m], ffn_in[:m], outs, stream, around)
        return mod

    def free(self) -> None:
        for blk in self.blocks:
            for w in blk.proj.values():
                w.free()
        for w in self.ada:
            w.free()
        if self.modset is not None:
            self.modset.free()


def alloc_outputs(dims: DitDims, rows: int, device) -> dict[str, torch.Tensor]:
    H, FF = dims.dim, dims.ffn
    out = {}
    for name in PROJ_NAMES:
        n = FF if name in FF13 else H
        out[name] = torch.empty((rows, n), dtype=torch.bfloat16, device=device)
    return out


__all__ = ["DitDims", "Layout", "DitProjectionSet", "projection_flops", "modulation_flops",
           "alloc_outputs", "module_names"]
