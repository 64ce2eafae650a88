"""TEST INFRASTRUCTURE — fp32 CPU forward of the Ming-Image DiT, the oracle of
the end-to-end bar (the GPU bf16 forward must stay within rel-L2 0.0158 of
it). Only tests/ import this module.

A torch fp32 restatement of the reference DiT over the REAL rows (pads
dropped, positions keep the padded offsets), following (vpipe-ming-image):
  timestep sinusoid            src/ming-dit.cc:1418-1437 (cos first; t = t_scale * (1 - sigma))
  t_embedder MLP               docs/MING-IMAGE.md:426-431 (Linear 256->1024, SiLU, Linear 1024->256)
  x / caption embed            src/ming-dit.cc:2283-2305 (stream A: RMSNorm + Linear; stream B copied)
  block order                  src/ming-dit.cc:2388-2447 (context refiner | noise refiner, layers)
  block math                   src/ming-dit.cc:2065-2263, docs/MING-IMAGE.md:432-448
                               (sandwich RMSNorms eps 1e-5, per-head q/k RMSNorm, tanh gates,
                               (1 + scale), unmodulated context refiner)
  RoPE                         src/ming-dit.cc:1443-1486 (interleaved pairs; f64 angles -> f32)
  layout / positions           src/ming-layout.cc:19-60 (image axis-0 = roundup32(cap_len) + 1)
  final layer                  src/ming-dit.cc:2553-2563 (LayerNorm eps 1e-6 * (1 + Linear(SiLU(temb))))
The parity of this restatement against the reference's own goldens is
unpinned: the goldens (tools/dump_ming_golden.py) are not in the reference
tree.
"""
from __future__ import annotations

import math

import numpy as np
import torch

SEQ_MULTIPLE = 32
X_EMBEDDER = "all_x_embedder.2-1"      # checkpoint names of the model-level Linears
FINAL = "all_final_layer.2-1"


def roundup(v: int, m: int) -> int:
    return (v + m - 1) // m * m


def positions(grid_h: int, grid_w: int, cap_len: int) -> np.ndarray:
    """[joint, 3] RoPE positions of [image rows | caption rows]."""
    img = grid_h * grid_w
    cap_total = roundup(cap_len, SEQ_MULTIPLE)
    pos = np.zeros((img + cap_len, 3), dtype=np.int64)
    hh, ww = np.meshgrid(np.arange(grid_h), np.arange(grid_w), indexing="ij")
    pos[:img, 0] = cap_total + 1
    pos[:img, 1] = hh.reshape(-1)
    pos[:img, 2] = ww.reshape(-1)
    pos[img:, 0] = np.arange(cap_len) + 1
    return pos


def rope_tables(pos: np.ndarray, head_dim: int, axes=(32, 48, 48), theta: float = 256.0):
    """cos / sin per row and per interleaved pair, f64 angles rounded to f32:
    returns two float32 arrays [rows, head_dim // 2]."""
    freqs, axis_of = [], []
    for a, d in enumerate(axes):
        for j in range(d // 2):
            freqs.append(1.0 / theta ** (2.0 * j / d))
            axis_of.append(a)
    freqs = np.array(freqs[: head_dim // 2], dtype=np.float64)
    axis_of = np.array(axis_of[: head_dim // 2])
    ang = pos[:, axis_of].astype(np.float64) * freqs[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def timestep_embedding(sigma: float, t_scale: float = 1000.0, dim: int = 256) -> np.ndarray:
    half = dim // 2
    t = t_scale * (1.0 - sigma)
    i = np.arange(half, dtype=np.float64)
    f = np.exp(-math.log(10000.0) * i / half)
    return np.concatenate([np.cos(t * f), np.sin(t * f)]).astype(np.float32)


def rms(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y * w if w is not None else y


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [rows, heads, hd]; cos/sin [rows, hd/2]; interleaved pairs."""
    x0, x1 = x[..., 0::2], x[..., 1::2]
    c, s = cos[:, None, :], sin[:, None, :]
    out = torch.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


class DitRef:
    """fp32 CPU forward. `w` maps the checkpoint's tensor names to float
    tensors (block projections already dequantized when a pack is tested)."""

    def __init__(self, w: dict, dim: int, n_heads: int, n_refiner: int, n_layers: int,
                 cap_feat_dim: int, eps: float = 1e-5, dtype=torch.float32):
        self.w = {k: torch.as_tensor(v).to(dtype) for k, v in w.items()}
        self.dim, self.nh, self.hd = dim, n_heads, dim // n_heads
        self.n_refiner, self.n_layers = n_refiner, n_layers
        self.cap_feat_dim = cap_feat_dim
        self.eps = eps
        self.dtype = dtype

    def lin(self, x, name, bias=True):
        y = x @ self.w[name + ".weight"].T
        if bias and (name + ".bias") in self.w:
            y = y + self.w[name + ".bias"]
        return y

    def block(self, x, pre, cos, sin, temb):
        w, eps, nh, hd = self.w, self.eps, self.nh, self.hd
        R = x.shape[0]
        if temb is not None:
            mods = self.lin(temb[None, :], pre + "adaLN_modulation.0")[0]
            s_msa, g_msa, s_mlp, g_mlp = mods.chunk(4)
        n1 = rms(x, w[pre + "attention_norm1.weight"], eps)
        if temb is not None:
            n1 = n1 * (1.0 + s_msa)
        q = self.lin(n1, pre + "attention.to_q", False).view(R, nh, hd)
        k = self.lin(n1, pre + "attention.to_k", False).view(R, nh, hd)
        v = self.lin(n1, pre + "attention.to_v", False).view(R, nh, hd)
        q = rope(rms(q, w[pre + "attention.norm_q.weight"], eps), cos, sin)
        k = rope(rms(k, w[pre + "attention.norm_k.weight"], eps), cos, sin)
        att = torch.nn.functional.scaled_dot_product_attention(
            q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None])
        a = att[0].transpose(0, 1).reshape(R, nh * hd)
        o = rms(self.lin(a, pre + "attention.to_out.0", False), w[pre + "attention_norm2.weight"],
                eps)
        x = x + (torch.tanh(g_msa) * o if temb is not None else o)
        n2 = rms(x, w[pre + "ffn_norm1.weight"], eps)
        if temb is not None:
            n2 = n2 * (1.0 + s_mlp)
        h = torch.nn.functional.silu(self.lin(n2, pre + "feed_forward.w1", False)) * \
            self.lin(n2, pre + "feed_forward.w3", False)
        f = rms(self.lin(h, pre + "feed_forward.w2", False), w[pre + "ffn_norm2.weight"], eps)
        return x + (torch.tanh(g_mlp) * f if temb is not None else f)

    def forward(self, latents, cap, query_rows: int, grid_h: int, grid_w: int, sigma: float,
                trace_dir: str | None = None):
        """latents [img, patch_dim]; cap [cap_len, >= dim] with stream A in
        rows [0, query_rows) x columns [0, cap_feat_dim). Returns [img, patch_dim].
        With trace_dir, writes the stages the reference traces
        (src/ming-dit.cc:2304, 2413, 2545) as raw float32 files <tag>.f32:
        embed, ctx, blk<L>."""
        def trace(tag, rows):
            if trace_dir is not None:
                import os
                os.makedirs(trace_dir, exist_ok=True)
                rows.detach().float().numpy().astype("float32").tofile(
                    os.path.join(trace_dir, tag + ".f32"))

        dt = self.dtype
        latents = torch.as_tensor(latents).to(dt)
        cap = torch.as_tensor(cap).to(dt)
        img = grid_h * grid_w
        cap_len = cap.shape[0]
        pos = positions(grid_h, grid_w, cap_len)
        c, s = rope_tables(pos, self.hd)
        cos, sin = torch.from_numpy(c).to(dt), torch.from_numpy(s).to(dt)
        emb = torch.from_numpy(timestep_embedding(sigma)).to(dt)
        te = torch.nn.functional.silu(self.lin(emb[None], "t_embedder.mlp.0"))
        temb = self.lin(te, "t_embedder.mlp.2")[0]
        x = self.lin(latents, X_EMBEDDER)
        x0, xs = x, []
        for i in range(self.n_refiner):
            x = self.block(x, f"noise_refiner.{i}.", cos[:img], sin[:img], temb)
            xs.append(x)
        ca = rms(cap[:query_rows, : self.cap_feat_dim], self.w["cap_embedder.0.weight"], self.eps)
        ca = self.lin(ca, "cap_embedder.1")
        cj = torch.cat([ca, cap[query_rows:, : self.dim]], dim=0)
        trace("embed", torch.cat([x0, cj], dim=0))
        for i in range(self.n_refiner):
            cj = self.block(cj, f"context_refiner.{i}.", cos[img:], sin[img:], None)
        trace("ctx", cj)
        for i in range(self.n_refiner):
            trace(f"blk{i}", torch.cat([xs[i], cj], dim=0))
        j = torch.cat([x, cj], dim=0)
        for i in range(self.n_layers):
            j = self.block(j, f"layers.{i}.", cos, sin, temb)
            trace(f"blk{self.n_refiner + i}", j)
        scale = self.lin(torch.nn.functional.silu(temb)[None], FINAL + ".adaLN_modulation.1")[0]
        xi = torch.nn.functional.layer_norm(j[:img], (self.dim,), eps=1e-6) * (1.0 + scale)
        return self.lin(xi, FINAL + ".linear")
