"""The Ming-Image DiT forward on one GPU. Through the mingproj kernels: every
block projection, the batched adaLN modulation, the q/k head RMSNorm + RoPE
(q/k/v epilogue, head-major outputs), the attention (head dim 128), the
SwiGLU (w1/w3 epilogue) and the sandwich norms with their gated residuals
(one pass each after to_out and w2). In torch bf16: the embedders and the
final layer — the DiT driver around the hot path.

Follows the reference's MingDitMetal::forward (vpipe-ming-image,
src/ming-dit.cc:1490-2642): one forward over the REAL rows [image | caption]
with pads dropped and positions keeping the padded offsets
(src/ming-layout.cc:19-60); precision as the reference's map
(docs/MING-IMAGE.md:786-799): bf16 activations, f32 norm statistics and
RoPE, timestep sinusoid f32 then bf16.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from .dit import DitDims, DitProjectionSet
from .pack import PROJ_NAMES, PackedWeight, bf16_bits_to_f32
from .packio import Pack
from .proj import Context

TRACE_ENV = "VPIPE_MING_DIT_TRACE"  # the reference's per-stage trace switch
X_EMBEDDER = "all_x_embedder.2-1"
FINAL = "all_final_layer.2-1"
SEQ_MULTIPLE = 32


@dataclass
class DitModelConfig:
    """The DiT's structural dimensions (ming::DitConfig, src/ming-config.h:34-56)."""
    dim: int = 3840
    n_heads: int = 30
    n_refiner: int = 2
    n_layers: int = 30
    cap_feat_dim: int = 2560
    patch_dim: int = 64
    time_freq: int = 256
    time_mid: int = 1024
    adaln: int = 256
    norm_eps: float = 1e-5
    rope_theta: float = 256.0
    t_scale: float = 1000.0
    axes: tuple = (32, 48, 48)

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @property
    def ffn(self) -> int:
        return int(self.dim / 3 * 8)

    def proj_dims(self) -> DitDims:
        return DitDims(dim=self.dim, n_heads=self.n_heads, n_refiner=self.n_refiner,
                       n_layers=self.n_layers, adaln=self.adaln)


def _bf16(a) -> torch.Tensor:
    """uint16 bf16 bits (numpy) or float array (f16 / f32) -> torch bf16 (CPU)."""
    if isinstance(a, torch.Tensor):
        return a.to(torch.bfloat16)
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16)


def rope_tables(positions: np.ndarray, head_dim: int, axes, theta: float):
    """cos / sin [rows, head_dim / 2] for interleaved pairs (f64 angles -> f32),
    as build_rope_ (src/ming-dit.cc:1443-1486)."""
    freqs, axis_of = [], []
    for a, d in enumerate(axes):
        for j in range(d // 2):
            freqs.append(1.0 / theta ** (2.0 * j / d))
            axis_of.append(a)
    freqs = np.array(freqs[: head_dim // 2], dtype=np.float64)
    axis_of = np.array(axis_of[: head_dim // 2])
    ang = positions[:, axis_of].astype(np.float64) * freqs[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def layout_positions(grid_h: int, grid_w: int, cap_len: int) -> np.ndarray:
    """[joint, 3] positions (build_layout, src/ming-layout.cc:19-60): the image
    sits at axis-0 position roundup32(cap_len) + 1; caption row i at i + 1."""
    img = grid_h * grid_w
    cap_total = (cap_len + SEQ_MULTIPLE - 1) // SEQ_MULTIPLE * SEQ_MULTIPLE
    pos = np.zeros((img + cap_len, 3), dtype=np.int64)
    hh, ww = np.meshgrid(np.arange(grid_h), np.arange(grid_w), indexing="ij")
    pos[:img, 0] = cap_total + 1
    pos[:img, 1] = hh.reshape(-1)
    pos[:img, 2] = ww.reshape(-1)
    pos[img:, 0] = np.arange(cap_len) + 1
    return pos


class DitForward:
    """One DiT on one device. `weights` is either a dict mapping checkpoint
    names to bf16 bit arrays (uint16) for dense tensors, where block
    projections may instead be PackedWeight (a w8/w4 pack), or an open
    mingproj.packio.Pack (a checkpoint or pack read by the library's own
    safetensors reader; projections uploaded as load_qw_ detects them)."""

    def __init__(self, ctx: Context, cfg: DitModelConfig, weights, device):
        self.ctx, self.cfg, self.dev = ctx, cfg, device
        dims = cfg.proj_dims()
        self.dims = dims
        self.proj = DitProjectionSet(ctx, dims)
        is_pack = isinstance(weights, Pack)

        def matrix(base: str):
            if is_pack:
                return weights.upload(ctx, base)
            v = weights[base + ".weight"] if (base + ".weight") in weights else weights[base]
            if isinstance(v, PackedWeight):
                return ctx.upload(v.n, v.k, v.bits, v.data, v.scales, v.biases, mode=v.mode)
            t = _bf16(v)
            return ctx.upload(t.shape[0], t.shape[1], 0, t.contiguous())

        def tensor(name: str):
            return _bf16(weights.array(name) if is_pack else weights[name])

        for b in range(dims.n_blocks):
            pre = dims.block_prefix(b)
            for name in PROJ_NAMES:
                self.proj.blocks[b].proj[name] = matrix(pre + name)
        # adaLN of the modulated blocks, in the order noise_refiner..., layers...
        ada, biases, an1, fn1 = [], [], [], []
        for b in range(cfg.n_refiner, dims.n_blocks):
            pre = dims.block_prefix(b)
            ada.append(matrix(pre + "adaLN_modulation.0"))
            biases.append(tensor(pre + "adaLN_modulation.0.bias").to(device))
            an1.append(tensor(pre + "attention_norm1.weight").to(device))
            fn1.append(tensor(pre + "ffn_norm1.weight").to(device))
        self.ada = ada
        self.modset = ctx.modulation_set(ada, biases, an1, fn1)
        self._keep = (biases, an1, fn1)
        # every other tensor as a device bf16 tensor
        self.t = {}
        names = weights.names() if is_pack else list(weights)
        for k in names:
            if not is_pack and isinstance(weights[k], PackedWeight):
                continue
            if any(k.startswith(dims.block_prefix(b) + n) for b in range(dims.n_blocks)
                   for n in PROJ_NAMES + ("adaLN_modulation.0",)):
                continue
            self.t[k] = tensor(k).to(device)
        self._init_caches()

    def _init_caches(self) -> None:
        self.cap_cache_entries = 4
        self._cap_cache: list[dict] = []
        self._cap_strengths: tuple | None = None
        self._tick = 0
        self._rope_cache: dict = {}
        self.last_cap_cache_hit = False

    @classmethod
    def synthetic(cls, ctx: Context, cfg: DitModelConfig, bits: int, seed: int,
                  device) -> "DitForward":
        """Seeded random weights of the model's shapes, made on the device (no
        checkpoint; for timing whole forwards): the block projections and the
        adaLN Linears as DitProjectionSet.synthetic makes them (w8 / w4 packs
        or dense bf16), every other matrix bf16 ~N(0, 1/k), biases
        ~N(0, 0.02^2) and norm gains ~1 + N(0, 0.1^2)."""
        self = cls.__new__(cls)
        self.ctx, self.cfg, self.dev = ctx, cfg, device
        self.dims = cfg.proj_dims()
        self.proj = DitProjectionSet.synthetic(ctx, self.dims, bits, seed, device)
        self.ada, self.modset = self.proj.ada, self.proj.modset
        gen = torch.Generator(device=device)
        gen.manual_seed(seed + 1)
        H, hd = cfg.dim, cfg.head_dim

        def lin(n, k):
            return (torch.randn((n, k), device=device, generator=gen) / math.sqrt(k)).to(
                torch.bfloat16)

        def vec(n, mean=0.0, std=0.02):
            return (mean + std * torch.randn(n, device=device, generator=gen)).to(torch.bfloat16)

        t = {X_EMBEDDER + ".weight": lin(H, cfg.patch_dim), X_EMBEDDER + ".bias": vec(H),
             "cap_embedder.0.weight": vec(cfg.cap_feat_dim, 1.0, 0.1),
             "cap_embedder.1.weight": lin(H, cfg.cap_feat_dim), "cap_embedder.1.bias": vec(H),
             "t_embedder.mlp.0.weight": lin(cfg.time_mid, cfg.time_freq),
             "t_embedder.mlp.0.bias": vec(cfg.time_mid),
             "t_embedder.mlp.2.weight": lin(cfg.adaln, cfg.time_mid),
             "t_embedder.mlp.2.bias": vec(cfg.adaln),
             FINAL + ".adaLN_modulation.1.weight": lin(H, cfg.adaln),
             FINAL + ".adaLN_modulation.1.bias": vec(H),
             FINAL + ".linear.weight": lin(cfg.patch_dim, H), FINAL + ".linear.bias": vec(cfg.patch_dim)}
        for b in range(self.dims.n_blocks):
            pre = self.dims.block_prefix(b)
            t[pre + "attention.norm_q.weight"] = vec(hd, 1.0, 0.1)
            t[pre + "attention.norm_k.weight"] = vec(hd, 1.0, 0.1)
            for nm in ("attention_norm1", "attention_norm2", "ffn_norm1", "ffn_norm2"):
                t[pre + nm + ".weight"] = vec(H, 1.0, 0.1)
        self.t = t
        self._keep = ()
        self._init_caches()
        return self

    # ---- pieces ------------------------------------------------------------
    def _rms(self, x: torch.Tensor, w: torch.Tensor | None, eps: float | None = None):
        eps = self.cfg.norm_eps if eps is None else eps
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        if w is not None:
            y = y * w.float()
        return y.to(torch.bfloat16)

    def _rope(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        x0, x1 = xf[..., 0::2], xf[..., 1::2]
        c, s = cos[:, None, :], sin[:, None, :]
        out = torch.empty_like(xf)
        out[..., 0::2] = x0 * c - x1 * s
        out[..., 1::2] = x0 * s + x1 * c
        return out.to(torch.bfloat16)

    def _linear(self, x: torch.Tensor, name: str) -> torch.Tensor:
        return F.linear(x, self.t[name + ".weight"], self.t.get(name + ".bias"))

    def _block(self, b: int, x: torch.Tensor, cos, sin, mod_idx: int | None, mods, nw1, nw3,
               nb: int = 1):
        """Block b over `nb` sequences of equal length stacked in x (updated in
        place): the projections run once over all rows, norms, gates and the
        attention per sequence (sequence i takes modulation row i)."""
        cfg, pre = self.cfg, self.dims.block_prefix(b)
        t = self.t
        R = x.shape[0] // nb
        # the kernels' tile and K-split choices follow one sequence's rows
        self.ctx.set_image_rows(R if nb > 1 else 0)
        H, nh, hd, FF = cfg.dim, cfg.n_heads, cfg.head_dim, cfg.ffn
        p = self.proj.blocks[b].proj
        modulated = mod_idx is not None
        segs = [slice(i * R, (i + 1) * R) for i in range(nb)]
        nrm = torch.empty_like(x)
        for i, sl in enumerate(segs):
            gain1 = nw1[mod_idx, i] if modulated else t[pre + "attention_norm1.weight"]
            self.ctx.rms_residual(x[sl], None, nrm_gain=gain1, eps=cfg.norm_eps, nrm=nrm[sl])
        qkv = [p["attention.to_q"], p["attention.to_k"], p["attention.to_v"]]
        if hd == 128:
            # one launch: q/k/v head-major, q and k through the head RMSNorm and
            # the rotary embedding in the projection epilogue; then the tcgen05
            # attention per sequence, writing its rows of the token-major to_out input
            cs, sn = (cos, sin) if nb == 1 else (cos.repeat(nb, 1), sin.repeat(nb, 1))
            q, k, v = self.ctx.linear_heads(
                qkv, nrm, norm_w=[t[pre + "attention.norm_q.weight"],
                                  t[pre + "attention.norm_k.weight"], None],
                eps=cfg.norm_eps, rope_cos=cs, rope_sin=sn)
            a = torch.empty((nb * R, H), dtype=torch.bfloat16, device=x.device)
            for sl in segs:
                self.ctx.attention(q[:, sl], k[:, sl], v[:, sl], out=a[sl])
        else:
            qa, ka, va = self.ctx.linear_shared(qkv, nrm)
            a = torch.empty((nb * R, H), dtype=torch.bfloat16, device=x.device)
            for sl in segs:
                q = self._rope(self._rms(qa[sl].reshape(R, nh, hd),
                                         t[pre + "attention.norm_q.weight"]), cos, sin)
                k = self._rope(self._rms(ka[sl].reshape(R, nh, hd),
                                         t[pre + "attention.norm_k.weight"]), cos, sin)
                v = va[sl].reshape(R, nh, hd)
                att = F.scaled_dot_product_attention(q.transpose(0, 1)[None],
                                                     k.transpose(0, 1)[None],
                                                     v.transpose(0, 1)[None])
                a[sl] = att[0].transpose(0, 1).reshape(R, H)
        o = self.ctx.linear(p["attention.to_out.0"], a)
        # one pass per sequence: x += [tanh(gate_msa) *] rms(o, norm2);
        # nrm = rms(x, ffn norm) (x is this block's own copy of the stream)
        for i, sl in enumerate(segs):
            gain3 = nw3[mod_idx, i] if modulated else t[pre + "ffn_norm1.weight"]
            self.ctx.rms_residual(x[sl], o[sl], t[pre + "attention_norm2.weight"],
                                  mods[mod_idx, i, H:2 * H] if modulated else None,
                                  gain3, eps=cfg.norm_eps, nrm=nrm[sl])
        # gate and up projections with the SwiGLU in their epilogue (one launch):
        # h = bf16(silu(g) * u) of the bf16 gate and up values, as gpu_ff computes it
        ld = (FF + 7) // 8 * 8
        h = torch.empty((nb * R, ld), dtype=torch.bfloat16, device=x.device)
        self.ctx.linear_swiglu(p["feed_forward.w1"], p["feed_forward.w3"], nrm, out=h[:, :FF])
        f = self.ctx.linear(p["feed_forward.w2"], h[:, :FF])
        for i, sl in enumerate(segs):
            self.ctx.rms_residual(x[sl], f[sl], t[pre + "ffn_norm2.weight"],
                                  mods[mod_idx, i, 3 * H:] if modulated else None,
                                  eps=cfg.norm_eps)
        return x

    # ---- per-stage trace -----------------------------------------------------
    def _trace_dir(self) -> str | None:
        """The per-stage dump directory, read from VPIPE_MING_DIT_TRACE as the
        reference's forward reads it (src/ming-dit.cc:1658-1687). When set, a
        single-image eager forward writes each stage's rows as raw float32
        files <dir>/<tag>.f32, the tags of the reference: `embed` (the joint
        rows after the x and caption embedders), `ctx` (the caption rows after
        the context refiner), `blk<L>` (the joint rows after block L of the
        noise refiners, then the main layers). It synchronises the device, so
        a traced run is not a timing run; a CUDA-graph capture never traces."""
        d = os.environ.get(TRACE_ENV)
        if not d or torch.cuda.is_current_stream_capturing():
            return None
        return d

    @staticmethod
    def _trace(d: str, tag: str, rows: torch.Tensor) -> None:
        os.makedirs(d, exist_ok=True)
        rows.float().cpu().numpy().astype(np.float32).tofile(os.path.join(d, tag + ".f32"))

    # ---- the forward -------------------------------------------------------
    @torch.no_grad()
    def forward(self, latents: torch.Tensor, cap: torch.Tensor, query_rows: int, grid_h: int,
                grid_w: int, sigma: float) -> torch.Tensor:
        """latents bf16 [img, patch_dim]; cap bf16 [cap_len, >= dim] (stream A in
        rows [0, query_rows) x columns [0, cap_feat_dim)). Returns bf16
        [img, patch_dim], the model output before the pipeline's negation."""
        return self.forward_batch(latents[None], [cap], query_rows, grid_h, grid_w, sigma)[0]

    @torch.no_grad()
    def forward_batch(self, latents: torch.Tensor, caps, query_rows: int, grid_h: int,
                      grid_w: int, sigmas) -> torch.Tensor:
        """A batch of B images of one layout in ONE pass (CFG: the conditional
        and the negative caption with the same latents):
        latents bf16 [B, img, patch_dim]; caps: B captions of the same shape;
        sigmas: one value or B values. Every projection runs over the B images'
        rows at once; the modulation takes B timestep rows in its one launch;
        norms, gates and attention stay per image, so image i's output is what
        forward() gives for it alone. Returns bf16 [B, img, patch_dim]."""
        B, sig = self._check_batch(latents, caps, sigmas)
        img = grid_h * grid_w
        cos, sin = self._rope_dev(grid_h, grid_w, caps[0].shape[0])
        self._tracing = self._trace_dir() if B == 1 else None
        if self._tracing:
            self._cap_cache.clear()  # the embedded caption rows are traced too
        try:
            cj = [self._context(cp, query_rows, cos[img:], sin[img:]) for cp in caps]
            return self._core(latents.to(self.dev), self._timestep_emb(sig).to(self.dev), cj,
                              cos, sin, img)
        finally:
            self._tracing = None

    def graph(self, batch: int, query_rows: int, grid_h: int, grid_w: int,
              cap_len: int) -> "ForwardGraph":
        """A CUDA-graph runner of forward_batch for one layout (see ForwardGraph)."""
        return ForwardGraph(self, batch, query_rows, grid_h, grid_w, cap_len)

    # ---- pieces of the forward ----------------------------------------------
    def _check_batch(self, latents, caps, sigmas):
        B = latents.shape[0]
        if len(caps) != B or any(c.shape != caps[0].shape for c in caps):
            raise ValueError("one caption per image, all of the same shape")
        sig = [float(sigmas)] * B if np.isscalar(sigmas) else [float(x) for x in sigmas]
        if len(sig) != B or B > 4:
            raise ValueError("one sigma per image; at most 4 images (the modulation's rows)")
        return B, sig

    def _rope_dev(self, grid_h: int, grid_w: int, cap_len: int):
        """f32 cos / sin [img + cap_len, head_dim / 2] of the layout, on the
        device (kept per layout: a denoising loop asks for the same one)."""
        key = (grid_h, grid_w, cap_len)
        hit = self._rope_cache.get(key)
        if hit is None:
            c, s = rope_tables(layout_positions(grid_h, grid_w, cap_len), self.cfg.head_dim,
                               self.cfg.axes, self.cfg.rope_theta)
            if len(self._rope_cache) >= 8:
                self._rope_cache.clear()
            hit = (torch.from_numpy(c).to(self.dev), torch.from_numpy(s).to(self.dev))
            self._rope_cache[key] = hit
        return hit

    def _timestep_emb(self, sig) -> torch.Tensor:
        """f32 [B, time_freq] sinusoids of t = t_scale * (1 - sigma), on the host
        (the reference's timestep embedding, f32 then bf16 on the device)."""
        cfg = self.cfg
        half = cfg.time_freq // 2
        f = np.exp(-math.log(10000.0) * np.arange(half, dtype=np.float64) / half)
        emb = np.stack([np.concatenate([np.cos(cfg.t_scale * (1.0 - sg) * f),
                                        np.sin(cfg.t_scale * (1.0 - sg) * f)]) for sg in sig])
        return torch.from_numpy(emb.astype(np.float32))

    def _core(self, lat: torch.Tensor, emb: torch.Tensor, cj, cos, sin, img: int) -> torch.Tensor:
        """The device part of one step: lat bf16 [B, img, patch_dim], emb f32
        [B, time_freq], cj: the B images' context rows [cap_len, dim]. Launches
        kernels only (no host synchronisation, no host-to-device copy), so a
        CUDA graph can hold it."""
        cfg = self.cfg
        B = lat.shape[0]
        emb = emb.to(torch.bfloat16)
        # the model-level dense layers (library GEMMs) run per image: a library
        # GEMM over B rows may pick another algorithm than over one, and image
        # i's bits must not depend on the batch; the modulation, projections
        # and norms are this library's kernels, row-independent by design
        temb = torch.cat([self._linear(F.silu(self._linear(emb[bi:bi + 1], "t_embedder.mlp.0")),
                                       "t_embedder.mlp.2") for bi in range(B)])
        mods, nw1, nw3 = self.ctx.modulation(self.modset, temb.contiguous())
        x = torch.cat([self._linear(lat[bi], X_EMBEDDER) for bi in range(B)])
        nref = cfg.n_refiner
        tr = getattr(self, "_tracing", None)
        if tr:
            self._trace(tr, "embed", torch.cat([x, self._trace_cap]))
        for i in range(nref):
            x = self._block(nref + i, x, cos[:img], sin[:img], i, mods, nw1, nw3, nb=B)
            if tr:
                self._trace(tr, f"blk{i}", torch.cat([x, cj[0]]))
        j = torch.cat([t for bi in range(B) for t in (x[bi * img:(bi + 1) * img], cj[bi])],
                      dim=0)
        for i in range(cfg.n_layers):
            j = self._block(2 * nref + i, j, cos, sin, nref + i, mods, nw1, nw3, nb=B)
            if tr:
                self._trace(tr, f"blk{nref + i}", j)
        self.ctx.set_image_rows(0)
        L = j.shape[0] // B
        out = []
        for bi in range(B):
            scale = self._linear(F.silu(temb[bi:bi + 1]), FINAL + ".adaLN_modulation.1")
            xi = F.layer_norm(j[bi * L:bi * L + img].float(), (cfg.dim,), eps=1e-6)
            xi = (xi * (1.0 + scale.float())).to(torch.bfloat16)
            out.append(self._linear(xi, FINAL + ".linear"))
        return torch.stack(out)

    def _context(self, cap: torch.Tensor, query_rows: int, cos, sin) -> torch.Tensor:
        """The caption rows after the context refiner, through the caption
        cache (the reference's, src/ming-dit.cc:1543-1577): keyed on the
        caption's exact bytes, its shape and the query-row split; the context
        rows' rotary positions depend on the caption alone, so one entry serves
        every image size; a few entries, least recently used replaced; an
        entry is stored only once its rows are complete. The context refiner's
        projections carry the adapters, so any change of a live strength drops
        every entry (set_lora_scale does, :3031-3038; here the strengths and
        the adapter bindings are compared with those the entries were made
        under)."""
        cfg, dev = self.cfg, self.dev
        strengths = (tuple(self.ctx.strength(i) for i in range(8)), self.proj.binding_version)
        if strengths != self._cap_strengths:
            self._cap_cache.clear()
            self._cap_strengths = strengths
        key = cap.to(dev)
        self._tick += 1
        for e in self._cap_cache:
            if (e["q"] == query_rows and e["key"].shape == key.shape and
                    torch.equal(e["key"].view(torch.int16), key.view(torch.int16))):
                e["tick"] = self._tick
                self.last_cap_cache_hit = True
                return e["out"]
        self.last_cap_cache_hit = False
        ca = self._rms(key[:query_rows, : cfg.cap_feat_dim], self.t["cap_embedder.0.weight"])
        ca = self._linear(ca, "cap_embedder.1")
        cj = torch.cat([ca, key[query_rows:, : cfg.dim]], dim=0)
        tr = getattr(self, "_tracing", None)
        if tr:
            self._trace_cap = cj.clone()
        for i in range(cfg.n_refiner):
            cj = self._block(i, cj, cos, sin, None, None, None, None)
        if tr:
            self._trace(tr, "ctx", cj)
        if self.cap_cache_entries > 0:
            if len(self._cap_cache) >= self.cap_cache_entries:
                self._cap_cache.remove(min(self._cap_cache, key=lambda e: e["tick"]))
            self._cap_cache.append({"key": key.clone(), "q": query_rows, "out": cj,
                                    "tick": self._tick})
        return cj

    def free(self) -> None:
        self.proj.free()
        for w in self.ada:
            w.free()
        self.modset.free()


class ForwardGraph:
    """forward_batch for one layout (B images of grid_h x grid_w patches,
    captions of cap_len rows, query_rows of them query rows) as ONE CUDA-graph
    replay per denoising step.

    The graph holds the per-step work: the timestep embedder, the batched
    modulation, the x embedder, every noise-refiner and main block
    (projections, norms, attention) and the final layer — the work the
    reference's forward launches one by one on every sampler step
    (src/ming-dit.cc:1490-2642). Outside it: the context refiner, whose rows
    depend on the caption alone and come through the caption cache (copied
    into the graph's input rows), and the timestep sinusoid, made on the host
    and copied in as f32.

    A graph keeps the LoRA strengths, row segments and bindings of its capture
    (Context.state_version): a call after any change of them captures again,
    after a warm-up on the new state. Inputs are copied into the graph's
    static buffers; the result is a copy of its static output, so image i's
    bits are those of forward_batch on the same inputs.
    """

    def __init__(self, fwd: DitForward, batch: int, query_rows: int, grid_h: int, grid_w: int,
                 cap_len: int, warmup: int = 2):
        if not 1 <= batch <= 4:
            raise ValueError("1 to 4 images (the modulation's rows)")
        cfg, dev = fwd.cfg, fwd.dev
        self.fwd, self.batch, self.query_rows = fwd, batch, query_rows
        self.img, self.cap_len, self.warmup = grid_h * grid_w, cap_len, warmup
        self.lat = torch.zeros((batch, self.img, cfg.patch_dim), dtype=torch.bfloat16, device=dev)
        self.emb = torch.zeros((batch, cfg.time_freq), dtype=torch.float32, device=dev)
        self.cj = torch.zeros((batch, cap_len, cfg.dim), dtype=torch.bfloat16, device=dev)
        self.cos, self.sin = fwd._rope_dev(grid_h, grid_w, cap_len)
        self.g: torch.cuda.CUDAGraph | None = None
        self.out: torch.Tensor | None = None
        self.version: int | None = None
        self.captures = 0
        self.replays = 0

    def _run(self) -> torch.Tensor:
        return self.fwd._core(self.lat, self.emb, self.cj, self.cos, self.sin, self.img)

    def _capture(self) -> None:
        self.g, self.out = None, None  # the old graph's memory pool goes first
        dev = self.fwd.dev
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            # warm-up: the library's buffers reach their sizes and the LoRA
            # stacks are built here, so the capture holds kernels only
            for _ in range(self.warmup):
                self._run()
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.out = self._run()
        self.g = g
        self.version = self.fwd.ctx.state_version()
        self.captures += 1

    @torch.no_grad()
    def __call__(self, latents: torch.Tensor, caps, sigmas) -> torch.Tensor:
        fwd = self.fwd
        B, sig = fwd._check_batch(latents, caps, sigmas)
        if (B != self.batch or tuple(latents.shape[1:]) != tuple(self.lat.shape[1:])
                or caps[0].shape[0] != self.cap_len):
            raise ValueError(f"this graph takes {self.batch} x {tuple(self.lat.shape[1:])} "
                             f"latents and captions of {self.cap_len} rows")
        for bi, cp in enumerate(caps):
            self.cj[bi].copy_(fwd._context(cp, self.query_rows, self.cos[self.img:],
                                           self.sin[self.img:]))
        self.lat.copy_(latents)
        self.emb.copy_(fwd._timestep_emb(sig))
        if self.g is None or fwd.ctx.state_version() != self.version:
            self._capture()
        self.g.replay()
        self.replays += 1
        return self.out.clone()

    def release(self) -> None:
        self.g, self.out = None, None


__all__ = ["DitForward", "DitModelConfig", "ForwardGraph", "layout_positions", "rope_tables"]
