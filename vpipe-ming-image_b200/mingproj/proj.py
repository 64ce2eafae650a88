"""Projection API over the mingproj C-ABI — the host-side mirror of the
reference's per-projection surface.

  reference (vpipe-ming-image)                      here
  -----------------------------------------------   --------------------------------
  QWeight + load_qw_ (src/ming-dit.cc:446-452,      Context.upload() -> Weight
    :802-831)
  Adapter::bind per projection (:2954-2968)         Weight.bind(slot, A, B)
  set_lora_scale / lora_scale (:3024-3039)          Context.set_strength / strength
  lin(x, xe, w, y, ye, M, N, K, lora::Stack)        Context.linear(w, x, out=y)
    (:1763-1771)
  q/k/v (w1/w3) lin calls on one `nrm`              Context.linear_shared(ws, x)
    (:2078-2080, :2155-2156)
  fill_mod (:2266-2273), all blocks at once         Context.modulation(set, temb)
  DitEngagement (src/ming-dit.h:55-103)             Context.engagement()

Device memory, streams and tensors are torch's; every computation is a call
into libmingproj.so. There is no CPU path here.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import (MP_GROUP, MP_MAX_SEGMENTS, MP_MAX_SLOTS, MP_OK, MP_QUANT_AFFINE,
                   MP_QUANT_SYMMETRIC, MPError)


def _ptr(t) -> C.c_void_p | None:
    if t is None:
        return None
    if isinstance(t, torch.Tensor):
        return C.c_void_p(t.data_ptr())
    if isinstance(t, np.ndarray):
        return t.ctypes.data_as(C.c_void_p)
    raise TypeError(f"unsupported buffer type {type(t)}")


def _contig(t):
    if t is None:
        return None
    if isinstance(t, torch.Tensor):
        return t.contiguous()
    return np.ascontiguousarray(t)


def _alloc_out(m: int, n: int, device) -> torch.Tensor:
    """bf16 [m, n] output view whose row pitch is rounded up to 8 elements (the
    kernels store rows with TMA, which wants 16-byte row strides)."""
    ld = (n + 7) // 8 * 8
    return torch.empty((m, ld), dtype=torch.bfloat16, device=device)[:, :n]


def _stream_handle(stream) -> C.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


@dataclass
class WeightInfo:
    n: int
    k: int
    bits: int
    mode: int


class Weight:
    """One uploaded projection weight (a QWeight) and its LoRA slots."""

    def __init__(self, ctx: "Context", handle: C.c_void_p, info: WeightInfo):
        self.ctx = ctx
        self.handle = handle
        self.info = info
        self.ranks = [0] * MP_MAX_SLOTS

    @property
    def n(self) -> int:
        return self.info.n

    @property
    def k(self) -> int:
        return self.info.k

    @property
    def bits(self) -> int:
        return self.info.bits

    def bind(self, slot: int, a, b) -> None:
        """a: bf16 [rank, k] (alpha folded in), b: bf16 [n, rank]; torch bf16
        tensors or uint16 numpy arrays, host or device."""
        a = _as_bf16_bits(a)
        b = _as_bf16_bits(b)
        rank = a.shape[0]
        if tuple(a.shape) != (rank, self.k) or tuple(b.shape) != (self.n, rank):
            raise MPError(_lib.MP_EINVAL,
                          f"LoRA factors {tuple(a.shape)} / {tuple(b.shape)} do not fit "
                          f"[{self.n}, {self.k}]")
        self.ctx._check(self.ctx.lib.mp_lora_bind(self.ctx.h, self.handle, slot, _ptr(a),
                                                   _ptr(b), rank))
        self.ranks[slot] = rank

    def unbind(self, slot: int) -> None:
        self.ctx._check(self.ctx.lib.mp_lora_unbind(self.ctx.h, self.handle, slot))
        self.ranks[slot] = 0

    def read_codes(self) -> np.ndarray:
        """The stored codes (or dense weight) bytes, read back from the device."""
        nbytes = self.n * self.k * (2 if self.bits == 0 else self.bits) // (1 if self.bits == 0 else 8)
        out = np.empty(nbytes, dtype=np.uint8)
        self.ctx._check(self.ctx.lib.mp_weight_read_codes(self.ctx.h, self.handle, _ptr(out),
                                                           nbytes))
        return out

    def free(self) -> None:
        if self.handle:
            self.ctx.lib.mp_weight_free(self.ctx.h, self.handle)
            self.handle = None


def _as_bf16_bits(t):
    """torch bf16 tensor -> same tensor (contiguous); numpy uint16 -> contiguous."""
    if isinstance(t, torch.Tensor):
        if t.dtype not in (torch.bfloat16, torch.int16, torch.uint16):
            raise TypeError(f"expected bf16 tensor, got {t.dtype}")
        return t.contiguous()
    a = np.ascontiguousarray(t)
    if a.dtype != np.uint16:
        raise TypeError(f"expected uint16 (bf16 bits), got {a.dtype}")
    return a


class ModSet:
    def __init__(self, ctx: "Context", handle: C.c_void_p, n_blocks: int, n: int, k: int):
        self.ctx, self.handle, self.n_blocks, self.n, self.k = ctx, handle, n_blocks, n, k

    def free(self):
        if self.handle:
            self.ctx.lib.mp_modulation_free(self.ctx.h, self.handle)
            self.handle = None


class Context:
    """One mingproj context bound to a CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = _lib.load()
        self.device = device
        h = C.c_void_p()
        rc = self.lib.mp_create(device, C.byref(h))
        if rc != MP_OK:
            raise MPError(rc, f"mp_create({device}) failed: {_lib.status_name(rc)}")
        self.h = h

    # -- plumbing --------------------------------------------------------
    def _check(self, rc: int) -> None:
        if rc != MP_OK:
            msg = self.lib.mp_last_error(self.h).decode()
            raise MPError(rc, f"{_lib.status_name(rc)}: {msg}")

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.mp_destroy(self.h)
            self.h = None

    def sync_check(self, stream=None) -> None:
        """Synchronizes and raises MPError(MP_ETIMEOUT) if a kernel gave up a
        bounded device-side wait."""
        self._check(self.lib.mp_sync_check(self.h, _stream_handle(stream)))

    def selftest_wait(self, limit_ns: int, stream=None) -> None:
        """Launches the failure-detection self-test: one bounded wait that can
        never complete. The next sync_check raises MPError(MP_ETIMEOUT)."""
        self._check(self.lib.mp_selftest_wait(self.h, limit_ns, _stream_handle(stream)))

    def set_wait_limit(self, ns: int) -> None:
        self._check(self.lib.mp_set_wait_limit(self.h, int(ns)))

    # -- weights -----------------------------------------------------------
    def upload(self, n: int, k: int, bits: int, data, scales=None, biases=None,
               mode: int = MP_QUANT_AFFINE) -> Weight:
        """data: U32 codes [n, k*bits/32] (numpy uint32 or torch int32) for
        bits 4/8, or bf16 [n, k] for bits 0. Host or device."""
        desc = _lib.WeightDesc(n, k, bits, MP_GROUP if bits else 0, mode)
        data = _contig(data)
        scales = _contig(scales)
        biases = _contig(biases)
        h = C.c_void_p()
        self._check(self.lib.mp_weight_upload(self.h, C.byref(desc), _ptr(data), _ptr(scales),
                                              _ptr(biases), C.byref(h)))
        return Weight(self, h, WeightInfo(n, k, bits, mode))

    # -- strengths ---------------------------------------------------------
    def set_strength(self, slot: int, s: float) -> None:
        self._check(self.lib.mp_set_strength(self.h, slot, float(s)))

    def strength(self, slot: int) -> float:
        v = C.c_float()
        self._check(self.lib.mp_get_strength(self.h, slot, C.byref(v)))
        return float(v.value)

    def state_version(self) -> int:
        """Advanced by every change of a strength, the row segments or a LoRA
        binding: a CUDA graph captured at one version is stale at another."""
        v = C.c_uint64()
        self._check(self.lib.mp_state_version(self.h, C.byref(v)))
        return int(v.value)

    def set_strengths_rows(self, strengths, row_starts) -> None:
        """strengths: [batch, 8] floats; row_starts: [batch + 1] token rows.
        Pass batch 0 (empty) to return to per-slot strengths."""
        s = np.ascontiguousarray(strengths, dtype=np.float32).reshape(-1, MP_MAX_SLOTS)
        r = np.ascontiguousarray(row_starts, dtype=np.int32)
        batch = s.shape[0]
        if batch > MP_MAX_SEGMENTS:
            raise MPError(_lib.MP_EINVAL, f"at most {MP_MAX_SEGMENTS} segments")
        self._check(self.lib.mp_set_strengths_rows(
            self.h, s.ctypes.data_as(C.POINTER(C.c_float)),
            r.ctypes.data_as(C.POINTER(C.c_int32)), batch))

    def set_image_rows(self, rows: int) -> None:
        """Rows of one image in the launches that follow (0: each launch is
        one image): a batch of equal-length images then has each image's bits
        of its own launch."""
        self._check(self.lib.mp_set_image_rows(self.h, int(rows)))

    def clear_strengths_rows(self) -> None:
        self._check(self.lib.mp_set_strengths_rows(self.h, None, None, 0))

    # -- projections -------------------------------------------------------
    def linear(self, w: Weight, x: torch.Tensor, out: torch.Tensor | None = None,
               stream=None) -> torch.Tensor:
        """y = x · deq(W)^T + sum_live s_i (x A_i^T) B_i^T; x bf16 [m, k] on the
        context's device (row stride a multiple of 8)."""
        m = x.shape[0]
        if out is None:
            out = _alloc_out(m, w.n, x.device)
        self._check(self.lib.mp_linear(self.h, w.handle, _ptr(x), x.stride(0), _ptr(out),
                                       out.stride(0), m, _stream_handle(stream)))
        return out

    def linear_shared(self, ws: list[Weight], x: torch.Tensor, outs=None, stream=None):
        m = x.shape[0]
        if outs is None:
            outs = [_alloc_out(m, w.n, x.device) for w in ws]
        n = len(ws)
        W = (C.c_void_p * n)(*[w.handle.value for w in ws])
        Y = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
        L = (C.c_int64 * n)(*[o.stride(0) for o in outs])
        self._check(self.lib.mp_linear_shared(self.h, W, Y, L, n, _ptr(x), x.stride(0), m,
                                              _stream_handle(stream)))
        return outs

    def linear_swiglu(self, w1: Weight, w3: Weight, x: torch.Tensor,
                      out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """h = bf16(silu(g) * u) with g = bf16(x W1^T + LoRA), u = bf16(x W3^T + LoRA):
        the FFN gate/up pair and its SwiGLU in one launch."""
        m = x.shape[0]
        if out is None:
            out = _alloc_out(m, w1.n, x.device)
        self._check(self.lib.mp_linear_swiglu(self.h, w1.handle, w3.handle, _ptr(x), x.stride(0),
                                              _ptr(out), out.stride(0), m,
                                              _stream_handle(stream)))
        return out

    def linear_heads(self, ws: list[Weight], x: torch.Tensor, norm_w=None, eps: float = 1e-5,
                     rope_cos: torch.Tensor | None = None, rope_sin: torch.Tensor | None = None,
                     outs=None, stream=None) -> list[torch.Tensor]:
        """q/k/v of one input in one launch, each returned head-major
        [n / 128, m, 128] bf16. norm_w[i] (bf16 [128] on the device, or None)
        applies member i's per-head RMSNorm and then the interleaved-pair
        rotary embedding with rope_cos / rope_sin (f32 [m, 64] on the device)."""
        m = x.shape[0]
        n = len(ws)
        if outs is None:
            outs = [torch.empty((w.n // 128, m, 128), dtype=torch.bfloat16, device=x.device)
                    for w in ws]
        W = (C.c_void_p * n)(*[w.handle.value for w in ws])
        Y = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
        keep = []
        NW = None
        if norm_w is not None:
            vals = []
            for g in norm_w:
                if g is None:
                    vals.append(None)
                else:
                    g = g.to(torch.bfloat16).contiguous()
                    keep.append(g)
                    vals.append(g.data_ptr())
            NW = (C.c_void_p * n)(*vals)
        tabs = []
        for tab in (rope_cos, rope_sin):
            if tab is None:
                tabs.append(None)
            else:
                tab = tab.to(torch.float32).contiguous()
                if tab.shape != (m, 64):
                    raise ValueError(f"rotary table shape {tuple(tab.shape)} != ({m}, 64)")
                keep.append(tab)
                tabs.append(_ptr(tab))
        self._check(self.lib.mp_linear_heads(self.h, W, Y, n, _ptr(x), x.stride(0), m, NW,
                                             float(eps), tabs[0], tabs[1],
                                             _stream_handle(stream)))
        if stream is not None:
            # converted gains and tables: their memory is not reused before the
            # launch on `stream` has read them (on the current stream the
            # allocator's stream order already guarantees it)
            for t in keep:
                t.record_stream(stream)
        return outs

    def attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  scale: float | None = None, out: torch.Tensor | None = None,
                  stream=None) -> torch.Tensor:
        """Non-causal attention over head-major q, k, v (bf16 [nh, s, 128], as
        linear_heads returns them, or one image's rows of a batch's head-major
        tensor: a [:, r0:r1, :] view); returns token-major bf16 [s, nh * 128]
        (into `out` when given, e.g. that image's rows of the batch)."""
        nh, s, hd = q.shape
        if hd != 128 or k.shape != q.shape or v.shape != q.shape:
            raise ValueError(f"q, k, v must be [nh, s, 128] alike (got {tuple(q.shape)}, "
                             f"{tuple(k.shape)}, {tuple(v.shape)})")
        if not all(t.stride(1) == 128 and t.stride(2) == 1 and t.stride(0) == q.stride(0)
                   for t in (q, k, v)):
            q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        if out is None:
            out = torch.empty((s, nh * 128), dtype=torch.bfloat16, device=q.device)
        sc = float(scale) if scale is not None else 1.0 / math.sqrt(hd)
        self._check(self.lib.mp_attention(self.h, _ptr(q), _ptr(k), _ptr(v), s, nh, q.stride(0),
                                          sc, _ptr(out), out.stride(0), _stream_handle(stream)))
        return out

    def rms_residual(self, x: torch.Tensor, o: torch.Tensor | None, o_gain=None, gate=None,
                     nrm_gain=None, eps: float = 1e-5, nrm: torch.Tensor | None = None,
                     stream=None) -> torch.Tensor | None:
        """The sandwich-norm residual step, one kernel: with `o`, x (bf16 [m, h],
        updated IN PLACE) += [tanh(gate) *] rms(o, o_gain); with `nrm_gain`,
        returns rms(x, nrm_gain) (into `nrm` when given). Gains and gate: bf16
        [h] on the device."""
        m, h = x.shape
        vecs = []
        for v in (o_gain, gate, nrm_gain):
            if v is None:
                vecs.append(None)
            else:
                v = v.to(torch.bfloat16).contiguous()
                vecs.append(v)
        if nrm_gain is not None and nrm is None:
            nrm = _alloc_out(m, h, x.device)
        self._check(self.lib.mp_rms_residual(
            self.h, _ptr(x), x.stride(0), _ptr(o), o.stride(0) if o is not None else 0,
            _ptr(vecs[0]), _ptr(vecs[1]), _ptr(nrm) if nrm_gain is not None else None,
            nrm.stride(0) if nrm_gain is not None else 0, _ptr(vecs[2]), h, m, float(eps),
            _stream_handle(stream)))
        if stream is not None:
            for v in vecs:
                if v is not None:
                    v.record_stream(stream)
        return nrm if nrm_gain is not None else None

    def linear_lora_static(self, w: Weight, x: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                           strength: float, out: torch.Tensor | None = None,
                           stream=None) -> torch.Tensor:
        """One adapter's fused projection without any device allocation in the
        library: the rank-space intermediate lives in the library's fixed
        device array (see mp_linear_lora_static). a: bf16 [rank, k], b: bf16
        [n, rank], both on the device; the slots bound to `w` are not applied."""
        m = x.shape[0]
        rank = a.shape[0] if a.dim() == 2 else -1
        for name, t, shape in (("a", a, (rank, w.k)), ("b", b, (w.n, rank))):
            if t.dim() != 2 or tuple(t.shape) != shape:
                raise ValueError(f"{name} must be [{shape[0]}, {shape[1]}], got {tuple(t.shape)}")
            if t.dtype != torch.bfloat16:
                raise ValueError(f"{name} must be bfloat16, got {t.dtype}")
            if t.device != x.device:
                raise ValueError(f"{name} is on {t.device}, x on {x.device}")
        if out is None:
            out = _alloc_out(m, w.n, x.device)
        a = a.contiguous()
        b = b.contiguous()
        self._check(self.lib.mp_linear_lora_static(
            self.h, w.handle, _ptr(x), x.stride(0), _ptr(a), _ptr(b), a.shape[0],
            float(strength), _ptr(out), out.stride(0), m, _stream_handle(stream)))
        return out

    # -- modulation ----------------------------------------------------------
    def modulation_set(self, ada: list[Weight], biases, an1=None, fn1=None) -> ModSet:
        nb = len(ada)
        biases = [_as_bf16_bits(b) for b in biases]
        an1 = [_as_bf16_bits(a) for a in an1] if an1 is not None else None
        fn1 = [_as_bf16_bits(a) for a in fn1] if fn1 is not None else None
        W = (C.c_void_p * nb)(*[w.handle.value for w in ada])
        Bp = (C.c_void_p * nb)(*[_ptr(b).value for b in biases])
        A1 = (C.c_void_p * nb)(*[_ptr(a).value for a in an1]) if an1 is not None else None
        F1 = (C.c_void_p * nb)(*[_ptr(a).value for a in fn1]) if fn1 is not None else None
        h = C.c_void_p()
        self._check(self.lib.mp_modulation_create(self.h, nb, W, Bp, A1, F1, C.byref(h)))
        return ModSet(self, h, nb, ada[0].n, ada[0].k)

    def modulation(self, mset: ModSet, temb: torch.Tensor, fold: bool = True, stream=None):
        """Returns (mods [n_blocks, m, 4H], nw1 [n_blocks, m, H] | None,
        nw3 [n_blocks, m, H] | None), all bf16."""
        m = temb.shape[0]
        H = mset.n // 4
        dev = temb.device
        mods = torch.empty((mset.n_blocks, m, mset.n), dtype=torch.bfloat16, device=dev)
        nw1 = torch.empty((mset.n_blocks, m, H), dtype=torch.bfloat16, device=dev) if fold else None
        nw3 = torch.empty((mset.n_blocks, m, H), dtype=torch.bfloat16, device=dev) if fold else None
        self._check(self.lib.mp_modulation_all(self.h, mset.handle, _ptr(temb.contiguous()), m,
                                               _ptr(mods), _ptr(nw1), _ptr(nw3),
                                               _stream_handle(stream)))
        return mods, nw1, nw3

    # -- engagement --------------------------------------------------------
    def engagement(self) -> dict:
        e = _lib.Engagement()
        self._check(self.lib.mp_engagement_get(self.h, C.byref(e)))
        return e.as_dict()

    def reset_engagement(self) -> None:
        self._check(self.lib.mp_engagement_reset(self.h))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["Context", "Weight", "ModSet", "MPError", "MP_QUANT_AFFINE", "MP_QUANT_SYMMETRIC"]
