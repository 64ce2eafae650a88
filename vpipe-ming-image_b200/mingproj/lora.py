"""Runtime-LoRA adapters: reading a .safetensors adapter, mapping its keys onto
this model's projection modules, and the binding rules of the reference's
`bind_loras_` (src/ming-dit.cc:2893-3005).

Module names are the model's own (src/ming-dit.cc:2893-2916), per block
  attention.to_q / to_k / to_v / to_out.0, feed_forward.w1 / w3 / w2
over context_refiner.<i>, noise_refiner.<i> and layers.<i>. Accepted spellings:
  * diffusers / peft: `<module>.lora_A.weight` [r, in], `<module>.lora_B.weight`
    [out, r], optionally under `transformer.` / `diffusion_model.` /
    `base_model.model.` prefixes and with peft's `.lora_A.<adapter>.` infix;
  * kohya: `lora_unet_<module with . -> _>.lora_down.weight` [r, in] and
    `.lora_up.weight` [out, r];
  * an alpha stated per module (`<prefix>.alpha`) or once in the file's
    metadata (`lora_alpha`, `alpha`, `ss_network_alpha`) is folded into A as
    alpha / rank; without one the factors are used as they are.
Binding rules (reference behaviour):
  * slots are POSITIONAL: an empty path leaves its slot empty (:2925-2928);
  * a module present by name at the wrong shape refuses the WHOLE slot
    (:2971-2983) — `skipped` > 0 and nothing bound;
  * an adapter that binds no module is reported, and the base model runs
    (:2995-3002);
  * adaLN and the model-level layers are never adapted (:467-469).
The exact rename table of the host's lora-names.h is not in the reference
tree; this list is a reading of the conventions above.
"""
from __future__ import annotations

import json
import re
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .pack import PROJ_NAMES, bf16_bits_to_f32, f32_to_bf16_bits

STACKS = ("context_refiner", "noise_refiner", "layers")
_PREFIXES = ("base_model.model.", "transformer.", "diffusion_model.", "model.")
_META_ALPHA_KEYS = ("lora_alpha", "alpha", "ss_network_alpha")

_DTYPES = {"BF16": (np.uint16, 2), "F16": (np.float16, 2), "F32": (np.float32, 4),
           "F64": (np.float64, 8), "U32": (np.uint32, 4), "I32": (np.int32, 4),
           "U8": (np.uint8, 1), "I64": (np.int64, 8)}


def read_safetensors(path) -> tuple[dict[str, np.ndarray], dict[str, str], dict[str, str]]:
    """Minimal safetensors reader: returns (tensors, dtypes, metadata). BF16
    tensors come back as uint16 bit patterns."""
    raw = Path(path).read_bytes()
    (hlen,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + hlen].decode("utf-8"))
    meta = header.pop("__metadata__", {}) or {}
    data = memoryview(raw)[8 + hlen:]
    out, dtypes = {}, {}
    for name, info in header.items():
        dt = info["dtype"]
        if dt not in _DTYPES:
            continue
        np_dt, _ = _DTYPES[dt]
        a, b = info["data_offsets"]
        arr = np.frombuffer(data[a:b], dtype=np_dt).reshape(info["shape"])
        out[name] = arr
        dtypes[name] = dt
    return out, dtypes, meta


def write_safetensors(path, tensors: dict[str, np.ndarray], dtypes: dict[str, str] | None = None,
                      metadata: dict[str, str] | None = None) -> None:
    """Writes tensors (uint16 arrays are written as BF16 unless `dtypes` says
    otherwise)."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        dt = (dtypes or {}).get(name)
        if dt is None:
            dt = {np.dtype(np.uint16): "BF16", np.dtype(np.float16): "F16",
                  np.dtype(np.float32): "F32", np.dtype(np.float64): "F64",
                  np.dtype(np.uint32): "U32", np.dtype(np.int32): "I32",
                  np.dtype(np.uint8): "U8", np.dtype(np.int64): "I64"}[arr.dtype]
        b = arr.tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def module_names(n_refiner: int = 2, n_layers: int = 30) -> list[str]:
    """Every adaptable module, in binding order: 7 x (2 refiner stacks + layers)."""
    names = []
    for stack, count in (("context_refiner", n_refiner), ("noise_refiner", n_refiner),
                         ("layers", n_layers)):
        for i in range(count):
            names += [f"{stack}.{i}.{p}" for p in PROJ_NAMES]
    return names


def module_capacity(n_refiner: int = 2, n_layers: int = 30) -> int:
    """MingDit::lora_module_capacity (src/ming-dit.cc:3123-3128)."""
    return 7 * (2 * n_refiner + n_layers)


def module_shape(name: str, dim: int, ffn: int) -> tuple[int, int]:
    """[out, in] of a projection module."""
    if name.endswith(("feed_forward.w1", "feed_forward.w3")):
        return ffn, dim
    if name.endswith("feed_forward.w2"):
        return dim, ffn
    return dim, dim


_RE_AB = re.compile(r"^(?P<mod>.+)\.lora_(?P<ab>A|B)(?:\.[^.]+)?\.weight$")
_RE_DOWNUP = re.compile(r"^(?P<mod>.+)\.lora_(?P<du>down|up)\.weight$")
_RE_ALPHA = re.compile(r"^(?P<mod>.+)\.alpha$")


def _strip_prefix(name: str) -> str:
    changed = True
    while changed:
        changed = False
        for p in _PREFIXES:
            if name.startswith(p):
                name = name[len(p):]
                changed = True
    return name


@dataclass
class Factors:
    a: np.ndarray  # bf16 bits [r, in], alpha folded in
    b: np.ndarray  # bf16 bits [out, r]

    @property
    def rank(self) -> int:
        return self.a.shape[0]


@dataclass
class Adapter:
    """One adapter file, parsed into module -> raw (A, B, alpha)."""
    path: str
    modules: dict[str, dict] = field(default_factory=dict)
    meta_alpha: float | None = None

    @classmethod
    def open(cls, path, known_modules: list[str] | None = None) -> "Adapter":
        tensors, dtypes, meta = read_safetensors(path)
        ad = cls(str(path))
        for key in _META_ALPHA_KEYS:
            if key in meta:
                try:
                    ad.meta_alpha = float(meta[key])
                    break
                except ValueError:
                    pass
        flat = {m.replace(".", "_"): m for m in (known_modules or module_names())}
        for name, arr in tensors.items():
            canon = _strip_prefix(name)
            mod = part = None
            m = _RE_AB.match(canon)
            if m:
                mod, part = m["mod"], m["ab"]
            else:
                m = _RE_DOWNUP.match(canon)
                if m:
                    mod, part = m["mod"], ("A" if m["du"] == "down" else "B")
                else:
                    m = _RE_ALPHA.match(canon)
                    if m:
                        mod, part = m["mod"], "alpha"
            if mod is None:
                continue
            if mod.startswith("lora_unet_"):
                mod = flat.get(mod[len("lora_unet_"):], mod)
            entry = ad.modules.setdefault(mod, {})
            if part == "alpha":
                entry["alpha"] = float(np.asarray(arr, dtype=np.float64 if dtypes[name] != "BF16"
                                                  else np.uint16).ravel()[0]) \
                    if dtypes[name] != "BF16" else float(bf16_bits_to_f32(arr).ravel()[0])
            else:
                entry[part] = (arr, dtypes[name])
        return ad

    def factors(self, module: str) -> Factors | None:
        e = self.modules.get(module)
        if not e or "A" not in e or "B" not in e:
            return None
        a = _to_f32(*e["A"])
        b = _to_f32(*e["B"])
        r = a.shape[0]
        alpha = e.get("alpha", self.meta_alpha)
        if alpha is not None and r > 0:
            a = a * np.float32(alpha / r)
        return Factors(f32_to_bf16_bits(a), f32_to_bf16_bits(b))


def _to_f32(arr: np.ndarray, dt: str) -> np.ndarray:
    if dt == "BF16":
        return bf16_bits_to_f32(arr)
    return np.asarray(arr, dtype=np.float32)


@dataclass
class SlotBinding:
    """What one slot bound: module -> Factors, and the counts the reference
    reports (lora_modules / lora_skipped, src/ming-dit.h:157-170)."""
    path: str
    bound: dict[str, Factors] = field(default_factory=dict)
    skipped: int = 0
    fit: int = 0
    message: str = ""

    @property
    def modules(self) -> int:
        return len(self.bound)


def bind_adapter(path, dim: int, ffn: int, n_refiner: int = 2, n_layers: int = 30) -> SlotBinding:
    """Binds one adapter against the model's module list; refuses the whole slot
    when any module matches by name at the wrong shape."""
    names = module_names(n_refiner, n_layers)
    ad = Adapter.open(path, names)
    sb = SlotBinding(str(path))
    fits = {}
    for name in names:
        f = ad.factors(name)
        if f is None:
            continue
        out, inp = module_shape(name, dim, ffn)
        if f.a.shape[1] != inp or f.b.shape[0] != out or f.b.shape[1] != f.a.shape[0]:
            sb.skipped += 1
            continue
        fits[name] = f
    sb.fit = len(fits)
    if sb.skipped > 0:
        sb.message = (f"lora '{path}' is NOT applied: {sb.skipped} module(s) matched by name at "
                      f"the wrong shape ({sb.fit} fit) -- it was trained against a different "
                      "model; the base model runs")
        return sb
    sb.bound = fits
    if not fits:
        sb.message = (f"lora '{path}' bound NO modules -- it is for a different model, or its "
                      "names are in a convention this family does not map; the base model runs")
    else:
        sb.message = f"runtime LoRA modules bound: {len(fits)}"
    return sb
