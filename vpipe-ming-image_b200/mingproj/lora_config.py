"""The caller-side runtime-LoRA configuration keys: which config key names
which adapter slot, what is forwarded, what is load-time and what is live.

Reference (vpipe-ming-image):
  the key table kCfgLoraKeys          src/ming-model-config-stage.h:33-56
  resolved_config: keys forwarded only when SET; a strength of 0 or below is
  a request, not an unset value       src/ming-model-config-stage.cc:177-208
  load: positional slots, strength default 1.0, paths resolved to adapter
  files, unresolvable paths and slots past the DiT's warned and dropped
                                      src/ming-generator.cc:233-278
  apply_lora_keys_ per request: an absent key keeps what is in force, a path
  that differs from the loaded one is warned (once) and IGNORED, only a
  changed strength reaches set_lora_scale
                                      src/ming-generator.cc:310-337

Slot i is configured by `lora` / `lora_scale` for i = 0 and `lora<i+1>` /
`lora<i+1>_scale` otherwise, eight slots in all. Paths are LOAD-time (they
bind into the blocks as the DiT is built); strengths are LIVE (each request
may re-set them; the projection launches read them by value).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Mapping

CFG_LORA_SLOTS = 8
CFG_LORA_KEYS: tuple[tuple[str, str], ...] = tuple(
    ("lora", "lora_scale") if i == 0 else (f"lora{i + 1}", f"lora{i + 1}_scale")
    for i in range(CFG_LORA_SLOTS))


def forwarded_config(config: Mapping | None) -> dict:
    """The LoRA keys a model-config stage forwards (resolved_config): only the
    keys that are SET, a path as a string and a strength as a float, so an
    unset key leaves the family's own value alone (0 and negative strengths
    are forwarded: they are requests)."""
    out: dict = {}
    if not isinstance(config, Mapping):
        return out
    for pk, sk in CFG_LORA_KEYS:
        if pk in config:
            v = config[pk]
            out[pk] = v if isinstance(v, str) else ""
        if sk in config:
            out[sk] = _as_real(config[sk], 1.0)
    return out


def _as_real(v, default: float) -> float:
    if isinstance(v, bool):
        return default
    if isinstance(v, (int, float)):
        return float(v)
    return default


@dataclass
class LoraSpec:
    """One slot's load-time request: the resolved adapter file ('' = empty
    slot) and its strength."""
    path: str = ""
    scale: float = 1.0


@dataclass
class LoraKeyState:
    """What the loaded DiT holds per slot (the generator's _lora_ref /
    _lora_scale) and the messages said so far."""
    slots: int = CFG_LORA_SLOTS
    refs: list[str] = field(default_factory=lambda: [""] * CFG_LORA_SLOTS)
    scales: list[float] = field(default_factory=lambda: [1.0] * CFG_LORA_SLOTS)
    warnings: list[str] = field(default_factory=list)
    infos: list[str] = field(default_factory=list)
    _warned: set = field(default_factory=set)

    def warn_once(self, msg: str) -> None:
        if msg not in self._warned:
            self._warned.add(msg)
            self.warnings.append(msg)


def load_specs(config: Mapping | None, resolve: Callable[[str], str | None],
               slots: int = CFG_LORA_SLOTS) -> tuple[list[LoraSpec] | None, LoraKeyState]:
    """The load-time reading of the keys: per slot the strength (`*_scale`,
    default 1.0) and the adapter file `resolve(ref)` finds for a non-empty
    `lora*` reference (None: not found; warned, the slot stays empty). Slots
    are positional: slot 1 is `lora2` whether or not `lora` is set. Keys for
    slots past `slots` (what this DiT runs at once) are warned and dropped.
    Returns (specs, state); specs is None when no slot resolved to a file."""
    slots = min(slots, CFG_LORA_SLOTS)
    st = LoraKeyState(slots=slots)
    if not isinstance(config, Mapping):
        return None, st
    for i in range(slots, CFG_LORA_SLOTS):
        if CFG_LORA_KEYS[i][0] in config:
            st.warnings.append(f"ming-image: `{CFG_LORA_KEYS[i][0]}` is set, but this host's DiT "
                               f"runs {slots} adapters at once; it is NOT applied")
    specs = [LoraSpec() for _ in range(slots)]
    any_file = False
    for i in range(slots):
        pk, sk = CFG_LORA_KEYS[i]
        if sk in config:
            st.scales[i] = _as_real(config[sk], 1.0)
        specs[i].scale = st.scales[i]
        if pk not in config:
            continue
        ref = config[pk] if isinstance(config[pk], str) else ""
        st.refs[i] = ref
        if not ref:
            continue
        f = resolve(ref)
        if not f:
            st.warnings.append(f"ming-image: `{pk}` '{ref}' did not resolve to an adapter file "
                               "(not found); it is NOT applied")
            continue
        specs[i].path = f
        any_file = True
    return (specs if any_file else None), st


def apply_keys(config: Mapping | None, st: LoraKeyState,
               set_strength: Callable[[int, float], None],
               modules: Callable[[int], int] | None = None) -> int:
    """One request's keys against the loaded DiT (apply_lora_keys_). An absent
    key keeps what is in force; a `lora*` path that differs from the loaded
    one is warned once and IGNORED (paths are load-time); a `*_scale` that
    differs from the strength in force is applied through
    `set_strength(slot, s)`. Returns the number of strengths changed."""
    if not isinstance(config, Mapping):
        return 0
    changed = 0
    for i in range(st.slots):
        pk, sk = CFG_LORA_KEYS[i]
        if pk in config:
            v = config[pk] if isinstance(config[pk], str) else ""
            if v != st.refs[i]:
                st.warn_once(f"the DiT is already loaded, so the model_config beat's `{pk}` "
                             f"'{v}' is IGNORED -- it is a load-time argument (loaded: "
                             f"'{st.refs[i]}'). `{sk}` still applies")
        if sk not in config:
            continue
        s = _as_real(config[sk], 1.0)
        if s == st.scales[i]:
            continue
        st.scales[i] = s
        set_strength(i, s)
        changed += 1
        n = modules(i) if modules is not None else 0
        if n > 0:
            st.infos.append(f"ming-image: `{sk}` -> {s:.3f} ({n} modules)")
    return changed


def bind_from_config(pset, config: Mapping | None, resolve: Callable[[str], str | None],
                     dim: int, ffn: int) -> LoraKeyState:
    """Load-time binding of a DitProjectionSet from the config keys: every
    resolved slot's adapter is parsed and bound with the whole-slot refusal
    rules of bind_adapter, and every slot's strength is set on the context
    (1.0 unless its `*_scale` says otherwise)."""
    from .lora import bind_adapter

    specs, st = load_specs(config, resolve)
    for i in range(st.slots):
        pset.ctx.set_strength(i, st.scales[i])
    if specs is None:
        return st
    for i, spec in enumerate(specs):
        if not spec.path:
            continue
        sb = bind_adapter(spec.path, dim, ffn, pset.dims.n_refiner, pset.dims.n_layers)
        n = pset.bind_slot(i, sb)
        if n == 0:
            st.warnings.append(sb.message)
        else:
            st.infos.append(f"runtime LoRA modules bound: {CFG_LORA_KEYS[i][0]} {n}")
    return st


__all__ = ["CFG_LORA_SLOTS", "CFG_LORA_KEYS", "LoraSpec", "LoraKeyState", "forwarded_config",
           "load_specs", "apply_keys", "bind_from_config"]
