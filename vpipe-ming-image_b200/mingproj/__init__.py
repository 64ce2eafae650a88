"""mingproj — B200 (sm_100a) kernels for the Ming-Image DiT's block-linear hot
path (the seven LoRA-able projections of every block and the adaLN
modulation), behind the C-ABI in include/mingproj.h.

Submodules:
  _lib    ctypes bindings of libmingproj.so
  proj    Context / Weight / ModSet: the per-projection API
  pack    the w8/w4 g64 pack format and seeded synthetic weights
  lora    adapter key parsing and slot binding (diffusers / peft / kohya)
  dit     the DiT projection set of all blocks, and the torch DiT driver
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
