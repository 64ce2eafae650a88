"""The C-ABI library loads without a GPU and exports every entry point that
include/mingproj.h declares; compute entry points refuse cleanly when no
device is usable (no CPU fallback)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from conftest import ROOT, gpu_available

HEADER = ROOT / "include" / "mingproj.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mp_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for need in ("mp_create", "mp_weight_upload", "mp_lora_bind", "mp_set_strength",
                 "mp_linear", "mp_linear_shared", "mp_modulation_all", "mp_engagement_get",
                 "mp_last_error"):
        assert need in syms


def test_library_exports_every_declared_symbol():
    from mingproj import _lib
    lib = _lib.load()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"not exported: {missing}"
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_status_strings():
    from mingproj import _lib
    lib = _lib.load()
    assert lib.mp_status_string(0) == b"MP_OK"
    assert lib.mp_status_string(4) == b"MP_ETIMEOUT"


@pytest.mark.skipif(gpu_available(), reason="checks the no-device refusal")
def test_no_device_refuses():
    from mingproj import _lib
    lib = _lib.load()
    h = C.c_void_p()
    rc = lib.mp_create(0, C.byref(h))
    assert rc == _lib.MP_ECUDA
    assert not h.value
    # Null-context calls are argument errors, never crashes.
    assert lib.mp_linear(None, None, None, 0, None, 0, 1, None) == _lib.MP_EINVAL
    assert lib.mp_set_strength(None, 0, 1.0) == _lib.MP_EINVAL


def test_product_path_raises_without_library(tmp_path, monkeypatch):
    from mingproj import _lib
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "absent.so")
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load()
