"""The C-ABI library loads and exports every symbol include/fade_b200.h declares (CPU)."""

from __future__ import annotations

import ctypes
import re

import pytest

from fade_b200 import _lib

from conftest import ROOT


def _declared_symbols() -> set[str]:
    txt = (ROOT / "include" / "fade_b200.h").read_text()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return set(re.findall(r"\b(fade_[a-z0-9_]+)\s*\(", txt))


def test_library_builds_and_exports_all_symbols():
    from fade_b200.csrc import build as b

    path = b.build()
    lib = ctypes.CDLL(str(path))
    declared = _declared_symbols()
    assert len(declared) >= 15
    missing = [s for s in sorted(declared) if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_header():
    from fade_b200 import _lib

    assert _declared_symbols() == set(_lib.symbols())


def test_status_strings_and_host_validation():
    """Entry points validate arguments on the host before touching a device."""
    from fade_b200 import _lib

    lib = _lib.load()
    assert lib.fade_status_string(0) == b"ok"
    assert b"group" in lib.fade_status_string(_lib.FADE_ERR_GROUP)
    v = _lib.View4(1, 1, 4, 3, 12, 12, 3, 1)  # odd D
    assert lib.fade_quant_int4_k(None, 0, v, None, None, None) == _lib.FADE_ERR_ODD_DIM
    v = _lib.View4(1, 1, 10, 8, 80, 80, 8, 1)
    assert lib.fade_quant_int2_grouped(None, 0, v, 4, None, None, None, None) == _lib.FADE_ERR_GROUP
    assert lib.fade_pack_codes(None, 2, 6, 2, None, None) == _lib.FADE_ERR_ODD_DIM
    d = _lib.DecodeDesc()
    d.dtype, d.B, d.Hq, d.Hkv, d.D, d.n_q = 0, 1, 4, 1, 96, 1
    assert lib.fade_decode_attn_workspace_size(ctypes.byref(d)) == 0  # D=96 not compiled
    assert lib.fade_version() >= 100


def test_middle_kernel_switch():
    """The middle-kernel choice is a host-side switch (no GPU needed)."""
    from fade_b200.attention import get_middle_kernel, set_middle_kernel

    assert get_middle_kernel() == "mma_sync"
    with pytest.raises(ValueError):
        set_middle_kernel("wgmma")
    assert _lib.load().fade_set_middle_kernel(7) == _lib.FADE_ERR_INVALID_ARG
    try:
        set_middle_kernel("tcgen05")
        assert get_middle_kernel() == "tcgen05"
    finally:
        set_middle_kernel("mma_sync")
    assert get_middle_kernel() == "mma_sync"
