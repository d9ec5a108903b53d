"""CPU checks of the C-ABI boundary: the library loads and exports what the header declares."""

import ctypes
import re
from pathlib import Path

import pytest

from boltz_lumi_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "boltz_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"BL_API\s+[\w\s\*]+?\b(bl_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "bl_layernorm" in names and "bl_last_error" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_error_path_without_gpu():
    """An invalid request fails on the host with a message, before any CUDA call."""
    lib = _lib.load()
    status = lib.bl_layernorm(None, 7, 4, 128, 0, None, None, ctypes.c_float(1e-5), None, 0, None)
    assert status == 1
    assert b"dtype" in lib.bl_last_error()
    with pytest.raises(RuntimeError, match="bl_gate_pack"):
        _lib.call("bl_gate_pack", None, None, 300, None, 4, 1, None, None, None)
    # The residual form of triangle attention needs linear_o's weight.
    with pytest.raises(RuntimeError, match="w_o is required"):
        _lib.call("bl_triangle_attention_residual", None, None, None, None, 512, 8, 1, None, 8, 64, None, 8, 1,
                  1e9, 4, 32, 8, 8, None, 128, None, None, None, 128, None)
