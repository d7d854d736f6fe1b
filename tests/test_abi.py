"""The C-ABI library loads and exports every symbol include/cachebridge_b200.h declares.

These tests run without a GPU: they only load the library and call entry
points whose argument validation fails before any CUDA call.
"""

from __future__ import annotations

import ctypes
import re

import pytest

from cachebridge_b200 import _native as nat
from conftest import ROOT

HEADER = ROOT / "include" / "cachebridge_b200.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^CB_API\s+(?:const\s+)?\w+\s*\**\s*(cb_\w+)\s*\(", text, re.M))


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == set(nat.EXPORTED_SYMBOLS)


def test_library_loads_and_exports_every_declared_symbol():
    lib = nat.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_version_and_status_strings():
    lib = nat.load()
    assert lib.cb_version() >= 100
    assert lib.cb_status_string(nat.CB_OK) == b"ok"
    assert b"invalid" in lib.cb_status_string(nat.CB_ERR_INVALID)


def test_argument_validation_without_gpu():
    lib = nat.load()
    rope = nat.CbRope()  # half_dim 0: rejected before any CUDA call
    rc = lib.cb_rope_table(None, ctypes.byref(rope), 0, 4, None, None, 4)
    assert rc == nat.CB_ERR_INVALID
    assert b"rope table" in lib.cb_last_error()
    rc = lib.cb_map_install(None, None, None, None, 0, 0, None, None, 1, None, 0, None, None)
    assert rc == nat.CB_ERR_INVALID
    out = ctypes.c_void_p()
    rc = lib.cb_mapper_create(ctypes.byref(out), 0, 0, 1, 128, 1, None, None, None, None, None)
    assert rc == nat.CB_ERR_UNSUPPORTED
    with pytest.raises(ValueError):
        nat.check(nat.CB_ERR_INVALID, "probe")
