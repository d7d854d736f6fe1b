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


@pytest.mark.parametrize(
    "call,status,message",
    [
        (lambda lib: lib.cb_map_install_noalloc(None, None, None, None, 1, 0, None, None, nat.CB_DTYPE_BF16, None),
         nat.CB_ERR_INVALID, b"null mapper"),
        (lambda lib: lib.cb_pack_rows(None, None, 128, 7, 1, None, None), nat.CB_ERR_UNSUPPORTED, b"dtype"),
        (lambda lib: lib.cb_pack_rows(None, None, 0, nat.CB_DTYPE_BF16, 1, None, None), nat.CB_ERR_INVALID,
         b"head_dim"),
        (lambda lib: lib.cb_pack_rows(None, None, 128, nat.CB_DTYPE_BF16, 1, None, None), nat.CB_ERR_INVALID,
         b"null row set"),
        (lambda lib: lib.cb_install_rows(None, None, None, 128, nat.CB_DTYPE_F32, 1, None), nat.CB_ERR_INVALID,
         b"null row set"),
        (lambda lib: lib.cb_chunk_signal(None, None, 1), nat.CB_ERR_INVALID, b"null flag"),
        (lambda lib: lib.cb_chunk_signal(None, ctypes.c_void_p(0x1004), 1), nat.CB_ERR_INVALID, b"aligned"),
        (lambda lib: lib.cb_chunk_wait(None, ctypes.c_void_p(0x1000), 1, 1000, None), nat.CB_ERR_INVALID,
         b"null flag or status"),
        (lambda lib: lib.cb_chunk_wait(None, ctypes.c_void_p(0x1000), 1, 0, ctypes.c_void_p(0x2000)),
         nat.CB_ERR_INVALID, b"timeout"),
        (lambda lib: lib.cb_copy_async(None, None, None, 16), nat.CB_ERR_INVALID, b"null copy pointer"),
        (lambda lib: lib.cb_ipc_export(None, None, None), nat.CB_ERR_INVALID, b"null pointer"),
        (lambda lib: lib.cb_ipc_open(None, 0, None), nat.CB_ERR_INVALID, b"null pointer"),
        (lambda lib: lib.cb_mapper_info(None, None, None, None, None, None), nat.CB_ERR_INVALID, b"null mapper"),
        (lambda lib: lib.cb_rope_table(None, ctypes.byref(nat.CbRope(half_dim=64)), -1, 4, None, None, 4),
         nat.CB_ERR_INVALID, b"rope table"),
    ],
)
def test_entry_points_reject_bad_arguments_before_any_cuda_call(call, status, message):
    lib = nat.load()
    assert call(lib) == status
    assert message in lib.cb_last_error()


def test_null_handles_are_no_ops():
    lib = nat.load()
    assert lib.cb_mapper_destroy(None) == nat.CB_OK
    assert lib.cb_ipc_close(None) == nat.CB_OK
    assert lib.cb_copy_async(None, None, None, 0) == nat.CB_OK
    assert lib.cb_mapper_workspace_bytes(None, nat.CB_DTYPE_BF16, 100) == 0
