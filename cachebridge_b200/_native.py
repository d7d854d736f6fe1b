"""ctypes binding of the C ABI in ``include/cachebridge_b200.h``.

The shared library ``libcachebridge_b200.so`` is built in-tree by
``cachebridge_b200.csrc.build``. There is no fallback: if the library is
missing or fails to load, every GPU entry point raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "libcachebridge_b200.so"

CB_OK = 0
CB_ERR_INVALID = -1
CB_ERR_UNSUPPORTED = -2
CB_ERR_CUDA = -3
CB_ERR_ALIAS = -4

CB_DEV_ERR_SLOT_RANGE = 1
CB_DEV_ERR_TIMEOUT = 2

CB_DTYPE_F32 = 0
CB_DTYPE_BF16 = 1

CB_INDEX_NONE = 0
CB_INDEX_I32 = 32
CB_INDEX_I64 = 64

CB_PATH_CUDA_CORE = 0
CB_PATH_TENSOR_CORE = 1
CB_PATH_TENSOR_MEMORY = 2

CB_MAX_LAYERS = 128
CB_NOALLOC_SCRATCH_BYTES = 64 << 20

# Every entry point declared in include/cachebridge_b200.h (checked by tests).
EXPORTED_SYMBOLS = (
    "cb_version",
    "cb_status_string",
    "cb_last_error",
    "cb_mapper_create",
    "cb_mapper_create_dense",
    "cb_mapper_destroy",
    "cb_mapper_info",
    "cb_mapper_workspace_bytes",
    "cb_mapper_path",
    "cb_rope_table",
    "cb_map_install",
    "cb_map_install_noalloc",
    "cb_derotate_keys",
    "cb_map_install_packed",
    "cb_pack_rows",
    "cb_install_rows",
    "cb_ipc_export",
    "cb_ipc_open",
    "cb_ipc_close",
    "cb_copy_async",
    "cb_chunk_signal",
    "cb_chunk_wait",
    "cb_enable_peer_access",
)


class CbRows(ctypes.Structure):
    """Mirror of ``struct cb_rows``."""

    _fields_ = [
        ("layers", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("k", ctypes.POINTER(ctypes.c_void_p)),
        ("v", ctypes.POINTER(ctypes.c_void_p)),
        ("row_stride", ctypes.c_int64),
        ("rows", ctypes.c_int64),
        ("head_offset", ctypes.c_int32),
        ("slot_dtype", ctypes.c_int32),
        ("slots", ctypes.c_void_p),
    ]


class CbRope(ctypes.Structure):
    """Mirror of ``struct cb_rope``."""

    _fields_ = [
        ("half_dim", ctypes.c_int32),
        ("magnitude", ctypes.c_float),
        ("inv_freq", ctypes.c_float * 128),
    ]


_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _declare(lib: ctypes.CDLL) -> None:
    c_int, c_i64, c_vp, c_float, c_size = (
        ctypes.c_int,
        ctypes.c_int64,
        ctypes.c_void_p,
        ctypes.c_float,
        ctypes.c_size_t,
    )
    rows_p = ctypes.POINTER(CbRows)
    rope_p = ctypes.POINTER(CbRope)
    lib.cb_version.restype = c_int
    lib.cb_status_string.restype = ctypes.c_char_p
    lib.cb_status_string.argtypes = [c_int]
    lib.cb_last_error.restype = ctypes.c_char_p
    lib.cb_mapper_create.restype = c_int
    lib.cb_mapper_create.argtypes = [
        ctypes.POINTER(c_vp), c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp
    ]
    lib.cb_mapper_create_dense.restype = c_int
    lib.cb_mapper_create_dense.argtypes = [
        ctypes.POINTER(c_vp), c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp
    ]
    lib.cb_mapper_destroy.restype = c_int
    lib.cb_mapper_destroy.argtypes = [c_vp]
    lib.cb_mapper_info.restype = c_int
    lib.cb_mapper_info.argtypes = [c_vp] + [ctypes.POINTER(c_int)] * 5
    lib.cb_mapper_workspace_bytes.restype = c_size
    lib.cb_mapper_workspace_bytes.argtypes = [c_vp, c_int, c_i64]
    lib.cb_mapper_path.restype = c_int
    lib.cb_mapper_path.argtypes = [c_vp, c_int, c_i64, c_i64, rope_p, c_int]
    lib.cb_rope_table.restype = c_int
    lib.cb_rope_table.argtypes = [c_vp, rope_p, c_i64, c_i64, c_vp, c_vp, c_i64]
    lib.cb_map_install.restype = c_int
    lib.cb_map_install.argtypes = [
        c_vp, c_vp, rows_p, rows_p, c_i64, c_i64, rope_p, rope_p, c_int, c_vp, c_size, c_vp, c_vp
    ]
    lib.cb_map_install_noalloc.restype = c_int
    lib.cb_map_install_noalloc.argtypes = [c_vp, c_vp, rows_p, rows_p, c_i64, c_i64, rope_p, rope_p, c_int, c_vp]
    lib.cb_derotate_keys.restype = c_int
    lib.cb_derotate_keys.argtypes = [c_vp, c_vp, rows_p, c_i64, c_i64, rope_p, c_vp, c_size, c_vp, c_vp]
    lib.cb_map_install_packed.restype = c_int
    lib.cb_map_install_packed.argtypes = [c_vp, c_vp, rows_p, rows_p, c_i64, c_i64, rope_p, c_vp, c_size, c_vp, c_vp]
    lib.cb_pack_rows.restype = c_int
    lib.cb_pack_rows.argtypes = [c_vp, rows_p, c_int, c_int, c_i64, c_vp, c_vp]
    lib.cb_install_rows.restype = c_int
    lib.cb_install_rows.argtypes = [c_vp, c_vp, rows_p, c_int, c_int, c_i64, c_vp]
    lib.cb_ipc_export.restype = c_int
    lib.cb_ipc_export.argtypes = [c_vp, c_vp, ctypes.POINTER(ctypes.c_uint64)]
    lib.cb_ipc_open.restype = c_int
    lib.cb_ipc_open.argtypes = [c_vp, c_int, ctypes.POINTER(c_vp)]
    lib.cb_copy_async.restype = c_int
    lib.cb_copy_async.argtypes = [c_vp, c_vp, c_vp, c_size]
    lib.cb_chunk_signal.restype = c_int
    lib.cb_chunk_signal.argtypes = [c_vp, c_vp, c_i64]
    lib.cb_chunk_wait.restype = c_int
    lib.cb_chunk_wait.argtypes = [c_vp, c_vp, c_i64, c_i64, c_vp]
    lib.cb_ipc_close.restype = c_int
    lib.cb_ipc_close.argtypes = [c_vp]
    lib.cb_enable_peer_access.restype = c_int
    lib.cb_enable_peer_access.argtypes = [c_int, c_int]


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIBRARY_PATH.exists():
                raise RuntimeError(
                    f"cachebridge_b200 native library not built ({LIBRARY_PATH}); "
                    "run `python -m cachebridge_b200.csrc.build` (requires nvcc)"
                )
            lib = ctypes.CDLL(str(LIBRARY_PATH))
            _declare(lib)
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    """Raise the reference's exception type for a failing C-ABI status."""
    if status == CB_OK:
        return
    lib = load()
    message = f"{what}: {lib.cb_last_error().decode(errors='replace')}"
    if status in (CB_ERR_INVALID, CB_ERR_ALIAS):
        raise ValueError(message)
    raise NativeError(status, message)


def pointer_array(pointers) -> ctypes.Array:
    """Host array of device pointers (``void* const*``) for a cb_rows field."""
    arr = (ctypes.c_void_p * len(pointers))()
    for i, p in enumerate(pointers):
        arr[i] = int(p)
    return arr
