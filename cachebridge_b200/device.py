"""Torch-facing wrappers of the C-ABI launches (rows, RoPE tables, status).

Everything here runs on CUDA devices only and launches on the caller's current
torch stream. Buffers handed to the kernels (RoPE tables, the key workspace,
the device status word) come from torch's caching allocator; the C-ABI calls
themselves never allocate.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _native as nat
from .rope import rope_parameters

_DTYPES = {torch.bfloat16: nat.CB_DTYPE_BF16, torch.float32: nat.CB_DTYPE_F32}


def storage_dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"unsupported KV storage dtype {dtype}; expected bfloat16 or float32") from None


def require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{what} must be a CUDA tensor (cachebridge_b200 runs on GPUs only)")


def slot_code(slots: torch.Tensor | None) -> int:
    if slots is None:
        return nat.CB_INDEX_NONE
    if slots.dtype == torch.int32:
        return nat.CB_INDEX_I32
    if slots.dtype == torch.int64:
        return nat.CB_INDEX_I64
    raise ValueError("one-dimensional integer pool indices required")


@dataclass
class RowSet:
    """Per-layer row buffers [rows, heads, head_dim] on one device.

    The C-ABI view of an SGLang ``MHATokenToKVPool`` (``_get_key_buffer(l)`` /
    ``_get_value_buffer(l)``) or of a dense page ``[2, layers, tokens, heads,
    head_dim]`` (row = token).
    """

    k: list
    v: list
    heads: int
    head_dim: int
    head_offset: int = 0
    slots: torch.Tensor | None = None
    _keep: list = field(default_factory=list, repr=False)
    # Validated layer geometry of a pool (from_pool): the row stride and the C
    # pointer arrays, shared by every RowSet of that pool.
    _layers_c: "_PoolLayers | None" = field(default=None, repr=False)

    @property
    def layers(self) -> int:
        return len(self.k)

    @property
    def device(self) -> torch.device:
        return self.k[0].device

    @property
    def dtype(self) -> torch.dtype:
        return self.k[0].dtype

    @property
    def rows(self) -> int:
        return int(self.k[0].shape[0])

    @staticmethod
    def from_pool(pool, slots=None, head_offset: int = 0) -> "RowSet":
        pl = _pool_layers(pool)
        return RowSet(pl.k, pl.v, pl.heads, pl.head_dim, head_offset, slots, _layers_c=pl)

    @staticmethod
    def from_page(page: torch.Tensor, head_offset: int = 0) -> "RowSet":
        if page.ndim != 5 or page.shape[0] != 2:
            raise ValueError("source page must be [2,layers,tokens,kv_heads,head_dim]")
        if not page.is_contiguous():
            page = page.contiguous()
        k = [page[0, l] for l in range(page.shape[1])]
        v = [page[1, l] for l in range(page.shape[1])]
        rs = RowSet(k, v, int(page.shape[3]), int(page.shape[4]), head_offset, None)
        rs._keep.append(page)
        return rs

    def validate(self) -> int:
        """Check layer geometry; return the common row stride (elements)."""
        stride = None
        for t in list(self.k) + list(self.v):
            require_cuda(t, "KV rows")
            if t.ndim != 3 or t.shape[1] != self.heads or t.shape[2] != self.head_dim:
                raise ValueError("pool layers must be [rows, heads, head_dim]")
            if t.stride(2) != 1 or t.stride(1) != self.head_dim:
                raise ValueError("pool rows must be contiguous [heads, head_dim]")
            if t.dtype != self.dtype or t.device != self.device or t.shape[0] != self.rows:
                raise ValueError("pool layers must share dtype, device and row count")
            if stride is None:
                stride = t.stride(0)
            elif t.stride(0) != stride:
                raise ValueError("pool layers must share one row stride")
        self._validate_slots()
        return int(stride)

    def _validate_slots(self) -> None:
        if self.slots is not None:
            require_cuda(self.slots, "slot indices")
            if self.slots.ndim != 1:
                raise ValueError("one-dimensional integer pool indices required")
            if not self.slots.is_contiguous():
                self.slots = self.slots.contiguous()

    def to_c(self) -> nat.CbRows:
        pl = self._layers_c
        if pl is not None and pl.k is self.k and pl.v is self.v:
            # A pool's layers, validated once when their views were cached.
            self._validate_slots()
            stride, karr, varr = pl.row_stride, pl.karr, pl.varr
        else:
            stride = self.validate()
            karr = nat.pointer_array([t.data_ptr() for t in self.k])
            varr = nat.pointer_array([t.data_ptr() for t in self.v])
            self._keep.extend([karr, varr])
        return nat.CbRows(
            layers=self.layers,
            heads=self.heads,
            k=ctypes.cast(karr, ctypes.POINTER(ctypes.c_void_p)),
            v=ctypes.cast(varr, ctypes.POINTER(ctypes.c_void_p)),
            row_stride=stride,
            rows=self.rows,
            head_offset=self.head_offset,
            slot_dtype=slot_code(self.slots),
            slots=None if self.slots is None else self.slots.data_ptr(),
        )


@dataclass
class _PoolLayers:
    """A pool's per-layer K/V views with their validated row stride and C
    pointer arrays. Building these walks every layer of the pool in Python
    (two views, a dozen attribute checks and a pointer per layer and kind,
    about 0.3 ms for a 64-layer pool), which a handoff would otherwise repeat
    for every chunk it maps; they are built once per pool and rebuilt only
    when its first layer's buffer moves."""

    key: tuple
    k: list
    v: list
    heads: int
    head_dim: int
    row_stride: int
    karr: ctypes.Array
    varr: ctypes.Array


def _pool_layers(pool) -> _PoolLayers:
    first = pool._get_key_buffer(pool.start_layer)
    key = (pool.start_layer, pool.layer_num, first.data_ptr(), tuple(first.shape), first.dtype, first.device)
    cached = getattr(pool, "_cb_pool_layers", None)
    if cached is not None and cached.key == key:
        return cached
    layers = range(pool.start_layer, pool.start_layer + pool.layer_num)
    k = [pool._get_key_buffer(l) for l in layers]
    v = [pool._get_value_buffer(l) for l in layers]
    heads, dim = k[0].shape[1:]
    stride = RowSet(k, v, int(heads), int(dim)).validate()
    pl = _PoolLayers(key, k, v, int(heads), int(dim), stride, nat.pointer_array([t.data_ptr() for t in k]),
                     nat.pointer_array([t.data_ptr() for t in v]))
    try:
        pool._cb_pool_layers = pl
    except AttributeError:  # a pool type that takes no new attributes: rebuilt per call
        pass
    return pl


@dataclass
class RawRows:
    """Per-layer row buffers given by raw device addresses (no torch tensors).

    For rows this process did not allocate, such as a peer GPU's target pool
    mapped through CUDA IPC (``cb_ipc_open``); ``device`` is the GPU whose
    kernels address them, ``slots`` live on that device. Same interface as
    ``RowSet`` towards the mapper and the C ABI.
    """

    k_ptrs: list
    v_ptrs: list
    heads: int
    head_dim: int
    rows: int
    row_stride: int
    dtype: torch.dtype
    device: torch.device
    head_offset: int = 0
    slots: torch.Tensor | None = None
    _keep: list = field(default_factory=list, repr=False)

    @property
    def layers(self) -> int:
        return len(self.k_ptrs)

    def to_c(self) -> nat.CbRows:
        if self.slots is not None:
            require_cuda(self.slots, "slot indices")
            if self.slots.ndim != 1:
                raise ValueError("one-dimensional integer pool indices required")
            if not self.slots.is_contiguous():
                self.slots = self.slots.contiguous()
        karr = nat.pointer_array(self.k_ptrs)
        varr = nat.pointer_array(self.v_ptrs)
        self._keep.extend([karr, varr])
        return nat.CbRows(
            layers=self.layers,
            heads=self.heads,
            k=ctypes.cast(karr, ctypes.POINTER(ctypes.c_void_p)),
            v=ctypes.cast(varr, ctypes.POINTER(ctypes.c_void_p)),
            row_stride=self.row_stride,
            rows=self.rows,
            head_offset=self.head_offset,
            slot_dtype=slot_code(self.slots),
            slots=None if self.slots is None else self.slots.data_ptr(),
        )


def current_stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_status_words: dict = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word the kernels OR their CB_DEV_ERR_* bits into."""
    key = torch.device(device).index
    word = _status_words.get(key)
    if word is None:
        # A normal (non-inference) tensor, so it can be cleared in or out of inference mode.
        with torch.inference_mode(False):
            word = torch.zeros(1, dtype=torch.int32, device=device)
        _status_words[key] = word
    return word


def read_status(device: torch.device, clear: bool = True) -> int:
    """Synchronize the current stream and return (then clear) the status bits."""
    word = status_word(device)
    value = int(word.item())
    if clear and value:
        word.zero_()
    return value


def raise_for_status(device: torch.device) -> None:
    bits = read_status(device)
    if bits & nat.CB_DEV_ERR_SLOT_RANGE:
        raise ValueError("a pool slot index was outside the pool (device check)")
    if bits & nat.CB_DEV_ERR_TIMEOUT:
        raise RuntimeError("a bounded pipeline wait expired inside a handoff kernel")
    if bits:
        raise RuntimeError(f"handoff kernel reported device status {bits}")


def rope_descriptor(head_dim: int, theta: float, scaling: dict | None) -> nat.CbRope:
    """``cb_rope`` for a model's RoPE (inv_freq and YaRN magnitude, rope.py:16-69)."""
    inv_freq, magnitude = rope_parameters(head_dim, theta, scaling)
    rope = nat.CbRope()
    rope.half_dim = head_dim // 2
    rope.magnitude = magnitude
    for i, v in enumerate(inv_freq.tolist()):
        rope.inv_freq[i] = v
    return rope


def rope_tables(
    device: torch.device,
    head_dim: int,
    theta: float,
    scaling: dict | None,
    position_start: int,
    n: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Frequency-major cos/sin tables ``[head_dim/2, n]`` (FP32) for positions
    ``position_start .. +n-1`` (entry ``[i, t]`` is frequency i of token t)."""
    lib = nat.load()
    rope = rope_descriptor(head_dim, theta, scaling)
    width = max(n, 1)
    cos = torch.empty((head_dim // 2, width), dtype=torch.float32, device=device)
    sin = torch.empty_like(cos)
    nat.check(
        lib.cb_rope_table(
            ctypes.c_void_p(current_stream_ptr(device)),
            ctypes.byref(rope),
            int(position_start),
            int(n),
            cos.data_ptr(),
            sin.data_ptr(),
            width,
        ),
        "cb_rope_table",
    )
    return cos, sin


def pack_rows(src: RowSet, n: int, out: torch.Tensor) -> torch.Tensor:
    """Gather rows ``src.slots[:n]`` of every layer into dense ``out``."""
    lib = nat.load()
    status = status_word(src.device)
    c = src.to_c()
    nat.check(
        lib.cb_pack_rows(
            ctypes.c_void_p(current_stream_ptr(src.device)),
            ctypes.byref(c),
            src.head_dim,
            storage_dtype_code(src.dtype),
            int(n),
            out.data_ptr(),
            status.data_ptr(),
        ),
        "cb_pack_rows",
    )
    return out


def install_rows(block: torch.Tensor, dst: RowSet, n: int) -> None:
    """Scatter dense ``block`` [2, layers, n, heads, dim] into rows ``dst.slots``."""
    lib = nat.load()
    status = status_word(dst.device)
    c = dst.to_c()
    nat.check(
        lib.cb_install_rows(
            ctypes.c_void_p(current_stream_ptr(dst.device)),
            block.data_ptr(),
            ctypes.byref(c),
            dst.head_dim,
            storage_dtype_code(dst.dtype),
            int(n),
            status.data_ptr(),
        ),
        "cb_install_rows",
    )
