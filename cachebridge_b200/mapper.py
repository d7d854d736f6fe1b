"""Reference-compatible ``PageMapper`` backed by the sm_100a handoff kernels.

Drop-in for ``cachebridge.mapper.PageMapper`` / ``cachebridge.online.mapping.PageMapper``
(src/cachebridge/mapper.py:27-239, src/cachebridge/online/mapping.py:7-33) for
the CacheBridge ("headwise") method: same constructor arguments, the same
``layer_NNN.safetensors`` format and validation errors, and the same
``map_page(source_page, *, position_start, source_head_offset, output_device,
output)`` contract. The arithmetic runs in one CUDA call per page
(``cb_map_install``); there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch
from safetensors.torch import load_file

from . import _native as nat
from .device import RowSet, current_stream_ptr, rope_descriptor, status_word, storage_dtype_code


@dataclass(frozen=True)
class LayerWeights:
    """One target layer's head-sliced mapper tensors (mapper.py:17-24)."""

    selected: torch.Tensor
    k_weight: torch.Tensor
    k_bias: torch.Tensor
    v_weight: torch.Tensor
    v_bias: torch.Tensor
    headwise: bool


def _pad_selected(layers: list[LayerWeights], head_dim: int):
    """Stack per-layer tensors into uniform [L_t][S] / [L_t][H][S*D][D] arrays.

    Layers with fewer selected source layers than the widest one are padded by
    repeating their first selected layer with all-zero weight rows, which adds
    exact zeros to the FP32 accumulation.
    """
    S = max(int(layer.selected.numel()) for layer in layers)
    L_t = len(layers)
    H = int(layers[0].k_bias.shape[0])
    D = head_dim
    selected = np.zeros((L_t, S), dtype=np.int64)
    kw = np.zeros((L_t, H, S * D, D), dtype=np.float32)
    vw = np.zeros_like(kw)
    kb = np.zeros((L_t, H, D), dtype=np.float32)
    vb = np.zeros_like(kb)
    for i, layer in enumerate(layers):
        sel = layer.selected.tolist()
        s = len(sel)
        selected[i, :s] = sel
        selected[i, s:] = sel[0]
        kw[i, :, : s * D] = layer.k_weight.float().cpu().numpy()
        vw[i, :, : s * D] = layer.v_weight.float().cpu().numpy()
        kb[i] = layer.k_bias.float().cpu().numpy()
        vb[i] = layer.v_bias.float().cpu().numpy()
    return S, selected, kw, kb, vw, vb


def _dense_source_heads(layers: list[LayerWeights], heads: int, head_dim: int) -> int:
    """Source heads per selected layer of dense (nv_transfer) layers, whose
    k_weight is [S * source_heads * D, heads, D] (mapper.py:182-203)."""
    found = None
    for layer in layers:
        s = int(layer.selected.numel())
        f = int(layer.k_weight.shape[0])
        if (layer.k_weight.ndim != 3 or tuple(layer.k_weight.shape[1:]) != (heads, head_dim)
                or tuple(layer.v_weight.shape) != tuple(layer.k_weight.shape) or f % (s * head_dim)):
            raise ValueError("NV Dense feature-width mismatch")
        hs = f // (s * head_dim)
        if found is not None and hs != found:
            raise ValueError("NV Dense feature-width mismatch")
        found = hs
    return found


def _pad_dense(layers: list[LayerWeights], source_heads: int, head_dim: int):
    """Uniform [L_t][S] selections and [L_t][S*Hs*D][H][D] weights; layers with
    fewer selected source layers repeat their first one with zero weights."""
    S = max(int(layer.selected.numel()) for layer in layers)
    L_t = len(layers)
    H = int(layers[0].k_bias.shape[0])
    block = source_heads * head_dim
    selected = np.zeros((L_t, S), dtype=np.int64)
    kw = np.zeros((L_t, S * block, H, head_dim), dtype=np.float32)
    vw = np.zeros_like(kw)
    kb = np.zeros((L_t, H, head_dim), dtype=np.float32)
    vb = np.zeros_like(kb)
    for i, layer in enumerate(layers):
        sel = layer.selected.tolist()
        s = len(sel)
        selected[i, :s] = sel
        selected[i, s:] = sel[0]
        kw[i, : s * block] = layer.k_weight.float().cpu().numpy()
        vw[i, : s * block] = layer.v_weight.float().cpu().numpy()
        kb[i] = layer.k_bias.float().cpu().numpy()
        vb[i] = layer.v_bias.float().cpu().numpy()
    return S, selected, kw, kb, vw, vb


class PageMapper:
    """Apply CacheBridge mapper files to SGLang pages on a B200.

    Input and output use the canonical page layout
    ``[2, layers, tokens, kv_heads, head_dim]``; keys are stored RoPE-applied
    and the mapper consumes content-space keys (mapper.py:27-33).
    """

    def __init__(
        self,
        mapper_dir: str | Path | None,
        *,
        method: str,
        source_rope_theta: float,
        target_rope_theta: float,
        source_rope_scaling: dict | None = None,
        target_rope_scaling: dict | None = None,
        device: str | torch.device = "cuda",
        target_tp_rank: int = 0,
        target_tp_size: int = 1,
    ) -> None:
        self.mapper_dir = Path(mapper_dir) if mapper_dir is not None else None
        self.method = method
        self.source_rope_theta = float(source_rope_theta)
        self.target_rope_theta = float(target_rope_theta)
        self.source_rope_scaling = source_rope_scaling
        self.target_rope_scaling = target_rope_scaling
        self.device = torch.device(device)
        self.target_tp_rank = int(target_tp_rank)
        self.target_tp_size = int(target_tp_size)
        self.target_head_start: int | None = None
        self.target_head_stop: int | None = None
        self._handle = None
        paths = sorted(self.mapper_dir.glob("layer_*.safetensors")) if mapper_dir is not None else []
        if mapper_dir is not None and not paths:
            raise FileNotFoundError(f"no layer_*.safetensors in {self.mapper_dir}")
        sources = [(str(path), load_file(path, device="cpu")) for path in paths]
        if mapper_dir is None:
            pending = getattr(self, "_pending_tensors", None)
            if not pending:
                raise FileNotFoundError("no mapper directory and no in-memory layers given")
            sources = [(f"layer_{i:03d}", t) for i, t in enumerate(pending)]
            del self._pending_tensors
        self.layers: list[LayerWeights] = []
        for path, tensors in sources:
            required = {"selected", "k_weight", "k_bias", "v_weight", "v_bias"}
            missing = required.difference(tensors)
            if missing:
                raise ValueError(f"{path} is missing tensors: {sorted(missing)}")
            headwise = "headwise" in tensors
            if headwise != (method == "cachebridge"):
                raise ValueError(f"{path} headwise={headwise} does not match method={method}")
            target_heads = int(tensors["k_bias"].shape[0])
            if target_heads % self.target_tp_size:
                raise ValueError(
                    f"target KV heads ({target_heads}) must divide target TP ({self.target_tp_size})"
                )
            per_rank = target_heads // self.target_tp_size
            start = self.target_tp_rank * per_rank
            stop = start + per_rank
            if self.target_head_start is None:
                self.target_head_start, self.target_head_stop = start, stop
            elif (self.target_head_start, self.target_head_stop) != (start, stop):
                raise ValueError("target-head geometry changes across mapper layers")
            heads = slice(start, stop)
            if headwise:
                kw, vw = tensors["k_weight"][heads], tensors["v_weight"][heads]
            else:
                kw, vw = tensors["k_weight"][:, heads], tensors["v_weight"][:, heads]
            self.layers.append(
                LayerWeights(
                    selected=tensors["selected"].long().cpu(),
                    k_weight=kw.contiguous(),
                    k_bias=tensors["k_bias"][heads].contiguous(),
                    v_weight=vw.contiguous(),
                    v_bias=tensors["v_bias"][heads].contiguous(),
                    headwise=headwise,
                )
            )
        self.dense = method != "cachebridge"
        if self.device.type != "cuda":
            raise ValueError("cachebridge_b200 runs on CUDA devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.head_dim = int(self.layers[0].k_bias.shape[1])
        self.heads = self.target_head_stop - self.target_head_start
        self.source_heads = self.heads  # source heads read per selected layer
        for layer in self.layers:
            sel = layer.selected
            if sel.ndim != 1 or sel.numel() == 0 or int(sel.min()) < 0:
                raise ValueError("mapper selected layer list must be non-empty and non-negative")
            if not self.dense and tuple(layer.k_weight.shape) != (self.heads, sel.numel() * self.head_dim,
                                                                  self.head_dim):
                raise ValueError("CacheBridge source-head geometry mismatch")
        if self.dense:
            self.source_heads = _dense_source_heads(self.layers, self.heads, self.head_dim)
        self.max_selected = max(int(layer.selected.max()) for layer in self.layers)
        lib = nat.load()
        handle = ctypes.c_void_p()
        if self.dense:
            S, selected, kw, kb, vw, vb = _pad_dense(self.layers, self.source_heads, self.head_dim)
            self.num_selected = S
            nat.check(
                lib.cb_mapper_create_dense(
                    ctypes.byref(handle), self.device.index, len(self.layers), self.heads, self.source_heads,
                    self.head_dim, S, selected.ctypes.data, kw.ctypes.data, kb.ctypes.data, vw.ctypes.data,
                    vb.ctypes.data,
                ),
                "cb_mapper_create_dense",
            )
        else:
            S, selected, kw, kb, vw, vb = _pad_selected(self.layers, self.head_dim)
            self.num_selected = S
            nat.check(
                lib.cb_mapper_create(
                    ctypes.byref(handle), self.device.index, len(self.layers), self.heads, self.head_dim, S,
                    selected.ctypes.data, kw.ctypes.data, kb.ctypes.data, vw.ctypes.data, vb.ctypes.data,
                ),
                "cb_mapper_create",
            )
        self._handle = handle

    @classmethod
    def from_tensors(cls, layers: list[dict], **kwargs) -> "PageMapper":
        """Build a mapper from in-memory per-layer tensor dicts (the contents of
        ``layer_NNN.safetensors`` files, in layer order) instead of a directory."""
        obj = cls.__new__(cls)
        obj._pending_tensors = list(layers)
        cls.__init__(obj, None, **kwargs)
        return obj

    @property
    def target_layers(self) -> int:
        return len(self.layers)

    def close(self) -> None:
        if self._handle is not None and self._handle.value:
            nat.load().cb_mapper_destroy(self._handle)
        self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------
    def rope_descriptors(self):
        """``(source, target)`` ``cb_rope`` descriptors, built once per mapper."""
        if getattr(self, "_ropes", None) is None:
            self._ropes = (rope_descriptor(self.head_dim, self.source_rope_theta, self.source_rope_scaling),
                           rope_descriptor(self.head_dim, self.target_rope_theta, self.target_rope_scaling))
        return self._ropes

    def kernel_path(self, n_tokens: int, position_start: int = 0, *, dtype=torch.bfloat16, ordered: bool = False) -> str:
        """Which kernel a map + install call of ``n_tokens`` runs:
        "tensor_memory" (map_install_tm_kernel), "tensor_core"
        (map_install_tc_kernel) or "cuda_core" (``cb_mapper_path``)."""
        code = nat.load().cb_mapper_path(self._handle, storage_dtype_code(dtype), int(n_tokens), int(position_start),
                                         ctypes.byref(self.rope_descriptors()[1]), int(bool(ordered)))
        if code < 0:
            nat.check(code, "cb_mapper_path")
        return {nat.CB_PATH_CUDA_CORE: "cuda_core", nat.CB_PATH_TENSOR_CORE: "tensor_core",
                nat.CB_PATH_TENSOR_MEMORY: "tensor_memory"}[code]

    def tensor_memory_path(self, n_tokens: int, position_start: int = 0) -> bool:
        return self.kernel_path(n_tokens, position_start) == "tensor_memory"

    def workspace_bytes(self, dtype: torch.dtype, n_tokens: int) -> int:
        return int(nat.load().cb_mapper_workspace_bytes(self._handle, storage_dtype_code(dtype), int(n_tokens)))

    def prepare(
        self, src: RowSet, dst: RowSet, n_tokens: int, position_start: int, *, tables=None, workspace=None
    ) -> "HandoffCall":
        """Validate one gather + map + install and marshal its C-ABI arguments.

        The returned ``HandoffCall`` launches on the current stream each time it
        is run. RoPE tables for positions ``position_start..+n-1`` are built once
        here on the current stream unless ``tables = (src_cos, src_sin, dst_cos,
        dst_sin)`` (each ``[n, head_dim/2]`` FP32) is given; ``workspace`` (a
        uint8 CUDA tensor of at least ``workspace_bytes``) may be shared across
        calls that never run concurrently.
        """
        if self._handle is None:
            raise RuntimeError("mapper is closed")
        if src.device != self.device:
            raise ValueError("source rows must live on the mapper's device")
        if dst.device.type != "cuda":
            raise ValueError("destination rows must be CUDA memory (local or a peer device)")
        if src.head_dim != self.head_dim or dst.head_dim != self.head_dim:
            raise ValueError("CacheBridge source-head geometry mismatch")
        if src.layers <= self.max_selected:
            raise ValueError("mapper selected layer exceeds source page depth")
        if dst.layers != self.target_layers or src.dtype != dst.dtype:
            raise ValueError("mapper output geometry/dtype mismatch")
        for rs in (src, dst):
            if rs.slots is not None and rs.slots.device != self.device:
                raise ValueError("pool, indices and workspace must share device and dtype as applicable")
        n = int(n_tokens)
        if (src.slots is not None and src.slots.numel() < n) or (dst.slots is not None and dst.slots.numel() < n):
            raise ValueError("invalid target range or non-CacheBridge method")
        return HandoffCall(self, src, dst, n, int(position_start), workspace=workspace)

    def map_install(self, src: RowSet, dst: RowSet, n_tokens: int, position_start: int) -> None:
        """Fused gather + map + install of ``n_tokens`` tokens.

        Source rows ``src.slots[t]`` (a source pool, or a dense page with no
        slots) are mapped to this rank's heads and written to ``dst`` rows
        ``dst.slots[t]`` at head ``dst.head_offset``. Asynchronous on the current
        stream; device-side slot or timeout errors land in the device status
        word (see ``device.raise_for_status``).
        """
        self.prepare(src, dst, n_tokens, position_start).run()

    @torch.inference_mode()
    def map_page(
        self,
        source_page: torch.Tensor,
        *,
        position_start: int,
        source_head_offset: int = 0,
        output_device: str | torch.device = "cpu",
        output: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Map one page; same contract as the reference's ``map_page``.

        ``source_page`` is ``[2, source_layers, tokens, source_heads, head_dim]``
        (keys RoPE-applied). A headwise mapper narrows the received shard to
        this rank's heads first (online/mapping.py:18-28); a dense one reads
        every source head. Returns (or fills ``output``
        with) ``[2, target_layers, tokens, heads, head_dim]`` in the page dtype.
        """
        if source_page.ndim != 5 or source_page.shape[0] != 2:
            raise ValueError("source page must be [2,layers,tokens,kv_heads,head_dim]")
        if self.dense:
            # Dense maps read every source head of the page (mapper.py:182-203).
            if source_page.shape[3] != self.source_heads:
                raise ValueError("NV Dense feature-width mismatch")
            start = 0
        else:
            start = self.target_head_start - source_head_offset
            stop = self.target_head_stop - source_head_offset
            if not 0 <= start < stop <= source_page.shape[3]:
                raise ValueError("Received source shard does not contain required heads")
        dtype = source_page.dtype
        storage_dtype_code(dtype)
        _, source_layers, tokens, _, head_dim = source_page.shape
        if self.max_selected >= source_layers:
            raise ValueError("mapper selected layer exceeds source page depth")
        if head_dim != self.head_dim:
            raise ValueError("CacheBridge source-head geometry mismatch")
        expected = (2, self.target_layers, tokens, self.heads, self.head_dim)
        if output is not None and (
            tuple(output.shape) != expected
            or output.dtype != dtype
            or output.device != torch.device(output_device)
        ):
            raise ValueError("preallocated mapper output geometry/dtype/device mismatch")
        page = source_page.to(self.device, non_blocking=True)
        if not page.is_contiguous():
            page = page.contiguous()
        direct = output is not None and output.device == self.device and output.is_contiguous()
        out = output if direct else torch.empty(expected, dtype=dtype, device=self.device)
        self.map_install(RowSet.from_page(page, head_offset=start), RowSet.from_page(out), tokens, position_start)
        if direct:
            return output
        if output is None:
            return out.to(output_device)
        output.copy_(out)
        return output


class HandoffCall:
    """One prepared ``cb_map_install`` (or its two phases) with marshalled arguments."""

    def __init__(self, mapper: PageMapper, src: RowSet, dst: RowSet, n: int, position_start: int, *,
                 workspace=None):
        self.mapper = mapper
        self.n = n
        self.position_start = position_start
        self.src, self.dst = src, dst
        self.src_c, self.dst_c = src.to_c(), dst.to_c()
        self.dtype = storage_dtype_code(src.dtype)
        self.tensor_core = mapper.head_dim == 128 and src.dtype == torch.bfloat16
        self.src_rope, self.dst_rope = mapper.rope_descriptors()
        dev = mapper.device
        ws_bytes = mapper.workspace_bytes(src.dtype, n)
        if workspace is None:
            workspace = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
        elif workspace.numel() < ws_bytes or workspace.device != dev:
            raise ValueError("workspace missing, too small or on the wrong device")
        self.workspace = workspace
        self.status = status_word(dev)
        # Processing order of the tokens on the tensor-core path (token_order
        # of the C ABI): None keeps 0..n-1. Results do not depend on it. On
        # B200, sorting by destination slot gained 1 % with 262144-slot pools
        # and lost 13 % when the slots cover the pool densely, so the default
        # is the natural order; callers may set an int32 permutation here.
        self.order = None

    def _order_ptr(self):
        return None if self.order is None else self.order.data_ptr()

    def _stream(self):
        return ctypes.c_void_p(current_stream_ptr(self.mapper.device))

    def run(self) -> None:
        """Both phases (``cb_map_install``)."""
        if not self.n:
            return
        nat.check(
            nat.load().cb_map_install(
                self.mapper._handle, self._stream(), ctypes.byref(self.src_c), ctypes.byref(self.dst_c), self.n,
                self.position_start, ctypes.byref(self.src_rope), ctypes.byref(self.dst_rope), self.dtype,
                self.workspace.data_ptr(), self.workspace.numel(), self._order_ptr(), self.status.data_ptr(),
            ),
            "cb_map_install",
        )

    def derotate(self) -> None:
        """Phase 1 of the tensor-core path (``cb_derotate_keys``): content-space
        keys into the workspace."""
        nat.check(
            nat.load().cb_derotate_keys(
                self.mapper._handle, self._stream(), ctypes.byref(self.src_c), self.n, self.position_start,
                ctypes.byref(self.src_rope), self.workspace.data_ptr(), self.workspace.numel(), self._order_ptr(),
                self.status.data_ptr(),
            ),
            "cb_derotate_keys",
        )

    def install(self) -> None:
        """Phase 2 of the tensor-core path (``cb_map_install_packed``)."""
        nat.check(
            nat.load().cb_map_install_packed(
                self.mapper._handle, self._stream(), ctypes.byref(self.src_c), ctypes.byref(self.dst_c), self.n,
                self.position_start, ctypes.byref(self.dst_rope), self.workspace.data_ptr(),
                self.workspace.numel(), self._order_ptr(), self.status.data_ptr(),
            ),
            "cb_map_install_packed",
        )
