"""A paged token KV pool with the SGLang ``MHATokenToKVPool`` duck type.

The handoff path addresses the target model's KV cache through the interface
the reference relies on (backends/sglang/runtime/source_mapper_adapter.py:389-425,
online/blocks.py:47-111): ``start_layer``, ``layer_num``, ``dtype``,
``_get_key_buffer(layer)`` / ``_get_value_buffer(layer)`` returning
``[rows, heads, head_dim]`` views, and
``set_kv_buffer(None, loc, k, v, layer_id_override=layer)``. SGLang's pool
lives in the (absent) engine; this class provides the same layout for the
tests, the benchmark and standalone users: one contiguous allocation per kind
``[layers, rows, heads, head_dim]`` (page_size = 1, slot = row).
"""

from __future__ import annotations

import torch

from .device import RowSet


class TokenKVPool:
    def __init__(self, *, layers: int, rows: int, heads: int, head_dim: int, dtype=torch.bfloat16,
                 device="cuda", start_layer: int = 0, fill: float | None = None):
        self.layer_num = int(layers)
        self.start_layer = int(start_layer)
        self.dtype = dtype
        self.device = torch.device(device)
        self.size = int(rows)
        shape = (self.layer_num, self.size, int(heads), int(head_dim))
        if fill is None:
            self.k_buffer = torch.empty(shape, dtype=dtype, device=self.device)
            self.v_buffer = torch.empty(shape, dtype=dtype, device=self.device)
        else:
            self.k_buffer = torch.full(shape, fill, dtype=dtype, device=self.device)
            self.v_buffer = torch.full(shape, fill, dtype=dtype, device=self.device)

    @property
    def heads(self) -> int:
        return int(self.k_buffer.shape[2])

    @property
    def head_dim(self) -> int:
        return int(self.k_buffer.shape[3])

    def _get_key_buffer(self, layer: int) -> torch.Tensor:
        return self.k_buffer[layer - self.start_layer]

    def _get_value_buffer(self, layer: int) -> torch.Tensor:
        return self.v_buffer[layer - self.start_layer]

    def set_kv_buffer(self, _layer, loc, cache_k, cache_v, layer_id_override=None):
        """SGLang semantics: ``k_buffer[layer][loc] = cache_k`` (and V)."""
        layer = layer_id_override - self.start_layer
        self.k_buffer[layer][loc] = cache_k.to(self.dtype)
        self.v_buffer[layer][loc] = cache_v.to(self.dtype)

    def rows(self, slots: torch.Tensor | None = None, head_offset: int = 0) -> RowSet:
        """C-ABI row-set view of this pool addressed through ``slots``."""
        return RowSet.from_pool(self, slots, head_offset)


def token_slots_from_pages(page_table, page_size: int, n_tokens: int | None = None) -> torch.Tensor:
    """Token slots of a request held in pages of ``page_size`` tokens.

    A paged SGLang pool still stores one row per token: token i of the request
    sits at row ``page_table[i // page_size] * page_size + i % page_size``
    (the ``req_to_token`` row the reference's adapter reads as
    ``device_indices``, backends/sglang/runtime/clean_adapter.py:370-380). The
    history must be non-empty and page-aligned, as the reference requires.
    Returns int64 slots on the page table's device.
    """
    pages = torch.as_tensor(page_table)
    if type(page_size) is not int or page_size <= 0:
        raise ValueError("page_size must be a positive integer")
    if pages.ndim != 1 or pages.dtype not in (torch.int32, torch.int64):
        raise ValueError("page_table must be a 1-D integer tensor")
    n = pages.numel() * page_size if n_tokens is None else int(n_tokens)
    if n == 0 or n % page_size:
        raise ValueError("Only nonempty page-aligned histories supported")
    if n > pages.numel() * page_size:
        raise ValueError("page_table holds fewer tokens than requested")
    used = pages[: n // page_size].long()
    if bool((used < 0).any()):
        raise ValueError("negative page index")
    offsets = torch.arange(page_size, device=used.device, dtype=torch.int64)
    return (used.unsqueeze(1) * page_size + offsets).reshape(-1)
