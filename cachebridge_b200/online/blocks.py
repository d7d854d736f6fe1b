"""Block primitives of the online handoff: pack, map+install, unpublished install.

Drop-in for ``cachebridge.online.blocks`` (src/cachebridge/online/blocks.py,
duplicated in backends/sglang/runtime/bounded_cachebridge_core.py):

- ``SourceLease``           single in-flight block ownership (blocks.py:11-43)
- ``pack_source_block``     gather pool rows into one contiguous workspace
                            (blocks.py:47-82), one ``cb_pack_rows`` launch instead
                            of 2*layers ``index_select`` launches
- ``map_write_block``       map a packed block and install it into target pool
                            rows (blocks.py:86-111), one fused launch pair instead
                            of map_page + per-layer ``set_kv_buffer``
- ``map_install_block``     the fully fused source-pool -> target-pool path (no
                            packed block at all): gather, map and install
- ``install_unpublished``   publish-after-vote transaction (blocks.py:114-171)
"""

from __future__ import annotations

import torch

from ..device import RowSet, pack_rows


class SourceLease:
    """Single in-flight block; release is legal only after consumer completion."""

    def __init__(self, acquire, release):
        self.acquire = acquire
        self.release = release
        self.active = False
        self.pending = False
        self.next_start = 0

    def begin(self):
        if self.active:
            raise RuntimeError("source lease already active")
        self.acquire()
        self.active = True
        self.next_start = 0

    def export(self, start, stop):
        ordered = self.active and not self.pending and start == self.next_start and stop > start
        if not ordered:
            raise RuntimeError("block ownership/order violation")
        self.pending = True
        self.next_start = stop

    def acknowledge(self, *, gpu_reads_complete):
        if not (self.active and self.pending and gpu_reads_complete):
            raise RuntimeError("consumer GPU completion required before buffer reuse")
        self.pending = False

    def close(self):
        if not self.active or self.pending:
            raise RuntimeError("cannot release source lease with outstanding GPU reads")
        self.release()
        self.active = False


@torch.inference_mode()
def pack_source_block(pool, indices, *, start, stop, workspace, block_tokens):
    """Pack pool rows ``indices[start:stop]`` into the prefix of ``workspace``.

    Returns a contiguous ``[2, layers, stop-start, heads, dim]`` view of the
    one-dimensional ``workspace`` (which must hold exactly one full block).
    """
    n = stop - start
    if not (0 <= start < stop <= len(indices)) or n > block_tokens:
        raise ValueError("invalid block span")
    layers = pool.layer_num
    first = pool._get_key_buffer(pool.start_layer)
    heads, dim = first.shape[1:]
    if workspace.ndim != 1 or workspace.numel() != 2 * layers * block_tokens * heads * dim or not workspace.is_contiguous():
        raise ValueError("workspace must be exactly one contiguous block")
    if workspace.device != first.device or workspace.dtype != first.dtype or indices.device != first.device:
        raise ValueError("pool, indices and workspace must share device and dtype as applicable")
    if indices.ndim != 1 or indices.dtype not in (torch.int32, torch.int64):
        raise ValueError("one-dimensional integer pool indices required")
    block = workspace[: 2 * layers * n * heads * dim].view(2, layers, n, heads, dim)
    src = RowSet.from_pool(pool, indices[start:stop])
    pack_rows(src, n, block)
    return block


@torch.inference_mode()
def map_write_block(mapper, block, target_pool, target_indices, *, start, source_head_offset):
    """Map a packed source block and install it at ``target_indices[start:start+n]``.

    Same arithmetic and positions as the reference (map_page at
    ``position_start=start``), fused with the install: mapped rows go straight
    from the kernel's registers to the target pool rows.
    """
    n = block.shape[2]
    if start < 0 or start + n > len(target_indices) or mapper.method != "cachebridge":
        raise ValueError("invalid target range or non-CacheBridge method")
    if block.ndim != 5 or block.shape[0] != 2:
        raise ValueError("source page must be [2,layers,tokens,kv_heads,head_dim]")
    if target_pool.layer_num != mapper.target_layers or target_pool.dtype != block.dtype:
        raise ValueError("mapper output geometry/dtype mismatch")
    head_start = mapper.target_head_start - source_head_offset
    if not 0 <= head_start < head_start + mapper.heads <= block.shape[3]:
        raise ValueError("Received source shard does not contain required heads")
    src = RowSet.from_page(block, head_offset=head_start)
    dst = RowSet.from_pool(target_pool, target_indices[start : start + n])
    if dst.heads != mapper.heads:
        raise ValueError("mapper output geometry/dtype mismatch")
    mapper.map_install(src, dst, n, position_start=start)


@torch.inference_mode()
def map_install_block(
    mapper,
    source_pool,
    source_indices,
    target_pool,
    target_indices,
    *,
    start,
    stop,
    source_head_offset=0,
    target_head_offset=0,
):
    """Fused pack + map + install of tokens ``[start, stop)`` of one request.

    Source rows ``source_indices[start:stop]`` of ``source_pool`` (which holds
    heads ``[source_head_offset, ...)`` of the source model) are mapped to this
    mapper's target heads and written to rows ``target_indices[start:stop]`` of
    ``target_pool`` at head ``target_head_offset``. ``target_pool`` may live on
    a peer GPU (its buffers opened through CUDA IPC).
    """
    n = stop - start
    if not (0 <= start < stop <= len(source_indices)) or stop > len(target_indices):
        raise ValueError("invalid block span")
    if target_pool.layer_num != mapper.target_layers or target_pool.dtype != source_pool.dtype:
        raise ValueError("mapper output geometry/dtype mismatch")
    # Headwise maps read this rank's heads of the source rows; dense maps all of them.
    head_start = 0 if mapper.dense else mapper.target_head_start - source_head_offset
    src = RowSet.from_pool(source_pool, source_indices[start:stop], head_offset=head_start)
    if not 0 <= head_start < head_start + mapper.source_heads <= src.heads:
        raise ValueError("Received source shard does not contain required heads")
    if hasattr(target_pool, "rows"):  # TokenKVPool, or a peer pool mapped through CUDA IPC
        dst = target_pool.rows(target_indices[start:stop], target_head_offset)
    else:
        dst = RowSet.from_pool(target_pool, target_indices[start:stop], head_offset=target_head_offset)
    if target_head_offset < 0 or target_head_offset + mapper.heads > dst.heads:
        raise ValueError("mapper output geometry/dtype mismatch")
    mapper.map_install(src, dst, n, position_start=start)


def install_unpublished(
    *,
    token_count,
    allocate,
    free,
    blocks,
    write,
    synchronize,
    ready_vote,
    publish,
    cancel_after_blocks=None,
):
    """Allocate, write ordered gap-free blocks, vote on all ranks, then publish.

    ``blocks`` yields ``(start, stop, value)``. Every rank reaches
    ``ready_vote`` even after a local failure; pages are freed exactly once on
    a local failure or a failed vote, never published while any rank is still
    writing, and kept (not freed) if the vote itself cannot complete, because a
    broken group cannot certify that all GPU writes stopped.
    """
    indices = None
    error = None
    written = 0
    cursor = 0
    try:
        indices = allocate(token_count)
        if indices is None:
            raise RuntimeError("target pool allocation failed")
        for start, stop, value in blocks:
            if start != cursor or not start < stop <= token_count or value.shape[2] != stop - start:
                raise ValueError("missing, duplicate or overlapping block")
            write(value, indices, start)
            synchronize()
            cursor = stop
            written += 1
            if cancel_after_blocks == written:
                raise RuntimeError("controlled cancellation before publication")
        if cursor != token_count:
            raise ValueError("incomplete prefix")
    except Exception as exc:  # noqa: BLE001 - every local failure must still vote
        error = exc
    synchronize()
    all_ready = ready_vote(error is None)  # a broken group propagates: pages stay owned
    if error is not None or not all_ready:
        if indices is not None:
            free(indices)
        raise RuntimeError("unpublished target transaction rolled back") from error
    publish(indices)
    return dict(tokens=cursor, blocks=written, published=True)
