"""Block primitives of the online handoff: pack, map+install, unpublished install.

Drop-in for ``cachebridge.online.blocks`` (src/cachebridge/online/blocks.py,
duplicated in backends/sglang/runtime/bounded_cachebridge_core.py):

- ``SourceLease``           single in-flight block ownership (blocks.py:11-43), a
                            one-buffer ``SlotLedger``
- ``pack_source_block``     gather pool rows into one contiguous workspace
                            (blocks.py:47-82), one ``cb_pack_rows`` launch instead
                            of 2*layers ``index_select`` launches
- ``map_write_block``       map a packed block and install it into target pool
                            rows (blocks.py:86-111), one fused launch pair instead
                            of map_page + per-layer ``set_kv_buffer``
- ``map_install_block``     the fully fused source-pool -> target-pool path (no
                            packed block at all): gather, map and install
- ``install_unpublished``   publish-after-vote transaction (blocks.py:114-171), run
                            on a ``HandoffTransaction`` (online/transaction.py)
"""

from __future__ import annotations

import torch

from ..device import RowSet, pack_rows
from .transaction import HandoffTransaction, SlotLedger


class SourceLease(SlotLedger):
    """Single in-flight block; release is legal only after consumer completion.

    The reference's one-buffer lease (online/blocks.py:11-43) as a
    ``SlotLedger`` of one buffer: ``begin`` opens it (restarting at token 0),
    ``export`` claims the buffer for the next ordered block, ``acknowledge``
    settles it once the consumer's GPU reads completed, ``close`` releases.
    The error messages are the reference's, which callers match on.
    """

    def __init__(self, acquire, release):
        super().__init__(1, acquire, release, restart_on_open=True, messages=dict(
            open="source lease already active", order="block ownership/order violation",
            settle="consumer GPU completion required before buffer reuse",
            close="cannot release source lease with outstanding GPU reads"))

    @property
    def active(self) -> bool:
        return self.is_open

    @property
    def pending(self) -> bool:
        return self.held[0]

    def begin(self):
        self.open()

    def export(self, start, stop):
        self.claim(0, start, stop)

    def acknowledge(self, *, gpu_reads_complete):
        self.settle(0, gpu_reads_complete=gpu_reads_complete)


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

    The reference's single-round contract (online/blocks.py:114-171), run on a
    ``HandoffTransaction``: ``blocks`` yields ``(start, stop, value)``; each
    block is checked for order before ``write(value, indices, start)`` and
    counted after ``synchronize()``; a cancellation point counts written
    blocks. Every rank reaches ``ready_vote`` even after a local failure. On a
    local failure or a failed vote the rows are freed exactly once and
    ``RuntimeError("unpublished target transaction rolled back")`` is raised;
    if ``synchronize`` or the vote itself raises, the exception propagates and
    the rows stay owned (a broken group cannot certify that GPU writes
    stopped). Returns ``{"tokens", "blocks", "published"}``.
    """
    txn = HandoffTransaction("install_unpublished", token_count, allocate=allocate, free=free,
                             cancel_after_chunks=cancel_after_blocks)
    indices = txn.begin()
    if txn.error is None:
        try:
            for start, stop, value in blocks:
                if start != txn.cursor or not start < stop <= token_count or value.shape[2] != stop - start:
                    raise ValueError("missing, duplicate or overlapping block")
                write(value, indices, start)
                synchronize()
                if not txn.chunk(start, stop):
                    break
        except Exception as exc:  # noqa: BLE001 - every local failure must still vote
            txn.fail(exc)
    synchronize()
    all_ready = ready_vote(txn.ready)  # raises through: the rows stay owned
    if not (txn.ready and all_ready):
        txn._free_once()
        raise RuntimeError("unpublished target transaction rolled back") from txn.error
    publish(indices)
    return dict(tokens=txn.cursor, blocks=txn.chunks, published=True)
