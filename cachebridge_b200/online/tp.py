"""Tensor-parallel handoff: source rank r maps its KV heads straight into the
target pool of rank r + world/2 over NVLink.

Equal source and target TP (world = 2 * tp): source rank r owns KV heads
``[r * H_r, (r + 1) * H_r)`` of both models, so the work shards by head with
no exchange step (reference: ``PageMapper`` head slice, src/cachebridge/mapper.py:81-92,
and ``source_head_offset = rank * H_r`` at
backends/sglang/runtime/source_mapper_adapter.py:754-760). The only transfer is
one point-to-point stream per pair: the fused map kernel stores every mapped
row directly into the peer's pool through a CUDA IPC mapping (no staging
buffer), replacing the reference's export -> ``cudaMemcpyPeerAsync`` span
loop (backends/sglang/runtime/peer_adapter.py:211-282, peer_runtime.py:55-64)
and its IPC export (bounded_handoff_channel.py:83-123).

Publication follows install_unpublished (src/cachebridge/online/blocks.py:114-171)
and the all-rank vote of source_mapper_adapter.py:543-548: every rank votes
after its stream work, and the prefix is published only if all ranks are
ready.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..device import RawRows, RowSet, status_word


@dataclass(frozen=True)
class PairPlan:
    """Role of one rank in a source-TP + target-TP handoff on one node."""

    world: int
    rank: int
    tp: int             # source TP = target TP = world / 2
    role: str           # "source" or "target"
    tp_rank: int        # head-shard index of this rank on its side
    peer: int           # the other rank of this pair
    heads_per_rank: int
    head_start: int     # first KV head (of the full model) owned by the pair


def pair_plan(world: int, rank: int, total_heads: int) -> PairPlan:
    """Ranks [0, world/2) are source ranks, [world/2, world) target ranks; rank r
    pairs with r + world/2 and both own heads [tp_rank*H_r, (tp_rank+1)*H_r)."""
    if world < 2 or world % 2:
        raise ValueError("a sharded handoff needs an even world size >= 2 (source TP + target TP)")
    if not 0 <= rank < world:
        raise ValueError("rank outside the world")
    tp = world // 2
    if total_heads % tp:
        raise ValueError("KV heads must divide evenly across the tensor-parallel ranks")
    h = total_heads // tp
    if rank < tp:
        return PairPlan(world, rank, tp, "source", rank, rank + tp, h, rank * h)
    return PairPlan(world, rank, tp, "target", rank - tp, rank - tp, h, (rank - tp) * h)


def chunk_spans(n_tokens: int, chunk: int) -> list[tuple[int, int]]:
    """Ordered, gap-free ``[start, stop)`` token spans of at most ``chunk`` tokens."""
    if n_tokens < 0 or chunk <= 0:
        raise ValueError("token count must be >= 0 and chunk > 0")
    return [(a, min(a + chunk, n_tokens)) for a in range(0, n_tokens, chunk)]


class PeerPool:
    """A target pool owned by another process, mapped into this one.

    Layout of the exporter's ``TokenKVPool``: one allocation per kind
    ``[layers, rows, heads, head_dim]``. The mapping is made in the context of
    the GPU whose kernels store into it (``device``) with lazy peer access, so
    the fused map kernel writes the peer's rows directly over NVLink.
    """

    def __init__(self, exported: dict, device: torch.device):
        from .. import _native as nat

        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.layer_num, self.size, h, d = exported["shape"]
        self.start_layer = exported["start_layer"]
        self.dtype = getattr(torch, exported["dtype"])
        self._heads, self._head_dim = h, d
        self._lib = nat.load()
        self._bases = []
        ptrs = []
        for handle, offset in (exported["k"], exported["v"]):
            base = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(handle, 64)
            nat.check(self._lib.cb_ipc_open(buf, self.device.index, ctypes.byref(base)), "cb_ipc_open")
            self._bases.append(base.value)
            ptrs.append(base.value + offset)
        self._k, self._v = ptrs
        self.elem = torch.tensor([], dtype=self.dtype).element_size()

    @property
    def heads(self) -> int:
        return self._heads

    @property
    def head_dim(self) -> int:
        return self._head_dim

    def rows(self, slots: torch.Tensor | None = None, head_offset: int = 0) -> RawRows:
        row = self._heads * self._head_dim
        layer_bytes = self.size * row * self.elem
        return RawRows(
            [self._k + l * layer_bytes for l in range(self.layer_num)],
            [self._v + l * layer_bytes for l in range(self.layer_num)],
            self._heads, self._head_dim, self.size, row, self.dtype, self.device, head_offset, slots,
        )

    def close(self) -> None:
        """Unmap the peer allocations (after every kernel that uses them finished)."""
        from .. import _native as nat

        with torch.cuda.device(self.device):
            for base in self._bases:
                nat.check(self._lib.cb_ipc_close(ctypes.c_void_p(base)), "cb_ipc_close")
        self._bases = []


def export_pool(pool) -> dict:
    """Picklable CUDA IPC description of a ``TokenKVPool``'s K and V buffers."""
    from .. import _native as nat

    lib = nat.load()
    out = dict(shape=tuple(pool.k_buffer.shape), start_layer=int(pool.start_layer),
               dtype=str(pool.dtype).replace("torch.", ""))
    for name, buf in (("k", pool.k_buffer), ("v", pool.v_buffer)):
        if not buf.is_contiguous():
            raise ValueError("exported pool buffers must be contiguous")
        handle = ctypes.create_string_buffer(64)
        offset = ctypes.c_uint64()
        nat.check(lib.cb_ipc_export(ctypes.c_void_p(buf.data_ptr()), handle, ctypes.byref(offset)), "cb_ipc_export")
        out[name] = (handle.raw, int(offset.value))
    return out


def open_pool(exported: dict, device: torch.device) -> PeerPool:
    """Map a peer's exported pool for kernels running on ``device``."""
    return PeerPool(exported, device)


def exchange_target_pools(plan: PairPlan, target_pool, group=None, device=None):
    """All ranks call this; target ranks export their pool and every source rank
    gets its peer's pool mapped for ``device`` (None on target ranks)."""
    payload = export_pool(target_pool) if plan.role == "target" else None
    gathered = [None] * plan.world
    dist.all_gather_object(gathered, payload, group=group)
    if plan.role != "source":
        return None
    exported = gathered[plan.peer]
    if exported is None:
        raise RuntimeError(f"target rank {plan.peer} exported no pool")
    return open_pool(exported, device)


def publication_vote(ready: bool | torch.Tensor, group=None, device=None) -> torch.Tensor:
    """All-rank MIN vote; returns a 1-element int32 tensor (1 = publish).

    With a CUDA ``device`` the vote is enqueued on the current stream after
    this rank's work (``ready`` may be a device tensor, e.g. a status check);
    with ``device=None`` it runs on the host (gloo). Every rank must call it the
    same number of times, failures included.
    """
    if isinstance(ready, torch.Tensor):
        vote = ready.to(torch.int32).reshape(1)
    else:
        vote = torch.tensor([1 if ready else 0], dtype=torch.int32, device=device)
    dist.all_reduce(vote, op=dist.ReduceOp.MIN, group=group)
    return vote


def device_ready(device: torch.device) -> torch.Tensor:
    """1 on the device when no handoff kernel on ``device`` flagged an error."""
    return (status_word(device) == 0).to(torch.int32)


class ShardedHandoff:
    """The source side of one pair: prepared map+install calls for a set of
    requests, chunked, writing into the peer target pool.

    ``requests`` is a list of ``(source_slots, target_slots)`` device index
    tensors (token t of a request sits at position t). All calls share one
    key workspace sized for the largest chunk, reused in stream order.
    """

    def __init__(self, mapper, source_pool, target_pool, requests, *, chunk: int,
                 source_head_offset: int = 0, target_head_offset: int = 0):
        self.mapper = mapper
        self.calls = []
        head_start = mapper.target_head_start - source_head_offset
        biggest = max((min(chunk, len(s)) for s, _ in requests), default=0)
        ws_bytes = max(mapper.workspace_bytes(source_pool.dtype, biggest), 16)
        self.workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=mapper.device)
        for src_slots, dst_slots in requests:
            if len(src_slots) != len(dst_slots):
                raise ValueError("source and target slot lists differ in length")
            for a, b in chunk_spans(len(src_slots), chunk):
                src = RowSet.from_pool(source_pool, src_slots[a:b], head_offset=head_start)
                dst = (target_pool.rows(dst_slots[a:b], target_head_offset) if isinstance(target_pool, PeerPool)
                       else RowSet.from_pool(target_pool, dst_slots[a:b], head_offset=target_head_offset))
                self.calls.append(mapper.prepare(src, dst, b - a, a, workspace=self.workspace))
        self.tokens = sum(len(s) for s, _ in requests)

    @property
    def launches(self) -> int:
        """Kernel launches per ``run`` (two per chunk on the tensor-core path)."""
        return sum(2 if c.tensor_core else 1 for c in self.calls)

    def run(self) -> None:
        """Enqueue every chunk on the current stream."""
        for call in self.calls:
            call.run()
