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

Publication goes through ``online.transaction``: each request is a
``HandoffTransaction`` (target rows allocated unpublished, chunks recorded in
order), and ``commit`` waits for the rank's GPU work, votes on all ranks and
publishes, rolls back or quarantines (src/cachebridge/online/blocks.py:114-171,
source_mapper_adapter.py:543-548 and :1145-1237).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..device import RawRows, RowSet, install_rows, status_word
from .transaction import SlotLedger


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


RAW = "raw"        # a chunk crosses NVLink as raw source rows; the target maps it
MAPPED = "mapped"  # the source maps the chunk; the target installs the mapped rows


def mixed_chunk_modes(lengths, chunk: int, source_block: str | None) -> list[str]:
    """Placement of every chunk of every request (requests in order, chunks
    in token order). ``source_block`` None maps every chunk on the target;
    "early" / "tail" map the first / last chunk of each request on the source
    and the rest on the target (the mixed per-block policy of
    backends/sglang/runtime/mixed_channel.py:50-104, whose source block index
    is 0 or the last)."""
    if source_block not in (None, "early", "tail"):
        raise ValueError("mixed source block must be None, 'early' or 'tail'")
    modes = []
    for n in lengths:
        spans = chunk_spans(n, chunk)
        pick = None if source_block is None else (0 if source_block == "early" else len(spans) - 1)
        modes.extend(MAPPED if i == pick else RAW for i in range(len(spans)))
    return modes


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


class _Mapped:
    """A peer allocation (or part of one) mapped into this process for ``device``."""

    def __init__(self, exported: tuple, device: torch.device):
        from .. import _native as nat

        handle, offset = exported
        self._lib = nat.load()
        self.device = device
        base = ctypes.c_void_p()
        nat.check(self._lib.cb_ipc_open(ctypes.create_string_buffer(handle, 64), device.index, ctypes.byref(base)),
                  "cb_ipc_open")
        self.base = base.value
        self.ptr = base.value + offset

    def close(self) -> None:
        from .. import _native as nat

        if self.base is not None:
            with torch.cuda.device(self.device):
                nat.check(self._lib.cb_ipc_close(ctypes.c_void_p(self.base)), "cb_ipc_close")
            self.base = None


def _export(t: torch.Tensor) -> tuple:
    from .. import _native as nat

    handle = ctypes.create_string_buffer(64)
    offset = ctypes.c_uint64()
    nat.check(nat.load().cb_ipc_export(ctypes.c_void_p(t.data_ptr()), handle, ctypes.byref(offset)), "cb_ipc_export")
    return handle.raw, int(offset.value)


class TargetPlacement:
    """Target-side placement for one source/target pair.

    The source rank gathers each chunk's raw source KV rows (its H_r heads of
    every source layer) into one of two receive slots on the target GPU:
    either stored straight into the peer slot by the gather kernel
    (``transport="peer_stores"``, the default: coalesced NVLink stores,
    691 GB/s at TP1+TP1), or staged locally and moved by one copy-engine
    transfer per chunk on a second stream (``"copy_engine"``: 603 GB/s). The target rank maps the received block into its own pool
    (``cb_map_install``: derotation, map, target RoPE, install through the
    slot table). Raw source rows are 2*L_s*H_r*D*2 bytes per token against
    2*L_t*H_r*D*2 mapped, so fewer bytes cross NVLink than with source-side
    placement. Slot reuse is ordered on the GPUs by int64 counters
    (``cb_chunk_signal`` / ``cb_chunk_wait``): the source waits until the
    target has consumed the chunk that last used a slot, the target waits
    until the chunk it maps has arrived.

    Reference: target placement of backends/sglang/runtime/receiver_mapping.py:89-242
    and native_source.py:29-108, with the double-buffered slots of
    source_mapper_adapter.py:197-232 / 282-324.

    Mixed placement (``mixed_source_block`` "early" or "tail"): one chunk of
    each request is mapped on the source instead, straight into the receive
    slot as a dense mapped page (the map kernel's stores go over NVLink), and
    the target installs it with one row scatter; the receive slots are sized
    for the larger of the raw and the mapped chunk. The source then needs the
    ``mapper`` too (peer stores only).

    Every rank of the pair builds one with the same ``requests`` (lists of
    ``(source_slots, target_slots)`` device tensors) and ``chunk``; the source
    passes ``source_pool``, the target ``mapper`` and ``target_pool``. The
    constructor is collective over ``group`` (all ranks of the world). On the
    target, the prepared calls read each request's target rows from a buffer
    of their own: ``set_target_rows`` replaces them (for rows allocated per
    handoff), ``target_slots`` starts them. Host-side ownership of the receive
    slots is kept in a ``SlotLedger``: a chunk claims its slot, and the slot
    is settled when the next chunk that uses it is queued behind the device
    wait for its consumption.
    """

    def __init__(self, plan: PairPlan, requests, *, chunk: int, source_layers: int, device: torch.device,
                 group=None, source_pool=None, mapper=None, target_pool=None, timeout_s: float = 10.0,
                 transport: str = "peer_stores", slots: int = 2, mixed_source_block: str | None = None):
        from .. import _native as nat
        from ..device import storage_dtype_code

        if transport not in ("copy_engine", "peer_stores"):
            raise ValueError("transport must be 'copy_engine' or 'peer_stores'")
        if slots < 2:
            raise ValueError("target placement needs at least two receive slots")
        self.SLOTS = slots  # receive slots on the target (chunks in flight)
        self.plan = plan
        self.transport = transport
        self.device = torch.device(device)
        self.lib = nat.load()
        self.timeout_ns = int(timeout_s * 1e9)
        self.chunks = [(q, a, b) for q, (s, _) in enumerate(requests) for a, b in chunk_spans(len(s), chunk)]
        self.modes = mixed_chunk_modes([len(s) for s, _ in requests], chunk, mixed_source_block)
        if mixed_source_block is not None and (mapper is None or transport != "peer_stores"):
            raise ValueError("mixed placement needs the mapper on both ranks and peer stores")
        self.counter = 0  # chunks enqueued so far, over all runs (the signalled values)
        self.last_use = [-1] * self.SLOTS  # counter of the chunk that last used each slot
        self.status = status_word(self.device)
        H, D = plan.heads_per_rank, None
        if plan.role == "source":
            D = source_pool.head_dim
            dtype = source_pool.dtype
        else:
            D = target_pool.head_dim
            dtype = target_pool.dtype
        self.dtype_code = storage_dtype_code(dtype)
        self.head_dim = D
        elem = torch.tensor([], dtype=dtype).element_size()
        target_layers = mapper.target_layers if mapper is not None else source_layers
        layers_in_slot = max(source_layers if RAW in self.modes else 0, target_layers if MAPPED in self.modes else 0)
        slot_elems = 2 * layers_in_slot * chunk * H * D
        self.slot_bytes = slot_elems * elem
        # Counters start at -1: nothing arrived, nothing consumed.
        flags = torch.full((self.SLOTS,), -1, dtype=torch.int64, device=self.device)
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        if plan.role == "target":
            self.recv = torch.empty((self.SLOTS, slot_elems), dtype=dtype, device=self.device)
            payload = dict(recv=_export(self.recv), ready=_export(flags), uuid=uuid, slots=self.SLOTS, chunk=chunk)
        else:
            payload = dict(consumed=_export(flags), uuid=uuid, slots=self.SLOTS, chunk=chunk)
        self.flags = flags
        self.ledger = SlotLedger(self.SLOTS, restart_on_open=True)
        self.request_tokens = [len(s) for s, _ in requests]
        self.bytes_per_token = {RAW: 2 * source_layers * H * D * elem, MAPPED: 2 * target_layers * H * D * elem}
        torch.cuda.synchronize(self.device)
        gathered = [None] * plan.world
        dist.all_gather_object(gathered, payload, group=group)
        peer = gathered[plan.peer]
        if (peer["slots"], peer["chunk"]) != (self.SLOTS, chunk):
            raise ValueError("source and target of a pair must use the same receive slots and chunk size")
        if peer["uuid"] == uuid:
            # The two sides wait on each other's kernels: they must be different GPUs.
            raise ValueError("source and target ranks of a pair share one GPU; target placement needs two")
        self._mapped = []
        if plan.role == "source":
            recv = _Mapped(peer["recv"], self.device)
            ready = _Mapped(peer["ready"], self.device)
            self._mapped = [recv, ready]
            self.peer_recv = [recv.ptr + s * self.slot_bytes for s in range(self.SLOTS)]
            self.peer_ready = [ready.ptr + 8 * s for s in range(self.SLOTS)]
            self.src_rows = []
            self.src_calls = {}
            for i, (q, a, b) in enumerate(self.chunks):
                rs = RowSet.from_pool(source_pool, requests[q][0][a:b])
                self.src_rows.append((rs, rs.to_c()))
                if self.modes[i] == MAPPED:
                    # Map on the source into the peer slot as a dense [2, L_t, n, H, D] page.
                    n, row = b - a, H * D
                    base = self.peer_recv[i % self.SLOTS]
                    page = RawRows([base + l * n * row * elem for l in range(target_layers)],
                                   [base + (target_layers + l) * n * row * elem for l in range(target_layers)],
                                   H, D, n, row, dtype, self.device)
                    self.src_calls[i] = mapper.prepare(rs, page, n, a)
            self.row_heads = source_pool.heads
            self.chunk_bytes = [2 * source_layers * (b - a) * H * D * elem for _, a, b in self.chunks]
            if transport == "copy_engine":
                # Packed chunks are staged locally, then one copy-engine transfer
                # per chunk moves them over NVLink on a second stream while the
                # next chunk is gathered.
                self.staging = torch.empty((self.SLOTS, slot_elems), dtype=dtype, device=self.device)
                self.copy_stream = torch.cuda.Stream(self.device)
                self.packed = [torch.cuda.Event() for _ in range(self.SLOTS)]
                self.copied = [torch.cuda.Event() for _ in range(self.SLOTS)]
                self.copied_recorded = [False] * self.SLOTS
        else:
            consumed = _Mapped(peer["consumed"], self.device)
            self._mapped = [consumed]
            self.peer_consumed = [consumed.ptr + 8 * s for s in range(self.SLOTS)]
            # One key workspace, sized for the largest chunk, shared in stream order.
            biggest = max((b - a for _, a, b in self.chunks), default=0)
            ws = torch.empty(max(mapper.workspace_bytes(dtype, biggest), 16), dtype=torch.uint8, device=self.device)
            self.workspace_bytes = ws.numel() + self.SLOTS * self.slot_bytes
            # Each request's target rows, read by its prepared calls.
            self.target_rows = [t.to(self.device, torch.int64).clone() for _, t in requests]
            self.calls = []
            self.installs = {}
            for i, (q, a, b) in enumerate(self.chunks):
                n = b - a
                if self.modes[i] == MAPPED:
                    # The source mapped this chunk: install the slot's page.
                    block = self.recv[i % self.SLOTS, : 2 * target_layers * n * H * D].view(2, target_layers, n, H, D)
                    self.installs[i] = (block, target_pool.rows(self.target_rows[q][a:b]))
                    self.calls.append(None)
                    continue
                page = self.recv[i % self.SLOTS, : 2 * source_layers * n * H * D].view(2, source_layers, n, H, D)
                self.calls.append(mapper.prepare(RowSet.from_page(page), target_pool.rows(self.target_rows[q][a:b]), n,
                                                 a, workspace=ws))

    @property
    def launches(self) -> int:
        """Kernel launches per ``run`` on this rank."""
        if self.plan.role == "source":
            return sum(4 if m == MAPPED else 3 for m in self.modes)
        return sum(3 if c is None else (4 if c.tensor_core else 3) for c in self.calls)

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def set_target_rows(self, request: int, rows: torch.Tensor) -> None:
        """Target rank: install request ``request`` into ``rows`` (a device
        index tensor of the request's length) from the next ``run`` on; the
        copy is queued on the current stream."""
        if self.plan.role != "target":
            raise RuntimeError("only the target rank owns target rows")
        if rows is None or rows.numel() != self.target_rows[request].numel():
            raise ValueError("target rows must match the request's token count")
        self.target_rows[request].copy_(rows, non_blocking=True)

    def run(self, transactions=None) -> None:
        """Enqueue every chunk of every request on the current stream.

        ``transactions`` (one ``HandoffTransaction`` per request, optional)
        receive each chunk as it is queued, with its logical bytes: raw source
        rows on either rank. The device pipeline queues every chunk even after
        a transaction failed, so both ranks' device handshakes stay paired;
        the failed transaction is rolled back at commit.
        """
        from .. import _native as nat

        st = self._stream()
        status = self.status.data_ptr()
        self.ledger.open()
        for i in range(len(self.chunks)):
            c = self.counter
            slot = i % self.SLOTS  # fixed per chunk: the target's prepared calls read it
            if self.ledger.held[slot]:
                # Its previous chunk's consumption is awaited on the device before reuse.
                self.ledger.settle(slot, gpu_reads_complete=True)
            q, a, b = self.chunks[i]
            self.ledger.claim(slot, self.ledger.next_start, self.ledger.next_start + (b - a))
            if transactions is not None:
                transactions[q].chunk(a, b, copy_bytes=(b - a) * self.bytes_per_token[self.modes[i]])
            if self.plan.role == "source" and self.transport == "copy_engine":
                self._send_staged(i, slot, c, st, status)
            elif self.plan.role == "source":
                # The chunk that last used this slot must have been consumed.
                nat.check(self.lib.cb_chunk_wait(st, ctypes.c_void_p(self.flags.data_ptr() + 8 * slot),
                                                 self.last_use[slot], self.timeout_ns, status), "cb_chunk_wait")
                if self.modes[i] == MAPPED:
                    self.src_calls[i].run()
                else:
                    rs, crow = self.src_rows[i]
                    nat.check(self.lib.cb_pack_rows(st, ctypes.byref(crow), self.head_dim, self.dtype_code,
                                                    rs.slots.numel(), ctypes.c_void_p(self.peer_recv[slot]), status),
                              "cb_pack_rows")
                nat.check(self.lib.cb_chunk_signal(st, ctypes.c_void_p(self.peer_ready[slot]), c),
                          "cb_chunk_signal")
            else:
                nat.check(self.lib.cb_chunk_wait(st, ctypes.c_void_p(self.flags.data_ptr() + 8 * slot), c,
                                                 self.timeout_ns, status), "cb_chunk_wait")
                if self.modes[i] == MAPPED:
                    block, dst = self.installs[i]
                    install_rows(block, dst, b - a)
                else:
                    self.calls[i].run()
                nat.check(self.lib.cb_chunk_signal(st, ctypes.c_void_p(self.peer_consumed[slot]), c),
                          "cb_chunk_signal")
            self.last_use[slot] = c
            self.counter += 1
        for slot in range(self.SLOTS):
            if self.ledger.held[slot]:
                self.ledger.settle(slot, gpu_reads_complete=True)  # awaited by the next run's device waits
        self.ledger.close()
        if self.plan.role == "source" and self.transport == "copy_engine":
            # Later work on the caller's stream (the vote) follows every transfer.
            current = torch.cuda.current_stream(self.device)
            for slot in range(self.SLOTS):
                if self.copied_recorded[slot]:
                    current.wait_event(self.copied[slot])

    def _send_staged(self, i: int, slot: int, c: int, st, status: int) -> None:
        """Gather chunk i into local staging slot `slot` on the caller's stream,
        then (copy stream) wait until the target consumed the receive slot's
        previous chunk, copy the chunk over NVLink and signal its arrival."""
        from .. import _native as nat

        current = torch.cuda.current_stream(self.device)
        if self.copied_recorded[slot]:
            current.wait_event(self.copied[slot])  # the staging slot's last transfer is done
        rs, crow = self.src_rows[i]
        staged = self.staging[slot].data_ptr()
        nat.check(self.lib.cb_pack_rows(st, ctypes.byref(crow), self.head_dim, self.dtype_code, rs.slots.numel(),
                                        ctypes.c_void_p(staged), status), "cb_pack_rows")
        self.packed[slot].record(current)
        cs = self.copy_stream
        cs.wait_event(self.packed[slot])
        cst = ctypes.c_void_p(cs.cuda_stream)
        nat.check(self.lib.cb_chunk_wait(cst, ctypes.c_void_p(self.flags.data_ptr() + 8 * slot), self.last_use[slot],
                                         self.timeout_ns, status), "cb_chunk_wait")
        nat.check(self.lib.cb_copy_async(cst, ctypes.c_void_p(self.peer_recv[slot]), ctypes.c_void_p(staged),
                                         self.chunk_bytes[i]), "cb_copy_async")
        nat.check(self.lib.cb_chunk_signal(cst, ctypes.c_void_p(self.peer_ready[slot]), c), "cb_chunk_signal")
        self.copied[slot].record(cs)
        self.copied_recorded[slot] = True

    def close(self) -> None:
        """Unmap the peer buffers (after this rank's stream work finished)."""
        for m in self._mapped:
            m.close()
        self._mapped = []
