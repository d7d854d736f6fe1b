"""Publication transactions of the online handoff.

A handoff installs rows into the target pool that no request may read until
every rank can vouch for its part. The rows are allocated unpublished, the
chunks of the history land in order and without gaps, every rank waits for
its own GPU work and votes, and only then are the rows published. The outcomes
and the obligations that come with them are the reference's
(src/cachebridge/online/blocks.py:114-171 install_unpublished;
backends/sglang/runtime/source_mapper_adapter.py:543-548 vote,
:1145-1237 commit, :824-825 and :1168-1171 quarantine):

  published    every rank is ready: the rows become visible to the cache.
  rolled_back  some rank reported a local failure (allocation, an ordering
               error, a device status bit, a cancellation): the rows are freed
               exactly once, on the rank that owns them.
  quarantined  some rank cannot certify that its GPU reads and writes have
               stopped, or the vote itself fails (a broken group proves
               nothing): the rows stay owned, nothing is freed or published,
               and the request needs reconciliation.

This module is engine-independent: ``SlotAllocator`` stands in for the
engine's token allocator, ``publish`` for its radix-cache insert. Several
requests are voted on together in one all-reduce.
"""

from __future__ import annotations

import time
import zlib
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch
import torch.distributed as dist

PUBLISHED = "published"
ROLLED_BACK = "rolled_back"
QUARANTINED = "quarantined"


class TransactionError(RuntimeError):
    """A transaction ended without publication; ``outcome`` says how."""

    def __init__(self, message: str, outcome: str, receipts=None):
        super().__init__(message)
        self.outcome = outcome
        self.receipts = receipts or []


class DeviceDataError(RuntimeError):
    """The device reported a data error (a status bit) but the GPU is usable:
    the rank's work has stopped, so a rollback is safe."""


# ---------------------------------------------------------------------------
# Target rows
# ---------------------------------------------------------------------------
class SlotAllocator:
    """Free rows of a token pool, kept on the device (page_size 1).

    ``allocate(n)`` hands out the next n free rows as a device index tensor
    (or None when fewer than n are free); ``free(indices)`` returns an
    allocation. Every allocation is returned exactly once: freeing rows that
    are not currently allocated raises. The initial order of the free list is
    a seeded permutation, so placements are random over the pool like a
    fragmented engine pool's.
    """

    def __init__(self, rows: int, *, device, seed: int | None = 0, reserved: int = 0):
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        order = torch.randperm(rows, generator=g) if g is not None else torch.arange(rows)
        order = order[order >= reserved] if reserved else order
        self.device = torch.device(device)
        self._free = order.to(self.device, torch.int64)
        self._head = 0  # rows before _head are handed out
        self._live: dict[int, int] = {}  # data_ptr -> length of each live allocation

    @classmethod
    def from_free_rows(cls, free_rows: torch.Tensor) -> "SlotAllocator":
        """An allocator over an explicit free list (e.g. a pool whose other
        rows hold other requests); rows are handed out in the list's order."""
        alloc = cls(0, device=free_rows.device, seed=None)
        alloc._free = free_rows.to(torch.int64)
        return alloc

    @property
    def free_rows(self) -> int:
        return self._free.numel() - self._head

    def allocate(self, n: int):
        if n <= 0 or n > self.free_rows:
            return None
        out = self._free[self._head : self._head + n]
        self._head += n
        self._live[out.data_ptr()] = n
        return out

    def free(self, indices: torch.Tensor) -> None:
        key = indices.data_ptr()
        if self._live.get(key) != indices.numel():
            raise RuntimeError("rows freed twice or never allocated")
        del self._live[key]
        rest = self._free[self._head :]
        # Returned rows go to the back of the free list (device-side copy).
        self._free = torch.cat((rest, indices.to(self.device, torch.int64)))
        self._head = 0


# ---------------------------------------------------------------------------
# Transfer buffers
# ---------------------------------------------------------------------------
class SlotLedger:
    """Ownership of reusable transfer buffers by the chunks of one handoff.

    A chunk claims a buffer that no earlier chunk still holds, and chunks are
    claimed in order without gaps. A buffer is settled (free again) only once
    the consumer's GPU reads of it are known to be complete; the ledger closes
    only when no buffer is held. ``acquire`` / ``release`` bracket the
    ownership of the source data the buffers are filled from (a radix-cache
    lock in the engine).
    """

    def __init__(self, buffers: int, acquire: Callable | None = None, release: Callable | None = None,
                 *, restart_on_open: bool = True, messages: dict | None = None):
        if buffers < 1:
            raise ValueError("a ledger needs at least one buffer")
        self._acquire = acquire or (lambda: None)
        self._release = release or (lambda: None)
        self._restart = restart_on_open
        self.held = [False] * buffers
        self.is_open = False
        self.next_start = 0
        self._msg = dict(open="ledger already open", order="chunk ownership/order violation",
                         settle="consumer GPU completion required before buffer reuse",
                         close="cannot close the ledger with buffers still held")
        self._msg.update(messages or {})

    def open(self) -> None:
        if self.is_open:
            raise RuntimeError(self._msg["open"])
        self._acquire()
        self.is_open = True
        if self._restart:
            self.next_start = 0

    def claim(self, buffer: int, start: int, stop: int) -> None:
        ok = self.is_open and not self.held[buffer] and start == self.next_start and stop > start
        if not ok:
            raise RuntimeError(self._msg["order"])
        self.held[buffer] = True
        self.next_start = stop

    def settle(self, buffer: int, *, gpu_reads_complete: bool) -> None:
        if not (self.is_open and self.held[buffer] and gpu_reads_complete):
            raise RuntimeError(self._msg["settle"])
        self.held[buffer] = False

    def close(self) -> None:
        if not self.is_open or any(self.held):
            raise RuntimeError(self._msg["close"])
        self._release()
        self.is_open = False


# ---------------------------------------------------------------------------
# Transactions
# ---------------------------------------------------------------------------
@dataclass
class HandoffTransaction:
    """One request's unpublished install as seen by one rank.

    A target rank passes ``allocate`` / ``free`` / ``publish``; a source rank
    passes none of them and only reports its chunks. ``chunk`` records each
    enqueued chunk and refuses an out-of-order or overlapping one (which marks
    the transaction failed). Byte counters feed the receipt.
    """

    request_id: str
    tokens: int
    rank: int = 0
    allocate: Callable | None = None
    free: Callable | None = None
    publish: Callable | None = None
    cancel_after_chunks: int | None = None
    indices: torch.Tensor | None = None
    cursor: int = 0
    chunks: int = 0
    copy_bytes: int = 0
    transfer_workspace_bytes: int = 0
    placement_runs: int = 0
    error: BaseException | None = None
    outcome: str | None = None
    completion_ns: int = 0
    _freed: bool = field(default=False, repr=False)

    def begin(self):
        """Allocate the unpublished target rows (target ranks); returns them."""
        if self.allocate is None:
            return None
        try:
            self.indices = self.allocate(self.tokens)
        except Exception as exc:  # noqa: BLE001 - a failed allocation is a local failure
            self.fail(exc)
            return None
        if self.indices is None:
            self.fail(RuntimeError("target pool allocation failed"))
        return self.indices

    def chunk(self, start: int, stop: int, *, copy_bytes: int = 0, runs: int = 1) -> bool:
        """Record tokens [start, stop) as enqueued; False once the transaction failed."""
        if self.error is not None:
            return False
        if start != self.cursor or not start < stop <= self.tokens:
            self.fail(ValueError("missing, duplicate or overlapping block"))
            return False
        self.cursor = stop
        self.chunks += 1
        self.copy_bytes += copy_bytes
        self.placement_runs += runs
        if self.cancel_after_chunks == self.chunks:
            self.fail(RuntimeError("controlled cancellation before publication"))
            return False
        return True

    def fail(self, exc: BaseException) -> None:
        if self.error is None:
            self.error = exc

    @property
    def ready(self) -> bool:
        if self.error is None and self.cursor != self.tokens:
            self.fail(ValueError("incomplete prefix"))
        return self.error is None

    def _free_once(self) -> None:
        if self.indices is not None and self.free is not None and not self._freed:
            self._freed = True
            self.free(self.indices)

    def receipt(self) -> dict:
        return dict(request_id=self.request_id, rank=self.rank, outcome=self.outcome, tokens=self.cursor,
                    blocks=self.chunks, logical_copy_bytes=self.copy_bytes,
                    target_transfer_workspace_bytes=self.transfer_workspace_bytes,
                    target_placement_runs=self.placement_runs,
                    certified_data_completion_ns=self.completion_ns,
                    error=None if self.error is None else repr(self.error))


def device_settle(device, stream=None) -> Callable[[], None]:
    """``settle`` for ``commit``: wait for the stream's work on ``device``, then
    read (and clear) its status word. A status bit raises ``DeviceDataError``
    (the work stopped: a rollback is safe); a CUDA error raises through (the
    rank cannot certify that its GPU work stopped)."""

    def settle() -> None:
        from ..device import read_status

        (stream or torch.cuda.current_stream(device)).synchronize()
        bits = read_status(device)
        if bits:
            raise DeviceDataError(f"handoff kernels reported device status {bits}")

    return settle


def gloo_vote(group=None) -> Callable[[Sequence[int]], list[int]]:
    """All-rank MIN of a vector of 0/1 flags over a (CPU) process group."""

    def vote(flags: Sequence[int]) -> list[int]:
        t = torch.tensor(list(flags), dtype=torch.int32)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
        return [int(x) for x in t.tolist()]

    return vote


def _identity(request_id: str) -> int:
    """31-bit identity of a request id, equal on every rank for equal ids."""
    return zlib.crc32(request_id.encode()) & 0x7FFFFFFF


def commit(transactions: Sequence[HandoffTransaction], *, settle: Callable[[], None],
           vote: Callable[[Sequence[int]], list[int]], expected_ids: Sequence[str] | None = None) -> list[dict]:
    """Certify, vote and publish a set of transactions on one rank.

    Every rank calls this with its transactions for the same requests, in the
    same order, whatever happened locally. ``settle`` waits for this rank's GPU
    work on the transactions and checks its device status: it raises
    ``DeviceDataError`` for a data error (the rank's work has stopped: safe to
    roll back) and anything else when it cannot certify that the work stopped.
    A transaction whose id differs from ``expected_ids`` (the caller's view of
    the request being committed), or from the id other ranks commit at the
    same position, is not ready.

    The first vote carries ready per transaction and safe for the rank. Not
    safe anywhere -> all quarantined. Not ready anywhere -> that transaction is
    rolled back (its rows freed once). The second vote is on the local
    publication of the rest:
    a publication that failed on any rank leaves the transaction quarantined.
    A vote that raises quarantines every transaction still open. Returns this
    rank's receipts; raises ``TransactionError`` (with the receipts) unless
    every transaction was published.
    """
    txns = list(transactions)
    if expected_ids is not None:
        if len(expected_ids) != len(txns):
            raise ValueError("one expected request id per transaction")
        for t, rid in zip(txns, expected_ids):
            if t.request_id != rid:
                t.fail(RuntimeError("source-mapped transaction identity mismatch"))
    safe = True
    try:
        settle()
    except DeviceDataError as exc:
        for t in txns:
            t.fail(exc)
    except Exception as exc:  # noqa: BLE001 - cannot certify that GPU work stopped
        safe = False
        for t in txns:
            t.fail(exc)
    now = time.perf_counter_ns()
    for t in txns:
        t.completion_ns = now
    k = len(txns)
    ids = [_identity(t.request_id) for t in txns]
    # One all-reduce (MIN): ready flags, the safe flag, and each identity as
    # +id and -id, whose minima give the smallest and the largest id.
    flags = [int(t.ready) for t in txns] + [int(safe)] + ids + [-i for i in ids]
    try:
        agreed = vote(flags)
    except Exception as exc:  # noqa: BLE001 - a broken group certifies nothing
        for t in txns:
            t.outcome = QUARANTINED
            t.fail(exc)
        raise TransactionError("publication vote failed; ownership retained", QUARANTINED,
                               [t.receipt() for t in txns]) from exc
    lo, neg_hi = agreed[k + 1 : 2 * k + 1], agreed[2 * k + 1 :]
    agreed = agreed[: k + 1]
    for i, t in enumerate(txns):
        if lo[i] != -neg_hi[i]:
            t.fail(RuntimeError("source-mapped transaction identity mismatch"))
            agreed[i] = 0
    if not agreed[-1]:
        for t in txns:
            t.outcome = QUARANTINED
        raise TransactionError("cannot certify source-mapped reads/pool writes", QUARANTINED,
                               [t.receipt() for t in txns])
    published_here = []
    for t, ok in zip(txns, agreed[:-1]):
        if not ok:
            t.outcome = ROLLED_BACK
            t._free_once()
            published_here.append(1)  # nothing to publish: agrees with any outcome
            continue
        try:
            if t.publish is not None:
                t.publish(t.indices)
            published_here.append(1)
        except Exception as exc:  # noqa: BLE001
            t.fail(exc)
            published_here.append(0)
    try:
        confirmed = vote(published_here)
    except Exception as exc:  # noqa: BLE001
        confirmed = [0] * len(txns)
        for t in txns:
            t.fail(exc)
    for t, ok in zip(txns, confirmed):
        if t.outcome == ROLLED_BACK:
            continue
        t.outcome = PUBLISHED if ok else QUARANTINED
    receipts = [t.receipt() for t in txns]
    outcomes = {t.outcome for t in txns}
    if outcomes != {PUBLISHED}:
        worst = QUARANTINED if QUARANTINED in outcomes else ROLLED_BACK
        msg = ("unpublished target transaction rolled back" if worst == ROLLED_BACK
               else "source-mapped publication failed; ownership retained")
        first_error = next((t.error for t in txns if t.error is not None), None)
        raise TransactionError(msg, worst, receipts) from first_error
    return receipts
