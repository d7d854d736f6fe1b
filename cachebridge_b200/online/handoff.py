"""Handoff coordination and a local endpoint served by the GPU handoff path.

``HandoffRequest`` and ``run_handoff`` keep the engine-independent protocol of
src/cachebridge/online/handoff.py:1-127: start the target, then the source;
collect both replies; then poll ``try_publish`` until every target rank
reports one consistent publication with complete GPU-completion receipts. A
stale, partial or unfenced publication is an error. A timeout leaves every
resource owned by the backend. ``run_handoff`` never frees pages.

``LocalHandoffEndpoint`` implements the endpoint protocol (``start`` /
``receive`` / ``try_publish``) for one process that holds the source pool,
the target pool and the mapper (one target rank). The source start enqueues
the whole history as ``map_install_block`` chunks of ``block_tokens`` on one
stream and records a CUDA event. ``try_publish`` answers "pending" until that
event completes. It then checks the device status word, publishes the target
slots exactly once and returns the receipt fields the coordinator requires.
They are derived from the GPU completion, so ``certified_data_completion_ns``
is the host time at which the completion was first observed.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, Protocol

import torch


class HandoffEndpoint(Protocol):
    def start(self, role, parameters): ...
    def receive(self, role, deadline): ...
    def try_publish(self, label, parameters): ...


RECEIPT_FIELDS = (
    "worker_done",
    "worker_thread_exited",
    "all_rank_ready",
    "original_commit_stack_called",
    "certified_data_completion_ns",
)


@dataclass(frozen=True)
class HandoffRequest:
    """One request's history handoff (online/handoff.py:14-52)."""

    request_id: str
    phase: str
    history_ids: tuple[int, ...]
    namespace: str
    target_ranks: int = 4
    block_tokens: int = 2048

    def __post_init__(self):
        for name in ("request_id", "phase", "namespace"):
            value = getattr(self, name)
            if not isinstance(value, str) or not value:
                raise ValueError("A handoff requires request, phase and namespace identities")
        ids = self.history_ids
        if not ids or any(type(i) is not int or i < 0 for i in ids):
            raise ValueError("history_ids must contain non-negative token IDs")
        for count in (self.target_ranks, self.block_tokens):
            if type(count) is not int or count <= 0:
                raise ValueError("Rank and block counts must be positive integers")

    def parameters(self) -> dict:
        return {
            "action": "online_stage_start",
            "phase": self.phase,
            "request_id": self.request_id,
            "history_ids": list(self.history_ids),
            "mapper_kind": "CacheBridge",
            "execution": "double",
            "block_tokens": self.block_tokens,
            "cache_namespace": self.namespace,
            "source_pipeline": "double",
            "instrument_gpu_stages": False,
        }


def _check_rows(rows, request: HandoffRequest, label: str) -> set:
    if len(rows) != request.target_ranks:
        raise RuntimeError("Stale or incomplete all-rank publication identity")
    for rank, row in enumerate(rows):
        identity = (row.get("phase"), row.get("transaction_phase"), row.get("request_id"), row.get("rank"))
        if identity != (label, request.phase, request.request_id, rank) or not row.get("all_rank_identity_valid"):
            raise RuntimeError("Stale or incomplete all-rank publication identity")
    return {row.get("outcome") for row in rows}


def run_handoff(endpoint: HandoffEndpoint, request: HandoffRequest, *, timeout=120, poll_interval=0.002) -> dict:
    """Start both peers, then require complete all-rank publication evidence
    (online/handoff.py:55-127). On failure every outstanding resource stays with
    the backend: a timeout does not prove that GPU work stopped."""
    if timeout <= 0 or poll_interval < 0:
        raise ValueError("Invalid handoff timeout or polling interval")
    parameters = request.parameters()
    began = time.perf_counter_ns()
    deadline = time.monotonic() + timeout
    endpoint.start("target", dict(parameters, action="online_stage_start"))
    endpoint.start("source", dict(parameters, action="online_stage_source"))
    replies = {role: endpoint.receive(role, deadline) for role in ("target", "source")}
    observations: list = []
    while True:
        if time.monotonic() > deadline:
            raise TimeoutError("mapper publication")
        label = f"{request.phase}-ready-{len(observations)}"
        rows = endpoint.try_publish(label, parameters)
        outcomes = _check_rows(rows, request, label)
        observations.append(rows)
        if outcomes == {"published"}:
            if not all(row.get(field) for row in rows for field in RECEIPT_FIELDS):
                raise RuntimeError("Publication lacks complete GPU-read and worker completion evidence")
            break
        if outcomes != {"pending"}:
            raise RuntimeError(f"Inconsistent publication outcomes: {outcomes}")
        time.sleep(poll_interval)
    return {
        "parameters": parameters,
        "replies": replies,
        "readiness": observations,
        "mapping_started_ns": began,
        "committed_ns": time.perf_counter_ns(),
    }


class LocalHandoffEndpoint:
    """The endpoint protocol served by this process's GPU path (one target rank).

    ``source_slots(request_id, n)`` returns the device index tensor of the
    request's n history rows in ``source_pool``. ``allocate(n)`` returns n free
    target rows (device index tensor) or None. ``publish(indices)`` hands them
    to the target's cache once the data is certified, and ``free(indices)``
    returns them after a failure. The mapper's heads must match both pools'.
    """

    def __init__(self, mapper, source_pool, target_pool, *, source_slots: Callable, allocate: Callable,
                 publish: Callable, free: Callable, source_head_offset: int = 0, target_head_offset: int = 0):
        self.mapper = mapper
        self.source_pool = source_pool
        self.target_pool = target_pool
        self.source_slots = source_slots
        self.allocate = allocate
        self.publish = publish
        self.free = free
        self.source_head_offset = source_head_offset
        self.target_head_offset = target_head_offset
        self.device = mapper.device
        self.stream = torch.cuda.Stream(self.device)
        self._reset()

    def _reset(self):
        self.request_id = None
        self.phase = None
        self.indices = None
        self.event = None
        self.completion_ns = 0
        self.outcome = None
        self.replies = {}

    def start(self, role, parameters):
        from ..device import read_status
        from .blocks import map_install_block
        from .tp import chunk_spans

        n = len(parameters["history_ids"])
        if role == "target":
            self._reset()
            self.request_id, self.phase = parameters["request_id"], parameters["phase"]
            self.indices = self.allocate(n)
            if self.indices is None:
                raise RuntimeError("target pool allocation failed")
            self.replies["target"] = {"ready": True, "role": "target", "tokens": n}
            return
        if role != "source" or self.indices is None or parameters["request_id"] != self.request_id:
            raise RuntimeError("the source may start only after its target transaction")
        src = self.source_slots(self.request_id, n)
        read_status(self.device)  # start from a clean device status word
        with torch.cuda.stream(self.stream):
            for a, b in chunk_spans(n, int(parameters["block_tokens"])):
                map_install_block(self.mapper, self.source_pool, src, self.target_pool, self.indices, start=a,
                                  stop=b, source_head_offset=self.source_head_offset,
                                  target_head_offset=self.target_head_offset)
            self.event = torch.cuda.Event()
            self.event.record(self.stream)
        self.replies["source"] = {"ready": True, "role": "source", "blocks": len(chunk_spans(n, int(parameters["block_tokens"])))}

    def receive(self, role, deadline):
        if role not in self.replies:
            raise RuntimeError(f"no {role} reply")
        return self.replies[role]

    def try_publish(self, label, parameters):
        from ..device import read_status

        row = {
            "phase": label,
            "transaction_phase": parameters["phase"],
            "request_id": parameters["request_id"],
            "rank": 0,
            "all_rank_identity_valid": parameters["request_id"] == self.request_id
            and parameters["phase"] == self.phase,
        }
        if self.outcome is None:
            if self.event is None or not self.event.query():
                return [dict(row, outcome="pending")]
            self.completion_ns = time.perf_counter_ns()
            if read_status(self.device):
                self.outcome = "failed"
                self.free(self.indices)
            else:
                self.publish(self.indices)
                self.outcome = "published"
        done = self.outcome == "published"
        return [dict(row, outcome=self.outcome, worker_done=True, worker_thread_exited=True, all_rank_ready=done,
                     original_commit_stack_called=done, certified_data_completion_ns=self.completion_ns)]
