"""Break-even admission for the live mapper, calibrated by measurement.

``LiveMapperCostPolicy`` keeps the gate of src/cachebridge/online/admission.py:83-103:
a request is mapped (instead of re-prefilled on the target) when its history
holds at least ``min_history_tokens`` tokens. ``calibrate_cost_policy`` sets
that threshold from measured times of this path: the handoff, and the
re-prefill it replaces. Each time is modelled as fixed + per-token, fitted
to one or more (tokens, ms) measurements. The threshold is the history
length from which the handoff is faster. ``policy_from_bench`` reads the
figures from a ``bench.py`` JSON line (``latency_p50_ms`` / tokens and
``reprefill_estimate``).

``OnlineMapperRouter``, ``LiveMapperMechanism`` and ``LiveMapperAdmission``
(below) route each cohort of arrivals to the live mapper, an idle cohort or
native re-prefill, and keep at most one unpublished mapper transaction.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Literal


@dataclass(frozen=True)
class MapperRequest:
    request_id: str
    history_tokens: int


@dataclass(frozen=True)
class LiveMapperCostPolicy:
    """Admit a request to the live mapper from ``min_history_tokens`` on."""

    min_history_tokens: int
    objective: Literal["ttft"] = "ttft"

    def validate(self) -> None:
        if self.min_history_tokens <= 0:
            raise ValueError("min_history_tokens must be positive")
        if self.objective != "ttft":
            raise ValueError("only the measured ttft objective is supported")

    def admits(self, request: MapperRequest) -> bool:
        return request.history_tokens >= self.min_history_tokens


@dataclass(frozen=True)
class CostModel:
    """time_ms(tokens) = fixed_ms + per_token_ms * tokens."""

    fixed_ms: float
    per_token_ms: float

    def time_ms(self, tokens: int) -> float:
        return self.fixed_ms + self.per_token_ms * tokens


def fit_cost(points) -> CostModel:
    """Least-squares line through (tokens, ms) points. A single point becomes
    a pure per-token cost (fixed part 0)."""
    pts = [(float(n), float(t)) for n, t in points]
    if not pts or any(n <= 0 or t < 0 for n, t in pts):
        raise ValueError("cost points need positive token counts and non-negative times")
    if len({n for n, _ in pts}) == 1:
        n = pts[0][0]
        return CostModel(0.0, sum(t for _, t in pts) / len(pts) / n)
    mn = sum(n for n, _ in pts) / len(pts)
    mt = sum(t for _, t in pts) / len(pts)
    slope = sum((n - mn) * (t - mt) for n, t in pts) / sum((n - mn) ** 2 for n, _ in pts)
    return CostModel(max(0.0, mt - slope * mn), max(0.0, slope))


def break_even_tokens(handoff: CostModel, reprefill: CostModel) -> int | None:
    """Smallest history length for which the handoff is faster than
    re-prefill, or None when it never is."""
    gain = reprefill.per_token_ms - handoff.per_token_ms
    extra = handoff.fixed_ms - reprefill.fixed_ms
    if gain <= 0:
        return None if extra >= 0 or gain < 0 else 1
    if extra < 0:
        return 1
    return max(1, math.floor(extra / gain) + 1)


def calibrate_cost_policy(handoff_points, reprefill_points) -> LiveMapperCostPolicy | None:
    """Policy from measured (tokens, ms) points of both options; None when
    the handoff never pays off."""
    tokens = break_even_tokens(fit_cost(handoff_points), fit_cost(reprefill_points))
    if tokens is None:
        return None
    policy = LiveMapperCostPolicy(tokens)
    policy.validate()
    return policy


def policy_from_bench(line: dict) -> LiveMapperCostPolicy | None:
    """Policy from one ``bench.py`` JSON line (N=1 or N>1)."""
    prefill = line["reprefill_estimate"]
    tokens = prefill["tokens_per_request"] * prefill["requests"]
    handoff_ms = line.get("latency_p50_ms", line["ms_per_step"])
    return calibrate_cost_policy([(tokens, handoff_ms)], [(tokens, prefill["ms"])])


# ---------------------------------------------------------------------------
# Live mapper routing and admission (src/cachebridge/online/admission.py:43-81,
# 106-394): a fail-closed capability contract, a router that picks exactly one
# serving path per cohort, and the single-unpublished-transaction state
# machine. Names, modes, reasons and messages are the reference's interface.
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class LiveMapperMechanism:
    """Capabilities required before mapper work may overlap target decode.

    A fail-closed contract: the mapper computes on the source ranks with two
    or more output slots, places rows directly into the target pool, holds no
    target workspace, and leaves allocation and publication to the target's
    scheduler. ``of_placement`` describes this package's sharded placements:
    source placement (``ShardedHandoff``) meets the contract; target placement
    (``TargetPlacement``) maps on the target with receive slots and a key
    workspace there, so it does not, and serves throughput cohorts instead.
    """

    mapper_compute_role: Literal["source", "target"] = "source"
    mapped_output_slots: int = 2
    direct_target_placement: bool = True
    target_mapper_workspace_bytes: int = 0
    target_transfer_workspace_bytes: int = 0
    scheduler_serialized_allocation: bool = True
    scheduler_serialized_publication: bool = True
    source_slot_gpu_ack: bool = True
    max_staged_transactions: int = 1

    def validate(self) -> None:
        for broken, message in _LIVE_RULES:
            if broken(self):
                raise ValueError(message)

    @classmethod
    def of_placement(cls, placement: str, *, slots: int = 2, target_workspace_bytes: int = 0,
                     target_transfer_bytes: int = 0) -> "LiveMapperMechanism":
        if placement == "source":
            return cls(mapped_output_slots=slots)
        if placement == "target":
            return cls(mapper_compute_role="target", mapped_output_slots=slots,
                       target_mapper_workspace_bytes=target_workspace_bytes,
                       target_transfer_workspace_bytes=target_transfer_bytes)
        raise ValueError("placement must be 'source' or 'target'")


# (violated?, message), checked in order.
_LIVE_RULES = (
    (lambda m: m.mapper_compute_role != "source", "live mapper compute must be source-isolated"),
    (lambda m: m.mapped_output_slots < 2, "live mapper requires at least two output slots"),
    (lambda m: not m.direct_target_placement, "live mapper requires direct target placement"),
    (lambda m: m.target_mapper_workspace_bytes != 0, "live mapper cannot allocate target mapper workspace"),
    (lambda m: m.target_transfer_workspace_bytes != 0, "live mapper cannot allocate target transfer workspace"),
    (lambda m: not m.scheduler_serialized_allocation, "target allocation must be scheduler-serialized"),
    (lambda m: not m.scheduler_serialized_publication, "target publication must be scheduler-serialized"),
    (lambda m: not m.source_slot_gpu_ack, "source slots require target GPU-complete ACKs"),
    (lambda m: m.max_staged_transactions != 1, "exactly one unpublished transaction is supported"),
)


@dataclass(frozen=True)
class RouterDecision:
    mode: Literal["cachebridge_live", "cachebridge_cohort", "native_reprefill", "backpressure"]
    reason: str
    requests: tuple
    canceled_request_ids: tuple
    decoder_active: bool
    service_class: Literal["latency", "throughput"]
    cohort_preformed: bool


class OnlineMapperRouter:
    """Route a cohort of arrivals to one serving path.

    With a validated live mechanism every cohort takes the live mapper
    (decoder activity, latency class and trickle arrival are no reason to drop
    KV reuse), unless a cost policy says some request is below break-even,
    which sends the whole cohort to native re-prefill. Without one, the
    idle-cohort rules apply: only an idle, preformed throughput cohort is
    mapped. Cancelled requests are removed first; an empty or oversized
    cohort is backpressured.
    """

    def __init__(self, *, max_cohort_requests: int = 4, live_mechanism: LiveMapperMechanism | None = None,
                 live_cost_policy: LiveMapperCostPolicy | None = None) -> None:
        if max_cohort_requests <= 0:
            raise ValueError("max_cohort_requests must be positive")
        if live_mechanism is not None:
            live_mechanism.validate()
        if live_cost_policy is not None:
            live_cost_policy.validate()
            if live_mechanism is None:
                raise ValueError("live cost policy requires a live mapper mechanism")
        self.max_cohort_requests = max_cohort_requests
        self.live_mechanism = live_mechanism
        self.live_cost_policy = live_cost_policy

    def _path(self, active, decoder_active, service_class, cohort_preformed) -> tuple[str, str]:
        if self.live_mechanism is not None:
            if self.live_cost_policy is not None and not all(self.live_cost_policy.admits(r) for r in active):
                return "native_reprefill", "below_live_mapper_break_even"
            return "cachebridge_live", "source_isolated_live_mapper"
        if decoder_active:
            return "native_reprefill", "decoder_active"
        if service_class == "latency":
            return "native_reprefill", "latency_service_class"
        if not cohort_preformed:
            return "native_reprefill", "trickle_arrival_no_wait"
        return "cachebridge_cohort", "idle_preformed_throughput_cohort"

    def route(self, requests, *, decoder_active: bool, service_class: Literal["latency", "throughput"],
              cohort_preformed: bool, canceled_request_ids=()) -> RouterDecision:
        cohort = tuple(requests)
        if not cohort:
            raise ValueError("route requires at least one request")
        ids = [r.request_id for r in cohort]
        if not all(ids):
            raise ValueError("request identity must be non-empty")
        if len(set(ids)) != len(ids):
            raise ValueError("request identities must be unique")
        canceled = tuple(canceled_request_ids)
        if len(set(canceled)) != len(canceled):
            raise ValueError("canceled request identities must be unique")
        unknown = set(canceled) - set(ids)
        if unknown:
            raise ValueError(f"unknown canceled request identities: {sorted(unknown)}")
        active = tuple(r for r in cohort if r.request_id not in set(canceled))
        context = (decoder_active, service_class, cohort_preformed)
        if not active:
            return RouterDecision("backpressure", "cohort_canceled", (), canceled, *context)
        if len(active) > self.max_cohort_requests:
            return RouterDecision("backpressure", "cohort_request_limit", active, canceled, *context)
        mode, reason = self._path(active, *context)
        return RouterDecision(mode, reason, active, canceled, *context)

    def dispatch(self, decision: RouterDecision, *, cachebridge_live=None, cachebridge_cohort, native_reprefill):
        """Invoke exactly one already-selected serving path."""
        handlers = {"cachebridge_live": cachebridge_live, "cachebridge_cohort": cachebridge_cohort,
                    "native_reprefill": native_reprefill}
        if decision.mode not in handlers:
            raise RuntimeError(f"cannot dispatch backpressured route: {decision.reason}")
        handler = handlers[decision.mode]
        if handler is None:
            raise RuntimeError("cachebridge_live callback is required")
        return handler(decision.requests)


@dataclass(frozen=True)
class LiveAdmissionPlan:
    admitted: bool
    reason: str
    request: MapperRequest
    required_target_tokens: int
    available_target_tokens: int
    decoder_active: bool


@dataclass(frozen=True)
class PublicationProof:
    gpu_reads_complete: bool
    tp_vote_passed: bool

    @classmethod
    def from_receipts(cls, receipts) -> "PublicationProof":
        """Proof from one request's ``commit`` receipts (online/transaction.py):
        the GPU work was settled and every rank's vote published it."""
        rows = list(receipts)
        settled = bool(rows) and all(r.get("certified_data_completion_ns") for r in rows)
        return cls(gpu_reads_complete=settled, tp_vote_passed=bool(rows) and
                   all(r.get("outcome") == "published" for r in rows))


class LiveMapperAdmission:
    """At most one unpublished mapper transaction, overlapping target decode.

    Phases: idle -> mapping (``begin``) -> source_ready
    (``mark_source_complete``) -> published (``publish`` with a proof of GPU
    completion and the TP vote) -> idle (``mark_submitted``). A safe rollback
    (reads complete, pages released) returns to idle from mapping or
    source_ready; anything unsafe quarantines the machine.
    """

    def __init__(self, *, mechanism: LiveMapperMechanism, query_reserve_tokens: int = 32) -> None:
        if query_reserve_tokens < 0:
            raise ValueError("query reserve must be non-negative")
        mechanism.validate()
        self.mechanism = mechanism
        self.query_reserve_tokens = query_reserve_tokens
        self._active: MapperRequest | None = None
        self._phase = "idle"
        self._decoder_active = False
        self._completed: list[str] = []
        self._error: str | None = None

    def plan(self, request: MapperRequest, *, available_target_tokens: int, decoder_active: bool) -> LiveAdmissionPlan:
        if not request.request_id:
            raise ValueError("request identity must be non-empty")
        if request.history_tokens <= 0:
            raise ValueError("history_tokens must be positive")
        required = request.history_tokens + self.query_reserve_tokens
        if self._phase != "idle":
            admitted, reason = False, "mapper_transaction_in_flight"
        elif required > available_target_tokens:
            admitted, reason = False, "target_token_backpressure"
        else:
            admitted, reason = True, "admitted_during_decode" if decoder_active else "admitted"
        return LiveAdmissionPlan(admitted, reason, request, required, available_target_tokens, decoder_active)

    def begin(self, plan: LiveAdmissionPlan) -> MapperRequest:
        if self._phase != "idle":
            raise RuntimeError(f"cannot begin while state={self._phase}")
        if not plan.admitted:
            raise RuntimeError(f"cannot execute rejected plan: {plan.reason}")
        if plan.request.request_id in self._completed:
            raise RuntimeError("request identity was already published")
        self._active, self._decoder_active, self._phase, self._error = plan.request, plan.decoder_active, "mapping", None
        return plan.request

    def _owner(self, request_id: str, phase: str) -> None:
        if self._phase != phase or self._active is None or self._active.request_id != request_id:
            raise RuntimeError("operation does not own the active mapper transaction")

    def mark_source_complete(self, request_id: str) -> None:
        self._owner(request_id, "mapping")
        self._phase = "source_ready"

    def publish(self, request_id: str, proof: PublicationProof) -> None:
        self._owner(request_id, "source_ready")
        if not (proof.gpu_reads_complete and proof.tp_vote_passed):
            self.quarantine("publication proof failed")
            raise RuntimeError("cannot publish without GPU completion and TP vote")
        self._phase = "published"

    def mark_submitted(self, request_id: str) -> None:
        self._owner(request_id, "published")
        self._completed.append(request_id)
        self._idle()

    def rollback(self, request_id: str, *, gpu_reads_complete: bool, target_pages_released: bool) -> None:
        if self._active is None or self._active.request_id != request_id:
            raise RuntimeError("rollback does not own the active transaction")
        if self._phase not in ("mapping", "source_ready"):
            raise RuntimeError(f"cannot roll back while state={self._phase}")
        if not (gpu_reads_complete and target_pages_released):
            self.quarantine("unsafe rollback")
            raise RuntimeError("rollback requires completed reads and released pages")
        self._idle()

    def _idle(self) -> None:
        self._active, self._decoder_active, self._phase = None, False, "idle"

    def quarantine(self, error) -> None:
        self._phase = "quarantined"
        self._error = str(error)

    def snapshot(self) -> dict:
        m = self.mechanism
        return dict(state=self._phase, active_request=None if self._active is None else self._active.request_id,
                    decoder_active_during_mapping=self._decoder_active, completed_request_ids=tuple(self._completed),
                    error=self._error, mapper_compute_role=m.mapper_compute_role,
                    mapped_output_slots=m.mapped_output_slots, max_staged_transactions=m.max_staged_transactions,
                    target_mapper_workspace_bytes=m.target_mapper_workspace_bytes,
                    target_transfer_workspace_bytes=m.target_transfer_workspace_bytes,
                    direct_target_placement=m.direct_target_placement,
                    scheduler_serialized_publication=m.scheduler_serialized_publication)
