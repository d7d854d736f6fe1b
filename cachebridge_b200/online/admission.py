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
