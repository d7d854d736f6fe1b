"""Measured break-even admission (online/admission.py:83-103 gate)."""

import pytest

from cachebridge_b200.online import admission as ad


def test_gate_matches_reference_semantics():
    policy = ad.LiveMapperCostPolicy(4096)
    policy.validate()
    assert policy.admits(ad.MapperRequest("a", 4096)) and not policy.admits(ad.MapperRequest("b", 4095))
    with pytest.raises(ValueError):
        ad.LiveMapperCostPolicy(0).validate()
    with pytest.raises(ValueError):
        ad.LiveMapperCostPolicy(1, objective="throughput").validate()


def test_fit_and_break_even():
    handoff = ad.fit_cost([(1024, 2.0 + 1024 * 0.001), (8192, 2.0 + 8192 * 0.001)])
    assert handoff.fixed_ms == pytest.approx(2.0) and handoff.per_token_ms == pytest.approx(0.001)
    reprefill = ad.CostModel(0.0, 0.05)
    n = ad.break_even_tokens(handoff, reprefill)
    assert handoff.time_ms(n) < reprefill.time_ms(n) and handoff.time_ms(n - 1) >= reprefill.time_ms(n - 1)
    assert ad.break_even_tokens(ad.CostModel(1.0, 0.1), ad.CostModel(0.0, 0.05)) is None
    assert ad.break_even_tokens(ad.CostModel(0.0, 0.01), ad.CostModel(1.0, 0.05)) == 1


def test_policy_from_bench_line():
    line = {"latency_p50_ms": 1.37, "ms_per_step": 1.37,
            "reprefill_estimate": {"ms": 448.0, "tokens_per_request": 8192, "requests": 1}}
    policy = ad.policy_from_bench(line)
    assert policy is not None and policy.min_history_tokens == 1
    slow = dict(line, latency_p50_ms=900.0)
    assert ad.policy_from_bench(slow) is None
