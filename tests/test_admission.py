"""Admission for the live mapper: the measured break-even gate
(online/admission.py:83-103), the router and the single-transaction live
admission (admission.py:43-81, 106-394), against the reference's behaviours."""

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


# ---- router and live admission (admission.py:43-81, 106-394 behaviours) ----
import dataclasses

from cachebridge_b200.online.admission import (
    LiveMapperAdmission,
    LiveMapperCostPolicy,
    LiveMapperMechanism,
    MapperRequest,
    OnlineMapperRouter,
    PublicationProof,
)


def _reqs(*sizes):
    return [MapperRequest(f"r{i}", n) for i, n in enumerate(sizes)]


def test_router_without_live_mechanism_maps_only_idle_preformed_throughput_cohorts():
    router = OnlineMapperRouter()
    d = router.route(_reqs(4096, 8192), decoder_active=False, service_class="throughput", cohort_preformed=True)
    assert (d.mode, d.reason) == ("cachebridge_cohort", "idle_preformed_throughput_cohort")
    for kwargs, reason in [
        (dict(decoder_active=True, service_class="throughput", cohort_preformed=True), "decoder_active"),
        (dict(decoder_active=False, service_class="latency", cohort_preformed=True), "latency_service_class"),
        (dict(decoder_active=False, service_class="throughput", cohort_preformed=False), "trickle_arrival_no_wait"),
    ]:
        d = router.route(_reqs(4096), **kwargs)
        assert (d.mode, d.reason) == ("native_reprefill", reason)


def test_router_with_live_mechanism_maps_during_decode_unless_below_break_even():
    live = OnlineMapperRouter(live_mechanism=LiveMapperMechanism())
    d = live.route(_reqs(300), decoder_active=True, service_class="latency", cohort_preformed=False)
    assert (d.mode, d.reason) == ("cachebridge_live", "source_isolated_live_mapper")
    gated = OnlineMapperRouter(live_mechanism=LiveMapperMechanism(), live_cost_policy=LiveMapperCostPolicy(1024))
    d = gated.route(_reqs(4096, 512), decoder_active=True, service_class="throughput", cohort_preformed=True)
    assert (d.mode, d.reason) == ("native_reprefill", "below_live_mapper_break_even")  # the whole cohort
    d = gated.route(_reqs(4096), decoder_active=True, service_class="throughput", cohort_preformed=True)
    assert d.mode == "cachebridge_live"
    with pytest.raises(ValueError, match="requires a live mapper mechanism"):
        OnlineMapperRouter(live_cost_policy=LiveMapperCostPolicy(1024))


def test_router_cancels_backpressures_and_dispatches_exactly_one_path():
    router = OnlineMapperRouter(max_cohort_requests=2)
    d = router.route(_reqs(10, 20, 30), decoder_active=False, service_class="throughput", cohort_preformed=True,
                     canceled_request_ids=["r1"])
    assert d.mode == "cachebridge_cohort" and [r.request_id for r in d.requests] == ["r0", "r2"]
    d = router.route(_reqs(10, 20, 30), decoder_active=False, service_class="throughput", cohort_preformed=True)
    assert (d.mode, d.reason) == ("backpressure", "cohort_request_limit")
    with pytest.raises(RuntimeError, match="cohort_request_limit"):
        router.dispatch(d, cachebridge_cohort=lambda r: 1, native_reprefill=lambda r: 2)
    d = router.route(_reqs(10), decoder_active=False, service_class="throughput", cohort_preformed=True,
                     canceled_request_ids=["r0"])
    assert (d.mode, d.reason) == ("backpressure", "cohort_canceled")
    d = router.route(_reqs(10), decoder_active=True, service_class="throughput", cohort_preformed=True)
    calls = []
    router.dispatch(d, cachebridge_cohort=lambda r: calls.append("cohort"), native_reprefill=lambda r: calls.append("native"))
    assert calls == ["native"]
    with pytest.raises(ValueError, match="unique"):
        router.route([MapperRequest("a", 1), MapperRequest("a", 2)], decoder_active=False,
                     service_class="throughput", cohort_preformed=True)


@pytest.mark.parametrize("field,value,message", [
    ("mapper_compute_role", "target", "source-isolated"),
    ("mapped_output_slots", 1, "two output slots"),
    ("direct_target_placement", False, "direct target placement"),
    ("target_mapper_workspace_bytes", 1, "target mapper workspace"),
    ("target_transfer_workspace_bytes", 1, "target transfer workspace"),
    ("scheduler_serialized_allocation", False, "allocation must be scheduler-serialized"),
    ("scheduler_serialized_publication", False, "publication must be scheduler-serialized"),
    ("source_slot_gpu_ack", False, "GPU-complete ACKs"),
    ("max_staged_transactions", 2, "exactly one unpublished"),
])
def test_live_mechanism_fails_closed(field, value, message):
    with pytest.raises(ValueError, match=message):
        dataclasses.replace(LiveMapperMechanism(), **{field: value}).validate()


def test_our_placements_against_the_live_contract():
    LiveMapperMechanism.of_placement("source").validate()  # ShardedHandoff: mapper on the source
    with pytest.raises(ValueError, match="source-isolated"):
        LiveMapperMechanism.of_placement("target", target_workspace_bytes=1 << 30).validate()


def test_live_admission_publishes_with_proof_and_serialises_ownership():
    adm = LiveMapperAdmission(mechanism=LiveMapperMechanism())
    req = MapperRequest("a", 8192)
    assert adm.plan(req, available_target_tokens=100, decoder_active=False).reason == "target_token_backpressure"
    plan = adm.plan(req, available_target_tokens=10000, decoder_active=True)
    assert plan.admitted and plan.reason == "admitted_during_decode" and plan.required_target_tokens == 8192 + 32
    adm.begin(plan)
    assert adm.plan(MapperRequest("b", 10), available_target_tokens=10000, decoder_active=False).reason == \
        "mapper_transaction_in_flight"
    with pytest.raises(RuntimeError, match="does not own"):
        adm.mark_source_complete("b")
    adm.mark_source_complete("a")
    receipts = [dict(outcome="published", certified_data_completion_ns=123) for _ in range(2)]
    adm.publish("a", PublicationProof.from_receipts(receipts))
    with pytest.raises(RuntimeError, match="state=published"):
        adm.rollback("a", gpu_reads_complete=True, target_pages_released=True)
    adm.mark_submitted("a")
    assert adm.snapshot()["state"] == "idle" and adm.snapshot()["completed_request_ids"] == ("a",)
    again = adm.plan(req, available_target_tokens=10000, decoder_active=False)
    with pytest.raises(RuntimeError, match="already published"):
        adm.begin(again)


def test_live_admission_quarantines_without_proof_and_rolls_back_safely():
    adm = LiveMapperAdmission(mechanism=LiveMapperMechanism())
    adm.begin(adm.plan(MapperRequest("a", 64), available_target_tokens=1000, decoder_active=False))
    adm.rollback("a", gpu_reads_complete=True, target_pages_released=True)
    assert adm.snapshot()["state"] == "idle"
    adm.begin(adm.plan(MapperRequest("b", 64), available_target_tokens=1000, decoder_active=False))
    adm.mark_source_complete("b")
    rolled = [dict(outcome="rolled_back", certified_data_completion_ns=1)]
    with pytest.raises(RuntimeError, match="GPU completion and TP vote"):
        adm.publish("b", PublicationProof.from_receipts(rolled))
    assert adm.snapshot()["state"] == "quarantined"
