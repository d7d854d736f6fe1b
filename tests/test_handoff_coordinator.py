"""Handoff coordination protocol (src/cachebridge/online/handoff.py) on the
host: both peers start before any wait, publication needs every target rank
with one consistent identity and complete GPU-completion receipts, and a
timeout keeps the backend's resources. A GPU test drives the local endpoint
end to end."""

from __future__ import annotations

import pytest
import torch

from cachebridge_b200.online import handoff as ho


class FakeEndpoint:
    """Two target ranks; the first poll is pending, later polls published."""

    def __init__(self, mutate=None):
        self.events = []
        self.polls = 0
        self.mutate = mutate

    def start(self, role, parameters):
        self.events.append(("start", role, parameters["action"]))

    def receive(self, role, deadline):
        assert [e[1] for e in self.events[:2]] == ["target", "source"]  # both started before any wait
        self.events.append(("receive", role))
        return {"role": role}

    def try_publish(self, label, parameters):
        self.polls += 1
        rows = []
        for rank in range(2):
            row = {"phase": label, "transaction_phase": parameters["phase"], "request_id": parameters["request_id"],
                   "rank": rank, "all_rank_identity_valid": True,
                   "outcome": "pending" if self.polls == 1 else "published"}
            row.update({field: 1 for field in ho.RECEIPT_FIELDS})
            rows.append(row)
        if self.mutate:
            self.mutate(rows)
        return rows


def _request():
    return ho.HandoffRequest("req-1", "phase-1", (5, 6, 7), "ns", target_ranks=2)


def test_request_validation_and_parameters():
    p = _request().parameters()
    assert p["history_ids"] == [5, 6, 7] and p["mapper_kind"] == "CacheBridge" and p["block_tokens"] == 2048
    for bad in (dict(request_id=""), dict(history_ids=()), dict(history_ids=(1, -2)), dict(target_ranks=0),
                dict(block_tokens=True)):
        kw = dict(request_id="r", phase="p", history_ids=(1,), namespace="n")
        kw.update(bad)
        with pytest.raises(ValueError):
            ho.HandoffRequest(**kw)


def test_publication_after_pending_with_complete_receipts():
    ep = FakeEndpoint()
    result = ho.run_handoff(ep, _request(), poll_interval=0)
    assert len(result["readiness"]) == 2
    assert [e for e in ep.events if e[0] == "start"] == [("start", "target", "online_stage_start"),
                                                         ("start", "source", "online_stage_source")]
    assert result["committed_ns"] >= result["mapping_started_ns"]


@pytest.mark.parametrize(
    "mutate",
    [
        lambda rows: rows.pop(),
        lambda rows: rows[1].update(request_id="other"),
        lambda rows: rows[0].update(transaction_phase="old"),
        lambda rows: rows[1].update(rank=0),
        lambda rows: rows[0].update(phase="phase-1-ready-9"),
        lambda rows: rows[0].update(all_rank_identity_valid=False),
        lambda rows: rows[1].update(outcome="failed"),
        lambda rows: rows[0].update(worker_done=False) if rows[0]["outcome"] == "published" else None,
        lambda rows: rows[1].update(certified_data_completion_ns=0) if rows[1]["outcome"] == "published" else None,
    ],
)
def test_stale_partial_or_unfenced_publication_is_rejected(mutate):
    with pytest.raises(RuntimeError):
        ho.run_handoff(FakeEndpoint(mutate), _request(), poll_interval=0)


def test_timeout_keeps_backend_ownership(monkeypatch):
    ticks = iter([0.0, 5.0])
    monkeypatch.setattr(ho.time, "monotonic", lambda: next(ticks))
    ep = FakeEndpoint()
    with pytest.raises(TimeoutError):
        ho.run_handoff(ep, _request(), timeout=1)
    assert ep.polls == 0 and len(ep.events) == 4  # both started and answered; nothing released


@pytest.mark.gpu
def test_local_endpoint_end_to_end(tmp_path, cuda_device):
    import cachebridge_b200 as cb
    from cachebridge_b200.online.blocks import map_install_block
    from test_gpu_parity import _random_mapper

    g = torch.Generator().manual_seed(3)
    L_s, L_t, H, D, rows, n = 6, 4, 2, 128, 4096, 700
    mapper = cb.PageMapper(_random_mapper(tmp_path, seed=8, L_s=L_s, L_t=L_t, H=H, D=D, S=2), method="cachebridge",
                           source_rope_theta=1e6, target_rope_theta=1e6, device=cuda_device)
    source = cb.TokenKVPool(layers=L_s, rows=rows, heads=H, head_dim=D, device=cuda_device)
    source.k_buffer.normal_(generator=torch.Generator(device=cuda_device).manual_seed(1))
    source.v_buffer.normal_(generator=torch.Generator(device=cuda_device).manual_seed(2))
    target = cb.TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=cuda_device, fill=-7.25)
    src_slots = torch.randperm(rows, generator=g)[:n].to(cuda_device)
    free = torch.randperm(rows, generator=g).to(cuda_device)
    published, freed = [], []
    ep = ho.LocalHandoffEndpoint(
        mapper, source, target, source_slots=lambda rid, k: src_slots[:k], allocate=lambda k: free[:k],
        publish=published.append, free=freed.append)
    req = ho.HandoffRequest("r1", "p1", tuple(range(n)), "ns", target_ranks=1, block_tokens=256)
    result = ho.run_handoff(ep, req, poll_interval=0)
    assert result["readiness"][-1][0]["outcome"] == "published"
    assert len(published) == 1 and torch.equal(published[0], free[:n]) and not freed
    expected = cb.TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=cuda_device, fill=-7.25)
    for a in range(0, n, 256):
        map_install_block(mapper, source, src_slots, expected, free[:n], start=a, stop=min(n, a + 256))
    torch.cuda.synchronize()
    assert torch.equal(target.k_buffer, expected.k_buffer) and torch.equal(target.v_buffer, expected.v_buffer)

    # A source slot outside the pool: reported on the device, the transaction fails and its rows are freed.
    bad = src_slots.clone()
    bad[10] = rows
    ep2 = ho.LocalHandoffEndpoint(
        mapper, source, target, source_slots=lambda rid, k: bad[:k], allocate=lambda k: free[:k],
        publish=published.append, free=freed.append)
    with pytest.raises(RuntimeError, match="Inconsistent publication outcomes"):
        ho.run_handoff(ep2, ho.HandoffRequest("r2", "p2", tuple(range(n)), "ns", target_ranks=1), poll_interval=0)
    assert len(published) == 1 and len(freed) == 1
