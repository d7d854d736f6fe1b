"""Host-side contracts of the handoff path (no GPU needed).

Mirrors the reference's CPU lifecycle tests: tests/test_blocks.py (lease,
unpublished-install transaction), tests/test_pipeline.py (two-slot lease, peer
byte geometry) and the PageMapper constructor's validation
(src/cachebridge/mapper.py:59-91).
"""

from __future__ import annotations

import pytest
import torch
from safetensors.torch import save_file

from cachebridge_b200 import PageMapper, contiguous_runs
from cachebridge_b200.online.blocks import SourceLease, install_unpublished
from peer_geometry_check import operations
from cachebridge_b200.online.pipeline import PipelinedSourceLease
from conftest import GOLDEN


def test_source_lease_requires_gpu_ack_before_reuse_or_release():
    events = []
    lease = SourceLease(lambda: events.append("lock"), lambda: events.append("unlock"))
    lease.begin()
    lease.export(0, 512)
    with pytest.raises(RuntimeError):
        lease.export(512, 513)
    with pytest.raises(RuntimeError):
        lease.close()
    with pytest.raises(RuntimeError):
        lease.acknowledge(gpu_reads_complete=False)
    lease.acknowledge(gpu_reads_complete=True)
    lease.export(512, 513)
    lease.acknowledge(gpu_reads_complete=True)
    lease.close()
    assert events == ["lock", "unlock"]


def test_two_live_slots_require_individual_completion():
    events = []
    lease = PipelinedSourceLease(lambda: events.append("acquire"), lambda: events.append("release"))
    lease.begin()
    lease.export(0, 0, 2048)
    lease.export(1, 2048, 4096)
    with pytest.raises(RuntimeError):
        lease.export(0, 4096, 4097)
    with pytest.raises(RuntimeError):
        lease.close()
    with pytest.raises(RuntimeError):
        lease.acknowledge(0, gpu_reads_complete=False)
    lease.acknowledge(0, gpu_reads_complete=True)
    lease.export(0, 4096, 4097)
    lease.acknowledge(1, gpu_reads_complete=True)
    with pytest.raises(RuntimeError):
        lease.close()
    lease.acknowledge(0, gpu_reads_complete=True)
    lease.close()
    assert events == ["acquire", "release"]


def _transaction(*, foreign_failure=False, cancel=None, broken_span=False):
    events = []
    value = torch.zeros(2, 1, 2, 1, 1)
    blocks = [(0, 2, value), (3 if broken_span else 2, 4, value)]
    kwargs = dict(
        token_count=4,
        allocate=lambda n: torch.tensor([5, 2, 9, 3]),
        free=lambda idx: events.append(("free", idx.tolist())),
        blocks=blocks,
        write=lambda value, idx, start: events.append(("write", start)),
        synchronize=lambda: events.append(("sync",)),
        ready_vote=lambda local: events.append(("vote", local)) or (local and not foreign_failure),
        publish=lambda idx: events.append(("publish", idx.tolist())),
        cancel_after_blocks=cancel,
    )
    return events, kwargs


def test_publish_only_after_complete_writes_and_ready_vote():
    events, kwargs = _transaction()
    result = install_unpublished(**kwargs)
    assert result == dict(tokens=4, blocks=2, published=True)
    assert events[-2][0] == "vote" and events[-1][0] == "publish"
    assert "free" not in [e[0] for e in events]


@pytest.mark.parametrize("options", [dict(cancel=1), dict(foreign_failure=True), dict(broken_span=True)])
def test_cancellation_or_foreign_failure_frees_unpublished_once(options):
    events, kwargs = _transaction(**options)
    with pytest.raises(RuntimeError, match="rolled back"):
        install_unpublished(**kwargs)
    assert [e[0] for e in events].count("free") == 1
    assert "publish" not in [e[0] for e in events]


def test_broken_vote_keeps_pages_owned():
    events, kwargs = _transaction()

    def fail(_):
        raise RuntimeError("distributed group unavailable")

    kwargs["ready_vote"] = fail
    with pytest.raises(RuntimeError, match="distributed group"):
        install_unpublished(**kwargs)
    assert "free" not in [e[0] for e in events]


@pytest.mark.parametrize("tokens", [1, 512, 2048, 4096])
def test_peer_geometry_covers_fragmented_destination_without_overlap(tokens):
    split = max(1, tokens // 2)
    runs = [(0, split, 5)]
    if split < tokens:
        runs.append((split, tokens, split + 20))
    row = 2 * 128 * 2
    copies = operations(0, tokens, runs, heads=2)
    assert sum(c[4] for c in copies) == 2 * 64 * tokens * row
    for kind in range(2):
        for layer in range(64):
            spans = [(s, d, z) for k, l, s, d, z in copies if (k, l) == (kind, layer)]
            cursor = (kind * 64 + layer) * tokens * row
            for (a, b, p), (s, d, z) in zip(runs, spans):
                assert (s, d, z) == (cursor, p * row, (b - a) * row)
                cursor += z
            assert cursor == (kind * 64 + layer + 1) * tokens * row


def test_peer_geometry_rejects_alias_and_unsupported_block():
    with pytest.raises(ValueError, match="alias"):
        operations(0, 8, [(0, 4, 5), (4, 8, 7)], heads=2)
    with pytest.raises(ValueError, match="unsupported"):
        operations(0, 4097, [(0, 4097, 0)], heads=2)
    with pytest.raises(ValueError, match="cover"):
        operations(0, 8, [(0, 4, 0)], heads=2)


def test_contiguous_runs():
    assert contiguous_runs([]) == []
    assert contiguous_runs([7]) == [(0, 1, 7)]
    assert contiguous_runs([5, 6, 7, 2, 9, 10]) == [(0, 3, 5), (3, 4, 2), (4, 6, 9)]


def _headwise_file(root, **over):
    t = dict(
        selected=torch.tensor([0]),
        k_weight=torch.eye(4).expand(2, 4, 4).contiguous(),
        k_bias=torch.zeros(2, 4),
        v_weight=torch.eye(4).expand(2, 4, 4).contiguous(),
        v_bias=torch.zeros(2, 4),
        headwise=torch.tensor(1, dtype=torch.int8),
    )
    t.update(over)
    t = {k: v for k, v in t.items() if v is not None}
    save_file(t, str(root / "layer_000.safetensors"))


def test_mapper_constructor_validation(tmp_path):
    kw = dict(method="cachebridge", source_rope_theta=1e4, target_rope_theta=1e4)
    with pytest.raises(FileNotFoundError):
        PageMapper(tmp_path, **kw)
    _headwise_file(tmp_path, v_bias=None)
    with pytest.raises(ValueError, match="missing tensors"):
        PageMapper(tmp_path, **kw)
    _headwise_file(tmp_path)
    with pytest.raises(ValueError, match="does not match method"):
        PageMapper(tmp_path, method="nv_transfer", source_rope_theta=1e4, target_rope_theta=1e4)
    with pytest.raises(ValueError, match="must divide target TP"):
        PageMapper(tmp_path, target_tp_size=3, **kw)
    with pytest.raises(ValueError, match="CUDA devices only"):
        PageMapper(tmp_path, device="cpu", **kw)


def test_mapper_rejects_head_geometry_drift(tmp_path):
    _headwise_file(tmp_path)
    t = dict(
        selected=torch.tensor([0]),
        k_weight=torch.zeros(4, 4, 4),
        k_bias=torch.zeros(4, 4),
        v_weight=torch.zeros(4, 4, 4),
        v_bias=torch.zeros(4, 4),
        headwise=torch.tensor(1, dtype=torch.int8),
    )
    save_file(t, str(tmp_path / "layer_001.safetensors"))
    with pytest.raises(ValueError, match="geometry changes"):
        PageMapper(tmp_path, method="cachebridge", source_rope_theta=1e4, target_rope_theta=1e4,
                   target_tp_rank=1, target_tp_size=2)


def test_golden_fixtures_present():
    assert (GOLDEN / "make_golden.py").exists()
    assert len(list(GOLDEN.glob("*/case.json"))) >= 12
