"""Host logic of the tensor-parallel handoff on CPU: pair plan, chunking, the
publication transaction (online/transaction.py) and the pool-handle exchange,
run as world_size-2 ``gloo`` process groups (no GPU).

Failures are made on the host (src/cachebridge/online/blocks.py:114-171,
backends/sglang/runtime/source_mapper_adapter.py:543-548, :1145-1237): a
cancellation after k chunks, a foreign rank whose device check fails, a rank
that cannot certify its GPU work, an identity mismatch, a failed publication,
and a rank that leaves so that the vote itself fails. Every rank must reach
the same outcome; freed rows are freed exactly once and quarantined rows
never.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cachebridge_b200.online import tp
from cachebridge_b200.online.blocks import install_unpublished
from cachebridge_b200.online.transaction import (
    PUBLISHED,
    QUARANTINED,
    ROLLED_BACK,
    DeviceDataError,
    HandoffTransaction,
    TransactionError,
    commit,
    gloo_vote,
)


def test_pair_plan_roles_heads_and_peers():
    plans = [tp.pair_plan(8, r, 8) for r in range(8)]
    assert [p.role for p in plans] == ["source"] * 4 + ["target"] * 4
    assert [p.peer for p in plans] == [4, 5, 6, 7, 0, 1, 2, 3]
    assert all(p.heads_per_rank == 2 for p in plans)
    assert [p.head_start for p in plans] == [0, 2, 4, 6, 0, 2, 4, 6]
    two = tp.pair_plan(2, 0, 8)
    assert (two.tp, two.heads_per_rank, two.peer) == (1, 8, 1)
    with pytest.raises(ValueError, match="even world"):
        tp.pair_plan(3, 0, 8)
    with pytest.raises(ValueError, match="divide evenly"):
        tp.pair_plan(6, 0, 8)


def test_chunk_spans_are_ordered_and_gap_free():
    for n, c in [(0, 2048), (1, 2048), (2048, 2048), (5000, 2048), (32768, 2048), (33, 7)]:
        spans = tp.chunk_spans(n, c)
        assert all(b - a <= c and b > a for a, b in spans)
        assert [a for a, _ in spans] == list(range(0, n, c))
        assert (spans[-1][1] if spans else 0) == n
    with pytest.raises(ValueError):
        tp.chunk_spans(10, 0)


def test_mixed_chunk_modes_put_one_chunk_per_request_on_the_source():
    lengths = [5000, 2048, 100]
    assert tp.mixed_chunk_modes(lengths, 2048, None) == [tp.RAW] * 5
    assert tp.mixed_chunk_modes(lengths, 2048, "early") == [tp.MAPPED, tp.RAW, tp.RAW, tp.MAPPED, tp.MAPPED]
    assert tp.mixed_chunk_modes(lengths, 2048, "tail") == [tp.RAW, tp.RAW, tp.MAPPED, tp.MAPPED, tp.MAPPED]
    with pytest.raises(ValueError, match="mixed source block"):
        tp.mixed_chunk_modes(lengths, 2048, "middle")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _commit_scenario(rank, scenario):
    """Two requests per rank; rank 1 is the target (owns rows), rank 0 the source."""
    freed, published = [], []
    target = rank == 1
    ids = ["req-a", "req-b"]
    if scenario == "identity" and rank == 0:
        ids = ["req-a", "req-x"]  # this rank commits another request at position 1
    txns = [HandoffTransaction(rid, 10, rank=rank, allocate=(lambda n: list(range(n))) if target else None,
                               free=freed.append if target else None,
                               publish=published.append if target else None,
                               cancel_after_chunks=2 if (scenario == "cancel" and rank == 0 and i == 0) else None)
            for i, rid in enumerate(ids)]
    for t in txns:
        t.begin()
        for a, b in tp.chunk_spans(10, 4):
            t.chunk(a, b, copy_bytes=(b - a) * 64)

    def settle():
        if scenario == "foreign_device" and rank == 0:
            raise DeviceDataError("slot outside the pool")
        if scenario == "uncertified" and rank == 0:
            raise RuntimeError("stream synchronize failed")

    vote = gloo_vote()
    if scenario == "publish_fails" and target:
        def bad_publish(indices):
            raise RuntimeError("radix insert refused")
        txns[1].publish = bad_publish
    if scenario == "vote_broken" and rank == 0:
        return ("left", 0, 0)  # this rank never votes: the other rank's vote fails
    try:
        receipts = commit(txns, settle=settle, vote=vote, expected_ids=["req-a", "req-b"] if rank == 1 else ids)
        outcome = [r["outcome"] for r in receipts]
    except TransactionError as exc:
        outcome = [r["outcome"] for r in exc.receipts]
    return (outcome, len(freed), len(published))


def _worker(rank, world, port, scenario, results):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    timeout = datetime.timedelta(seconds=5 if scenario == "vote_broken" else 60)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
    try:
        if scenario.startswith("commit:"):
            results[rank] = _commit_scenario(rank, scenario.split(":", 1)[1])
            return
        plan = tp.pair_plan(world, rank, 8)
        if scenario == "vote":
            all_ok = int(tp.publication_vote(True).item())
            one_bad = int(tp.publication_vote(rank != 1).item())
            results[rank] = (all_ok, one_bad)
        elif scenario == "transaction":
            freed, published = [], []

            def write(value, indices, start):
                if rank == 1 and start >= 4:
                    raise RuntimeError("rank 1 lost its peer mapping")

            blocks = [(a, b, torch.zeros(2, 1, b - a)) for a, b in tp.chunk_spans(10, 4)]
            outcome = "published"
            try:
                install_unpublished(
                    token_count=10, allocate=lambda n: list(range(n)), free=freed.append, blocks=blocks,
                    write=write, synchronize=lambda: None,
                    ready_vote=lambda ok: bool(tp.publication_vote(ok).item()), publish=published.append,
                )
            except RuntimeError as exc:
                outcome = str(exc)
            results[rank] = (outcome, len(freed), len(published))
        elif scenario == "exchange":
            # Stand-in payloads: the exchange logic, not CUDA IPC, is under test.
            tp.export_pool = lambda pool: ("pool-of", rank)
            tp.open_pool = lambda exported, device: exported
            opened = tp.exchange_target_pools(plan, object() if plan.role == "target" else None)
            results[rank] = opened
    finally:
        if not (scenario == "commit:vote_broken" and rank == 0):
            dist.destroy_process_group()


def _run(scenario, world=2):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert codes == [0] * world, f"worker exit codes {codes}"
        return dict(results)


def test_publication_vote_is_all_rank_min():
    res = _run("vote")
    assert res == {0: (1, 0), 1: (1, 0)}


def test_one_rank_failure_rolls_back_every_rank():
    res = _run("transaction")
    for rank in (0, 1):
        outcome, freed, published = res[rank]
        assert "rolled back" in outcome
        assert freed == 1 and published == 0  # freed exactly once, never published


def test_source_rank_opens_its_peer_target_pool():
    res = _run("exchange", world=4)
    assert res[0] == ("pool-of", 2) and res[1] == ("pool-of", 3)
    assert res[2] is None and res[3] is None


def test_commit_publishes_when_every_rank_is_ready():
    res = _run("commit:all_ready")
    assert res[0] == ([PUBLISHED, PUBLISHED], 0, 0)  # the source owns no rows
    assert res[1] == ([PUBLISHED, PUBLISHED], 0, 2)


def test_commit_rolls_back_a_cancelled_request_on_every_rank():
    res = _run("commit:cancel")
    assert res[0][0] == [ROLLED_BACK, PUBLISHED] and res[1][0] == [ROLLED_BACK, PUBLISHED]
    assert res[1][1:] == (1, 1)  # the target frees the cancelled rows once and publishes the other


def test_commit_rolls_back_when_a_foreign_rank_reports_a_device_error():
    res = _run("commit:foreign_device")
    for rank in (0, 1):
        assert res[rank][0] == [ROLLED_BACK, ROLLED_BACK]
    assert res[1][1:] == (2, 0)


def test_commit_quarantines_when_a_rank_cannot_certify_its_gpu_work():
    res = _run("commit:uncertified")
    for rank in (0, 1):
        assert res[rank][0] == [QUARANTINED, QUARANTINED]
    assert res[1][1:] == (0, 0)  # nothing freed, nothing published: ownership kept


def test_commit_rolls_back_on_identity_mismatch():
    res = _run("commit:identity")
    for rank in (0, 1):
        assert res[rank][0] == [PUBLISHED, ROLLED_BACK]
    assert res[1][1:] == (1, 1)


def test_commit_quarantines_a_request_whose_publication_failed():
    res = _run("commit:publish_fails")
    for rank in (0, 1):
        assert res[rank][0] == [PUBLISHED, QUARANTINED]
    assert res[1][1:] == (0, 1)  # quarantined rows are not freed


def test_commit_quarantines_when_the_vote_fails():
    res = _run("commit:vote_broken")
    assert res[0] == ("left", 0, 0)
    assert res[1] == ([QUARANTINED, QUARANTINED], 0, 0)
