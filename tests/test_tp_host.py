"""Host logic of the tensor-parallel handoff on CPU: pair plan, chunking, the
all-rank publication vote and the pool-handle exchange, run as world_size-2
``gloo`` process groups (no GPU).

Failures are made on the host: one rank reports a local error and the vote
must roll back the transaction on every rank (src/cachebridge/online/blocks.py:114-171,
backends/sglang/runtime/source_mapper_adapter.py:543-548).
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


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scenario, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
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
