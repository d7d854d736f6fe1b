"""Property tests (hypothesis) of the host-side helpers of the handoff path:
chunk spans, the TP pair plan, contiguous slot runs and paged token rows."""

from __future__ import annotations

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from cachebridge_b200 import contiguous_runs, token_slots_from_pages
from cachebridge_b200.online.tp import chunk_spans, pair_plan

PROFILE = settings(max_examples=150, deadline=None)


@PROFILE
@given(st.integers(0, 200_000), st.integers(1, 70_000))
def test_chunk_spans_tile_the_history_in_order(n, chunk):
    spans = chunk_spans(n, chunk)
    assert sum(b - a for a, b in spans) == n
    assert all(0 < b - a <= chunk for a, b in spans)
    assert all(spans[i][1] == spans[i + 1][0] for i in range(len(spans) - 1))
    assert not spans or (spans[0][0] == 0 and spans[-1][1] == n)


@PROFILE
@given(st.sampled_from([2, 4, 8]), st.data())
def test_pair_plan_pairs_every_source_with_one_target(world, data):
    total = data.draw(st.sampled_from([h for h in (2, 4, 8, 16) if h % (world // 2) == 0]))
    plans = [pair_plan(world, r, total) for r in range(world)]
    tp = world // 2
    for p in plans:
        assert plans[p.peer].peer == p.rank
        assert {p.role, plans[p.peer].role} == {"source", "target"}
        assert p.head_start == plans[p.peer].head_start == p.tp_rank * p.heads_per_rank
        assert p.heads_per_rank * tp == total
    sources = sorted(p.head_start for p in plans if p.role == "source")
    assert sources == list(range(0, total, total // tp))


@PROFILE
@given(st.lists(st.integers(0, 5000), min_size=0, max_size=300, unique=True))
def test_contiguous_runs_reassemble_the_slot_list(slots):
    runs = contiguous_runs(slots)
    rebuilt = [p + i for a, b, p in runs for i in range(b - a)]
    assert rebuilt == slots
    assert all(a < b for a, b, _ in runs)
    # maximal: consecutive runs never continue each other
    assert all(runs[i][2] + (runs[i][1] - runs[i][0]) != runs[i + 1][2] for i in range(len(runs) - 1))


@PROFILE
@given(st.sampled_from([1, 2, 16, 64]), st.integers(1, 40), st.integers(0, 10_000))
def test_paged_token_rows_are_distinct_and_page_local(page_size, n_pages, seed):
    g = torch.Generator().manual_seed(seed)
    pages = torch.randperm(4 * n_pages + 8, generator=g)[:n_pages]
    slots = token_slots_from_pages(pages, page_size)
    assert slots.numel() == n_pages * page_size
    assert slots.unique().numel() == slots.numel()
    assert torch.equal(slots // page_size, pages.repeat_interleave(page_size))
    assert torch.equal(slots % page_size, torch.arange(page_size).repeat(n_pages))
    if page_size > 1:
        assert len(contiguous_runs(slots.tolist())) <= n_pages
