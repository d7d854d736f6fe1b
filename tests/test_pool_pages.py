"""Token slots of paged pools (page_size > 1): the row of token i is
page_table[i // page_size] * page_size + i % page_size, and histories must be
non-empty and page-aligned (backends/sglang/runtime/clean_adapter.py:370-373)."""

from __future__ import annotations

import pytest
import torch

from cachebridge_b200 import contiguous_runs, token_slots_from_pages


def test_slots_follow_the_page_table():
    pages = torch.tensor([7, 2, 9])
    slots = token_slots_from_pages(pages, 4)
    assert slots.dtype == torch.int64
    assert slots.tolist() == [28, 29, 30, 31, 8, 9, 10, 11, 36, 37, 38, 39]
    assert token_slots_from_pages(pages, 4, 8).tolist() == [28, 29, 30, 31, 8, 9, 10, 11]
    # page runs appear as contiguous slot runs
    assert contiguous_runs(slots.tolist()) == [(0, 4, 28), (4, 8, 8), (8, 12, 36)]


def test_page_size_one_is_the_identity():
    pages = torch.randperm(50, generator=torch.Generator().manual_seed(3))[:20].to(torch.int32)
    assert torch.equal(token_slots_from_pages(pages, 1), pages.long())


def test_shuffled_free_page_list_gives_distinct_rows():
    g = torch.Generator().manual_seed(11)
    free = torch.randperm(4096, generator=g)
    slots = [token_slots_from_pages(free[q * 64:(q + 1) * 64], 16) for q in range(4)]
    flat = torch.cat(slots)
    assert flat.numel() == 4 * 64 * 16 and flat.unique().numel() == flat.numel()
    assert int(flat.max()) < 4096 * 16


@pytest.mark.parametrize(
    "pages,page_size,n,message",
    [
        (torch.tensor([1, 2]), 16, 20, "page-aligned"),
        (torch.tensor([1, 2]), 16, 0, "page-aligned"),
        (torch.tensor([1, 2]), 16, 48, "fewer tokens"),
        (torch.tensor([1, -2]), 16, None, "negative"),
        (torch.tensor([[1, 2]]), 16, None, "1-D"),
        (torch.tensor([1.0, 2.0]), 16, None, "1-D integer"),
        (torch.tensor([1, 2]), 0, None, "positive"),
    ],
)
def test_invalid_page_tables_are_rejected(pages, page_size, n, message):
    with pytest.raises(ValueError, match=message):
        token_slots_from_pages(pages, page_size, n)
