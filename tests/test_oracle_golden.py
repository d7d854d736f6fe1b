"""The CPU oracle reproduces the reference's own outputs (golden fixtures).

Pins ``oracle/`` to the reference: every fixture under tests/golden/ was
produced by running the reference implementation (tests/golden/make_golden.py).
"""

from __future__ import annotations

import json

import pytest
import torch

from conftest import DENSE_CASES, GOLDEN, MAPPER_CASES, load_case, oracle_kwargs
from oracle import mapper_oracle as orc


@pytest.mark.parametrize("name", MAPPER_CASES + DENSE_CASES)
def test_oracle_matches_reference_map_page(name):
    d, params, t = load_case(name)
    layers, head_range = orc.load_layers(d, tp_rank=params.get("tp_rank", 0), tp_size=params.get("tp_size", 1))
    out = orc.map_page(layers, t["page"], head_range=head_range, **oracle_kwargs(params))
    expected = t["expected"]
    assert out.shape == expected.shape and out.dtype == expected.dtype
    torch.testing.assert_close(out, expected, atol=0, rtol=0)
    if "known_answer" in t:
        torch.testing.assert_close(out.float(), t["known_answer"].float(), atol=1e-5, rtol=1e-5)


def test_oracle_input_page_is_unmodified():
    d, params, t = load_case("qwen_mini_bf16")
    layers, head_range = orc.load_layers(d, tp_rank=params["tp_rank"], tp_size=params["tp_size"])
    page = t["page"].clone()
    orc.map_page(layers, page, head_range=head_range, **oracle_kwargs(params))
    assert torch.equal(page, t["page"])


def test_oracle_compact_shard_equals_full_page():
    # tests/test_fitting.py:189-194: a compact shard with source_head_offset maps bit-exactly.
    for rank in range(2):
        d, params, t = load_case(f"fit_tp_rank{rank}")
        layers, head_range = orc.load_layers(d, tp_rank=rank, tp_size=2)
        full = orc.map_page(layers, t["page"], head_range=head_range, **oracle_kwargs(params))
        kw = oracle_kwargs(params)
        kw["source_head_offset"] = rank * 2
        compact = orc.map_page(layers, t["page"][:, :, :, rank * 2 : rank * 2 + 2], head_range=head_range, **kw)
        assert torch.equal(full, compact)


def test_oracle_pack_matches_reference():
    _, params, t = load_case("pack_blocks")
    k = torch.arange(3 * 700 * 2 * 4).reshape(3, 700, 2, 4).float()
    v = -k
    for start, stop in params["spans"]:
        packed = orc.pack(list(k), list(v), t["indices"], start, stop)
        assert torch.equal(packed, t[f"packed_{start}_{stop}"])


def test_oracle_contiguous_runs():
    assert orc.contiguous_runs([]) == []
    assert orc.contiguous_runs([5, 6, 7, 2, 9, 10]) == [(0, 3, 5), (3, 4, 2), (4, 6, 9)]


def test_peer_geometry_matches_reference_fixture():
    import hashlib

    from peer_geometry_check import operations

    cases = json.loads((GOLDEN / "peer_geometry" / "case.json").read_text())
    for c in cases:
        runs = [tuple(r) for r in c["runs"]]
        ops = operations(c["start"], c["stop"], runs, heads=c["heads"])
        assert len(ops) == c["count"]
        blob = json.dumps([list(o) for o in ops]).encode()
        assert hashlib.sha256(blob).hexdigest() == c["sha256"]
        if "ops" in c:
            assert [list(o) for o in ops] == c["ops"]
