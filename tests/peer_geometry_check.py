"""Test-side restatement of the reference's peer-copy span geometry.

A checker, not product code: ``operations`` restates
src/cachebridge/online/peer_geometry.py:4-54 (= backends/sglang/runtime/
peer_geometry.py:4-54), the byte spans ``(kind, layer, src_offset,
dst_offset, size)`` that place one mapped block against fragmented target
runs, with the reference's guards and messages. The B200 path installs the
same bytes with one kernel launch (``cb_install_rows``); the tests pin this
restatement to the fixture made by running the reference and use it to check
that the kernel's placement covers exactly the reference's bytes.
"""

from __future__ import annotations


def operations(start, stop, runs, *, layers=64, heads=4, dim=128, itemsize=2, max_tokens=4096):
    """Return the copy list; raise ``ValueError`` on unsupported or aliasing input."""
    if not 0 <= start < stop or stop - start > max_tokens or (layers, dim, itemsize) != (64, 128, 2) or heads not in (2, 4):
        raise ValueError("unsupported fixed peer-copy geometry")
    n = stop - start
    row = heads * dim * itemsize
    expect = 0
    covered = 0
    spans = []
    for run in runs:
        a, b, p = run
        if not all(isinstance(x, int) for x in run) or a != expect or not a < b or p < 0:
            raise ValueError("invalid ordered logical partition")
        expect = b
        spans.append((p, p + b - a))
        covered += max(0, min(stop, b) - max(start, a))
    spans.sort()
    for (_, end), (begin, _) in zip(spans, spans[1:]):
        if end > begin:
            raise ValueError("target pages alias")
    if covered != n:
        raise ValueError("target runs do not cover exactly one block")
    ops = []
    for layer in range(layers):
        for a, b, p in runs:
            left, right = max(start, a), min(stop, b)
            if left >= right:
                continue
            for kind in (0, 1):
                src = ((kind * layers + layer) * n + left - start) * row
                ops.append((kind, layer, src, (p + left - a) * row, (right - left) * row))
    if sum(op[4] for op in ops) != 2 * layers * n * row:
        raise ValueError("copy-byte invariant")
    return ops
