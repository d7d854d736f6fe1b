"""Direct install of mapped blocks into unpublished target pool rows.

``DirectMappedPoolCodec`` is the drop-in for ``_DirectMappedPoolCodec``
(backends/sglang/runtime/source_mapper_adapter.py:366-428) and its certified
peer-copy wrapper (backends/sglang/runtime/peer_adapter.py:172-441): the same
``select`` / ``copy`` / ``synchronize`` / ``workspace_bytes`` / ``runs``
surface, but ``copy`` installs a whole block with ONE ``cb_install_rows``
launch (a row scatter through the slot table, reading the mapped block over
NVLink when it lives on the source GPU) instead of 2 * layers * runs
``copy_`` / ``cudaMemcpyPeerAsync`` calls.
"""

from __future__ import annotations

import torch

from .device import RowSet, install_rows, raise_for_status


def contiguous_runs(values) -> list[tuple[int, int, int]]:
    """``(logical_start, logical_stop, physical_start)`` runs of a slot list
    (source_mapper_adapter.py:349-363). Used for receipts; the install kernel
    does not need them."""
    values = [int(v) for v in values]
    runs: list[tuple[int, int, int]] = []
    begin = 0
    for i in range(1, len(values) + 1):
        if i == len(values) or values[i] != values[i - 1] + 1:
            runs.append((begin, i, values[begin]))
            begin = i
    return runs if values else []


class DirectMappedPoolCodec:
    """Install mapped ``[2, layers, n, heads, dim]`` blocks at ``indices[start:stop]``."""

    def __init__(self, device, pool, indices, *, head_offset: int = 0):
        self.device = torch.device(device)
        self.pool = pool
        self.indices = indices
        self.head_offset = int(head_offset)
        self._runs = None
        self.start = None
        self.stop = None
        self.install_stream = torch.cuda.Stream(device=self.device)

    @property
    def runs(self) -> list[tuple[int, int, int]]:
        """``contiguous_runs`` of the slot list (for receipts). Computed on first
        use: it copies the indices to the host, which the install itself
        never needs."""
        if self._runs is None:
            self._runs = contiguous_runs(self.indices.detach().cpu().tolist())
        return self._runs

    @property
    def workspace_bytes(self) -> int:
        return 0

    def select(self, start, stop):
        self.start, self.stop = start, stop

    def allocate(self, elements):
        return None

    def copy(self, remote, local, elements):
        """Install the selected span from flat ``remote`` storage; returns after GPU completion."""
        if self.start is None or self.stop is None:
            raise RuntimeError("mapped target span was not selected")
        n = self.stop - self.start
        layers = self.pool.layer_num
        heads = self.pool._get_key_buffer(self.pool.start_layer).shape[1] - self.head_offset
        dim = self.pool._get_key_buffer(self.pool.start_layer).shape[2]
        expected = 2 * layers * n * heads * dim
        if elements != expected:
            raise ValueError("mapped target block geometry mismatch")
        block = remote[:elements]
        dst = RowSet.from_pool(self.pool, self.indices[self.start : self.stop], head_offset=self.head_offset)
        self.install_stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.install_stream):
            install_rows(block, dst, n)
        # The ACK may be sent only after all reads of `remote` and pool writes complete.
        self.install_stream.synchronize()
        with torch.cuda.device(self.device):
            raise_for_status(self.device)
        self.start = self.stop = None
        return remote[:elements]

    def synchronize(self):
        self.install_stream.synchronize()
