"""Two-slot source lease (drop-in for src/cachebridge/online/pipeline.py:7-43).

One instance per handoff. It launches nothing: callers own the GPU fences and
acknowledge a slot only once the consumer's reads of it completed on the GPU.
It is a ``SlotLedger`` (online/transaction.py) of ``slots`` buffers that keeps
its token cursor across ``begin`` calls; the messages are the reference's.
"""

from .transaction import SlotLedger


class PipelinedSourceLease(SlotLedger):
    """Hold one source lock while at most one export per output slot is live."""

    def __init__(self, acquire, release, slots=2):
        super().__init__(slots, acquire, release, restart_on_open=False, messages=dict(
            open="pipelined source lease already active", order="pipelined block ownership/order violation",
            settle="slot-local GPU completion required before reuse",
            close="cannot release source lease with live output slots"))

    @property
    def active(self) -> bool:
        return self.is_open

    @property
    def pending(self) -> list:
        return self.held

    def begin(self):
        self.open()

    def export(self, slot, start, stop):
        self.claim(slot, start, stop)

    def acknowledge(self, slot, *, gpu_reads_complete):
        self.settle(slot, gpu_reads_complete=gpu_reads_complete)
