"""cachebridge_b200: the CacheBridge online handoff hot path on NVIDIA B200 (sm_100a).

Mapper apply (headwise ridge-map K/V maps with RoPE removal/re-application) fused
with the paged-KV install, behind the reference's ``PageMapper`` / online block
interface. GPU kernels are reached through the C ABI in
``include/cachebridge_b200.h``; there is no CPU fallback.
"""

from .device import RowSet, raise_for_status, read_status
from .install import DirectMappedPoolCodec, contiguous_runs
from .mapper import LayerWeights, PageMapper
from .pool import TokenKVPool, token_slots_from_pages

__all__ = [
    "DirectMappedPoolCodec",
    "LayerWeights",
    "PageMapper",
    "RowSet",
    "TokenKVPool",
    "contiguous_runs",
    "raise_for_status",
    "read_status",
    "token_slots_from_pages",
]
