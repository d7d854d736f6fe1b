"""``cachebridge.online.mapping.PageMapper`` drop-in (src/cachebridge/online/mapping.py:7-33).

The head narrowing of a received source shard is part of
``cachebridge_b200.mapper.PageMapper.map_page``, so both reference entry points
resolve to the same class, as the reference's modularity test requires
(tests/test_backend_modularity.py:112-124).
"""

from ..mapper import PageMapper

__all__ = ["PageMapper"]
