"""TEST INFRASTRUCTURE ONLY: CPU oracle of the CacheBridge handoff hot path.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / ``--impl reference`` arm, always as the checker or the timed CPU
baseline, never by the ``cachebridge_b200`` package.
"""
