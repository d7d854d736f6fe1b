"""Compatibility import (src/cachebridge/online/mapper.py)."""

from .mapping import PageMapper

__all__ = ["PageMapper"]
