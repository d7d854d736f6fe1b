"""Split-half (Qwen) RoPE parameters for the handoff kernels.

The kernels take, per token, ``cos[t][i]`` and ``sin[t][i]`` for the first half
of the head dimension (the reference duplicates the phase with
``cat(phase, phase)``, src/cachebridge/rope.py:70-71). This module computes the
per-frequency inputs of those tables on the host exactly as the reference does
(src/cachebridge/rope.py:16-72): ``inv_freq = 1 / theta**(2i/D)`` in FP32,
optionally adjusted by YaRN, and the YaRN attention magnitude. The per-token
tables themselves are produced on the GPU by ``cb_rope_table``.
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np
import torch


def _scaling_key(scaling: dict | None):
    if scaling is None:
        return None
    return tuple(sorted(scaling.items()))


@lru_cache(maxsize=64)
def _rope_parameters_cached(head_dim: int, theta: float, scaling_key) -> tuple[np.ndarray, float]:
    scaling = None if scaling_key is None else dict(scaling_key)
    return _rope_parameters(head_dim, theta, scaling)


def _rope_parameters(head_dim: int, theta: float, scaling: dict | None) -> tuple[np.ndarray, float]:
    if head_dim % 2:
        raise ValueError("RoPE head dimension must be even")
    frequency_ids = torch.arange(0, head_dim, 2).float()
    inv_freq = 1.0 / (theta ** (frequency_ids / head_dim))
    magnitude = 1.0
    if scaling is not None:
        rope_type = scaling.get("rope_type", scaling.get("type"))
        if rope_type != "yarn":
            raise ValueError(f"unsupported RoPE scaling type: {rope_type!r}")
        factor = float(scaling["factor"])
        original = int(scaling["original_max_position_embeddings"])
        beta_fast = float(scaling.get("beta_fast", 32))
        beta_slow = float(scaling.get("beta_slow", 1))
        extrapolation = float(scaling.get("extrapolation_factor", 1))
        attention = float(scaling.get("attn_factor", 1))
        if factor <= 1 or original <= 0:
            raise ValueError("YaRN factor must exceed one and original window must be positive")

        # Dimension index whose wavelength completes `rotations` turns over the
        # original context window (the YaRN correction range).
        def dim_for(rotations: float) -> float:
            return head_dim * math.log(original / (rotations * 2 * math.pi)) / (2 * math.log(theta))

        low = max(math.floor(dim_for(beta_fast)), 0)
        high = min(math.ceil(dim_for(beta_slow)), head_dim - 1)
        if low == high:
            high += 0.001
        ramp = torch.clamp((torch.arange(head_dim // 2).float() - low) / (high - low), 0, 1)
        keep = (1 - ramp) * extrapolation
        inv_freq = (inv_freq / factor) * (1 - keep) + inv_freq * keep
        magnitude = (0.1 * math.log(factor) + 1.0) * attention
    return inv_freq.numpy().astype(np.float32), float(magnitude)


def rope_parameters(head_dim: int, theta: float, scaling: dict | None = None) -> tuple[np.ndarray, float]:
    """Return ``(inv_freq[head_dim // 2] float32, magnitude)`` for qwen_rope."""
    return _rope_parameters_cached(int(head_dim), float(theta), _scaling_key(scaling))
