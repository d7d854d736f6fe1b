"""bench.py's torch restatement of the reference's GPU path (the baseline the
fused kernels are timed against) computes the reference's mapping: checked on
the CPU against the oracle, with the install placing rows bit-exactly."""

from __future__ import annotations

import torch

import bench
from cachebridge_b200 import TokenKVPool
from conftest import rel_frobenius
from oracle import mapper_oracle as orc

CANARY = -7.25


def test_torch_reference_handoff_matches_oracle():
    g = torch.Generator().manual_seed(31)
    L_s, L_t, H, D, S, n, rows, theta, start = 6, 4, 2, 128, 2, 50, 160, 1e6, 7
    layers = bench.random_layers(L_s=L_s, L_t=L_t, H=H, D=D, S=S, seed=3)
    src_slots = torch.randperm(rows, generator=g)[:n]
    dst_slots = torch.randperm(rows, generator=g)[:n]
    src_pool = TokenKVPool(layers=L_s, rows=rows, heads=H, head_dim=D, device="cpu", fill=0.0)
    src_pool.k_buffer.copy_(torch.randn(src_pool.k_buffer.shape, generator=g).bfloat16())
    src_pool.v_buffer.copy_(torch.randn(src_pool.v_buffer.shape, generator=g).bfloat16())
    dst_pool = TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device="cpu", fill=CANARY)

    mapped = bench.torch_reference_handoff(layers, src_pool, src_slots, dst_pool, dst_slots, theta=theta,
                                           position_start=start)

    page = orc.pack(list(src_pool.k_buffer), list(src_pool.v_buffer), src_slots, 0, n)
    ref_layers = [dict(selected=t["selected"].tolist(), k_weight=t["k_weight"], k_bias=t["k_bias"],
                       v_weight=t["v_weight"], v_bias=t["v_bias"]) for t in layers]
    f32 = orc.map_page_f32(ref_layers, page, position_start=start, head_range=(0, H), source_theta=theta,
                           target_theta=theta)
    assert mapped.shape == f32.shape and mapped.dtype == torch.bfloat16
    assert rel_frobenius(mapped.float(), f32) < 3e-3
    assert float(((mapped.float() - f32).abs() / f32.abs().clamp_min(1.0)).max()) < 2e-2
    assert torch.equal(dst_pool.k_buffer[:, dst_slots], mapped[0])
    assert torch.equal(dst_pool.v_buffer[:, dst_slots], mapped[1])
    untouched = torch.ones(rows, dtype=torch.bool)
    untouched[dst_slots] = False
    assert bool((dst_pool.k_buffer[:, untouched].float() == CANARY).all())
    assert bool((dst_pool.v_buffer[:, untouched].float() == CANARY).all())
