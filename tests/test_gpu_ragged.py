"""Ragged serving batch (the ragged TP4 configuration, reduced sizes) on one GPU.

A target pool is 70 % occupied by other requests' rows (seeded random
allocation). Twelve requests with LogNormal history lengths are installed
into the free rows through ``map_install_block``. Half of them then get a
suffix appended: more tokens mapped at the following positions into further
free rows. Checked:
  - every request's rows, history and suffix, match the oracle's FP32
    evaluation of its whole sequence within the BF16 bound;
  - occupied rows keep their bytes and never-allocated rows keep the canary
    (bit-exact).
Lengths are LogNormal(ln 384, 1.0) clipped to [32, 2048] (the full
configuration uses ln 4096 and [256, 32768]); the suffix is 96 tokens (full: 1024).
"""

from __future__ import annotations

import math

import pytest
import torch

from cachebridge_b200 import PageMapper, TokenKVPool, raise_for_status
from cachebridge_b200.online.blocks import map_install_block
from oracle import mapper_oracle as orc
from test_gpu_parity import _random_mapper, check_bf16

pytestmark = pytest.mark.gpu

CANARY = -7.25


def test_ragged_batch_with_suffix_append(tmp_path, cuda_device):
    g = torch.Generator().manual_seed(55)
    L_s, L_t, H, D, S, theta = 8, 6, 2, 128, 2, 1e6
    rows, n_req, suffix = 32768, 12, 96
    mapper_dir = _random_mapper(tmp_path, seed=21, L_s=L_s, L_t=L_t, H=H, D=D, S=S)
    mapper = PageMapper(mapper_dir, method="cachebridge", source_rope_theta=theta, target_rope_theta=theta,
                        device=cuda_device)
    lengths = [int(min(2048, max(32, round(math.exp(math.log(384) + torch.randn(1, generator=g).item())))))
               for _ in range(n_req)]
    with_suffix = [q % 2 == 0 for q in range(n_req)]
    totals = [n + (suffix if s else 0) for n, s in zip(lengths, with_suffix)]

    # Target pool: 70 % of the rows belong to other requests.
    target = TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=cuda_device, fill=CANARY)
    perm = torch.randperm(rows, generator=g)
    occupied = perm[: int(0.7 * rows)]
    free = perm[int(0.7 * rows):]
    resident_k = torch.randn(L_t, len(occupied), H, D, generator=g).bfloat16().to(cuda_device)
    resident_v = torch.randn(L_t, len(occupied), H, D, generator=g).bfloat16().to(cuda_device)
    occ = occupied.to(cuda_device)
    target.k_buffer[:, occ] = resident_k
    target.v_buffer[:, occ] = resident_v
    assert sum(totals) <= len(free)

    # Source pool holding every request's full sequence (history + suffix), RoPE-applied.
    src_rows = sum(totals) + 512
    source = TokenKVPool(layers=L_s, rows=src_rows, heads=H, head_dim=D, device=cuda_device, fill=0.0)
    src_perm = torch.randperm(src_rows, generator=g)
    pages, src_idx, dst_idx = [], [], []
    cursor = 0
    for total in totals:
        s_slots = src_perm[cursor:cursor + total]
        d_slots = free[cursor:cursor + total]
        cursor += total
        content = torch.randn(2, L_s, total, H, D, generator=g)
        content *= torch.exp(0.5 * torch.randn(2, L_s, 1, H, D, generator=g))
        cos, sin = orc.qwen_rope(torch.arange(total), head_dim=D, theta=theta)
        page = content.clone()
        page[0] = orc.apply_rope(content[0], cos, sin)
        page = page.bfloat16()
        loc = s_slots.to(cuda_device)
        for l in range(L_s):
            source.k_buffer[l][loc] = page[0, l].to(cuda_device)
            source.v_buffer[l][loc] = page[1, l].to(cuda_device)
        pages.append(page)
        src_idx.append(loc)
        dst_idx.append(d_slots.to(cuda_device))

    # Histories first (every request), then the suffixes (half of them).
    for q in range(n_req):
        map_install_block(mapper, source, src_idx[q], target, dst_idx[q], start=0, stop=lengths[q])
    for q in range(n_req):
        if with_suffix[q]:
            map_install_block(mapper, source, src_idx[q], target, dst_idx[q], start=lengths[q],
                              stop=lengths[q] + suffix)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)

    layers, head_range = orc.load_layers(mapper_dir)
    for q in range(n_req):
        f32 = orc.map_page_f32(layers, pages[q], head_range=head_range, position_start=0, source_theta=theta,
                               target_theta=theta)
        got = torch.stack([target.k_buffer[:, dst_idx[q]], target.v_buffer[:, dst_idx[q]]])
        check_bf16(got, f32)
    assert torch.equal(target.k_buffer[:, occ], resident_k) and torch.equal(target.v_buffer[:, occ], resident_v)
    never = free[sum(totals):].to(cuda_device)
    assert bool((target.k_buffer[:, never].float() == CANARY).all())
    assert bool((target.v_buffer[:, never].float() == CANARY).all())
