"""Paged pools (page_size 16) on Llama-3.1-8B -> 70B shapes: 32 -> 80 layers,
8 KV heads, head_dim 128, S=4 selected source layers, maps (512 x 128).

Each request's pages come from a seeded shuffled free-page list; its token
rows follow from the page table (token_slots_from_pages) and are installed by
map_install_block in 2048-token blocks, as the online path does. Checked:
every installed row against the oracle's FP32 evaluation within the BF16
bound of the GPU parity tests, and every row of every unused page keeps its
canary bytes (bit-exact). The full-size case holds 4 requests of 16384
tokens; there the oracle checks one 128-token window per request and
placement is checked for every row.
"""

from __future__ import annotations

import pytest
import torch

from cachebridge_b200 import PageMapper, TokenKVPool, raise_for_status, token_slots_from_pages
from cachebridge_b200.online.blocks import map_install_block
from cachebridge_b200.online.tp import chunk_spans
from oracle import mapper_oracle as orc
from test_gpu_parity import CANARY, _random_mapper, check_bf16

pytestmark = pytest.mark.gpu

L_S, L_T, H, D, S, THETA, PAGE = 32, 80, 8, 128, 4, 5e5, 16


def _history(gen, n, device):
    """RoPE-applied BF16 source page [2, L_s, n, H, D] built on the device."""
    content = torch.randn(2, L_S, n, H, D, device=device, generator=gen)
    content *= torch.exp(0.5 * torch.randn(2, L_S, 1, H, D, device=device, generator=gen))
    cos, sin = orc.qwen_rope(torch.arange(n, device=device), head_dim=D, theta=THETA)
    content[0] = orc.apply_rope(content[0], cos, sin)
    return content.bfloat16()


def _run(tmp_path, device, *, n, requests, pages, windows):
    g = torch.Generator().manual_seed(4000 + n)
    gen = torch.Generator(device=device).manual_seed(n)
    mapper_dir = _random_mapper(tmp_path, seed=40, L_s=L_S, L_t=L_T, H=H, D=D, S=S)
    mapper = PageMapper(mapper_dir, method="cachebridge", source_rope_theta=THETA, target_rope_theta=THETA,
                        device=device)
    rows = pages * PAGE
    src_pool = TokenKVPool(layers=L_S, rows=rows, heads=H, head_dim=D, device=device, fill=0.0)
    dst_pool = TokenKVPool(layers=L_T, rows=rows, heads=H, head_dim=D, device=device, fill=CANARY)
    src_free = torch.randperm(pages, generator=g)
    dst_free = torch.randperm(pages, generator=g)
    per = n // PAGE
    checks = []
    for q in range(requests):
        src_idx = token_slots_from_pages(src_free[q * per:(q + 1) * per].to(device), PAGE)
        dst_idx = token_slots_from_pages(dst_free[q * per:(q + 1) * per].to(device), PAGE)
        page = _history(gen, n, device)
        for l in range(L_S):
            src_pool.k_buffer[l][src_idx] = page[0, l]
            src_pool.v_buffer[l][src_idx] = page[1, l]
        a, b = windows(q)
        checks.append((page[:, :, a:b].cpu(), dst_idx[a:b], a))
        del page
        for start, stop in chunk_spans(n, 2048):
            map_install_block(mapper, src_pool, src_idx, dst_pool, dst_idx, start=start, stop=stop)
    torch.cuda.synchronize()
    raise_for_status(device)

    layers, head_range = orc.load_layers(mapper_dir)
    for window, loc, a in checks:
        f32 = orc.map_page_f32(layers, window, head_range=head_range, position_start=a, source_theta=THETA,
                               target_theta=THETA)
        got = torch.stack([dst_pool.k_buffer[:, loc], dst_pool.v_buffer[:, loc]])
        check_bf16(got, f32)
    used = torch.zeros(rows, dtype=torch.bool, device=device)
    used[token_slots_from_pages(dst_free[: requests * per].to(device), PAGE)] = True
    for buf in (dst_pool.k_buffer, dst_pool.v_buffer):
        for l in range(L_T):
            assert bool((buf[l][~used] == CANARY).all()), "a row of an unused page changed"
            assert not bool((buf[l][used] == CANARY).all(dim=-1).any()), "an installed row was not written"


def test_paged_llama_shapes_every_row(tmp_path, cuda_device):
    """4 requests of 320 tokens (20 pages each) in a 192-page pool; the oracle
    checks every installed row."""
    _run(tmp_path, cuda_device, n=320, requests=4, pages=192, windows=lambda q: (0, 320))


def test_paged_llama_full_size(tmp_path, cuda_device):
    """The configuration's 4 requests of 16384 tokens (1024 pages each) in a
    6144-page pool."""
    _run(tmp_path, cuda_device, n=16384, requests=4, pages=6144,
         windows=lambda q: (2048 * (q + 1) + 64 * q, 2048 * (q + 1) + 64 * q + 128))
