"""Full-size value parity: every mapped row of a BASELINE configuration against
the FP32 evaluation of the reference algorithm on the same GPU.

  - config 2 (Qwen3-14B -> 32B shapes): all 8192 tokens x 64 layers x 8 heads
    x K/V of one handoff;
  - config 4 (Llama-3.1-8B -> 70B shapes, S = 4, page_size 16 pages from a
    shuffled free-page list): one whole 16384-token request.

The FP32 evaluation is bench.reference_map_fp32, the restatement of
PageMapper.map_page that tests/test_bench_torch_reference.py pins to the
oracle. Tolerance (bench.value_parity): relative Frobenius error <= 5e-3 and
max |ours - f32| <= max |bf16(f32) - f32| + one BF16 ulp of max |f32|, i.e.
the kernels may differ from the reference's own stored BF16 values by at most
one ulp of the largest value. Both figures are printed (-s shows them).
Placement is checked bit-exactly on every pool row against its canary.
"""

from __future__ import annotations

import pytest
import torch

import bench
import cachebridge_b200 as cb

pytestmark = pytest.mark.gpu


def _run(device, *, L_s, L_t, H, D, S, theta, n, rows, src_slots, dst_slots, seed):
    layers = bench.random_layers(L_s=L_s, L_t=L_t, H=H, D=D, S=S, seed=seed)
    mapper = cb.PageMapper.from_tensors(layers, method="cachebridge", source_rope_theta=theta,
                                        target_rope_theta=theta, device=device)
    src_pool = cb.TokenKVPool(layers=L_s, rows=rows, heads=H, head_dim=D, device=device, fill=0.0)
    dst_pool = cb.TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=device, fill=bench.CANARY)
    bench.fill_source_rows(src_pool, src_slots, positions=torch.arange(n), theta=theta, seed=seed + 1, device=device)
    mapper.map_install(src_pool.rows(src_slots), dst_pool.rows(dst_slots), n, 0)
    torch.cuda.synchronize(device)
    cb.raise_for_status(device)
    mask = torch.zeros(rows, dtype=torch.bool, device=device)
    mask[dst_slots] = True
    placement = bench.rows_written(dst_pool, mask, bench.CANARY)
    block = torch.stack((src_pool.k_buffer[:, src_slots], src_pool.v_buffer[:, src_slots]))
    del src_pool
    f32 = bench.reference_map_fp32(layers, block, theta=theta, position_start=0)
    del block
    ours = torch.stack((dst_pool.k_buffer[:, dst_slots], dst_pool.v_buffer[:, dst_slots]))
    values = bench.value_parity(ours, f32)
    del f32, ours, dst_pool
    torch.cuda.empty_cache()
    return mapper.kernel_path(n), placement, values


def test_config2_every_row_matches_the_fp32_reference(cuda_device):
    q = bench.QWEN
    n, rows = 8192, 24576
    g = torch.Generator().manual_seed(5)
    src = torch.randperm(rows, generator=g)[:n].to(cuda_device)
    dst = torch.randperm(rows, generator=g)[:n].to(cuda_device)
    path, placement, values = _run(cuda_device, L_s=q["L_s"], L_t=q["L_t"], H=q["H"], D=q["D"], S=q["S"],
                                   theta=q["theta"], n=n, rows=rows, src_slots=src, dst_slots=dst, seed=11)
    print(f"config 2 ({path}): {values} placement {placement}")
    assert path == "tensor_memory"
    assert placement["ok"], placement
    assert values["ok"], values


def test_config4_whole_request_matches_the_fp32_reference(cuda_device):
    c = bench.LLAMA
    n, ps = c["tokens"], c["page_size"]
    pages = 2 * n // ps
    rows = pages * ps
    g = torch.Generator().manual_seed(41)
    src = cb.token_slots_from_pages(torch.randperm(pages, generator=g)[: n // ps], ps).to(cuda_device)
    dst = cb.token_slots_from_pages(torch.randperm(pages, generator=g)[: n // ps], ps).to(cuda_device)
    path, placement, values = _run(cuda_device, L_s=c["L_s"], L_t=c["L_t"], H=c["H"], D=c["D"], S=c["S"],
                                   theta=c["theta"], n=n, rows=rows, src_slots=src, dst_slots=dst, seed=13)
    print(f"config 4 ({path}): {values} placement {placement}")
    assert path == "tensor_memory"
    assert placement["ok"], placement
    assert values["ok"], values
