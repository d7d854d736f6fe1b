"""Dense (nv_transfer) mapper on the tensor-core path: every target head reads
all source heads of each selected source layer (src/cachebridge/mapper.py:182-203).

Tolerance: the BF16 bound of the GPU parity tests (relative Frobenius
<= 5e-3, max |Δ| / max(1, |y|) <= 2e-2) against the oracle's FP32
evaluation, and against the reference's own BF16 output for the golden case.
"""

from __future__ import annotations

import pytest
import torch

from cachebridge_b200 import PageMapper, TokenKVPool, raise_for_status
from cachebridge_b200._native import NativeError
from cachebridge_b200.online.blocks import map_install_block
from conftest import load_case, oracle_kwargs
from oracle import mapper_oracle as orc
from test_gpu_parity import CANARY, _check_install, _content_pool, check_bf16

pytestmark = pytest.mark.gpu


def _dense_dir(tmp_path, *, seed, L_s, L_t, Hs, H, D, S):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    F = S * Hs * D
    for l in range(L_t):
        t = {"selected": torch.randperm(L_s, generator=g)[:S].long()}
        for kind in ("k", "v"):
            t[f"{kind}_weight"] = (torch.randn(F, H, D, generator=g) / F**0.5).bfloat16().float()
            t[f"{kind}_bias"] = (torch.randn(H, D, generator=g) * 0.1).bfloat16().float()
        save_file(t, str(tmp_path / f"layer_{l:03d}.safetensors"))
    return tmp_path


def test_dense_map_page_matches_reference(cuda_device):
    d, params, t = load_case("dense_mini_bf16")
    mapper = PageMapper(d, method="nv_transfer", source_rope_theta=params["source_theta"],
                        target_rope_theta=params["target_theta"], device=cuda_device,
                        target_tp_rank=params["tp_rank"], target_tp_size=params["tp_size"])
    assert mapper.dense and mapper.source_heads == t["page"].shape[3]
    out = mapper.map_page(t["page"].to(cuda_device), position_start=params["position_start"],
                          output_device=cuda_device)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    assert out.shape == t["expected"].shape and out.dtype == t["expected"].dtype
    layers, head_range = orc.load_layers(d, tp_rank=params["tp_rank"], tp_size=params["tp_size"])
    f32 = orc.map_page_f32(layers, t["page"], head_range=head_range, **oracle_kwargs(params))
    check_bf16(out, f32)
    check_bf16(out, t["expected"].float())
    with pytest.raises(ValueError, match="feature-width"):
        mapper.map_page(t["page"][:, :, :, :2].to(cuda_device), position_start=0, output_device=cuda_device)


def test_dense_needs_head_dim_128():
    d, params, _ = load_case("dense_small_f32")  # head_dim 64: the B200 dense path is BF16 / 128 only
    with pytest.raises(NativeError, match="head_dim 128"):
        PageMapper(d, method="nv_transfer", source_rope_theta=params["source_theta"],
                   target_rope_theta=params["target_theta"], device="cuda:0")


@pytest.mark.parametrize(
    "L_s,L_t,Hs,H,S,n",
    [
        (6, 3, 2, 2, 2, 300),    # 4 feature blocks: weights resident in shared memory
        (12, 4, 8, 8, 2, 600),   # config-2 heads: 16 blocks, weights streamed per m-tile
        (5, 2, 3, 2, 1, 129),    # more source than target heads
    ],
)
def test_dense_pool_to_pool_install(tmp_path, cuda_device, L_s, L_t, Hs, H, S, n):
    g = torch.Generator().manual_seed(90 + n)
    D = 128
    mapper_dir = _dense_dir(tmp_path, seed=n, L_s=L_s, L_t=L_t, Hs=Hs, H=H, D=D, S=S)
    start = 57
    positions = torch.arange(start, start + n)
    src_rows, dst_rows = 2 * n + 64, 3 * n + 32
    src_slots = torch.randperm(src_rows, generator=g)[:n]
    dst_slots = torch.randperm(dst_rows, generator=g)[:n]
    src_pool, page = _content_pool(g, layers=L_s, rows=src_rows, heads=Hs, D=D, dtype=torch.bfloat16, theta=1e6,
                                   positions=positions, slots=src_slots, device=cuda_device)
    dst_pool = TokenKVPool(layers=L_t, rows=dst_rows, heads=H, head_dim=D, device=cuda_device, fill=CANARY)
    mapper = PageMapper(mapper_dir, method="nv_transfer", source_rope_theta=1e6, target_rope_theta=1e6,
                        device=cuda_device)
    pad = torch.zeros(start, dtype=torch.long)
    map_install_block(mapper, src_pool, torch.cat([pad, src_slots]).to(cuda_device), dst_pool,
                      torch.cat([pad, dst_slots]).to(cuda_device), start=start, stop=start + n)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    layers, head_range = orc.load_layers(mapper_dir)
    f32 = orc.map_page_f32(layers, page, head_range=head_range, position_start=start, source_theta=1e6,
                           target_theta=1e6)
    _check_install(dst_pool, dst_slots, f32, dtype=torch.bfloat16)
