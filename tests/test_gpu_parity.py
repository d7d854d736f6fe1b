"""GPU parity: the sm_100a handoff kernels against the reference and the oracle.

Tolerance (stated once, used everywhere below):
  - FP32 storage (CUDA-core kernel): |ours - reference| <= 1e-5 (abs and rel),
    the reference's own example tolerance (examples/fit_and_map.py:44).
  - BF16 storage (tcgen05 kernel: BF16 operands incl. the source-RoPE-removed
    keys, FP32 accumulation, BF16 output): against the FP32 evaluation of the
    mapper (the oracle before its final cast)
        relative Frobenius error          <= 5e-3
        max |ours - f32| / max(1, |f32|)  <= 2e-2
    i.e. the 2e-2 max-abs bound of the north star, normalised for |y| > 1
    where one BF16 storage ulp alone exceeds 2e-2 (the reference's own BF16
    output misses a plain 2e-2 absolute bound there too).
  - Placement (which rows are written, and that all other rows keep their
    canary bytes) is checked bit-exactly.
"""

from __future__ import annotations

import pytest
import torch

from cachebridge_b200 import PageMapper, TokenKVPool, raise_for_status
from cachebridge_b200.install import DirectMappedPoolCodec
from cachebridge_b200.online.blocks import map_install_block, map_write_block, pack_source_block
from conftest import MAPPER_CASES, load_case, oracle_kwargs, rel_frobenius
from oracle import mapper_oracle as orc

pytestmark = pytest.mark.gpu

CANARY = -7.25


def check_bf16(ours: torch.Tensor, f32: torch.Tensor) -> None:
    ours = ours.float().cpu()
    f32 = f32.float().cpu()
    rf = rel_frobenius(ours, f32)
    norm_err = float(((ours - f32).abs() / f32.abs().clamp_min(1.0)).max())
    assert rf <= 5e-3, f"relative Frobenius {rf:.3e}"
    assert norm_err <= 2e-2, f"normalised max error {norm_err:.3e}"


def make_mapper(d, params, device):
    return PageMapper(
        d,
        method="cachebridge",
        source_rope_theta=params["source_theta"],
        target_rope_theta=params["target_theta"],
        source_rope_scaling=params.get("source_scaling"),
        target_rope_scaling=params.get("target_scaling"),
        device=device,
        target_tp_rank=params.get("tp_rank", 0),
        target_tp_size=params.get("tp_size", 1),
    )


@pytest.mark.parametrize("name", MAPPER_CASES)
def test_map_page_matches_reference(name, cuda_device):
    d, params, t = load_case(name)
    mapper = make_mapper(d, params, cuda_device)
    page = t["page"]
    out = mapper.map_page(
        page.to(cuda_device),
        position_start=params["position_start"],
        source_head_offset=params.get("source_head_offset", 0),
        output_device=cuda_device,
    )
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    expected = t["expected"]
    assert out.shape == expected.shape and out.dtype == expected.dtype
    if page.dtype == torch.float32:
        torch.testing.assert_close(out.cpu(), expected, atol=1e-5, rtol=1e-5)
    else:
        layers, head_range = orc.load_layers(d, tp_rank=params.get("tp_rank", 0), tp_size=params.get("tp_size", 1))
        f32 = orc.map_page_f32(layers, page, head_range=head_range, **oracle_kwargs(params))
        check_bf16(out, f32)
        # and against the reference's own BF16 output (both rounded to BF16)
        check_bf16(out, expected.float())


def test_map_page_fills_caller_output_and_keeps_input(cuda_device):
    d, params, t = load_case("qwen_mini_bf16")
    mapper = make_mapper(d, params, cuda_device)
    page = t["page"].to(cuda_device)
    before = page.clone()
    output = torch.empty(tuple(t["expected"].shape), dtype=page.dtype, device=cuda_device)
    result = mapper.map_page(page, position_start=params["position_start"], output_device=cuda_device, output=output)
    torch.cuda.synchronize()
    assert result.data_ptr() == output.data_ptr()
    assert torch.equal(page, before)
    with pytest.raises(ValueError, match="preallocated"):
        mapper.map_page(page, position_start=0, output_device=cuda_device, output=output[:, :1])
    with pytest.raises(ValueError, match="required heads"):
        mapper.map_page(page[:, :, :, :1], position_start=0, source_head_offset=0)


def test_compact_shard_is_bit_exact_with_full_page(cuda_device):
    # tests/test_fitting.py:189-194 on the device path.
    for rank in range(2):
        d, params, t = load_case(f"fit_tp_rank{rank}")
        mapper = make_mapper(d, params, cuda_device)
        page = t["page"].to(cuda_device)
        full = mapper.map_page(page, position_start=103, output_device=cuda_device)
        compact = mapper.map_page(
            page[:, :, :, rank * 2 : rank * 2 + 2].contiguous(),
            position_start=103,
            source_head_offset=rank * 2,
            output_device=cuda_device,
        )
        assert torch.equal(full, compact)


def _random_mapper(tmp_path, *, seed, L_s, L_t, H, D, S, bf16=True, w_var=None):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    for l in range(L_t):
        sel = torch.randperm(L_s, generator=g)[:S]
        t = {}
        for kind in ("k", "v"):
            w = torch.randn(H, S * D, D, generator=g) * (w_var or 1.0 / (S * D)) ** 0.5
            b = torch.randn(H, D, generator=g) * 0.1
            if bf16:
                w, b = w.bfloat16().float(), b.bfloat16().float()
            t[f"{kind}_weight"], t[f"{kind}_bias"] = w, b
        t["selected"] = sel.long()
        t["headwise"] = torch.tensor(True)
        save_file(t, str(tmp_path / f"layer_{l:03d}.safetensors"))
    return tmp_path


def _content_pool(g, *, layers, rows, heads, D, dtype, theta, positions, slots, device, scaling=None):
    """Source pool whose rows `slots` hold a RoPE-applied synthetic history."""
    n = len(positions)
    content = torch.randn(2, layers, n, heads, D, generator=g)
    content *= torch.exp(0.5 * torch.randn(2, layers, 1, heads, D, generator=g))
    cos, sin = orc.qwen_rope(positions, head_dim=D, theta=theta, scaling=scaling)
    page = content.clone()
    page[0] = orc.apply_rope(content[0], cos, sin)
    page = page.to(dtype)
    pool = TokenKVPool(layers=layers, rows=rows, heads=heads, head_dim=D, dtype=dtype, device=device, fill=0.0)
    loc = slots.to(device)
    for l in range(layers):
        pool.k_buffer[l][loc] = page[0, l].to(device)
        pool.v_buffer[l][loc] = page[1, l].to(device)
    return pool, page


def _check_install(pool, loc, expected_f32, *, dtype, head_offset=0, heads=None):
    """Rows `loc` of pool match the mapped page; every other row keeps the canary."""
    heads = heads or expected_f32.shape[3]
    k = pool.k_buffer.float().cpu()
    v = pool.v_buffer.float().cpu()
    loc = loc.cpu().long()
    got = torch.stack([k[:, loc, head_offset : head_offset + heads], v[:, loc, head_offset : head_offset + heads]])
    if dtype == torch.float32:
        torch.testing.assert_close(got, expected_f32, atol=1e-5, rtol=1e-5)
    else:
        check_bf16(got, expected_f32)
    mask = torch.ones(pool.size, dtype=torch.bool)
    mask[loc] = False
    for buf in (k, v):
        assert bool((buf[:, mask] == CANARY).all()), "an untouched slot changed"
        if head_offset or heads < buf.shape[2]:
            other = torch.ones(buf.shape[2], dtype=torch.bool)
            other[head_offset : head_offset + heads] = False
            assert bool((buf[:, loc][:, :, other] == CANARY).all()), "an untouched head changed"


@pytest.mark.parametrize(
    "L_s,L_t,H,D,S,n,dtype",
    [
        (4, 6, 2, 64, 2, 512, torch.float32),     # CPU toy configuration (fp32)
        (40, 64, 8, 128, 2, 600, torch.bfloat16),  # Qwen3-14B -> 32B shapes, partial m-tile
        (32, 80, 8, 128, 4, 257, torch.bfloat16),  # Llama-3.1-8B -> 70B shapes (S=4)
        (12, 5, 2, 128, 1, 129, torch.bfloat16),
        (12, 4, 2, 128, 3, 1, torch.bfloat16),
        (12, 3, 2, 128, 5, 300, torch.bfloat16),   # streamed weights (S > 4)
        (12, 3, 2, 128, 8, 130, torch.bfloat16),   # the reference recipe's S=8
    ],
)
def test_fused_pool_to_pool_install(tmp_path, cuda_device, L_s, L_t, H, D, S, n, dtype):
    g = torch.Generator().manual_seed(1000 + S * 7 + n)
    mapper_dir = _random_mapper(tmp_path, seed=S + n, L_s=L_s, L_t=L_t, H=H, D=D, S=S)
    theta = 1e6
    start = 3 * n + 11
    positions = torch.arange(start, start + n)
    src_rows, dst_rows = 2 * n + 64, 4 * n + 128
    src_slots = torch.randperm(src_rows, generator=g)[:n]
    dst_slots = torch.randperm(dst_rows, generator=g)[:n]
    src_pool, page = _content_pool(g, layers=L_s, rows=src_rows, heads=H, D=D, dtype=dtype, theta=theta,
                                   positions=positions, slots=src_slots, device=cuda_device)
    dst_pool = TokenKVPool(layers=L_t, rows=dst_rows, heads=H, head_dim=D, dtype=dtype, device=cuda_device, fill=CANARY)
    mapper = PageMapper(mapper_dir, method="cachebridge", source_rope_theta=theta, target_rope_theta=theta,
                        device=cuda_device)
    # The request's history spans logical tokens [start, start+n): index arrays cover it.
    pad = torch.zeros(start, dtype=torch.long)
    src_idx = torch.cat([pad, src_slots]).to(cuda_device)
    dst_idx = torch.cat([pad, dst_slots]).to(cuda_device)
    map_install_block(mapper, src_pool, src_idx, dst_pool, dst_idx, start=start, stop=start + n)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    layers, head_range = orc.load_layers(mapper_dir)
    f32 = orc.map_page_f32(layers, page, head_range=head_range, position_start=start, source_theta=theta,
                           target_theta=theta)
    _check_install(dst_pool, dst_slots, f32, dtype=dtype)


def test_tp_head_offsets_int32_slots(tmp_path, cuda_device):
    """Rank 1 of TP2: reads source heads 2-3 of a 4-head pool, writes heads 2-3 of the target rows."""
    g = torch.Generator().manual_seed(5)
    L_s, L_t, H, D, n = 10, 6, 4, 128, 333
    mapper_dir = _random_mapper(tmp_path, seed=9, L_s=L_s, L_t=L_t, H=H, D=D, S=2)
    positions = torch.arange(0, n)
    src_slots = torch.randperm(1000, generator=g)[:n].int()
    dst_slots = torch.randperm(2000, generator=g)[:n].int()
    src_pool, page = _content_pool(g, layers=L_s, rows=1000, heads=H, D=D, dtype=torch.bfloat16, theta=1e6,
                                   positions=positions, slots=src_slots.long(), device=cuda_device)
    dst_pool = TokenKVPool(layers=L_t, rows=2000, heads=H, head_dim=D, device=cuda_device, fill=CANARY)
    mapper = PageMapper(mapper_dir, method="cachebridge", source_rope_theta=1e6, target_rope_theta=1e6,
                        device=cuda_device, target_tp_rank=1, target_tp_size=2)
    map_install_block(mapper, src_pool, src_slots.to(cuda_device), dst_pool, dst_slots.to(cuda_device),
                      start=0, stop=n, source_head_offset=0, target_head_offset=2)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    layers, head_range = orc.load_layers(mapper_dir, tp_rank=1, tp_size=2)
    f32 = orc.map_page_f32(layers, page, head_range=head_range, position_start=0, source_theta=1e6, target_theta=1e6)
    _check_install(dst_pool, dst_slots, f32, dtype=torch.bfloat16, head_offset=2, heads=2)


def test_out_of_range_slot_is_reported_not_faulted(tmp_path, cuda_device):
    mapper_dir = _random_mapper(tmp_path, seed=3, L_s=4, L_t=2, H=2, D=128, S=2)
    src_pool = TokenKVPool(layers=4, rows=64, heads=2, head_dim=128, device=cuda_device, fill=0.5)
    dst_pool = TokenKVPool(layers=2, rows=64, heads=2, head_dim=128, device=cuda_device, fill=CANARY)
    mapper = PageMapper(mapper_dir, method="cachebridge", source_rope_theta=1e4, target_rope_theta=1e4,
                        device=cuda_device)
    src = torch.arange(10, device=cuda_device)
    dst = torch.arange(10, device=cuda_device)
    dst[3] = 64  # one past the end of the pool
    map_install_block(mapper, src_pool, src, dst_pool, dst, start=0, stop=10)
    torch.cuda.synchronize()
    with pytest.raises(ValueError, match="outside the pool"):
        raise_for_status(cuda_device)
    # rows 10.. were never addressed and keep the canary
    assert bool((dst_pool.k_buffer[:, 10:].float() == CANARY).all())
    # empty span is a no-op
    with pytest.raises(ValueError):
        map_install_block(mapper, src_pool, src, dst_pool, dst, start=0, stop=0)


def test_pack_source_block_matches_reference(cuda_device):
    _, params, t = load_case("pack_blocks")
    k = torch.arange(3 * 700 * 2 * 4).reshape(3, 700, 2, 4).float().to(cuda_device)
    pool = TokenKVPool(layers=3, rows=700, heads=2, head_dim=4, dtype=torch.float32, device=cuda_device)
    pool.k_buffer.copy_(k)
    pool.v_buffer.copy_(-k)
    indices = t["indices"].to(cuda_device)
    workspace = torch.empty(2 * 3 * 512 * 2 * 4, device=cuda_device)
    for start, stop in params["spans"]:
        packed = pack_source_block(pool, indices, start=start, stop=stop, workspace=workspace, block_tokens=512)
        assert packed.is_contiguous() and packed.data_ptr() == workspace.data_ptr()
        assert torch.equal(packed.cpu(), t[f"packed_{start}_{stop}"])
    with pytest.raises(ValueError, match="workspace"):
        pack_source_block(pool, indices, start=0, stop=4, workspace=workspace[:-1], block_tokens=512)


@pytest.mark.parametrize("heads", [2, 3, 8, 16])
def test_pack_rows_of_every_length_is_a_gather(cuda_device, heads):
    """Row gather of pools whose rows are 512 B (four rows per warp), 768 B
    (a ragged vector count), 2 KB and 4 KB (several rounds of four vectors
    per lane): bit-identical to the torch gather of the same slots."""
    g = torch.Generator().manual_seed(heads)
    layers, rows, n = 5, 3000, 777
    pool = TokenKVPool(layers=layers, rows=rows, heads=heads, head_dim=128, device=cuda_device)
    pool.k_buffer.normal_(generator=torch.Generator(device=cuda_device).manual_seed(heads))
    pool.v_buffer.normal_(generator=torch.Generator(device=cuda_device).manual_seed(heads + 1))
    indices = torch.randperm(rows, generator=g)[:n].to(cuda_device)
    workspace = torch.empty(2 * layers * n * heads * 128, dtype=torch.bfloat16, device=cuda_device)
    packed = pack_source_block(pool, indices, start=0, stop=n, workspace=workspace, block_tokens=n)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    ref = torch.stack((pool.k_buffer[:, indices], pool.v_buffer[:, indices]))
    assert torch.equal(packed.reshape(ref.shape), ref)


def test_install_codec_places_rows_bit_exactly(cuda_device):
    g = torch.Generator().manual_seed(21)
    layers, heads, D, n = 64, 2, 128, 700
    pool = TokenKVPool(layers=layers, rows=4096, heads=heads, head_dim=D, device=cuda_device, fill=CANARY)
    indices = torch.randperm(4096, generator=g)[:n].to(cuda_device)
    codec = DirectMappedPoolCodec(cuda_device, pool, indices)
    block = torch.randn(2, layers, 512, heads, D, generator=g).bfloat16().to(cuda_device)
    codec.select(0, 512)
    codec.copy(block.reshape(-1), None, block.numel())
    rest = torch.randn(2, layers, n - 512, heads, D, generator=g).bfloat16().to(cuda_device)
    codec.select(512, n)
    codec.copy(rest.reshape(-1), None, rest.numel())
    expected = torch.cat([block, rest], dim=2).cpu()
    got = torch.stack([pool.k_buffer[:, indices], pool.v_buffer[:, indices]]).cpu()
    assert torch.equal(got, expected)
    mask = torch.ones(4096, dtype=torch.bool)
    mask[indices.cpu()] = False
    assert bool((pool.k_buffer[:, mask.to(cuda_device)].float() == CANARY).all())
    assert codec.workspace_bytes == 0 and len(codec.runs) >= 1


def test_map_write_block_installs_packed_block(cuda_device):
    d, params, t = load_case("qwen_mini_bf16")
    mapper = make_mapper(d, params, cuda_device)
    page = t["page"].to(cuda_device)
    n = page.shape[2]
    pool = TokenKVPool(layers=mapper.target_layers, rows=4096, heads=mapper.heads, head_dim=128, device=cuda_device,
                       fill=CANARY)
    start = params["position_start"]
    idx = torch.zeros(start + n, dtype=torch.long)
    idx[start:] = t["slots"][:n]
    map_write_block(mapper, page, pool, idx.to(cuda_device), start=start, source_head_offset=0)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    layers, head_range = orc.load_layers(d, tp_rank=1, tp_size=2)
    f32 = orc.map_page_f32(layers, t["page"], head_range=head_range, **oracle_kwargs(params))
    _check_install(pool, t["slots"][:n], f32, dtype=torch.bfloat16)


@pytest.mark.parametrize(
    "theta,scaling,start",
    [
        (1e6, None, 0),
        (1e4, None, 32000),
        (1e6, {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 32768}, 40000),
    ],
)
def test_rope_table_matches_qwen_rope(cuda_device, theta, scaling, start):
    from cachebridge_b200.device import rope_tables

    n, D = 257, 128
    cos, sin = rope_tables(cuda_device, D, theta, scaling, start, n)
    ref_cos, ref_sin = orc.qwen_rope(torch.arange(start, start + n), head_dim=D, theta=theta, scaling=scaling)
    # frequency-major [D/2, n] against the reference's [n, D] (first half)
    torch.testing.assert_close(cos.cpu().T, ref_cos[:, : D // 2], atol=2e-6, rtol=0)
    torch.testing.assert_close(sin.cpu().T, ref_sin[:, : D // 2], atol=2e-6, rtol=0)


def test_padded_destination_rows(tmp_path, cuda_device):
    """Destination rows padded by 16 bytes (not 32-byte aligned) get the same
    bytes as an aligned pool, and the padding keeps its canary."""
    from cachebridge_b200.device import RowSet

    g = torch.Generator().manual_seed(41)
    L_s, L_t, H, D, n, rows = 6, 4, 2, 128, 300, 700
    mapper_dir = _random_mapper(tmp_path, seed=12, L_s=L_s, L_t=L_t, H=H, D=D, S=2)
    src_slots = torch.randperm(rows, generator=g)[:n]
    dst_slots = torch.randperm(rows, generator=g)[:n]
    src_pool, _ = _content_pool(g, layers=L_s, rows=rows, heads=H, D=D, dtype=torch.bfloat16, theta=1e6,
                                positions=torch.arange(n), slots=src_slots, device=cuda_device)
    mapper = PageMapper(mapper_dir, method="cachebridge", source_rope_theta=1e6, target_rope_theta=1e6,
                        device=cuda_device)
    aligned = TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=cuda_device, fill=CANARY)
    stride = H * D + 8  # 16 bytes of padding per row
    flat = torch.full((2, L_t, 8 + rows * stride), CANARY, dtype=torch.bfloat16, device=cuda_device)
    views = [[flat[kind, l, 8:].as_strided((rows, H, D), (stride, D, 1)) for l in range(L_t)] for kind in range(2)]
    padded = RowSet(views[0], views[1], H, D, 0, dst_slots.to(cuda_device))
    src = src_pool.rows(src_slots.to(cuda_device))
    mapper.map_install(src, aligned.rows(dst_slots.to(cuda_device)), n, 0)
    mapper.map_install(src, padded, n, 0)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    for kind, buf in ((0, aligned.k_buffer), (1, aligned.v_buffer)):
        got = torch.stack([views[kind][l] for l in range(L_t)])
        assert torch.equal(got[:, dst_slots.to(cuda_device)], buf[:, dst_slots.to(cuda_device)])
        mask = torch.ones(rows, dtype=torch.bool, device=cuda_device)
        mask[dst_slots.to(cuda_device)] = False
        assert bool((got[:, mask].float() == CANARY).all()), "an untouched row changed"
        pad = flat[kind, :, 8:].reshape(L_t, rows, stride)[:, :, H * D :]
        assert bool((pad.float() == CANARY).all()) and bool((flat[kind, :, :8].float() == CANARY).all())


@pytest.mark.parametrize("start", [0, 389_000, 600_000])
def test_target_rope_at_far_positions(tmp_path, cuda_device, start):
    """Target RoPE in the tensor-core epilogue: phases below 4e5 rad take the
    reduced hardware sin/cos, larger ones sincosf; both against the oracle."""
    g = torch.Generator().manual_seed(77 + start)
    L_s, L_t, H, D, S, n = 6, 3, 2, 128, 2, 200
    mapper_dir = _random_mapper(tmp_path, seed=31, L_s=L_s, L_t=L_t, H=H, D=D, S=S)
    positions = torch.arange(start, start + n)
    src_slots = torch.randperm(400, generator=g)[:n]
    dst_slots = torch.randperm(400, generator=g)[:n]
    src_pool, page = _content_pool(g, layers=L_s, rows=400, heads=H, D=D, dtype=torch.bfloat16, theta=1e6,
                                   positions=positions, slots=src_slots, device=cuda_device)
    dst_pool = TokenKVPool(layers=L_t, rows=400, heads=H, head_dim=D, device=cuda_device, fill=CANARY)
    mapper = PageMapper(mapper_dir, method="cachebridge", source_rope_theta=1e6, target_rope_theta=1e6,
                        device=cuda_device)
    mapper.map_install(src_pool.rows(src_slots.to(cuda_device)), dst_pool.rows(dst_slots.to(cuda_device)), n, start)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    layers, head_range = orc.load_layers(mapper_dir)
    f32 = orc.map_page_f32(layers, page, head_range=head_range, position_start=start, source_theta=1e6,
                           target_theta=1e6)
    _check_install(dst_pool, dst_slots, f32, dtype=torch.bfloat16)


def test_config2_full_size_properties(tmp_path, cuda_device):
    """Qwen3-14B -> 32B shapes at the full 8192-token history: every target
    row lands at its slot and nothing else changes (bit-exact), and a token
    window of every layer and head matches the oracle within the BF16 bound."""
    g = torch.Generator().manual_seed(2024)
    L_s, L_t, H, D, S, n, rows = 40, 64, 8, 128, 2, 8192, 12288
    mapper_dir = _random_mapper(tmp_path, seed=77, L_s=L_s, L_t=L_t, H=H, D=D, S=S)
    src_slots = torch.randperm(rows, generator=g)[:n]
    dst_slots = torch.randperm(rows, generator=g)[:n]
    positions = torch.arange(n)
    src_pool, page = _content_pool(g, layers=L_s, rows=rows, heads=H, D=D, dtype=torch.bfloat16, theta=1e6,
                                   positions=positions, slots=src_slots, device=cuda_device)
    dst_pool = TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=cuda_device, fill=CANARY)
    mapper = PageMapper(mapper_dir, method="cachebridge", source_rope_theta=1e6, target_rope_theta=1e6,
                        device=cuda_device)
    mapper.map_install(src_pool.rows(src_slots.to(cuda_device)), dst_pool.rows(dst_slots.to(cuda_device)), n, 0)
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    untouched = torch.ones(rows, dtype=torch.bool, device=cuda_device)
    untouched[dst_slots.to(cuda_device)] = False
    for buf in (dst_pool.k_buffer, dst_pool.v_buffer):
        assert bool((buf[:, untouched].float() == CANARY).all()), "an untouched row changed"
        assert not bool((buf[:, ~untouched].float() == CANARY).all(dim=-1).any()), "a target row was not written"
    a, b = 5000, 5256  # a window away from the start (large phases, several m-tiles in)
    layers, head_range = orc.load_layers(mapper_dir)
    f32 = orc.map_page_f32(layers, page[:, :, a:b].contiguous(), head_range=head_range, position_start=a,
                           source_theta=1e6, target_theta=1e6)
    loc = dst_slots[a:b].to(cuda_device)
    got = torch.stack([dst_pool.k_buffer[:, loc], dst_pool.v_buffer[:, loc]])
    check_bf16(got, f32)


def test_token_order_does_not_change_results(tmp_path, cuda_device):
    """The processing order of tokens (cb_map_install's token_order) changes
    only which tokens share a 128-token tile: pools written with a
    destination-sorted order and a random order are bit-identical (both run
    map_install_tc_kernel, the kernel that takes an order). Without an order
    the call runs map_install_tm_kernel, whose FP32 bias add and RoPE
    recurrence round differently: its rows match the oracle within the BF16
    tolerance. An order entry outside [0, n) is reported on the device."""
    g = torch.Generator().manual_seed(8)
    L_s, L_t, H, D, S, n, rows = 8, 4, 2, 128, 2, 700, 1500
    mapper_dir = _random_mapper(tmp_path, seed=4, L_s=L_s, L_t=L_t, H=H, D=D, S=S)
    src_slots = torch.randperm(rows, generator=g)[:n].to(cuda_device)
    dst_slots = torch.randperm(rows, generator=g)[:n].to(cuda_device)
    src_pool, page = _content_pool(g, layers=L_s, rows=rows, heads=H, D=D, dtype=torch.bfloat16, theta=1e6,
                                   positions=torch.arange(n), slots=src_slots.cpu(), device=cuda_device)
    mapper = PageMapper(mapper_dir, method="cachebridge", source_rope_theta=1e6, target_rope_theta=1e6,
                        device=cuda_device)
    orders = {"sorted": torch.argsort(dst_slots).to(torch.int32), "none": None,
              "random": torch.randperm(n, generator=g).to(torch.int32).to(cuda_device)}
    pools = {}
    for name, order in orders.items():
        pool = TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=cuda_device, fill=CANARY)
        call = mapper.prepare(src_pool.rows(src_slots), pool.rows(dst_slots), n, 17)
        call.order = order
        call.run()
        pools[name] = pool
    torch.cuda.synchronize()
    raise_for_status(cuda_device)
    assert torch.equal(pools["random"].k_buffer, pools["sorted"].k_buffer)
    assert torch.equal(pools["random"].v_buffer, pools["sorted"].v_buffer)
    layers, head_range = orc.load_layers(mapper_dir)
    f32 = orc.map_page_f32(layers, page, position_start=17, head_range=head_range, source_theta=1e6,
                           target_theta=1e6)
    for name in ("none", "sorted"):
        _check_install(pools[name], dst_slots, f32, dtype=torch.bfloat16)
    bad = torch.arange(n, dtype=torch.int32, device=cuda_device)
    bad[5] = n  # one past the end
    pool = TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=cuda_device, fill=CANARY)
    call = mapper.prepare(src_pool.rows(src_slots), pool.rows(dst_slots), n, 17)
    call.order = bad
    call.run()
    torch.cuda.synchronize()
    with pytest.raises(ValueError, match="outside the pool"):
        raise_for_status(cuda_device)
