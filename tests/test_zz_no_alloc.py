"""cb_map_install_noalloc: the map + install call that takes its key workspace
from the library's fixed per-device array instead of from the caller.

Checked through the C ABI against cb_map_install (caller workspace) on the
same inputs, for two calls in a row that share the array. Both calls run the
same deterministic kernels on the same inputs, so the written rows must be
bit-identical (a scratch-sharing fault that perturbs a few values, such as a
stale key row of the first request read during the second, fails this), and
untouched rows must keep their canary. The file sorts last so that it runs
after every other test, and it also runs alone in a fresh process (where its
first call performs the per-device set-up).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from cachebridge_b200 import PageMapper, TokenKVPool, raise_for_status
from cachebridge_b200 import _native as nat
from cachebridge_b200.device import RowSet, current_stream_ptr

pytestmark = pytest.mark.gpu

CANARY = -7.25
L_S, L_T, H, D, S = 24, 12, 4, 128, 2


def _mapper_dir(tmp_path, seed):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    for l in range(L_T):
        t = {"selected": torch.randperm(L_S, generator=g)[:S].long(), "headwise": torch.tensor(True)}
        for kind in ("k", "v"):
            t[f"{kind}_weight"] = (torch.randn(H, S * D, D, generator=g) / (S * D) ** 0.5).bfloat16().float()
            t[f"{kind}_bias"] = (torch.randn(H, D, generator=g) * 0.1).bfloat16().float()
        save_file(t, str(tmp_path / f"layer_{l:03d}.safetensors"))
    return tmp_path


def _noalloc(mapper, src: RowSet, dst: RowSet, n: int, position_start: int) -> int:
    """One cb_map_install_noalloc call on the current stream; returns its status."""
    call = mapper.prepare(src, dst, n, position_start)  # marshalled C-ABI arguments
    return nat.load().cb_map_install_noalloc(
        mapper._handle, ctypes.c_void_p(current_stream_ptr(mapper.device)), ctypes.byref(call.src_c),
        ctypes.byref(call.dst_c), n, position_start, ctypes.byref(call.src_rope), ctypes.byref(call.dst_rope),
        call.dtype, call.status.data_ptr(),
    )


def test_noalloc_matches_caller_workspace_on_two_calls(tmp_path, cuda_device):
    g = torch.Generator().manual_seed(77)
    mapper = PageMapper(_mapper_dir(tmp_path, 5), method="cachebridge", source_rope_theta=1e6,
                        target_rope_theta=1e6, device=cuda_device)
    src_rows, dst_rows = 1500, 2000
    src = TokenKVPool(layers=L_S, rows=src_rows, heads=H, head_dim=D, dtype=torch.bfloat16, device=cuda_device,
                      fill=0.0)
    src.k_buffer.copy_(torch.randn(src.k_buffer.shape, generator=g).to(cuda_device, torch.bfloat16))
    src.v_buffer.copy_(torch.randn(src.v_buffer.shape, generator=g).to(cuda_device, torch.bfloat16))
    # Two requests of different lengths and positions, mapped back to back.
    requests = [(600, 311), (257, 4099)]
    pools = {}
    for name in ("workspace", "noalloc"):
        pools[name] = TokenKVPool(layers=L_T, rows=dst_rows, heads=H, head_dim=D, dtype=torch.bfloat16,
                                  device=cuda_device, fill=CANARY)
    plans = []
    for n, start in requests:
        src_slots = torch.randperm(src_rows, generator=g)[:n].to(cuda_device)
        dst_slots = torch.randperm(dst_rows, generator=g)[:n].to(cuda_device)
        plans.append((n, start, src_slots, dst_slots))
        assert nat.CB_NOALLOC_SCRATCH_BYTES >= mapper.workspace_bytes(torch.bfloat16, n)

    for n, start, src_slots, dst_slots in plans:
        mapper.map_install(RowSet.from_pool(src, src_slots), RowSet.from_pool(pools["workspace"], dst_slots), n,
                           start)
    for n, start, src_slots, dst_slots in plans:
        rc = _noalloc(mapper, RowSet.from_pool(src, src_slots), RowSet.from_pool(pools["noalloc"], dst_slots), n,
                      start)
        assert rc == nat.CB_OK, nat.load().cb_last_error().decode()
    torch.cuda.synchronize()
    raise_for_status(cuda_device)

    ref, got = pools["workspace"], pools["noalloc"]
    written = torch.zeros(dst_rows, dtype=torch.bool)
    for n, start, src_slots, dst_slots in plans:
        loc = dst_slots.cpu()
        written[loc] = True
        for a, b in ((got.k_buffer, ref.k_buffer), (got.v_buffer, ref.v_buffer)):
            assert torch.equal(a[:, loc.to(cuda_device)], b[:, loc.to(cuda_device)]), "written rows differ"
    for buf in (got.k_buffer, got.v_buffer):
        assert bool((buf[:, (~written).to(cuda_device)].float() == CANARY).all()), "an untouched row changed"


def test_noalloc_rejects_tokens_beyond_its_scratch(tmp_path, cuda_device):
    mapper = PageMapper(_mapper_dir(tmp_path, 6), method="cachebridge", source_rope_theta=1e6,
                        target_rope_theta=1e6, device=cuda_device)
    per_token = mapper.workspace_bytes(torch.bfloat16, 1)
    limit = nat.CB_NOALLOC_SCRATCH_BYTES // per_token
    n = limit + 1
    src = TokenKVPool(layers=L_S, rows=8, heads=H, head_dim=D, dtype=torch.bfloat16, device=cuda_device, fill=0.0)
    dst = TokenKVPool(layers=L_T, rows=8, heads=H, head_dim=D, dtype=torch.bfloat16, device=cuda_device,
                      fill=CANARY)
    slots = torch.zeros(n, dtype=torch.int64, device=cuda_device)
    rc = _noalloc(mapper, RowSet.from_pool(src, slots), RowSet.from_pool(dst, slots), n, 0)
    assert rc == nat.CB_ERR_UNSUPPORTED
    msg = nat.load().cb_last_error().decode()
    assert f"at most {limit} tokens" in msg and str(nat.CB_NOALLOC_SCRATCH_BYTES) in msg
    torch.cuda.synchronize()
    assert bool((dst.k_buffer.float() == CANARY).all()) and bool((dst.v_buffer.float() == CANARY).all())
