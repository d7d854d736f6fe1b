"""Failure detection without a GPU fault: a bounded device-side wait on a flag
that nothing sets gives up, reports CB_DEV_ERR_TIMEOUT through the status
word, and leaves the context usable (the next launches run normally)."""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

from cachebridge_b200 import _native as nat
from cachebridge_b200.device import read_status, status_word

pytestmark = pytest.mark.gpu


def test_bounded_chunk_wait_times_out_and_context_survives(cuda_device):
    lib = nat.load()
    flag = torch.full((1,), -1, dtype=torch.int64, device=cuda_device)  # nothing will ever set it
    status = status_word(cuda_device)
    read_status(cuda_device)  # start clean
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    t0 = time.perf_counter()
    nat.check(lib.cb_chunk_wait(stream, ctypes.c_void_p(flag.data_ptr()), 0, int(0.2e9), ctypes.c_void_p(status.data_ptr())),
              "cb_chunk_wait")
    torch.cuda.synchronize(cuda_device)
    waited = time.perf_counter() - t0
    assert 0.15 < waited < 10.0
    assert read_status(cuda_device) & nat.CB_DEV_ERR_TIMEOUT
    # The context still works: a signal followed by a satisfied wait completes cleanly.
    nat.check(lib.cb_chunk_signal(stream, ctypes.c_void_p(flag.data_ptr()), 5), "cb_chunk_signal")
    nat.check(lib.cb_chunk_wait(stream, ctypes.c_void_p(flag.data_ptr()), 5, int(1e9), ctypes.c_void_p(status.data_ptr())),
              "cb_chunk_wait")
    torch.cuda.synchronize(cuda_device)
    assert read_status(cuda_device) == 0 and int(flag.item()) == 5
    assert float((torch.ones(4, device=cuda_device) * 2).sum()) == 8.0


def test_kernels_skip_work_after_a_device_timeout(cuda_device):
    """Once a bounded wait has flagged CB_DEV_ERR_TIMEOUT in a status word, a
    map + install and a row install given that word do nothing (the rows keep
    their canary), so a chunk whose receive slot never filled is not written;
    after the word is read and cleared the same calls write the rows."""
    from cachebridge_b200 import PageMapper, TokenKVPool
    from cachebridge_b200.device import RowSet, install_rows

    lib = nat.load()
    g = torch.Generator().manual_seed(3)
    L_s, L_t, H, D, S, n, rows = 6, 4, 2, 128, 2, 300, 512
    layers = []
    for _ in range(L_t):
        t = dict(selected=torch.randperm(L_s, generator=g)[:S].long(), headwise=torch.tensor(True))
        for kind in ("k", "v"):
            t[f"{kind}_weight"] = (torch.randn(H, S * D, D, generator=g) / (S * D) ** 0.5).bfloat16().float()
            t[f"{kind}_bias"] = (torch.randn(H, D, generator=g) * 0.1).bfloat16().float()
        layers.append(t)
    mapper = PageMapper.from_tensors(layers, method="cachebridge", source_rope_theta=1e6, target_rope_theta=1e6,
                                     device=cuda_device)
    canary = -7.25
    src = TokenKVPool(layers=L_s, rows=rows, heads=H, head_dim=D, device=cuda_device, fill=0.0)
    src.k_buffer.copy_(torch.randn(src.k_buffer.shape, generator=g).to(cuda_device, torch.bfloat16))
    src.v_buffer.copy_(torch.randn(src.v_buffer.shape, generator=g).to(cuda_device, torch.bfloat16))
    dst = TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=cuda_device, fill=canary)
    src_slots = torch.randperm(rows, generator=g)[:n].to(cuda_device)
    dst_slots = torch.randperm(rows, generator=g)[:n].to(cuda_device)
    block = torch.randn((2, L_t, n, H, D), generator=g).to(cuda_device, torch.bfloat16)

    status = status_word(cuda_device)
    read_status(cuda_device)
    flag = torch.full((1,), -1, dtype=torch.int64, device=cuda_device)  # nothing will ever set it
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    nat.check(lib.cb_chunk_wait(stream, ctypes.c_void_p(flag.data_ptr()), 0, int(0.05e9),
                                ctypes.c_void_p(status.data_ptr())), "cb_chunk_wait")
    mapper.map_install(RowSet.from_pool(src, src_slots), RowSet.from_pool(dst, dst_slots), n, 0)
    install_rows(block, RowSet.from_pool(dst, dst_slots), n)
    torch.cuda.synchronize(cuda_device)
    assert bool((dst.k_buffer.float() == canary).all()) and bool((dst.v_buffer.float() == canary).all())
    assert read_status(cuda_device) & nat.CB_DEV_ERR_TIMEOUT  # read and cleared

    mapper.map_install(RowSet.from_pool(src, src_slots), RowSet.from_pool(dst, dst_slots), n, 0)
    torch.cuda.synchronize(cuda_device)
    assert read_status(cuda_device) == 0
    written = dst.k_buffer[:, dst_slots].float()
    assert not bool((written == canary).any())
