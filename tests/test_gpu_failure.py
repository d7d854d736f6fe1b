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
