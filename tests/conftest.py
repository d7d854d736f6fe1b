"""Shared pytest configuration and fixture loaders."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest
import torch
from safetensors.torch import load_file

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"

MAPPER_CASES = [
    "ref_headwise_tp_slice",
    "ref_yarn_identity",
    "fit_and_map",
    "fit_tp_rank0",
    "fit_tp_rank1",
    "cfg1_toy",
    "qwen_mini_bf16",
    "llama_mini_s4",
    "yarn_d128_f32",
    "qwen_s8_compact",
]

# Dense (nv_transfer) mapper fixtures, produced by the reference's dense branch.
DENSE_CASES = ["dense_mini_bf16", "dense_small_f32"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_case(name: str):
    """(case directory, call parameters, tensors) of one golden fixture."""
    d = GOLDEN / name
    params = json.loads((d / "case.json").read_text())
    tensors = load_file(str(d / "case.safetensors")) if (d / "case.safetensors").exists() else {}
    return d, params, tensors


def oracle_kwargs(params: dict) -> dict:
    return dict(
        position_start=params["position_start"],
        source_head_offset=params.get("source_head_offset", 0),
        source_theta=params["source_theta"],
        target_theta=params["target_theta"],
        source_scaling=params.get("source_scaling"),
        target_scaling=params.get("target_scaling"),
    )


def rel_frobenius(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
