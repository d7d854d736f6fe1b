"""Mapper artifact verification (src/cachebridge/artifacts.py:17-81) on CPU."""

import json

import pytest
import torch
from safetensors.torch import save_file

from cachebridge_b200.artifacts import file_sha256, verify_descriptor


def _instance(tmp_path, *, layers=3, heads=2, dim=8, S=2, source_layers=5, mutate=None):
    d = tmp_path / "mapper"
    d.mkdir()
    g = torch.Generator().manual_seed(0)
    total = 0
    for l in range(layers):
        t = {"selected": torch.randperm(source_layers, generator=g)[:S].long(), "headwise": torch.tensor(True)}
        for kind in ("k", "v"):
            t[f"{kind}_weight"] = torch.randn(heads, S * dim, dim, generator=g)
            t[f"{kind}_bias"] = torch.randn(heads, dim, generator=g)
            total += (t[f"{kind}_weight"].numel() + t[f"{kind}_bias"].numel()) * 4
        if mutate:
            mutate(l, t)
        save_file(t, str(d / f"layer_{l:03d}.safetensors"))
    desc = {"mapper_id": "m-1", "mapper_dir": "mapper", "target_layers": layers, "source_layers": source_layers,
            "kv_heads": heads, "head_dim": dim, "logical_parameter_bytes": total,
            "file_hashes": {f"layer_{l:03d}.safetensors": file_sha256(d / f"layer_{l:03d}.safetensors")
                            for l in range(layers)}}
    p = tmp_path / "descriptor.json"
    p.write_text(json.dumps(desc))
    return p, d, desc


def test_valid_instance_passes(tmp_path):
    p, d, desc = _instance(tmp_path)
    out = verify_descriptor(p)
    assert out["status"] == "passed" and out["layers"] == 3
    assert out["logical_parameter_bytes"] == desc["logical_parameter_bytes"]
    assert out["mapper_dir"] == str(d.resolve()) and out["quality"] == "unmeasured"


def test_missing_extra_and_tampered_layers(tmp_path):
    p, d, desc = _instance(tmp_path)
    (d / "layer_003.safetensors").write_bytes(b"x")
    with pytest.raises(ValueError, match="noncontiguous"):
        verify_descriptor(p)
    (d / "layer_003.safetensors").unlink()
    raw = bytearray((d / "layer_001.safetensors").read_bytes())
    raw[-1] ^= 1
    (d / "layer_001.safetensors").write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="hash mismatch: layer_001"):
        verify_descriptor(p)


@pytest.mark.parametrize(
    "mutate,message",
    [
        (lambda l, t: t.pop("headwise"), "schema"),
        (lambda l, t: t.update(selected=torch.tensor([1, 1])), "support"),
        (lambda l, t: t.update(selected=torch.tensor([0, 9])), "out of range"),
        (lambda l, t: t.update(k_bias=torch.zeros(2, 7)), "geometry"),
        (lambda l, t: t["v_weight"].view(-1).__setitem__(0, float("nan")), "finite"),
        (lambda l, t: t.update(k_weight=t["k_weight"].double()), "finite FP32"),
    ],
)
def test_invalid_tensors_are_rejected(tmp_path, mutate, message):
    p, _, _ = _instance(tmp_path, mutate=lambda l, t: mutate(l, t) if l == 1 else None)
    with pytest.raises(ValueError, match=message):
        verify_descriptor(p)


def test_parameter_byte_total(tmp_path):
    p, _, desc = _instance(tmp_path)
    desc["logical_parameter_bytes"] += 4
    p.write_text(json.dumps(desc))
    with pytest.raises(ValueError, match="byte mismatch"):
        verify_descriptor(p)
    assert verify_descriptor(p, check_tensors=False)["logical_parameter_bytes"] == desc["logical_parameter_bytes"]
