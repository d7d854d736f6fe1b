"""Mapper artifact verification before upload (src/cachebridge/artifacts.py:17-81).

A mapper instance is a descriptor JSON plus ``layer_NNN.safetensors`` files.
``verify_descriptor`` checks, before any tensor reaches a GPU:

- the layer set is exactly ``layer_000 .. layer_{target_layers-1}``, both in
  the descriptor and on disk;
- every file's SHA-256 matches the descriptor;
- with ``check_tensors``, each file has the head-local schema, a duplicate-free
  int64 source-layer support inside ``[0, source_layers)``, the declared
  geometry, finite FP32 coefficients, and a parameter byte total equal to
  ``logical_parameter_bytes``.

Failures raise ``ValueError`` with the reference's messages, because callers
match on them.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

SCHEMA = frozenset({"selected", "headwise", "k_weight", "k_bias", "v_weight", "v_bias"})


def file_sha256(path) -> str:
    digest = hashlib.sha256()
    with open(path, "rb") as stream:
        while chunk := stream.read(1 << 23):
            digest.update(chunk)
    return digest.hexdigest()


def _check_layer(values: dict, desc: dict) -> int:
    """Validate one layer's tensors; return its parameter bytes."""
    import torch

    if set(values) != SCHEMA or not bool(values["headwise"]):
        raise ValueError("Invalid head-local mapper schema")
    sel = values["selected"]
    if sel.ndim != 1 or sel.dtype != torch.int64 or sel.unique().numel() != sel.numel():
        raise ValueError("Invalid source-layer support")
    if sel.numel() == 0 or int(sel.min()) < 0 or int(sel.max()) >= desc.get("source_layers", 40):
        raise ValueError("Source-layer support out of range")
    heads, dim = desc.get("kv_heads", 8), desc.get("head_dim", 128)
    total = 0
    for kind in ("k", "v"):
        w, b = values[f"{kind}_weight"], values[f"{kind}_bias"]
        if tuple(w.shape) != (heads, sel.numel() * dim, dim) or tuple(b.shape) != (heads, dim):
            raise ValueError("Mapper geometry mismatch")
        finite = bool(torch.isfinite(w).all()) and bool(torch.isfinite(b).all())
        if w.dtype != torch.float32 or b.dtype != torch.float32 or not finite:
            raise ValueError("Mapper coefficients must be finite FP32")
        total += w.numel() * w.element_size() + b.numel() * b.element_size()
    return total


def verify_descriptor(path, *, check_tensors: bool = True) -> dict:
    path = Path(path).expanduser().resolve()
    desc = json.loads(path.read_text())
    root = Path(desc["mapper_dir"])
    if not root.is_absolute():
        root = path.parent / root
    root = root.resolve()
    depth = desc.get("target_layers", 64)
    names = {f"layer_{i:03d}.safetensors" for i in range(depth)}
    on_disk = {p.name for p in root.glob("layer_*.safetensors")}
    if set(desc["file_hashes"]) != names or on_disk != names:
        raise ValueError("Missing, extra or noncontiguous mapper layers")
    tensor_bytes = 0
    for name, digest in desc["file_hashes"].items():
        if file_sha256(root / name) != digest:
            raise ValueError(f"Mapper hash mismatch: {name}")
        if check_tensors:
            from safetensors.torch import load_file

            tensor_bytes += _check_layer(load_file(str(root / name)), desc)
    if check_tensors and tensor_bytes != desc["logical_parameter_bytes"]:
        raise ValueError("Logical parameter byte mismatch")
    return {
        "status": "passed",
        "mapper_id": desc["mapper_id"],
        "mapper_dir": str(root),
        "layers": depth,
        "logical_parameter_bytes": tensor_bytes if check_tensors else desc["logical_parameter_bytes"],
        "descriptor_sha256": file_sha256(path),
        "quality": desc.get("quality", "unmeasured"),
    }
