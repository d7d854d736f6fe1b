"""TEST INFRASTRUCTURE ONLY — CPU (FP32) restatement of the CacheBridge hot path.

This is the parity oracle for the sm_100a kernels. It restates, in plain
PyTorch on the CPU, the reference's algorithm for the online handoff path:

  qwen_rope                 src/cachebridge/rope.py:16-72
  rotate_half/apply/remove  src/cachebridge/rope.py:9-13, 75-89
  PageMapper.map_page       src/cachebridge/mapper.py:116-181 (headwise branch),
                            182-203 (dense nv_transfer branch)
                            and 207-239 (stack, target RoPE, cast to page dtype),
                            after the head narrowing of online/mapping.py:7-33
  pack_source_block         src/cachebridge/online/blocks.py:47-82
  set_kv_buffer install     k_buffer[l][loc] = k (the fake SGLang pool of
                            tests/test_blocks.py:36-41; map_write_block
                            online/blocks.py:86-111)

Parity pin: tests/test_oracle_golden.py checks every function here against
golden vectors produced by running the reference itself
(tests/golden/make_golden.py, committed fixtures under tests/golden/).

It is used only by tests/, __graft_entry__.smoke() and bench.py (CPU baseline
and the ``--impl reference`` arm). Nothing in the ``cachebridge_b200`` package
imports it.
"""

from __future__ import annotations

import math
from pathlib import Path

import torch
from safetensors.torch import load_file


# --------------------------------------------------------------------------
# RoPE (rope.py:9-89)
# --------------------------------------------------------------------------
def qwen_rope(positions: torch.Tensor, *, head_dim: int, theta: float, scaling: dict | None = None):
    """cos, sin ``[tokens, head_dim]`` FP32 with the duplicated half (rope.py:16-72)."""
    if head_dim % 2:
        raise ValueError("RoPE head dimension must be even")
    ids = torch.arange(0, head_dim, 2, device=positions.device).float()
    inv = 1.0 / (theta ** (ids / head_dim))
    magnitude = 1.0
    if scaling is not None:
        kind = scaling.get("rope_type", scaling.get("type"))
        if kind != "yarn":
            raise ValueError(f"unsupported RoPE scaling type: {kind!r}")
        factor = float(scaling["factor"])
        window = int(scaling["original_max_position_embeddings"])
        fast = float(scaling.get("beta_fast", 32))
        slow = float(scaling.get("beta_slow", 1))
        extra = float(scaling.get("extrapolation_factor", 1))
        attn = float(scaling.get("attn_factor", 1))
        if factor <= 1 or window <= 0:
            raise ValueError("YaRN factor must exceed one and original window must be positive")

        def corr(rot):
            return head_dim * math.log(window / (rot * 2 * math.pi)) / (2 * math.log(theta))

        lo = max(math.floor(corr(fast)), 0)
        hi = min(math.ceil(corr(slow)), head_dim - 1)
        if lo == hi:
            hi += 0.001
        ramp = torch.clamp((torch.arange(head_dim // 2, device=positions.device).float() - lo) / (hi - lo), 0, 1)
        mask = (1 - ramp) * extra
        inv = (inv / factor) * (1 - mask) + inv * mask
        magnitude = (0.1 * math.log(factor) + 1.0) * attn
    phase = positions.float().unsqueeze(-1) * inv.unsqueeze(0)
    phase = torch.cat((phase, phase), dim=-1)
    return phase.cos() * magnitude, phase.sin() * magnitude


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    a, b = x.chunk(2, dim=-1)
    return torch.cat((-b, a), dim=-1)


def _view(cos: torch.Tensor) -> tuple:
    return (1, cos.shape[0], 1, cos.shape[1])


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    c = cos.reshape(_view(cos)).to(x)
    s = sin.reshape(_view(sin)).to(x)
    return x * c + rotate_half(x) * s


def remove_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    c = cos.reshape(_view(cos)).to(x)
    s = sin.reshape(_view(sin)).to(x)
    scale = c.square() + s.square()
    return (x * c - rotate_half(x) * s) / scale.clamp_min(torch.finfo(x.dtype).tiny)


# --------------------------------------------------------------------------
# Mapper weights
# --------------------------------------------------------------------------
def load_layers(mapper_dir, *, tp_rank: int = 0, tp_size: int = 1):
    """Head-sliced FP32 mapper tensors per target layer (mapper.py:59-110)."""
    layers = []
    head_range = None
    for path in sorted(Path(mapper_dir).glob("layer_*.safetensors")):
        t = load_file(str(path))
        heads = int(t["k_bias"].shape[0])
        per = heads // tp_size
        rng = (tp_rank * per, tp_rank * per + per)
        head_range = head_range or rng
        sl = slice(*rng)
        headwise = "headwise" in t
        layers.append(
            dict(
                selected=t["selected"].long().tolist(),
                # headwise [H, S*D, D] sliced by head; dense [F, H, D] by column (mapper.py:97-107)
                k_weight=(t["k_weight"][sl] if headwise else t["k_weight"][:, sl]).float(),
                k_bias=t["k_bias"][sl].float(),
                v_weight=(t["v_weight"][sl] if headwise else t["v_weight"][:, sl]).float(),
                v_bias=t["v_bias"][sl].float(),
                headwise=headwise,
            )
        )
    return layers, head_range


# --------------------------------------------------------------------------
# map_page (mapper.py:116-239 + online/mapping.py:7-33)
# --------------------------------------------------------------------------
@torch.inference_mode()
def map_page_f32(
    layers,
    page: torch.Tensor,
    *,
    position_start: int,
    head_range: tuple[int, int],
    source_head_offset: int = 0,
    source_theta: float,
    target_theta: float,
    source_scaling: dict | None = None,
    target_scaling: dict | None = None,
) -> torch.Tensor:
    """FP32 mapped page ``[2, L_t, n, H_r, D]`` before the storage-dtype cast.

    Headwise layers read this rank's heads of the page (online/mapping.py:18-28);
    dense (nv_transfer) layers read every source head (mapper.py:182-203)."""
    dense = bool(layers) and not layers[0].get("headwise", True)
    if not dense:
        start = head_range[0] - source_head_offset
        stop = head_range[1] - source_head_offset
        if not 0 <= start < stop <= page.shape[3]:
            raise ValueError("Received source shard does not contain required heads")
        page = page[:, :, :, start:stop, :]
    _, L_s, n, _, D = page.shape
    positions = torch.arange(position_start, position_start + n, dtype=torch.long)
    scos, ssin = qwen_rope(positions, head_dim=D, theta=source_theta, scaling=source_scaling)
    keys = remove_rope(page[0].float(), scos, ssin)
    values = page[1].float()
    out_k, out_v = [], []
    for layer in layers:
        sel = layer["selected"]
        if not sel or max(sel) >= L_s:
            raise ValueError("mapper selected layer exceeds source page depth")
        if layer.get("headwise", True):
            xk = torch.cat([keys[i] for i in sel], dim=-1)
            xv = torch.cat([values[i] for i in sel], dim=-1)
            out_k.append(torch.einsum("thf,hfd->thd", xk, layer["k_weight"]) + layer["k_bias"])
            out_v.append(torch.einsum("thf,hfd->thd", xv, layer["v_weight"]) + layer["v_bias"])
        else:
            xk = torch.cat([keys[i].reshape(n, -1) for i in sel], dim=-1)
            xv = torch.cat([values[i].reshape(n, -1) for i in sel], dim=-1)
            if xk.shape[-1] != layer["k_weight"].shape[0]:
                raise ValueError("NV Dense feature-width mismatch")
            h, d = layer["k_bias"].shape
            out_k.append((xk @ layer["k_weight"].reshape(xk.shape[-1], -1) + layer["k_bias"].reshape(-1)).reshape(n, h, d))
            out_v.append((xv @ layer["v_weight"].reshape(xv.shape[-1], -1) + layer["v_bias"].reshape(-1)).reshape(n, h, d))
    tk = torch.stack(out_k, dim=0)
    tv = torch.stack(out_v, dim=0)
    tcos, tsin = qwen_rope(positions, head_dim=tk.shape[-1], theta=target_theta, scaling=target_scaling)
    tk = apply_rope(tk, tcos, tsin)
    return torch.stack((tk, tv), dim=0)


def map_page(layers, page: torch.Tensor, **kw) -> torch.Tensor:
    """Mapped page in the page's dtype (mapper.py:216-219 / 237-238 cast)."""
    return map_page_f32(layers, page, **kw).to(page.dtype)


# --------------------------------------------------------------------------
# Pool gather / install (online/blocks.py:47-111 with a fake pool)
# --------------------------------------------------------------------------
def pack(pool_k, pool_v, indices: torch.Tensor, start: int, stop: int) -> torch.Tensor:
    """``[2, layers, stop-start, heads, dim]`` rows gathered at indices[start:stop]."""
    loc = indices[start:stop].long()
    return torch.stack(
        [torch.stack([k[loc] for k in pool_k]), torch.stack([v[loc] for v in pool_v])]
    )


def install(pool_k, pool_v, loc: torch.Tensor, mapped: torch.Tensor, head_offset: int = 0) -> None:
    """``k_buffer[l][loc, heads] = mapped[0, l]`` (SGLang set_kv_buffer semantics)."""
    loc = loc.long()
    h = mapped.shape[3]
    for l in range(mapped.shape[1]):
        pool_k[l][loc, head_offset : head_offset + h] = mapped[0, l]
        pool_v[l][loc, head_offset : head_offset + h] = mapped[1, l]


def contiguous_runs(values) -> list[tuple[int, int, int]]:
    """(logical_start, logical_stop, physical_start) runs of a slot list
    (backends/sglang/runtime/source_mapper_adapter.py:349-363)."""
    values = [int(v) for v in values]
    runs = []
    if not values:
        return runs
    begin = 0
    for i in range(1, len(values)):
        if values[i] != values[i - 1] + 1:
            runs.append((begin, i, values[begin]))
            begin = i
    runs.append((begin, len(values), values[begin]))
    return runs
