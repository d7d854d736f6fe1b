#!/usr/bin/env python
"""Benchmark of the CacheBridge online handoff hot path on B200.

Metric: mapped+installed KV tokens/s, plus p50 handoff latency
at an 8K-token history. One "step" is one handoff: every token of the history
is gathered from the source pool, mapped by the CacheBridge mapper (40 -> 64
layers, 8 KV heads, S=2) and installed into the target pool rows of its page
table.

  N=1  (default)  Qwen3-14B->32B shapes on one GPU: one
                  8192-token request, page_size=1 pools of 262144 slots, seeded
                  random source and target slot lists. The line also carries the
                  latency through run_handoff, a parity check of the installed
                  rows, and BASELINE config 4 (Llama-3.1-8B->70B, S=4, paged) as
                  configs.cfg4.
  N>1  (torchrun) the sharded handoff, source TP N/2 + target TP N/2: rank r <
                  N/2 gathers its heads' raw source rows of every 2048-token
                  chunk into receive slots on target rank r + N/2 (peer stores,
                  CUDA IPC, NVLink); the target maps and installs them into rows
                  it allocates per handoff, and every request is published by
                  the all-rank transaction (online/transaction.py). --config 3:
                  16 x 32768-token requests; --config 5: 64 ragged requests into
                  a 70%-occupied pool with suffix appends. Every target rank
                  checks placement and a value window after the timed steps.
  --impl reference  the reference algorithm on the host CPU (the oracle
                  restatement of src/cachebridge/mapper.py map_page + pool
                  install), on the same config.

All inputs are synthetic and seeded; mapper weights are random-init (bf16
values), source KV ~ N(0,1) x per-channel LogNormal(0, 0.5) with keys stored
RoPE-applied. Inputs are larger than L2 (1.3 GB read + 2.1 GB written per
step), so no L2 flush is needed between steps.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
METRIC = "mapped+installed KV tokens/s; p50 handoff latency at 8K-token history"
UNIT = "tokens/s"

# Qwen3-14B -> Qwen3-32B mapper shapes
QWEN = dict(L_s=40, L_t=64, H=8, D=128, S=2, theta=1e6)
CANARY = -7.25  # value of target pool rows no handoff writes


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ----------------------------------------------------------------------------
# synthetic workload
# ----------------------------------------------------------------------------
def random_layers(*, L_s, L_t, H, D, S, seed):
    """Seeded headwise mapper layers: S distinct source layers per target layer,
    W ~ N(0, 1/(S*D)) and b ~ N(0, 0.01), rounded to bf16 values (stored FP32)."""
    g = torch.Generator().manual_seed(seed)
    layers = []
    for _ in range(L_t):
        sel = torch.randperm(L_s, generator=g)[:S]
        t = dict(selected=sel.long(), headwise=torch.tensor(True))
        for kind in ("k", "v"):
            t[f"{kind}_weight"] = (torch.randn(H, S * D, D, generator=g) / math.sqrt(S * D)).bfloat16().float()
            t[f"{kind}_bias"] = (torch.randn(H, D, generator=g) * 0.1).bfloat16().float()
        layers.append(t)
    return layers


def fill_source_rows(pool, slots, *, positions, theta, seed, device):
    """Write a synthetic RoPE-applied history into pool rows `slots`."""
    from cachebridge_b200.rope import rope_parameters

    g = torch.Generator(device=device).manual_seed(seed)
    H, D = pool.heads, pool.head_dim
    inv, mag = rope_parameters(D, theta)
    inv = torch.from_numpy(inv).to(device)
    phase = positions.to(device).float()[:, None] * inv[None, :]
    cos, sin = (phase.cos() * mag)[:, None, :], (phase.sin() * mag)[:, None, :]
    n = len(slots)
    chunk = 4096
    for l in range(pool.layer_num):
        scale_k = torch.exp(0.5 * torch.randn(1, H, D, generator=g, device=device))
        scale_v = torch.exp(0.5 * torch.randn(1, H, D, generator=g, device=device))
        for a in range(0, n, chunk):
            b = min(n, a + chunk)
            k = torch.randn(b - a, H, D, generator=g, device=device) * scale_k
            v = torch.randn(b - a, H, D, generator=g, device=device) * scale_v
            x0, x1 = k[..., : D // 2], k[..., D // 2 :]
            c, s = cos[a:b], sin[a:b]
            k = torch.cat((x0 * c - x1 * s, x1 * c + x0 * s), dim=-1)
            pool.k_buffer[l][slots[a:b]] = k.to(pool.dtype)
            pool.v_buffer[l][slots[a:b]] = v.to(pool.dtype)


def algorithmic_work(*, n, L_t, H, D, S, used, idx_bytes=8):
    """Per-handoff algorithmic bytes and flops (source rows read once, target rows
    written once, weights once, two slot tables)."""
    bytes_ = n * (2 * used * H * D * 2 + 2 * L_t * H * D * 2) + 2 * L_t * H * (S * D * D + D) * 2 + 2 * n * idx_bytes
    flops = 4 * L_t * H * S * D * D * n
    return bytes_, flops


def measured_peak(key, fallback):
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())[key])
    except Exception:
        return fallback


def measured_peaks():
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def profiled_traffic(name):
    p = ROOT / "profiles" / f"{name}.json"
    try:
        return json.loads(p.read_text())
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a timed region."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"],
                stdout=self.out, stderr=subprocess.DEVNULL,
            )
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.out.flush()
        rows = []
        for line in Path(self.out.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), max=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], pcap=parts[8]))
            except ValueError:
                continue
        os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        busy = [r for r in rows if r["power"] > 300] or rows
        reasons = sorted({name for r in busy for name, key in
                          (("hw_slowdown", "hw"), ("hw_thermal_slowdown", "hwt"),
                           ("sw_thermal_slowdown", "swt"), ("sw_power_cap", "pcap"))
                          if r[key].lower() == "active"})
        return {"sm_mhz": statistics.median(r["sm"] for r in busy), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": reasons, "samples": len(busy), "power_w_max": max(r["power"] for r in rows)}


# ----------------------------------------------------------------------------
# Re-prefill estimate (what the handoff saves)
# ----------------------------------------------------------------------------
QWEN32B = dict(layers=64, hidden=5120, q_heads=64, kv_heads=8, head_dim=128, mlp=25600)


def reprefill_estimate(device, *, tokens, requests, tp, reps=3):
    """Time one Qwen3-32B-shaped decoder layer's prefill over ``tokens`` on
    this rank's tensor-parallel shard (bf16 torch.matmul for QKV, output and
    the gated MLP; causal SDPA with grouped KV heads; random weights), then
    scale to all layers and ``requests`` requests. Norms, RoPE and the two
    per-layer TP all-reduces are left out, so the estimate is a lower bound
    on the real re-prefill time."""
    import torch.nn.functional as F

    c = QWEN32B
    nq, nkv, d = c["q_heads"] // tp, c["kv_heads"] // tp, c["head_dim"]
    inter = c["mlp"] // tp
    g = torch.Generator(device=device).manual_seed(123)

    def w(*shape):
        return (torch.randn(*shape, generator=g, device=device) * 0.02).to(torch.bfloat16)

    wqkv, wo = w(c["hidden"], (nq + 2 * nkv) * d), w(nq * d, c["hidden"])
    wgu, wdown = w(c["hidden"], 2 * inter), w(inter, c["hidden"])
    x = w(tokens, c["hidden"])

    def layer(x):
        qkv = x @ wqkv
        q, k, v = qkv.split([nq * d, nkv * d, nkv * d], dim=-1)
        q = q.view(tokens, nq, d).transpose(0, 1)[None]
        k = k.view(tokens, nkv, d).transpose(0, 1)[None]
        v = v.view(tokens, nkv, d).transpose(0, 1)[None]
        att = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        h = x + att[0].transpose(0, 1).reshape(tokens, nq * d) @ wo
        gate, up = (h @ wgu).chunk(2, dim=-1)
        return h + (F.silu(gate) * up) @ wdown

    with torch.inference_mode():
        for _ in range(2):
            layer(x)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        a.record()
        for _ in range(reps):
            layer(x)
        b.record()
        b.synchronize()
    per_layer = a.elapsed_time(b) / reps
    return dict(ms=per_layer * c["layers"] * requests, per_layer_ms=per_layer, tokens_per_request=tokens,
                requests=requests, layers=c["layers"], tp=tp,
                model="Qwen3-32B-shaped proxy: hidden 5120, 64 q / 8 kv heads, head_dim 128, MLP 25600, "
                      "random bf16 weights; norms, RoPE and TP all-reduces omitted (lower bound)")


# ----------------------------------------------------------------------------
# The reference's torch path on this GPU (the baseline the fused kernels replace)
# ----------------------------------------------------------------------------
def reference_map_fp32(layers, block, *, theta, position_start=0, bf16_keys=False):
    """The reference's PageMapper.map_page on a packed block, before its cast.

    ``block`` is ``[2, L_s, n, H, D]`` (keys RoPE-applied, any device). RoPE is
    removed from the keys of every source layer in FP32,
    (x*cos - rot(x)*sin) / max(cos^2 + sin^2, tiny) (rope.py:82-89); per target
    layer the selected layers are concatenated along features and mapped with
    einsum('thf,hfd->thd') and the FP32 weights plus bias (mapper.py:153-181);
    the keys get the target RoPE (mapper.py:207-239). Returns FP32
    ``[2, L_t, n, H, D]``. ``bf16_keys`` rounds the derotated keys to BF16
    before the einsum, as the kernels do with their tensor-core operand (the
    reference keeps them in FP32); it measures that one rounding on its own.
    """
    dev = block.device
    n, D = block.shape[2], block.shape[4]
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device=dev).float() / D))
    phase = (torch.arange(n, device=dev) + position_start).float()[:, None] * inv[None, :]
    phase = torch.cat((phase, phase), dim=-1)
    cos, sin = phase.cos()[None, :, None, :], phase.sin()[None, :, None, :]

    def rot(x):
        a, b = x.chunk(2, dim=-1)
        return torch.cat((-b, a), dim=-1)

    keys = block[0].float()
    keys = (keys * cos - rot(keys) * sin) / torch.clamp_min(cos * cos + sin * sin, torch.finfo(torch.float32).tiny)
    if bf16_keys:
        keys = keys.to(torch.bfloat16).float()
    values = block[1].float()
    out_k, out_v = [], []
    for t in layers:
        sel = t["selected"].tolist()
        wk, bk = t["k_weight"].to(dev), t["k_bias"].to(dev)
        wv, bv = t["v_weight"].to(dev), t["v_bias"].to(dev)
        xk = torch.cat([keys[s] for s in sel], dim=-1)
        xv = torch.cat([values[s] for s in sel], dim=-1)
        out_k.append(torch.einsum("thf,hfd->thd", xk, wk) + bk)
        out_v.append(torch.einsum("thf,hfd->thd", xv, wv) + bv)
    k = torch.stack(out_k)
    k = k * cos + rot(k) * sin
    return torch.stack((k, torch.stack(out_v)))


def torch_reference_handoff(layers, src_pool, src_slots, dst_pool, dst_slots, *, theta, position_start=0):
    """One handoff the way the reference runs it with torch on a GPU.

    pack_source_block: one index_select per source layer and kind into a
    [2, L_s, n, H, D] block (online/blocks.py:47-82); PageMapper.map_page in
    FP32 (``reference_map_fp32``) and the cast to the pool dtype
    (mapper.py:207-239); install: k_buffer[l][loc] = k per target layer
    (SGLang set_kv_buffer, blocks.py:86-111). Returns the mapped
    [2, L_t, n, H, D] block.
    """
    dev = src_pool.k_buffer.device
    n = len(src_slots)
    L_s, H, D = src_pool.layer_num, src_pool.heads, src_pool.head_dim
    block = torch.empty((2, L_s, n, H, D), dtype=src_pool.dtype, device=dev)
    for l in range(L_s):
        torch.index_select(src_pool.k_buffer[l], 0, src_slots, out=block[0, l])
        torch.index_select(src_pool.v_buffer[l], 0, src_slots, out=block[1, l])
    mapped = reference_map_fp32(layers, block, theta=theta, position_start=position_start).to(dst_pool.dtype)
    for l in range(dst_pool.layer_num):
        dst_pool.k_buffer[l][dst_slots] = mapped[0, l]
        dst_pool.v_buffer[l][dst_slots] = mapped[1, l]
    return mapped


# ----------------------------------------------------------------------------
# Parity checks carried by the bench line
# ----------------------------------------------------------------------------
def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Spacing of BF16 numbers at |x| (8 significant bits), at least the
    smallest normal spacing."""
    e = torch.floor(torch.log2(x.abs().clamp_min(2.0 ** -126)))
    return torch.exp2(e - 7)


def value_parity(ours: torch.Tensor, f32: torch.Tensor) -> dict:
    """Our BF16 rows against the FP32 evaluation of the reference algorithm.

    The reference itself stores bf16(f32): its own max-abs against f32 is
    ``ref_bf16_max_abs``. Passing requires relative Frobenius error <= 5e-3
    and max |ours - f32| <= ref_bf16_max_abs + ulp_bf16(max |f32|): the
    kernels' BF16 operands and output rounding may cost at most one BF16 ulp
    of the largest value beyond the reference's own rounding. ``max_ulps`` is
    the largest per-element distance from the reference's stored value, in
    BF16 ulps at that value, over the elements with |y| >= 1 (informational;
    near zero, where cancellation leaves |y| far below its inputs, one ulp is
    tiny).
    """
    ours = ours.float()
    f32 = f32.float()
    ref = f32.to(torch.bfloat16).float()
    err = (ours - f32).abs()
    ref_err = (ref - f32).abs()
    rel = float((ours - f32).double().norm() / f32.double().norm().clamp_min(1e-30))
    max_abs, ref_max = float(err.max()), float(ref_err.max())
    y_max = float(f32.abs().max())
    bound = ref_max + float(bf16_ulp(torch.tensor(y_max)))
    big = f32.abs() >= 1.0
    ulps = float(((ours - ref).abs() / bf16_ulp(ref))[big].max()) if bool(big.any()) else 0.0
    return dict(rel_frobenius=rel, max_abs=max_abs, ref_bf16_max_abs=ref_max, max_abs_bound=bound, y_max=y_max,
                max_ulps=ulps, elements=int(ours.numel()), ok=bool(rel <= 5e-3 and max_abs <= bound))


def rows_written(pool, rows_mask: torch.Tensor, canary: float) -> dict:
    """Placement, bit-exact: in every layer and kind, a row holds anything but
    the canary exactly when ``rows_mask`` marks it (no written row left at the
    canary, no other row touched)."""
    bad = 0
    canary_t = torch.tensor(canary, dtype=pool.dtype, device=pool.k_buffer.device)
    for buf in (pool.k_buffer, pool.v_buffer):
        for l in range(buf.shape[0]):
            changed = (buf[l] != canary_t).flatten(1).any(dim=1)
            bad += int((changed != rows_mask).sum())
    return dict(rows=int(rows_mask.sum()), mismatched_rows=bad, ok=bad == 0)


def torch_reference_timing(layers, src_pool, src_slots, dst_pool, dst_slots, *, theta, reps=3):
    """Device time of torch_reference_handoff (CUDA events, after one warm-up
    run), and how far its mapped rows are from the rows the fused kernels
    installed in ``dst_pool`` before this call (relative Frobenius error and
    max |difference|, both against BF16 outputs)."""
    dev = src_pool.k_buffer.device
    gpu_layers = [{k: (v.to(dev) if k != "selected" else v) for k, v in t.items()} for t in layers]
    # The fused kernels' rows, read before the torch path overwrites them.
    ours = torch.stack((dst_pool.k_buffer[:, dst_slots], dst_pool.v_buffer[:, dst_slots]))
    mapped = torch_reference_handoff(gpu_layers, src_pool, src_slots, dst_pool, dst_slots, theta=theta)
    err2 = ref2 = max_abs = 0.0
    for kind in range(2):
        for l in range(mapped.shape[1]):
            m, o = mapped[kind, l].float(), ours[kind, l].float()
            err2 += float((m - o).square().sum())
            ref2 += float(m.square().sum())
            max_abs = max(max_abs, float((m - o).abs().max()))
    rel = math.sqrt(err2 / ref2)
    del ours, mapped
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    a.record()
    for _ in range(reps):
        torch_reference_handoff(gpu_layers, src_pool, src_slots, dst_pool, dst_slots, theta=theta)
    b.record()
    b.synchronize()
    torch.cuda.empty_cache()
    return a.elapsed_time(b) / reps, rel, max_abs


# ----------------------------------------------------------------------------
# CPU reference (oracle restatement of the reference's torch CPU path)
# ----------------------------------------------------------------------------
def cpu_reference_tokens_per_s(layers, *, n_sample, reps, seed=7, heads=None):
    """Time the reference algorithm (map_page + SGLang-style install) on the
    host, for the first ``heads`` KV heads (all by default)."""
    from oracle import mapper_oracle as orc

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    L_s, D = QWEN["L_s"], QWEN["D"]
    H = heads or QWEN["H"]
    page = (torch.randn(2, L_s, n_sample, H, D, generator=g)).bfloat16()
    head_range = (0, H)
    ref_layers = [dict(selected=t["selected"].tolist(), k_weight=t["k_weight"][:H], k_bias=t["k_bias"][:H],
                       v_weight=t["v_weight"][:H], v_bias=t["v_bias"][:H]) for t in layers]
    L_t = len(ref_layers)
    pool_k = [torch.zeros(2 * n_sample, H, D, dtype=torch.bfloat16) for _ in range(L_t)]
    pool_v = [torch.zeros(2 * n_sample, H, D, dtype=torch.bfloat16) for _ in range(L_t)]
    loc = torch.randperm(2 * n_sample, generator=g)[:n_sample]
    times = []
    for r in range(reps + 1):
        t0 = time.perf_counter()
        out = orc.map_page(ref_layers, page, position_start=r * n_sample, head_range=head_range,
                           source_theta=QWEN["theta"], target_theta=QWEN["theta"])
        orc.install(pool_k, pool_v, loc, out)
        times.append(time.perf_counter() - t0)
    best = statistics.median(times[1:]) if reps else times[0]
    return n_sample / best, torch.get_num_threads()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    layers = random_layers(L_s=QWEN["L_s"], L_t=QWEN["L_t"], H=QWEN["H"], D=QWEN["D"], S=QWEN["S"], seed=11)
    n_sample = args.ref_tokens
    from oracle import mapper_oracle as orc  # noqa: F401  (the timed CPU implementation)

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(3)
    L_s, H, D = QWEN["L_s"], QWEN["H"], QWEN["D"]
    page = torch.randn(2, L_s, n_sample, H, D, generator=g).bfloat16()
    ref_layers = [dict(selected=t["selected"].tolist(), k_weight=t["k_weight"], k_bias=t["k_bias"],
                       v_weight=t["v_weight"], v_bias=t["v_bias"]) for t in layers]
    pool_k = [torch.zeros(2 * n_sample, H, D, dtype=torch.bfloat16) for _ in range(len(ref_layers))]
    pool_v = [torch.zeros(2 * n_sample, H, D, dtype=torch.bfloat16) for _ in range(len(ref_layers))]
    loc = torch.randperm(2 * n_sample, generator=g)[:n_sample]

    def step(i):
        out = orc.map_page(ref_layers, page, position_start=(i * n_sample) % 8192, head_range=(0, H),
                           source_theta=QWEN["theta"], target_theta=QWEN["theta"])
        orc.install(pool_k, pool_v, loc, out)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    times = []
    for i in range(args.steps):
        s0 = time.perf_counter()
        step(i)
        times.append(time.perf_counter() - s0)
    elapsed = time.perf_counter() - t0
    value = n_sample * args.steps / elapsed
    cores = torch.get_num_threads()
    line = dict(
        impl="reference", metric=METRIC, value=value, unit=UNIT, n_gpus=args.gpus, steps=args.steps,
        warmup=args.warmup, ms_per_step=1e3 * elapsed / args.steps, higher_is_better=True,
        scaling="weak" if args.gpus == 1 else "strong", vs_baseline=None, dtype="f32", data="synthetic",
        config=dict(workload=("qwen3-14b->32b single-GPU handoff (BASELINE config 2)" if args.gpus == 1 else
                              f"qwen3-14b->32b {'ragged serving batch (BASELINE config 5)' if args.config == 5 else 'sharded handoff (BASELINE config 3)'}"
                              f", TP{args.gpus // 2}+TP{args.gpus // 2}")
                    + ", reference algorithm on host CPU, bounded sample", tokens_per_step=n_sample,
                    source_layers=L_s, target_layers=QWEN["L_t"], kv_heads=H, head_dim=D, selected=QWEN["S"]),
        cpu_baseline=dict(value=value, unit=UNIT, cores=cores, kind="port",
                          sample=f"{n_sample} of the 8192 history tokens per step (one reference block), "
                                 "all 40->64 layers and 8 heads, FP32 torch on host cores"),
        e2e=dict(value=value, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0),
        latency_p50_ms=1e3 * statistics.median(times),
    )
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------
# N = 1: single-GPU handoff of one 8192-token history
# ----------------------------------------------------------------------------
def handoff_latency(mapper, src_pool, src_slots, dst_pool, *, rows, n, block_tokens, runs, warmup, seed=21):
    """Host-clock latency of whole handoffs through the public coordinator:
    ``run_handoff`` over a ``LocalHandoffEndpoint`` (online/handoff.py), from
    the call until the prefix is published (target rows allocated from a
    free list, every chunk mapped and installed, GPU completion observed,
    device status checked, rows published). The source KV is resident; after
    each handoff the published rows are returned to the free list (the
    engine's later eviction, outside the timed call)."""
    from cachebridge_b200.online.handoff import HandoffRequest, LocalHandoffEndpoint, run_handoff
    from cachebridge_b200.online.transaction import SlotAllocator

    alloc = SlotAllocator(rows, device=src_pool.k_buffer.device, seed=seed)
    published = []
    endpoint = LocalHandoffEndpoint(mapper, src_pool, dst_pool, source_slots=lambda rid, k: src_slots[:k],
                                    allocate=alloc.allocate, publish=published.append, free=alloc.free)
    history = tuple(range(n))
    times = []
    for i in range(warmup + runs):
        req = HandoffRequest(request_id=f"bench-{i}", phase=f"p{i}", history_ids=history, namespace="bench",
                             target_ranks=1, block_tokens=block_tokens)
        t0 = time.perf_counter()
        run_handoff(endpoint, req, timeout=60, poll_interval=0.0)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
        alloc.free(published.pop())
    return dict(p50_ms=1e3 * statistics.median(times), min_ms=1e3 * min(times), runs=runs,
                block_tokens=block_tokens,
                path="run_handoff(LocalHandoffEndpoint): allocate target rows, map_install_block per chunk, "
                     "GPU completion, device status, publish")


def run_single(args):
    import cachebridge_b200 as cb
    from cachebridge_b200.online.blocks import map_write_block

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, rows = args.tokens, args.pool_slots
    L_s, L_t, H, D, S, theta = (QWEN[k] for k in ("L_s", "L_t", "H", "D", "S", "theta"))
    layers = random_layers(L_s=L_s, L_t=L_t, H=H, D=D, S=S, seed=11)
    mapper = cb.PageMapper.from_tensors(layers, method="cachebridge", source_rope_theta=theta,
                                        target_rope_theta=theta, device=dev)
    used = len({int(x) for t in layers for x in t["selected"]})
    g = torch.Generator().manual_seed(5)
    src_slots = torch.randperm(rows, generator=g)[:n].to(dev)
    dst_slots = torch.randperm(rows, generator=g)[:n].to(dev)
    log(f"allocating pools: source {L_s}x{rows} rows, target {L_t}x{rows} rows")
    src_pool = cb.TokenKVPool(layers=L_s, rows=rows, heads=H, head_dim=D, device=dev, fill=0.0)
    dst_pool = cb.TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=dev, fill=CANARY)
    fill_source_rows(src_pool, src_slots, positions=torch.arange(n), theta=theta, seed=9, device=dev)
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        call = mapper.prepare(src_pool.rows(src_slots), dst_pool.rows(dst_slots), n, position_start=0)
    launches_per_step = 2  # key gather/derotation + fused map/install
    bytes_alg, flops = algorithmic_work(n=n, L_t=L_t, H=H, D=D, S=S, used=used)

    def step():
        call.derotate()
        call.install()

    # ---- parity of the installed rows (first handoff into a canary pool) -----
    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    cb.raise_for_status(dev)
    mask = torch.zeros(rows, dtype=torch.bool, device=dev)
    mask[dst_slots] = True
    placement = rows_written(dst_pool, mask, CANARY)
    block = torch.stack((src_pool.k_buffer[:, src_slots], src_pool.v_buffer[:, src_slots]))
    f32 = reference_map_fp32(layers, block, theta=theta, position_start=0)
    ours = torch.stack((dst_pool.k_buffer[:, dst_slots], dst_pool.v_buffer[:, dst_slots]))
    values = value_parity(ours, f32)
    del ours
    # The kernels' one rounding step the reference does not have: derotated
    # keys rounded to BF16 before the GEMM. The same FP32 algorithm with only
    # that rounding added, against the FP32 result, on the mapped keys.
    f32_k = reference_map_fp32(layers, block, theta=theta, position_start=0, bf16_keys=True)[0]
    dk = f32_k - f32[0]
    key_rounding = dict(max_abs=float(dk.abs().max()),
                        rel_frobenius=float(dk.double().norm() / f32[0].double().norm().clamp_min(1e-30)),
                        ref_bf16_max_abs_keys=float((f32[0].to(torch.bfloat16).float() - f32[0]).abs().max()),
                        what="FP32 reference with the derotated keys rounded to BF16 before the einsum, "
                             "against the FP32 reference (mapped keys, all tokens, layers and heads)")
    values["key_rounding"] = key_rounding
    del block, f32, f32_k, dk, mask
    torch.cuda.empty_cache()
    parity = dict(placement=placement, values=values, ok=bool(placement["ok"] and values["ok"]),
                  scope=f"all {n} tokens x {L_t} layers x {H} heads x K/V against the FP32 restatement of the "
                        "reference algorithm on this GPU; every pool row checked against its canary")
    log(f"parity: {parity}")

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
    stream.synchronize()
    cb.raise_for_status(dev)

    # ---- device-resident timing (value, per-kernel) --------------------------
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for k in range(args.steps):
                ev[k][0].record(stream)
                call.derotate()
                ev[k][1].record(stream)
                call.install()
                ev[k][2].record(stream)
            end.record(stream)
        end.synchronize()
    cb.raise_for_status(dev)
    total_ms = start.elapsed_time(end)
    step_ms = [ev[k][0].elapsed_time(ev[k][2]) for k in range(args.steps)]
    tc_ms = [ev[k][1].elapsed_time(ev[k][2]) for k in range(args.steps)]
    pre_ms = [ev[k][0].elapsed_time(ev[k][1]) for k in range(args.steps)]
    value = n * args.steps / (total_ms / 1e3)

    # ---- latency through the public coordinator (host clock) -----------------
    latency = handoff_latency(mapper, src_pool, src_slots, dst_pool, rows=rows, n=n,
                              block_tokens=args.latency_block_tokens, runs=args.latency_runs, warmup=3)

    # ---- end to end through the public API, host buffers ---------------------
    block_host = torch.empty((2, L_s, n, H, D), dtype=torch.bfloat16).pin_memory()
    for l in range(L_s):  # the history as a packed source block (pack_source_block layout)
        block_host[0, l].copy_(src_pool.k_buffer[l][src_slots].cpu())
        block_host[1, l].copy_(src_pool.v_buffer[l][src_slots].cpu())
    idx_host = dst_slots.cpu().pin_memory()
    status_host = torch.empty(1, dtype=torch.int32).pin_memory()
    block_dev = torch.empty_like(block_host, device=dev)
    idx_dev = torch.empty_like(idx_host, device=dev)
    status = cb.device.status_word(dev)

    def e2e_step():
        block_dev.copy_(block_host, non_blocking=True)
        idx_dev.copy_(idx_host, non_blocking=True)
        map_write_block(mapper, block_dev, dst_pool, idx_dev, start=0, source_head_offset=0)
        status_host.copy_(status, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(2):
            e2e_step()
    stream.synchronize()
    e2e_times = []
    with torch.cuda.stream(stream):
        for _ in range(args.e2e_steps):
            t0 = time.perf_counter()
            e2e_step()
            stream.synchronize()
            if int(status_host.item()):
                raise RuntimeError(f"device status {int(status_host.item())}")
            e2e_times.append(time.perf_counter() - t0)
    e2e_value = n / statistics.mean(e2e_times)
    h2d = block_host.numel() * 2 + idx_host.numel() * 8
    del block_dev, block_host

    # ---- the reference's torch path on this GPU (same pools and slot lists) ------
    try:
        ref_ms, ref_rel, ref_max = torch_reference_timing(layers, src_pool, src_slots, dst_pool, dst_slots,
                                                          theta=theta)
        ref_tps = n / (ref_ms / 1e3)
        torch_ref = dict(ms=ref_ms, tokens_per_s=ref_tps, value_over_torch=value / ref_tps,
                         rel_frobenius_vs_kernels=ref_rel, max_abs_vs_kernels=ref_max,
                         path="pack_source_block (index_select per layer) + PageMapper.map_page (FP32, einsum "
                              "per target layer) + per-layer set_kv_buffer, restated in torch on this GPU")
    except Exception as exc:  # a failed baseline must not hide the bench line
        torch_ref = dict(error=f"{type(exc).__name__}: {exc}"[:300])
        torch.cuda.empty_cache()

    # ---- re-prefill estimate of the same history on this GPU ---------------------
    prefill = reprefill_estimate(dev, tokens=n, requests=1, tp=1)
    prefill["handoff_ms"] = statistics.median(step_ms)
    prefill["handoff_faster"] = prefill["handoff_ms"] < prefill["ms"]

    # ---- CPU baseline (reference algorithm on host cores, bounded sample) -------
    cpu_value, cores = cpu_reference_tokens_per_s(layers, n_sample=args.cpu_tokens, reps=2)

    hbm_peak, tc_peak, peak_kind = measured_peaks()
    tc_sustained = measured_peak("bf16_tflops_sustained", 1400.0)
    # The handoff's algorithmic bytes are moved by its two launches together
    # (key gather/derotation, then the fused map/install), so the roofline is
    # taken over one handoff: both launches' device time. Per kernel: the
    # derotation reads and writes U*H*256 B of keys per token; the map reads
    # those keys and the source values and writes the target rows.
    step_avg_s = statistics.mean(step_ms) / 1e3
    achieved = bytes_alg / step_avg_s / 1e9
    key_bytes = n * used * H * D * 2
    derot_bytes = 2 * key_bytes + n * 8
    map_bytes = bytes_alg  # the workspace keys replace the source keys one for one
    pre_s, map_s = statistics.mean(pre_ms) / 1e3, statistics.mean(tc_ms) / 1e3
    traffic = profiled_traffic("handoff_cfg2_traffic")
    kernel_name = "map_install_tm_kernel" if mapper.tensor_memory_path(n, 0) else "map_install_tc_kernel"
    del src_pool, dst_pool, call
    torch.cuda.empty_cache()

    cfg4 = run_cfg4(args, dev) if not args.skip_cfg4 else None

    line = dict(
        metric=METRIC, value=value, unit=UNIT, n_gpus=1, steps=args.steps, warmup=args.warmup,
        ms_per_step=total_ms / args.steps, higher_is_better=True, scaling="weak", vs_baseline=None,
        dtype="bf16", data="synthetic",
        config=dict(workload="qwen3-14b->32b single-GPU handoff (BASELINE config 2)", history_tokens=n,
                    source_layers=L_s, target_layers=L_t, kv_heads=H, head_dim=D, selected=S,
                    pool_slots=rows, page_size=1, slot_lists="seeded random", l2="inputs larger than L2",
                    parallelism="single GPU (source and target pools on one device)"),
        latency_p50_ms=latency["p50_ms"],
        latency=latency,
        device_ms=dict(p50=statistics.median(step_ms), mean=statistics.mean(step_ms),
                       what="CUDA events around one handoff's two launches"),
        roofline=dict(bound="hbm", achieved=achieved, peak=hbm_peak, unit="GB/s", frac=achieved / hbm_peak,
                      traffic=None if traffic is None else traffic.get("dram_bytes_per_step"),
                      kernel=f"derotate_pack_kernel + {kernel_name} (one handoff)",
                      algorithmic_bytes=bytes_alg, peak_source=peak_kind,
                      tensor_tflops=flops / step_avg_s / 1e12, tensor_frac=flops / step_avg_s / 1e12 / tc_peak,
                      roofline_ms=1e3 * max(bytes_alg / (hbm_peak * 1e9), flops / (tc_peak * 1e12)),
                      kernels={
                          "derotate_pack_kernel": dict(ms=1e3 * pre_s, algorithmic_bytes=derot_bytes,
                                                       gbs=derot_bytes / pre_s / 1e9,
                                                       frac=derot_bytes / pre_s / 1e9 / hbm_peak),
                          kernel_name: dict(ms=1e3 * map_s, algorithmic_bytes=map_bytes,
                                            gbs=map_bytes / map_s / 1e9, frac=map_bytes / map_s / 1e9 / hbm_peak,
                                            tensor_frac_sustained=flops / map_s / 1e12 / tc_sustained),
                      }),
        kernels_ms=dict(map_install=statistics.mean(tc_ms), derotate_pack=statistics.mean(pre_ms)),
        parity=parity,
        cpu_baseline=dict(value=cpu_value, unit=UNIT, cores=cores, kind="port",
                          sample=f"{args.cpu_tokens}-token block of the same workload (40->64 layers, 8 heads), "
                                 "reference torch algorithm restated in oracle/, FP32 on host cores"),
        e2e=dict(value=e2e_value, unit=UNIT, h2d_bytes_per_step=h2d, d2h_bytes_per_step=4,
                 path="map_write_block(pinned host source block -> device, install into the target pool)",
                 latency_p50_ms=1e3 * statistics.median(e2e_times)),
        gpu_launches=launches_per_step * args.steps,
        clocks=clocks.summary(),
        reprefill_estimate=prefill,
        torch_gpu_reference=torch_ref,
        configs=dict(cfg4=cfg4),
    )
    print(json.dumps(line), flush=True)
    return 0 if parity["ok"] and (cfg4 is None or cfg4.get("parity", {}).get("ok", True)) else 1


# ----------------------------------------------------------------------------
# BASELINE config 4 on the same GPU: Llama-3.1-8B -> 70B shapes, S = 4, paged
# ----------------------------------------------------------------------------
LLAMA = dict(L_s=32, L_t=80, H=8, D=128, S=4, theta=5e5, page_size=16, requests=4, tokens=16384)


def run_cfg4(args, dev):
    """Tensor-bound configuration: 4 requests of 16384 tokens, 32 -> 80
    layers, S = 4 (512 x 128 maps), page_size-16 pools whose pages come from
    a seeded shuffled free-page list (source and target). One step maps all 4
    requests (two launches each). Reports tokens/s, the tensor roofline against
    the measured dense bf16 peaks, HBM bytes, per-kernel times (the kernel the
    call selects, and the general kernel for comparison, forced by passing an
    identity token order), and a parity window of one request."""
    import cachebridge_b200 as cb

    c = LLAMA
    L_s, L_t, H, D, S, theta, ps = (c[k] for k in ("L_s", "L_t", "H", "D", "S", "theta", "page_size"))
    n, nreq = args.cfg4_tokens, args.cfg4_requests
    pages = 2 * nreq * n // ps
    rows = pages * ps
    layers = random_layers(L_s=L_s, L_t=L_t, H=H, D=D, S=S, seed=13)
    mapper = cb.PageMapper.from_tensors(layers, method="cachebridge", source_rope_theta=theta,
                                        target_rope_theta=theta, device=dev)
    used = len({int(x) for t in layers for x in t["selected"]})
    g = torch.Generator().manual_seed(41)
    src_pages, dst_pages = torch.randperm(pages, generator=g), torch.randperm(pages, generator=g)
    per = n // ps
    src = [cb.token_slots_from_pages(src_pages[q * per:(q + 1) * per], ps).to(dev) for q in range(nreq)]
    dst = [cb.token_slots_from_pages(dst_pages[q * per:(q + 1) * per], ps).to(dev) for q in range(nreq)]
    log(f"config 4: pools of {rows} rows ({pages} pages of {ps}), source {L_s} layers, target {L_t} layers")
    src_pool = cb.TokenKVPool(layers=L_s, rows=rows, heads=H, head_dim=D, device=dev, fill=0.0)
    dst_pool = cb.TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=dev, fill=CANARY)
    for q in range(nreq):
        fill_source_rows(src_pool, src[q], positions=torch.arange(n), theta=theta, seed=50 + q, device=dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        calls = [mapper.prepare(src_pool.rows(src[q]), dst_pool.rows(dst[q]), n, 0) for q in range(nreq)]

    def timed(steps):
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps * nreq)]
        with torch.cuda.stream(stream):
            for k in range(steps):
                for q, call in enumerate(calls):
                    e = evs[k * nreq + q]
                    e[0].record(stream)
                    call.derotate()
                    e[1].record(stream)
                    call.install()
                    e[2].record(stream)
        stream.synchronize()
        cb.raise_for_status(dev)
        pre = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
        mp = sum(e[1].elapsed_time(e[2]) for e in evs) / steps
        return pre, mp

    with torch.cuda.stream(stream):
        calls[0].run()
    stream.synchronize()
    cb.raise_for_status(dev)
    # Parity of request 0 against the FP32 restatement on a 2048-token window,
    # and placement of its rows (the other requests' rows are still canary).
    a = min(4096, n // 2)
    b = min(a + 2048, n)
    block = torch.stack((src_pool.k_buffer[:, src[0][a:b]], src_pool.v_buffer[:, src[0][a:b]]))
    f32 = reference_map_fp32(layers, block, theta=theta, position_start=a)
    ours = torch.stack((dst_pool.k_buffer[:, dst[0][a:b]], dst_pool.v_buffer[:, dst[0][a:b]]))
    values = value_parity(ours, f32)
    mask = torch.zeros(rows, dtype=torch.bool, device=dev)
    mask[dst[0]] = True
    placement = rows_written(dst_pool, mask, CANARY)
    del block, f32, ours
    timed(2)
    pre_ms, map_ms = timed(args.cfg4_steps)
    for call in calls:  # the general kernel for comparison (an identity order selects it)
        call.order = torch.arange(n, dtype=torch.int32, device=dev)
    timed(1)
    pre_g, map_g = timed(args.cfg4_steps)
    step_ms = pre_ms + map_ms
    tokens = n * nreq
    bytes_alg, flops = algorithmic_work(n=tokens, L_t=L_t, H=H, D=D, S=S, used=used)
    hbm_peak, tc_burst, _ = measured_peaks()
    tc_sust = measured_peak("bf16_tflops_sustained", 1400.0)
    tflops = flops / (step_ms / 1e3) / 1e12
    out = dict(
        workload=f"llama-3.1-8b->70b handoff (BASELINE config 4): {nreq} x {n} tokens, 32 -> 80 layers, 8 heads, S=4, "
                 "page_size 16, pages from a seeded shuffled free-page list", tokens_per_step=tokens,
        value=tokens / (step_ms / 1e3), unit=UNIT, ms_per_step=step_ms,
        kernels_ms=dict(derotate_pack=pre_ms, map_install=map_ms,
                        map_kernel="map_install_tm_kernel" if mapper.tensor_memory_path(n, 0) else "map_install_tc_kernel"),
        general_kernel_ms=dict(derotate_pack=pre_g, map_install_tc_kernel=map_g),
        roofline=dict(bound="tensor", achieved=tflops, unit="TFLOP/s", peak_sustained=tc_sust,
                      frac_sustained=tflops / tc_sust, peak_burst=tc_burst, frac_burst=tflops / tc_burst,
                      roofline_ms_sustained=1e3 * flops / (tc_sust * 1e12),
                      roofline_ms_burst=1e3 * flops / (tc_burst * 1e12), flops=flops,
                      algorithmic_bytes=bytes_alg, hbm_gbs=bytes_alg / (step_ms / 1e3) / 1e9,
                      hbm_roofline_ms=1e3 * bytes_alg / (hbm_peak * 1e9)),
        parity=dict(values=values, placement=placement, ok=bool(values["ok"] and placement["ok"]),
                    scope=f"request 0: tokens {a}..{b - 1} x 80 layers x 8 heads x K/V against the FP32 restatement; "
                          "every pool row against its canary after request 0's install"),
    )
    log(f"config 4: {json.dumps(out)[:400]}")
    del src_pool, dst_pool, calls
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------
# N > 1: sharded handoff (source TP N/2 + target TP N/2 over NVLink)
# ----------------------------------------------------------------------------
OCCUPIED = -3.0  # rows of other requests already in the target pool (config 5)
SUFFIX = 5.0     # rows the target appends after publication (config 5)


def sharded_workload(args, world):
    """Request lengths and pool sizing of the sharded configurations.

    config 3: 16 requests x 32768 tokens; the target pool holds them plus
    ``pool_slack`` free rows. config 5: 64 ragged requests (scaled by N/8
    below 8 GPUs), lengths ~ LogNormal(ln 4096, 1) clipped to [256, 32768],
    into a target pool that is 70 % occupied by other requests' rows, with a
    1024-token suffix appended to every other request after publication.
    """
    if args.config == 5:
        g = torch.Generator().manual_seed(555)
        count = max(2, 64 * world // 8)
        lengths = torch.exp(math.log(4096) + torch.randn(count, generator=g)).clamp(256, 32768).round().long()
        lengths = [int(x) for x in lengths]
        suffix = [1024 if q % 2 == 0 else 0 for q in range(count)]
        need = sum(lengths) + sum(suffix)
        rows = int(math.ceil(need / 0.3 * 1.02))
        return dict(lengths=lengths, suffix=suffix, rows=rows, occupied=0.7,
                    workload=f"qwen3-14b->32b ragged serving batch (BASELINE config 5): {count} requests, "
                             "lengths LogNormal(ln 4096, 1) clipped [256, 32768], 70% occupied target pool, "
                             "1024-token suffix appended to every other request after publication")
    lengths = [args.request_tokens] * args.requests
    return dict(lengths=lengths, suffix=[0] * len(lengths), rows=sum(lengths) + args.pool_slack, occupied=0.0,
                workload=f"qwen3-14b->32b sharded handoff (BASELINE config 3)")


def run_sharded(args):
    import datetime

    import torch.distributed as dist

    import cachebridge_b200 as cb
    from cachebridge_b200.online import tp
    from cachebridge_b200.online.transaction import (PUBLISHED, HandoffTransaction, SlotAllocator, commit,
                                                     device_settle, gloo_vote)

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch one rank per GPU with torchrun")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    host_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))
    L_s, L_t, H, D, S, theta = (QWEN[k] for k in ("L_s", "L_t", "H", "D", "S", "theta"))
    plan = tp.pair_plan(world, rank, H)
    Hr = plan.heads_per_rank
    work = sharded_workload(args, world)
    lengths, suffix, rows = work["lengths"], work["suffix"], work["rows"]
    n_req, total, chunk = len(lengths), sum(lengths), args.chunk
    target = plan.role == "target"
    # Source rows of each request: a seeded random placement in the source pool.
    g = torch.Generator().manual_seed(1000 + plan.tp_rank)
    src_rows = total + args.pool_slack
    src_perm = torch.randperm(src_rows, generator=g)[:total]
    offsets = [0]
    for n in lengths:
        offsets.append(offsets[-1] + n)
    requests = [(src_perm[offsets[q]:offsets[q + 1]].to(dev), torch.zeros(lengths[q], dtype=torch.int64, device=dev))
                for q in range(n_req)]
    mapper = src_pool = dst_pool = alloc = None
    layers = random_layers(L_s=L_s, L_t=L_t, H=H, D=D, S=S, seed=11)
    occupied_mask = None
    if target:
        mapper = cb.PageMapper.from_tensors(layers, method="cachebridge", source_rope_theta=theta,
                                            target_rope_theta=theta, device=dev, target_tp_rank=plan.tp_rank,
                                            target_tp_size=plan.tp)
        log(f"rank {rank}: target pool {L_t} layers x {rows} rows x {Hr} heads")
        dst_pool = cb.TokenKVPool(layers=L_t, rows=rows, heads=Hr, head_dim=D, device=dev, fill=CANARY)
        # The free list: every row, or (config 5) the 30 % not held by other requests.
        order = torch.randperm(rows, generator=torch.Generator().manual_seed(2000 + plan.tp_rank))
        n_occ = int(rows * work["occupied"])
        alloc = SlotAllocator.from_free_rows(order[n_occ:].to(dev))
        if n_occ:
            occupied_mask = torch.zeros(rows, dtype=torch.bool, device=dev)
            occupied_mask[order[:n_occ].to(dev)] = True
    else:
        log(f"rank {rank}: source pool {L_s} layers x {src_rows} rows x {Hr} heads")
        src_pool = cb.TokenKVPool(layers=L_s, rows=src_rows, heads=Hr, head_dim=D, device=dev)
        gd = torch.Generator(device=dev).manual_seed(17 + plan.tp_rank)
        for buf in (src_pool.k_buffer, src_pool.v_buffer):
            buf.normal_(generator=gd)
            buf.mul_(torch.exp(0.5 * torch.randn(L_s, 1, Hr, D, generator=gd, device=dev)).to(buf.dtype))
    torch.cuda.synchronize()
    if args.mixed and mapper is None:  # mixed placement maps some chunks on the source
        mapper = cb.PageMapper.from_tensors(layers, method="cachebridge", source_rope_theta=theta,
                                            target_rope_theta=theta, device=dev, target_tp_rank=plan.tp_rank,
                                            target_tp_size=plan.tp)
    placement = tp.TargetPlacement(plan, requests, chunk=chunk, source_layers=L_s, device=dev, group=host_group,
                                   source_pool=src_pool, mapper=mapper, target_pool=dst_pool,
                                   transport=args.transport, slots=args.slots, mixed_source_block=args.mixed)
    vote = gloo_vote(host_group)
    settle = device_settle(dev)

    def occupy():
        # Other requests' rows (config 5): a pattern the handoff must not touch.
        if occupied_mask is not None:
            for buf in (dst_pool.k_buffer, dst_pool.v_buffer):
                for l in range(L_t):
                    buf[l][occupied_mask] = OCCUPIED

    occupy()

    def handoff(tag):
        """One handoff of every request: allocate target rows, run the
        pipeline, then commit (settle, vote, publish). Returns the
        transactions; raises if any was not published."""
        txns = [HandoffTransaction(f"{tag}-r{q}", lengths[q], rank=rank,
                                   allocate=alloc.allocate if target else None, free=alloc.free if target else None,
                                   publish=(lambda idx: None) if target else None)
                for q in range(n_req)]
        if target:
            for q, t in enumerate(txns):
                rows_q = t.begin()
                if rows_q is not None:
                    placement.set_target_rows(q, rows_q)
        placement.run(txns)
        commit(txns, settle=settle, vote=vote)
        return txns

    def evict(txns):
        # The engine later frees the published rows (outside the timed handoff).
        if target:
            for t in txns:
                if t.outcome == PUBLISHED:
                    alloc.free(t.indices)

    for w in range(args.warmup):
        evict(handoff(f"warm{w}"))

    # ---- timed: device events over the steps, host latency per handoff -------
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    lat = []
    dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clocks:
        ev[0].record()
        for k in range(args.steps):
            t0 = time.perf_counter()
            txns = handoff(f"step{k}")
            lat.append(1e3 * (time.perf_counter() - t0))
            ev[k + 1].record()
            evict(txns)
        ev[-1].synchronize()
    per_step = torch.tensor([ev[k].elapsed_time(ev[k + 1]) for k in range(args.steps)] +
                            [ev[0].elapsed_time(ev[-1])] + lat, device=dev)
    dist.all_reduce(per_step, op=dist.ReduceOp.MAX)
    step_ms = per_step[:args.steps].tolist()
    total_ms = float(per_step[args.steps])
    lat_max = per_step[args.steps + 1:].tolist()

    # ---- end to end: slot tables from pinned host memory each handoff -------
    host_idx = [s.cpu().pin_memory() for s, _ in requests]

    def e2e_handoff(tag):
        for hs, (ds, _) in zip(host_idx, requests):
            ds.copy_(hs, non_blocking=True)
        return handoff(tag)

    evict(e2e_handoff("e2e-warm"))
    e_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    dist.barrier()
    torch.cuda.synchronize()
    e_ev[0].record()
    for k in range(args.e2e_steps):
        evict(e2e_handoff(f"e2e{k}"))
    e_ev[1].record()
    e_ev[1].synchronize()
    e2e_ms = torch.tensor([e_ev[0].elapsed_time(e_ev[1]) / args.e2e_steps], device=dev)
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)

    # ---- parity: one more handoff into a canary pool, checked on every target rank ----
    if target:
        dst_pool.k_buffer.fill_(CANARY)
        dst_pool.v_buffer.fill_(CANARY)
        occupy()
    txns = handoff("parity")
    win = min(256, lengths[0])
    w0 = int(torch.randint(0, lengths[0] - win + 1, (1,), generator=torch.Generator().manual_seed(7)))
    window = torch.empty((2, L_s, win, Hr, D), dtype=torch.bfloat16, device=dev)
    if not target:
        rows_w = requests[0][0][w0:w0 + win]
        window.copy_(torch.stack((src_pool.k_buffer[:, rows_w], src_pool.v_buffer[:, rows_w])))
        dist.send(window, dst=plan.peer)
    else:
        dist.recv(window, src=plan.peer)
    check = None
    if target:
        mask = torch.zeros(rows, dtype=torch.bool, device=dev)
        for t in txns:
            mask[t.indices] = True
        if occupied_mask is not None:
            mask |= occupied_mask
        placed = rows_written(dst_pool, mask, CANARY)
        mine = [{k: (v.float() if torch.is_tensor(v) and v.is_floating_point() else v) for k, v in
                 dict(selected=lw.selected, k_weight=lw.k_weight, k_bias=lw.k_bias, v_weight=lw.v_weight,
                      v_bias=lw.v_bias).items()} for lw in mapper.layers]
        f32 = reference_map_fp32(mine, window, theta=theta, position_start=w0)
        loc = txns[0].indices[w0:w0 + win]
        ours = torch.stack((dst_pool.k_buffer[:, loc], dst_pool.v_buffer[:, loc]))
        values = value_parity(ours, f32)
        check = dict(rank=rank, placement=placed, values=values, window=[w0, w0 + win])
        if work["occupied"]:
            check["occupied_untouched"] = all(bool((buf[l][occupied_mask] == OCCUPIED).all())
                                              for buf in (dst_pool.k_buffer, dst_pool.v_buffer) for l in range(L_t))
        if any(suffix):
            # The target engine appends new tokens after publication: the
            # published prefix rows and every other row keep their bytes.
            before = [buf[l][mask].float().sum(dim=(1, 2)) for buf in (dst_pool.k_buffer, dst_pool.v_buffer)
                      for l in range(L_t)]
            grown = mask.clone()
            for q, extra in enumerate(suffix):
                if extra:
                    new_rows = alloc.allocate(extra)
                    for buf in (dst_pool.k_buffer, dst_pool.v_buffer):
                        for l in range(L_t):
                            buf[l][new_rows] = SUFFIX
                    grown[new_rows] = True
            after = [buf[l][mask].float().sum(dim=(1, 2)) for buf in (dst_pool.k_buffer, dst_pool.v_buffer)
                     for l in range(L_t)]
            check["prefix_unchanged_after_suffix"] = all(torch.equal(a, b) for a, b in zip(before, after))
            check["placement_after_suffix"] = rows_written(dst_pool, grown, CANARY)
        check["ok"] = bool(placed["ok"] and values["ok"] and check.get("occupied_untouched", True)
                           and check.get("prefix_unchanged_after_suffix", True)
                           and check.get("placement_after_suffix", {"ok": True})["ok"])
    checks = [None] * world
    dist.all_gather_object(checks, check, group=host_group)
    parity_ok = all(c["ok"] for c in checks if c is not None)

    # Re-prefill estimate on the target TP group (every rank runs its shard; max over ranks).
    prefill = reprefill_estimate(dev, tokens=max(lengths), requests=1, tp=plan.tp)
    prefill_ms = torch.tensor([prefill["per_layer_ms"]], device=dev)
    dist.all_reduce(prefill_ms, op=dist.ReduceOp.MAX)
    per_layer_full = float(prefill_ms)
    prefill["per_layer_ms"] = per_layer_full
    # Ragged requests: the layer time of the longest request scaled by
    # (n / longest)^2 per request, a lower bound (the linear part of the work
    # shrinks more slowly than that).
    prefill["ms"] = sum(per_layer_full * prefill["layers"] * (n / max(lengths)) ** 2 for n in lengths) \
        if args.config == 5 else per_layer_full * prefill["layers"] * n_req
    prefill["requests"] = n_req
    prefill["handoff_ms"] = total_ms / args.steps
    prefill["handoff_faster"] = prefill["handoff_ms"] < prefill["ms"]

    # CPU baseline: this rank's share (H_r heads) of the work, on a 2048-token sample.
    cpu = None
    if rank == 0:
        cpu_value, cores = cpu_reference_tokens_per_s(layers, n_sample=args.cpu_tokens, reps=1, heads=Hr)
        cpu = dict(value=cpu_value, unit=UNIT, cores=cores, kind="port", extrapolated=True,
                   sample=f"{args.cpu_tokens} tokens of one request, one rank's share ({Hr} of {H} heads), "
                          "reference torch algorithm restated in oracle/, FP32 on host cores; extrapolated: one "
                          f"rank's share of a {max(lengths)}-token request would take "
                          f"{max(lengths) / cpu_value:.1f} s")

    launches = torch.tensor([placement.launches * args.steps], device=dev)
    dist.all_reduce(launches)
    clk = clocks.summary()
    value = total * args.steps / (total_ms / 1e3)
    # Bytes that must cross NVLink per pair per handoff: the raw source rows.
    shard_bytes = total * 2 * L_s * Hr * D * 2
    nvlink_peak = 900.0  # NVLink 5, per direction per GPU (nominal)
    achieved = shard_bytes / (statistics.mean(step_ms) / 1e3) / 1e9
    if rank == 0:
        h2d = sum(s.numel() * s.element_size() for s in host_idx)
        line = dict(
            metric=METRIC, value=value, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
            ms_per_step=total_ms / args.steps, higher_is_better=True, scaling="strong", vs_baseline=None,
            dtype="bf16", data="synthetic",
            config=dict(workload=work["workload"] + f", TP{plan.tp}+TP{plan.tp}", requests=n_req,
                        tokens_per_step=total, request_tokens=(lengths[0] if args.config == 3 else None),
                        chunk_tokens=chunk, source_layers=L_s, target_layers=L_t, kv_heads=H, heads_per_rank=Hr,
                        head_dim=D, selected=S, target_pool_slots=rows, page_size=1,
                        target_rows="allocated per handoff from a seeded free list (publication transaction)",
                        transport_mode=args.transport, receive_slots=args.slots, mixed_source_block=args.mixed,
                        l2="inputs larger than L2",
                        parallelism=f"src tp{plan.tp} -> dst tp{plan.tp}"),
            latency_p50_ms=statistics.median(lat_max),
            latency=dict(what="host clock per handoff, max over ranks: target rows allocated, every chunk queued, "
                              "GPU work settled, all-rank vote, rows published", p50_ms=statistics.median(lat_max),
                         min_ms=min(lat_max)),
            device_ms=dict(p50=statistics.median(step_ms), what="CUDA events between handoffs, max over ranks"),
            roofline=dict(bound="nvlink", achieved=achieved, peak=nvlink_peak, unit="GB/s",
                          frac=achieved / nvlink_peak, traffic=None,
                          kernel=("copy-engine transfers" if args.transport == "copy_engine"
                                  else "copy_rows_kernel peer stores") + " (one pair, per direction)",
                          shard_bytes_per_pair=shard_bytes,
                          peak_source="NVLink 5 nominal 900 GB/s per direction per GPU",
                          roofline_ms=1e3 * shard_bytes / (nvlink_peak * 1e9)),
            parity=dict(ok=parity_ok, ranks=[c for c in checks if c is not None],
                        scope="per target rank: every pool row against its canary (and the occupied rows' "
                              "pattern), plus a 256-token window of request 0 x all layers x its heads against the "
                              "FP32 restatement of the reference algorithm on the GPU"),
            cpu_baseline=cpu,
            e2e=dict(value=total / (float(e2e_ms) / 1e3), unit=UNIT, h2d_bytes_per_step=h2d, d2h_bytes_per_step=0,
                     path="source slot tables H2D + handoff (allocate, TargetPlacement.run, commit with host vote)",
                     ms_per_step=float(e2e_ms)),
            gpu_launches=int(launches.item()),
            clocks=clk,
            reprefill_estimate=prefill,
        )
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    placement.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0 if parity_ok else 1


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[3, 5], default=3,
                    help="N>1: BASELINE config 3 (16 x 32K) or config 5 (64 ragged requests, 70%% occupied pool)")
    ap.add_argument("--tokens", type=int, default=8192, help="history tokens (N=1)")
    ap.add_argument("--pool-slots", type=int, default=262144)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-tokens", type=int, default=2048)
    ap.add_argument("--ref-tokens", type=int, default=2048)
    ap.add_argument("--latency-runs", type=int, default=20, help="N=1: handoffs timed through run_handoff")
    ap.add_argument("--latency-block-tokens", type=int, default=2048, help="N=1: block_tokens of those handoffs")
    ap.add_argument("--cfg4-steps", type=int, default=5, help="N=1: timed steps of the config-4 sub-record")
    ap.add_argument("--cfg4-tokens", type=int, default=LLAMA["tokens"],
                    help="N=1: tokens per config-4 request (smaller only for profiling captures)")
    ap.add_argument("--cfg4-requests", type=int, default=LLAMA["requests"],
                    help="N=1: config-4 requests per step (fewer only for profiling captures)")
    ap.add_argument("--skip-cfg4", action="store_true", help="N=1: leave out the config-4 sub-record")
    ap.add_argument("--requests", type=int, default=16, help="requests per step (N>1, config 3)")
    ap.add_argument("--request-tokens", type=int, default=32768, help="history tokens per request (N>1, config 3)")
    ap.add_argument("--chunk", type=int, default=2048, help="tokens per map+install call (N>1)")
    ap.add_argument("--pool-slack", type=int, default=4096, help="free pool rows beyond the requests (N>1)")
    ap.add_argument("--slots", type=int, default=2, help="N>1 target placement: receive slots (chunks in flight)")
    ap.add_argument("--mixed", choices=["early", "tail"], default=None,
                    help="N>1: map the first or last chunk of each request on the source (mixed placement)")
    ap.add_argument("--transport", choices=["copy_engine", "peer_stores"], default="peer_stores",
                    help="N>1 target placement: staged chunks moved by the copy engine, or gather-kernel peer stores")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        log("warm-up raised to 3 steps (timing rule)")
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.gpus == 1 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        return run_single(args)
    return run_sharded(args)


if __name__ == "__main__":
    sys.exit(main())
