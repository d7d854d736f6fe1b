#!/usr/bin/env python
"""Benchmark of the CacheBridge online handoff hot path on B200.

Metric: mapped+installed KV tokens/s, plus p50 handoff latency
at an 8K-token history. One "step" is one handoff: every token of the history
is gathered from the source pool, mapped by the CacheBridge mapper (40 -> 64
layers, 8 KV heads, S=2) and installed into the target pool rows of its page
table.

  N=1  (default)  Qwen3-14B->32B shapes on one GPU: one 8192-token request, page_size=1 pools
                  of 262144 slots, seeded random source and target slot lists.
  N>1  (torchrun) the sharded handoff (16 x 32768-token requests, at TP4, TP2 or TP1): source TP
                  N/2 + target TP N/2; rank r < N/2 maps its heads for 16 x
                  32768-token requests and stores them straight into the peer
                  target rank's pool (CUDA IPC pointers, NVLink), in
                  double-buffered 2048-token chunks; the prefix is published
                  after an all-rank vote.
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
def torch_reference_handoff(layers, src_pool, src_slots, dst_pool, dst_slots, *, theta, position_start=0):
    """One handoff the way the reference runs it with torch on a GPU.

    pack_source_block: one index_select per source layer and kind into a
    [2, L_s, n, H, D] block (online/blocks.py:47-82). PageMapper.map_page in
    FP32: RoPE removed from the keys of every source layer,
    (x*cos - rot(x)*sin) / max(cos^2 + sin^2, tiny) (rope.py:82-89); per target
    layer the selected layers concatenated along features and
    einsum('thf,hfd->thd') with the FP32 weights plus bias (mapper.py:153-181);
    target RoPE on the keys and the cast to the pool dtype (mapper.py:207-239).
    Install: k_buffer[l][loc] = k per target layer (SGLang set_kv_buffer,
    blocks.py:86-111). Returns the mapped [2, L_t, n, H, D] block.
    """
    dev = src_pool.k_buffer.device
    n = len(src_slots)
    L_s, H, D = src_pool.layer_num, src_pool.heads, src_pool.head_dim
    block = torch.empty((2, L_s, n, H, D), dtype=src_pool.dtype, device=dev)
    for l in range(L_s):
        torch.index_select(src_pool.k_buffer[l], 0, src_slots, out=block[0, l])
        torch.index_select(src_pool.v_buffer[l], 0, src_slots, out=block[1, l])
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device=dev).float() / D))
    phase = (torch.arange(n, device=dev) + position_start).float()[:, None] * inv[None, :]
    phase = torch.cat((phase, phase), dim=-1)
    cos, sin = phase.cos()[None, :, None, :], phase.sin()[None, :, None, :]

    def rot(x):
        a, b = x.chunk(2, dim=-1)
        return torch.cat((-b, a), dim=-1)

    keys = block[0].float()
    keys = (keys * cos - rot(keys) * sin) / torch.clamp_min(cos * cos + sin * sin, torch.finfo(torch.float32).tiny)
    values = block[1].float()
    out_k, out_v = [], []
    for t in layers:
        sel = t["selected"].tolist()
        xk = torch.cat([keys[s] for s in sel], dim=-1)
        xv = torch.cat([values[s] for s in sel], dim=-1)
        out_k.append(torch.einsum("thf,hfd->thd", xk, t["k_weight"]) + t["k_bias"])
        out_v.append(torch.einsum("thf,hfd->thd", xv, t["v_weight"]) + t["v_bias"])
    k = torch.stack(out_k)
    k = k * cos + rot(k) * sin
    mapped = torch.stack((k, torch.stack(out_v))).to(dst_pool.dtype)
    for l in range(dst_pool.layer_num):
        dst_pool.k_buffer[l][dst_slots] = mapped[0, l]
        dst_pool.v_buffer[l][dst_slots] = mapped[1, l]
    return mapped


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
def cpu_reference_tokens_per_s(layers, *, n_sample, reps, seed=7):
    """Time the reference algorithm (map_page + SGLang-style install) on the host."""
    from oracle import mapper_oracle as orc

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    L_s, H, D = QWEN["L_s"], QWEN["H"], QWEN["D"]
    page = (torch.randn(2, L_s, n_sample, H, D, generator=g)).bfloat16()
    head_range = (0, H)
    ref_layers = [dict(selected=t["selected"].tolist(), k_weight=t["k_weight"], k_bias=t["k_bias"],
                       v_weight=t["v_weight"], v_bias=t["v_bias"]) for t in layers]
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
                              f"qwen3-14b->32b sharded handoff (BASELINE config 3), TP{args.gpus // 2}+TP{args.gpus // 2}")
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
    dst_pool = cb.TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=dev)
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

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
    stream.synchronize()
    cb.raise_for_status(dev)

    # ---- device-resident timing (value, latency, per-kernel) -----------------
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
    # The handoff's algorithmic bytes are moved by its two launches together
    # (key gather/derotation, then the fused map/install), so the roofline is
    # taken over one handoff: both launches' device time.
    step_avg_s = statistics.mean(step_ms) / 1e3
    achieved = bytes_alg / step_avg_s / 1e9
    traffic = profiled_traffic("handoff_cfg2_traffic")
    line = dict(
        metric=METRIC, value=value, unit=UNIT, n_gpus=1, steps=args.steps, warmup=args.warmup,
        ms_per_step=total_ms / args.steps, higher_is_better=True, scaling="weak", vs_baseline=None,
        dtype="bf16", data="synthetic",
        config=dict(workload="qwen3-14b->32b single-GPU handoff (BASELINE config 2)", history_tokens=n,
                    source_layers=L_s, target_layers=L_t, kv_heads=H, head_dim=D, selected=S,
                    pool_slots=rows, page_size=1, slot_lists="seeded random", l2="inputs larger than L2",
                    parallelism="single GPU (source and target pools on one device)"),
        latency_p50_ms=statistics.median(step_ms),
        roofline=dict(bound="hbm", achieved=achieved, peak=hbm_peak, unit="GB/s", frac=achieved / hbm_peak,
                      traffic=None if traffic is None else traffic.get("dram_bytes_per_step"),
                      kernel="derotate_pack_kernel + map_install_tc_kernel (one handoff)",
                      algorithmic_bytes=bytes_alg, peak_source=peak_kind,
                      tensor_tflops=flops / step_avg_s / 1e12, tensor_frac=flops / step_avg_s / 1e12 / tc_peak,
                      roofline_ms=1e3 * max(bytes_alg / (hbm_peak * 1e9), flops / (tc_peak * 1e12))),
        kernels_ms=dict(map_install_tc=statistics.mean(tc_ms), derotate_pack=statistics.mean(pre_ms)),
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
    )
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------
# N > 1: sharded handoff (source TP N/2 + target TP N/2 over NVLink)
# ----------------------------------------------------------------------------
def run_sharded(args):
    import datetime

    import torch.distributed as dist

    import cachebridge_b200 as cb
    from cachebridge_b200.online import tp
    from cachebridge_b200.online.blocks import map_install_block

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch one rank per GPU with torchrun")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    host_group = dist.new_group(backend="gloo")
    L_s, L_t, H, D, S, theta = (QWEN[k] for k in ("L_s", "L_t", "H", "D", "S", "theta"))
    plan = tp.pair_plan(world, rank, H)
    Hr = plan.heads_per_rank
    n_req, n_tok, chunk = args.requests, args.request_tokens, args.chunk
    total = n_req * n_tok
    rows = total + args.pool_slack
    target_side = args.placement == "target"
    # Both ranks of a pair draw the same slot lists.
    g = torch.Generator().manual_seed(1000 + plan.tp_rank)
    src_perm = torch.randperm(rows, generator=g)[:total]
    dst_perm = torch.randperm(rows, generator=g)[:total]
    requests = [(src_perm[q * n_tok:(q + 1) * n_tok].to(dev), dst_perm[q * n_tok:(q + 1) * n_tok].to(dev))
                for q in range(n_req)]
    mapper = src_pool = dst_pool = None
    if plan.role == "target" or not target_side:
        # The rank that maps: the target (target placement) or the source.
        layers = random_layers(L_s=L_s, L_t=L_t, H=H, D=D, S=S, seed=11)
        mapper = cb.PageMapper.from_tensors(layers, method="cachebridge", source_rope_theta=theta,
                                            target_rope_theta=theta, device=dev, target_tp_rank=plan.tp_rank,
                                            target_tp_size=plan.tp)
    if plan.role == "source":
        log(f"rank {rank}: source pool {L_s} layers x {rows} rows x {Hr} heads")
        src_pool = cb.TokenKVPool(layers=L_s, rows=rows, heads=Hr, head_dim=D, device=dev)
        gd = torch.Generator(device=dev).manual_seed(17 + plan.tp_rank)
        for buf in (src_pool.k_buffer, src_pool.v_buffer):
            buf.normal_(generator=gd)
            buf.mul_(torch.exp(0.5 * torch.randn(L_s, 1, Hr, D, generator=gd, device=dev)).to(buf.dtype))
    else:
        log(f"rank {rank}: target pool {L_t} layers x {rows} rows x {Hr} heads")
        dst_pool = cb.TokenKVPool(layers=L_t, rows=rows, heads=Hr, head_dim=D, device=dev)
    torch.cuda.synchronize()
    peer_pool = placement = handoff = None
    if target_side:
        placement = tp.TargetPlacement(plan, requests, chunk=chunk, source_layers=L_s, device=dev, group=host_group,
                                       source_pool=src_pool, mapper=mapper, target_pool=dst_pool,
                                       transport=args.transport, slots=args.slots)
        runner = placement
    else:
        peer_pool = tp.exchange_target_pools(plan, dst_pool, group=host_group, device=dev)
        if plan.role == "source":
            handoff = tp.ShardedHandoff(mapper, src_pool, peer_pool, requests, chunk=chunk,
                                        source_head_offset=plan.head_start)
        runner = handoff
    ones = torch.ones(1, dtype=torch.int32, device=dev)

    def step():
        if runner is not None:
            runner.run()
            ready = tp.device_ready(dev)
        else:
            ready = ones.clone()
        return tp.publication_vote(ready, device=dev)

    for _ in range(args.warmup):
        vote = step()
    torch.cuda.synchronize()
    if int(vote.item()) != 1:
        raise RuntimeError("warm-up handoff was not published (a rank reported a device error)")

    # ---- device-resident timing ------------------------------------------------
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clocks:
        ev[0].record()
        for k in range(args.steps):
            vote = step()
            ev[k + 1].record()
        ev[-1].synchronize()
    published = int(vote.item())
    per_step = torch.tensor([ev[k].elapsed_time(ev[k + 1]) for k in range(args.steps)] +
                            [ev[0].elapsed_time(ev[-1]), float(published == 1)], device=dev)
    dist.all_reduce(per_step[:-1], op=dist.ReduceOp.MAX)
    dist.all_reduce(per_step[-1:], op=dist.ReduceOp.MIN)
    step_ms, total_ms, all_published = per_step[:-2].tolist(), float(per_step[-2]), float(per_step[-1])
    if all_published != 1.0:
        raise RuntimeError("sharded handoff was not published on every rank")

    # ---- end to end through the public API --------------------------------------
    # Per step: every request's slot tables come from pinned host memory, the
    # handoff runs through the public entry points (TargetPlacement.run, or
    # map_install_block per chunk for source placement), and the publication
    # vote is read back to the host.
    host_idx = [(s.cpu().pin_memory(), t.cpu().pin_memory()) for s, t in requests]
    vote_host = torch.empty(1, dtype=torch.int32).pin_memory()

    def e2e_step():
        for (hs, ht), (ds, dt) in zip(host_idx, requests):
            ds.copy_(hs, non_blocking=True)
            dt.copy_(ht, non_blocking=True)
        if target_side:
            placement.run()
            ready = tp.device_ready(dev)
        elif plan.role == "source":
            for ds, dt in requests:
                for a, b in tp.chunk_spans(n_tok, chunk):
                    map_install_block(mapper, src_pool, ds, peer_pool, dt, start=a, stop=b,
                                      source_head_offset=plan.head_start, target_head_offset=0)
            ready = tp.device_ready(dev)
        else:
            ready = ones.clone()
        vote_host.copy_(tp.publication_vote(ready, device=dev), non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    dist.barrier()
    torch.cuda.synchronize()
    e_ev[0].record()
    for _ in range(args.e2e_steps):
        e2e_step()
    e_ev[1].record()
    e_ev[1].synchronize()
    e2e_ms = torch.tensor([e_ev[0].elapsed_time(e_ev[1]) / args.e2e_steps], device=dev)
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    if int(vote_host.item()) != 1:
        raise RuntimeError("end-to-end handoff was not published")

    # Re-prefill estimate on the target TP group (every rank runs its shard; max over ranks).
    prefill = reprefill_estimate(dev, tokens=n_tok, requests=n_req, tp=plan.tp)
    prefill_ms = torch.tensor([prefill["per_layer_ms"]], device=dev)
    dist.all_reduce(prefill_ms, op=dist.ReduceOp.MAX)
    prefill["per_layer_ms"] = float(prefill_ms)
    prefill["ms"] = prefill["per_layer_ms"] * prefill["layers"] * n_req
    prefill["handoff_ms"] = total_ms / args.steps
    prefill["handoff_faster"] = prefill["handoff_ms"] < prefill["ms"]

    launches = torch.tensor([runner.launches * args.steps if runner is not None else 0], device=dev)
    dist.all_reduce(launches)
    clk = clocks.summary()
    value = total * args.steps / (total_ms / 1e3)
    # Bytes that must cross NVLink per pair per step: raw source rows (target
    # placement) or mapped target rows (source placement).
    shard_bytes = total * 2 * (L_s if target_side else L_t) * Hr * D * 2
    nvlink_peak = 770.0  # measured peer copy per direction on this pool's B200s (GB/s)
    achieved = shard_bytes / (statistics.mean(step_ms) / 1e3) / 1e9
    if rank == 0:
        h2d = sum(s.numel() * s.element_size() + t.numel() * t.element_size() for s, t in host_idx)
        transport = (("source rows gathered locally, moved by one copy-engine transfer per chunk into the target "
                      "GPU's receive slots (CUDA IPC), mapped and installed on the target" if args.transport == "copy_engine"
                      else "source rows packed into the target GPU's receive slots (peer stores, CUDA IPC), mapped "
                      "and installed on the target") if target_side else
                     "map kernel stores into the peer target pool (CUDA IPC, NVLink)")
        line = dict(
            metric=METRIC, value=value, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
            ms_per_step=total_ms / args.steps, higher_is_better=True, scaling="strong", vs_baseline=None,
            dtype="bf16", data="synthetic",
            config=dict(workload=f"qwen3-14b->32b sharded handoff (BASELINE config 3), TP{plan.tp}+TP{plan.tp}",
                        requests=n_req, request_tokens=n_tok, chunk_tokens=chunk, source_layers=L_s,
                        transport_mode=args.transport if target_side else "peer_stores",
                        receive_slots=args.slots if target_side else None,
                        target_layers=L_t, kv_heads=H, heads_per_rank=Hr, head_dim=D, selected=S,
                        pool_slots=rows, page_size=1, slot_lists="seeded random", placement=args.placement,
                        transport=transport, l2="inputs larger than L2",
                        parallelism=f"src tp{plan.tp} -> dst tp{plan.tp}"),
            latency_p50_ms=statistics.median(step_ms),
            roofline=dict(bound="nvlink", achieved=achieved, peak=nvlink_peak, unit="GB/s",
                          frac=achieved / nvlink_peak, traffic=None,
                          kernel=(("copy-engine transfers" if args.transport == "copy_engine" else "copy_rows_kernel peer stores")
                                  if target_side else "map_install_tc_kernel peer stores") + " (one pair, per direction)",
                          shard_bytes_per_pair=shard_bytes, peak_source="recipe-measured peer copy"),
            cpu_baseline=None,
            e2e=dict(value=total / (float(e2e_ms) / 1e3), unit=UNIT, h2d_bytes_per_step=h2d,
                     d2h_bytes_per_step=4,
                     path=("slot tables H2D + TargetPlacement.run + vote D2H" if target_side else
                           "slot tables H2D + map_install_block per chunk into the peer pool + vote D2H"),
                     ms_per_step=float(e2e_ms)),
            gpu_launches=int(launches.item()),
            clocks=clk,
            reprefill_estimate=prefill,
        )
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    if peer_pool is not None:
        peer_pool.close()
    if placement is not None:
        placement.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=8192, help="history tokens (N=1)")
    ap.add_argument("--pool-slots", type=int, default=262144)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-tokens", type=int, default=2048)
    ap.add_argument("--ref-tokens", type=int, default=2048)
    ap.add_argument("--requests", type=int, default=16, help="requests per step (N>1)")
    ap.add_argument("--request-tokens", type=int, default=32768, help="history tokens per request (N>1)")
    ap.add_argument("--chunk", type=int, default=2048, help="tokens per map+install call (N>1)")
    ap.add_argument("--pool-slack", type=int, default=4096, help="free pool rows beyond the requests (N>1)")
    ap.add_argument("--slots", type=int, default=2, help="N>1 target placement: receive slots (chunks in flight)")
    ap.add_argument("--transport", choices=["copy_engine", "peer_stores"], default="peer_stores",
                    help="N>1 target placement: staged chunks moved by the copy engine, or gather-kernel peer stores")
    ap.add_argument("--placement", choices=["target", "source"], default="target",
                    help="N>1: map on the target GPU (raw source rows cross NVLink) or on the source GPU")
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
