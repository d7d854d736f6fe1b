"""Sharded handoff on two GPUs, both placements:
  - source placement: rank 0 maps into rank 1's pool through CUDA IPC peer
    stores (NVLink);
  - target placement: rank 0 packs raw source rows into rank 1's receive
    slots (staged and moved by the copy engine, or stored straight into the
    peer slot), rank 1 maps them into its own pool (device-side chunk
    handshake). Each request is a HandoffTransaction, published by commit
    (device settle + all-rank host vote);
  - mixed placement: the first ("early") or last ("tail") chunk of each
    request is mapped on the source into the receive slot and installed by
    the target, the other chunks as in target placement.
The target rank checks every installed row against the CPU oracle (the FP32
restatement of the reference algorithm, BF16 tolerance of the GPU parity
tests), every other row against its canary, and, as a cross-check, that a
local run of the same kernels on the same inputs is bit-identical.

Needs two visible GPUs; skipped otherwise. NVLS is off (peer loads only).
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

CANARY = -7.25


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layers(L_s, L_t, H, D, S, seed):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(L_t):
        t = dict(selected=torch.randperm(L_s, generator=g)[:S].long(), headwise=torch.tensor(True))
        for kind in ("k", "v"):
            t[f"{kind}_weight"] = (torch.randn(H, S * D, D, generator=g) / (S * D) ** 0.5).bfloat16().float()
            t[f"{kind}_bias"] = (torch.randn(H, D, generator=g) * 0.1).bfloat16().float()
        out.append(t)
    return out


def _worker(rank, port, placement, results):
    import datetime

    import torch.distributed as dist

    import cachebridge_b200 as cb
    from cachebridge_b200.device import status_word
    from cachebridge_b200.online import tp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60), device_id=dev)
    host = dist.new_group(backend="gloo")
    try:
        L_s, L_t, H, D, S, rows = 6, 4, 2, 128, 2, 2048
        plan = tp.pair_plan(2, rank, H)
        g = torch.Generator().manual_seed(3)
        src_perm = torch.randperm(rows, generator=g)[:900]
        dst_perm = torch.randperm(rows, generator=g)[:900]
        # 600 + 300 tokens in 256-token chunks: 5 chunks, an odd count over 2 slots.
        requests = [(src_perm[:600].to(dev), dst_perm[:600].to(dev)), (src_perm[600:].to(dev), dst_perm[600:].to(dev))]
        layers = _layers(L_s, L_t, H, D, S, seed=5)
        mapper = cb.PageMapper.from_tensors(layers, method="cachebridge", source_rope_theta=1e6,
                                            target_rope_theta=1e6, device=dev)
        src_pool = cb.TokenKVPool(layers=L_s, rows=rows, heads=H, head_dim=D, device=dev)
        gd = torch.Generator(device=dev).manual_seed(11)
        src_pool.k_buffer.normal_(generator=gd)
        src_pool.v_buffer.normal_(generator=gd)
        target = cb.TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=dev, fill=CANARY)
        torch.cuda.synchronize()
        peer = None
        if placement == "source":
            peer = tp.exchange_target_pools(plan, target if plan.role == "target" else None, group=host, device=dev)
        else:
            transport = "copy_engine" if placement == "target_copy_engine" else "peer_stores"
            slots = 3 if placement == "target_3slots" else 2
            mixed = placement.split("_", 1)[1] if placement.startswith("mixed_") else None
            peer = tp.TargetPlacement(plan, requests, chunk=256, source_layers=L_s, device=dev, group=host,
                                      source_pool=src_pool if plan.role == "source" else None,
                                      mapper=mapper if (plan.role == "target" or mixed) else None,
                                      target_pool=target if plan.role == "target" else None, timeout_s=20.0,
                                      transport=transport, slots=slots, mixed_source_block=mixed)
        # Every rank reaches the vote, a local failure included (it votes 0).
        error = None
        if placement == "source":
            ready = torch.ones(1, dtype=torch.int32, device=dev)
            try:
                if plan.role == "source":
                    tp.ShardedHandoff(mapper, src_pool, peer, requests, chunk=256).run()
                ready = tp.device_ready(dev)
            except Exception as exc:  # noqa: BLE001
                error = repr(exc)
                ready = torch.zeros(1, dtype=torch.int32, device=dev)
            bits = int(status_word(dev).item())  # this rank's device status before the vote
            vote = int(tp.publication_vote(ready, device=dev).item())
        else:
            from cachebridge_b200.online.transaction import (HandoffTransaction, TransactionError, commit,
                                                             device_settle, gloo_vote)

            bits = 0
            vote = 1
            for rep in range(2):  # two handoffs: the slot counters carry over
                txns = [HandoffTransaction(f"req{q}-{rep}", len(s), rank=rank,
                                           allocate=(lambda n, r=t: r) if plan.role == "target" else None)
                        for q, (s, t) in enumerate(requests)]
                for t in txns:
                    t.begin()
                try:
                    peer.run(txns)
                    receipts = commit(txns, settle=device_settle(dev), vote=gloo_vote(host))
                    assert all(r["blocks"] == len(tp.chunk_spans(r["tokens"], 256)) for r in receipts)
                except TransactionError as exc:
                    error, vote = repr(exc), 0
                    break
        if vote != 1:  # not published: every rank stops here
            results[rank] = (vote, error, bits)
            return
        if plan.role == "target":
            from oracle import mapper_oracle as orc

            ref_layers = [dict(selected=t["selected"].tolist(), k_weight=t["k_weight"], k_bias=t["k_bias"],
                               v_weight=t["v_weight"], v_bias=t["v_bias"]) for t in layers]
            worst_rel, worst_norm = 0.0, 0.0
            for s_slots, d_slots in requests:  # each request's history starts at position 0
                page = torch.stack((src_pool.k_buffer[:, s_slots], src_pool.v_buffer[:, s_slots])).cpu()
                f32 = orc.map_page_f32(ref_layers, page, position_start=0, head_range=(0, H), source_theta=1e6,
                                       target_theta=1e6)
                got = torch.stack((target.k_buffer[:, d_slots], target.v_buffer[:, d_slots])).float().cpu()
                worst_rel = max(worst_rel, float((got - f32).norm() / f32.norm()))
                worst_norm = max(worst_norm, float(((got - f32).abs() / f32.abs().clamp_min(1.0)).max()))
            oracle_ok = worst_rel <= 5e-3 and worst_norm <= 2e-2
            local = cb.TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=dev, fill=CANARY)
            tp.ShardedHandoff(mapper, src_pool, local, requests, chunk=256).run()
            torch.cuda.synchronize()
            cb.raise_for_status(dev)
            same = torch.equal(target.k_buffer, local.k_buffer) and torch.equal(target.v_buffer, local.v_buffer)
            mask = torch.ones(rows, dtype=torch.bool, device=dev)
            mask[dst_perm.to(dev)] = False
            untouched = bool((target.k_buffer[:, mask].float() == CANARY).all()) and bool(
                (target.v_buffer[:, mask].float() == CANARY).all())
            written = not bool((target.k_buffer[:, dst_perm.to(dev)].float() == CANARY).any())
            results[rank] = (vote, same, untouched, written, oracle_ok, worst_rel, worst_norm)
        else:
            results[rank] = (vote,)
        if peer is not None:
            torch.cuda.synchronize()
            peer.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("placement", ["source", "target", "target_copy_engine", "target_3slots", "mixed_early",
                                       "mixed_tail"])
def test_sharded_install_is_bit_exact(placement):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, port, placement, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=180)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert codes == [0, 0], f"worker exit codes {codes}"
        res = dict(results)
    assert res[0] == (1,)
    vote, same, untouched, written, oracle_ok, rel, norm = res[1]
    assert vote == 1 and untouched and written
    assert oracle_ok, f"against the oracle: relative Frobenius {rel:.3e}, normalised max {norm:.3e}"
    assert same
