"""Sharded handoff on two GPUs: source rank 0 maps into target rank 1's pool
through CUDA IPC peer stores (NVLink); rank 1 maps the same inputs locally and
the two pools must be bit-identical, untouched rows keeping their canary.

Needs two visible GPUs; skipped otherwise.
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


def _worker(rank, port, results):
    import datetime

    import torch.distributed as dist

    import cachebridge_b200 as cb
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
        requests = [(src_perm[:700].to(dev), dst_perm[:700].to(dev)), (src_perm[700:].to(dev), dst_perm[700:].to(dev))]
        layers = _layers(L_s, L_t, H, D, S, seed=5)
        mapper = cb.PageMapper.from_tensors(layers, method="cachebridge", source_rope_theta=1e6,
                                            target_rope_theta=1e6, device=dev)
        src_pool = cb.TokenKVPool(layers=L_s, rows=rows, heads=H, head_dim=D, device=dev)
        gd = torch.Generator(device=dev).manual_seed(11)
        src_pool.k_buffer.normal_(generator=gd)
        src_pool.v_buffer.normal_(generator=gd)
        target = cb.TokenKVPool(layers=L_t, rows=rows, heads=H, head_dim=D, device=dev, fill=CANARY)
        torch.cuda.synchronize()
        peer = tp.exchange_target_pools(plan, target if plan.role == "target" else None, group=host, device=dev)
        # Every rank reaches the vote, a local failure included (it votes 0).
        error = None
        ready = torch.ones(1, dtype=torch.int32, device=dev)
        if plan.role == "source":
            try:
                tp.ShardedHandoff(mapper, src_pool, peer, requests, chunk=256).run()
                ready = tp.device_ready(dev)
            except Exception as exc:  # noqa: BLE001
                error = repr(exc)
                ready = torch.zeros(1, dtype=torch.int32, device=dev)
        vote = int(tp.publication_vote(ready, device=dev).item())
        if vote != 1:  # not published: every rank stops here
            results[rank] = (vote, error)
            return
        if plan.role == "target":
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
            results[rank] = (vote, same, untouched, written)
        else:
            results[rank] = (vote,)
        if peer is not None:
            torch.cuda.synchronize()
            peer.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_source_rank_installs_into_peer_pool_bit_exactly():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, port, results)) for r in range(2)]
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
    vote, same, untouched, written = res[1]
    assert vote == 1 and same and untouched and written
