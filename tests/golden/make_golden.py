"""Generate golden vectors by running the reference CacheBridge implementation.

Run in the build container, where the reference source tree is importable:

    PYTHONDONTWRITEBYTECODE=1 PYTHONPATH=<reference>/src \
        python tests/golden/make_golden.py <reference> [dense]

Each case directory under tests/golden/ holds the mapper files in the
reference's ``layer_NNN.safetensors`` format, ``case.safetensors`` (inputs and
the reference's outputs) and ``case.json`` (call parameters). The reference is
not needed afterwards: tests read only the committed fixtures.

Inputs are seeded synthetic tensors shaped like the benchmark configurations
(reduced token / layer counts so fixtures stay small) plus re-creations of the
inputs of the reference's own known-answer tests (tests/test_mapper.py,
tests/test_fitting.py, tests/test_blocks.py, examples/fit_and_map.py).
"""

from __future__ import annotations

import hashlib
import json
import shutil
import sys
from pathlib import Path
from types import SimpleNamespace

import torch
from safetensors.torch import save_file

HERE = Path(__file__).resolve().parent


def _reference(root: str):
    sys.path.insert(0, str(Path(root) / "src"))
    from cachebridge.mapper import PageMapper as BaseMapper  # noqa: F401
    from cachebridge.online.mapping import PageMapper
    from cachebridge.online.blocks import pack_source_block
    from cachebridge.online.peer_geometry import operations
    from cachebridge.offline.fitting import fit_layer
    from cachebridge.rope import apply_rope, qwen_rope

    return SimpleNamespace(
        PageMapper=PageMapper,
        pack_source_block=pack_source_block,
        operations=operations,
        fit_layer=fit_layer,
        apply_rope=apply_rope,
        qwen_rope=qwen_rope,
    )


def _case_dir(name: str) -> Path:
    d = HERE / name
    if d.exists():
        shutil.rmtree(d)
    d.mkdir(parents=True)
    return d


def _write_layers(d: Path, layers: list[dict]) -> None:
    for i, t in enumerate(layers):
        save_file({k: v.contiguous() for k, v in t.items()}, str(d / f"layer_{i:03d}.safetensors"))


def _random_layers(g, *, L_s, L_t, H, D, S, w_var, b_var, bf16_weights):
    """Seeded headwise layers; S distinct source layers per target layer."""
    layers = []
    for _ in range(L_t):
        sel = torch.randperm(L_s, generator=g)[:S].sort().values
        sel = sel[torch.randperm(S, generator=g)]  # arbitrary order, as fitted recipes allow
        kw = torch.randn(H, S * D, D, generator=g) * w_var**0.5
        vw = torch.randn(H, S * D, D, generator=g) * w_var**0.5
        kb = torch.randn(H, D, generator=g) * b_var**0.5
        vb = torch.randn(H, D, generator=g) * b_var**0.5
        if bf16_weights:
            # Exactly representable in bf16; stored as bf16 on disk (the reference
            # loads with .float(), mapper.py:175-180), as FP32 otherwise.
            kw, vw, kb, vb = (x.bfloat16() for x in (kw, vw, kb, vb))
        layers.append(
            dict(selected=sel.long(), k_weight=kw, k_bias=kb, v_weight=vw, v_bias=vb,
                 headwise=torch.tensor(True))
        )
    return layers


def _source_page(ref, g, *, L_s, n, H, D, theta, scaling, position_start, dtype, lognormal):
    """Content-space K/V ~N(0,1) (optionally x per-channel LogNormal(0,0.5)); K stored RoPE-applied."""
    content = torch.randn(2, L_s, n, H, D, generator=g)
    if lognormal:
        scale = torch.exp(0.5 * torch.randn(2, L_s, 1, H, D, generator=g))
        content = content * scale
    pos = torch.arange(position_start, position_start + n)
    cos, sin = ref.qwen_rope(pos, head_dim=D, theta=theta, scaling=scaling)
    page = content.clone()
    page[0] = ref.apply_rope(content[0], cos, sin)
    return page.to(dtype)


def _run_mapper(ref, d, params, page, output_dtype=None):
    mapper = ref.PageMapper(
        d,
        method="cachebridge",
        source_rope_theta=params["source_theta"],
        target_rope_theta=params["target_theta"],
        source_rope_scaling=params.get("source_scaling"),
        target_rope_scaling=params.get("target_scaling"),
        target_tp_rank=params.get("tp_rank", 0),
        target_tp_size=params.get("tp_size", 1),
    )
    return mapper.map_page(
        page,
        position_start=params["position_start"],
        source_head_offset=params.get("source_head_offset", 0),
    )


def _save(d: Path, params: dict, tensors: dict) -> None:
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(d / "case.safetensors"))
    (d / "case.json").write_text(json.dumps(params, indent=1, sort_keys=True) + "\n")


def random_case(ref, name, *, seed, L_s, L_t, H, D, S, n, dtype, position_start, source_theta,
                target_theta, source_scaling=None, target_scaling=None, tp_rank=0, tp_size=1,
                source_head_offset=0, page_heads=None, w_var=None, b_var=0.01, lognormal=False,
                bf16_weights=False, pool_rows=None):
    g = torch.Generator().manual_seed(seed)
    d = _case_dir(name)
    layers = _random_layers(g, L_s=L_s, L_t=L_t, H=H, D=D, S=S, w_var=w_var or 1.0 / (S * D),
                            b_var=b_var, bf16_weights=bf16_weights)
    _write_layers(d, layers)
    page_heads = page_heads or H
    page = _source_page(ref, g, L_s=L_s, n=n, H=page_heads, D=D, theta=source_theta,
                        scaling=source_scaling, position_start=position_start, dtype=dtype,
                        lognormal=lognormal)
    params = dict(position_start=position_start, source_theta=source_theta, target_theta=target_theta,
                  source_scaling=source_scaling, target_scaling=target_scaling, tp_rank=tp_rank,
                  tp_size=tp_size, source_head_offset=source_head_offset)
    out = _run_mapper(ref, d, params, page)
    tensors = dict(page=page, expected=out)
    if pool_rows:
        slots = torch.randperm(pool_rows, generator=g)[:n]
        tensors["slots"] = slots.long()
        params["pool_rows"] = pool_rows
    _save(d, params, tensors)
    return out


def dense_case(ref, name, *, seed, L_s, L_t, Hs, H, D, S, n, dtype, position_start, theta, tp_rank=0,
               tp_size=1, bf16_weights=False):
    """Dense (nv_transfer) layers: k_weight [S*Hs*D, H, D] without a headwise
    key, mapped by the reference's PageMapper(method="nv_transfer")."""
    g = torch.Generator().manual_seed(seed)
    d = _case_dir(name)
    F = S * Hs * D
    layers = []
    for _ in range(L_t):
        sel = torch.randperm(L_s, generator=g)[:S]
        t = dict(selected=sel.long())
        for kind in ("k", "v"):
            w = torch.randn(F, H, D, generator=g) / F**0.5
            b = torch.randn(H, D, generator=g) * 0.1
            if bf16_weights:
                w, b = w.bfloat16(), b.bfloat16()
            t[f"{kind}_weight"], t[f"{kind}_bias"] = w, b
        layers.append(t)
    _write_layers(d, layers)
    page = _source_page(ref, g, L_s=L_s, n=n, H=Hs, D=D, theta=theta, scaling=None,
                        position_start=position_start, dtype=dtype, lognormal=True)
    mapper = ref.PageMapper(d, method="nv_transfer", source_rope_theta=theta, target_rope_theta=theta,
                            target_tp_rank=tp_rank, target_tp_size=tp_size)
    out = mapper.map_page(page, position_start=position_start)
    params = dict(position_start=position_start, source_theta=theta, target_theta=theta, source_scaling=None,
                  target_scaling=None, tp_rank=tp_rank, tp_size=tp_size, source_head_offset=0,
                  method="nv_transfer")
    _save(d, params, dict(page=page, expected=out))
    return out


def dense_cases(ref):
    # Dense maps read every source head: 4 source heads, 4 target heads, TP rank 1 of 2.
    dense_case(ref, "dense_mini_bf16", seed=31, L_s=5, L_t=2, Hs=4, H=4, D=128, S=2, n=96,
               dtype=torch.bfloat16, position_start=700, theta=1e6, tp_rank=1, tp_size=2, bf16_weights=True)
    # FP32 storage, different source and target head counts (oracle pin; the B200 dense path is BF16 only).
    dense_case(ref, "dense_small_f32", seed=32, L_s=3, L_t=2, Hs=3, H=2, D=64, S=1, n=20,
               dtype=torch.float32, position_start=3, theta=1e4)


def reference_unit_cases(ref):
    """Re-creations of tests/test_mapper.py:66-105 (headwise identity, TP slice, YaRN)."""
    # tests/test_mapper.py:38-50 headwise identity mapper, 10-18 rotated page (seed 7).
    d = _case_dir("ref_headwise_tp_slice")
    eye = torch.eye(4).expand(2, 4, 4).contiguous()
    _write_layers(d, [dict(selected=torch.tensor([0]), k_weight=eye, k_bias=torch.zeros(2, 4),
                           v_weight=eye.clone(), v_bias=torch.zeros(2, 4),
                           headwise=torch.tensor(1, dtype=torch.int8))])
    torch.manual_seed(7)
    content = torch.randn(1, 3, 2, 4)
    values = torch.randn(1, 3, 2, 4)
    cos, sin = ref.qwen_rope(torch.arange(3), head_dim=4, theta=10_000)
    page = torch.stack((ref.apply_rope(content, cos, sin), values), dim=0)
    params = dict(position_start=0, source_theta=10_000.0, target_theta=10_000.0, tp_rank=1, tp_size=2,
                  source_head_offset=0)
    out = _run_mapper(ref, d, params, page)
    assert out.shape == (2, 1, 3, 1, 4)
    _save(d, params, dict(page=page, expected=out, known_answer=page[:, :, :, 1:2].clone()))

    d = _case_dir("ref_yarn_identity")
    _write_layers(d, [dict(selected=torch.tensor([0]), k_weight=eye, k_bias=torch.zeros(2, 4),
                           v_weight=eye.clone(), v_bias=torch.zeros(2, 4),
                           headwise=torch.tensor(1, dtype=torch.int8))])
    scaling = {"rope_type": "yarn", "factor": 2.0, "original_max_position_embeddings": 32}
    torch.manual_seed(11)
    content = torch.randn(1, 3, 2, 4)
    values = torch.randn(1, 3, 2, 4)
    cos, sin = ref.qwen_rope(torch.arange(40, 43), head_dim=4, theta=10_000, scaling=scaling)
    page = torch.stack((ref.apply_rope(content, cos, sin), values), dim=0)
    params = dict(position_start=40, source_theta=10_000.0, target_theta=10_000.0,
                  source_scaling=scaling, target_scaling=scaling)
    out = _run_mapper(ref, d, params, page)
    _save(d, params, dict(page=page, expected=out, known_answer=page.clone()))


def fit_cases(ref):
    """examples/fit_and_map.py:18-49 (seed 42) and tests/test_fitting.py:153-195 (seed 14)."""
    rng = torch.Generator().manual_seed(42)
    source = torch.randn(2, 3, 256, 2, 4, generator=rng)
    target = 0.6 * source[:, 0] + 0.3 * source[:, 2] + 0.1
    weights, _ = ref.fit_layer(source[:, :, :192], target[:, :192], selected=[0, 2], ridge=1e-4)
    d = _case_dir("fit_and_map")
    _write_layers(d, [weights])
    page = source[:, :, 192:].clone()
    cos, sin = ref.qwen_rope(torch.arange(192, 256), head_dim=4, theta=10000)
    page[0] = ref.apply_rope(page[0], cos, sin)
    expected = target[:, None, 192:].clone()
    tcos, tsin = ref.qwen_rope(torch.arange(192, 256), head_dim=4, theta=1000000)
    expected[0] = ref.apply_rope(expected[0], tcos, tsin)
    params = dict(position_start=192, source_theta=10000.0, target_theta=1000000.0)
    out = _run_mapper(ref, d, params, page)
    torch.testing.assert_close(out, expected, atol=1e-5, rtol=1e-5)
    _save(d, params, dict(page=page, expected=out, known_answer=expected))

    rng = torch.Generator().manual_seed(14)
    source = torch.randn(2, 3, 128, 4, 4, generator=rng)
    target = 0.7 * source[:, 2] - 0.2 * source[:, 0] + 0.13
    weights, _ = ref.fit_layer(source[:, :, :96], target[:, :96], selected=[2, 0], ridge=1e-4, chunk_rows=17)
    page = source[:, :, 96:].clone()
    cos, sin = ref.qwen_rope(torch.arange(103, 135), head_dim=4, theta=10000)
    page[0] = ref.apply_rope(page[0], cos, sin)
    for rank in range(2):
        d = _case_dir(f"fit_tp_rank{rank}")
        _write_layers(d, [weights])
        params = dict(position_start=103, source_theta=10000.0, target_theta=1000000.0, tp_rank=rank,
                      tp_size=2, source_head_offset=0)
        full = _run_mapper(ref, d, params, page)
        compact_params = dict(params, source_head_offset=rank * 2)
        compact = _run_mapper(ref, d, compact_params, page[:, :, :, rank * 2 : rank * 2 + 2].contiguous())
        assert torch.equal(full, compact)
        _save(d, params, dict(page=page, expected=full))


def pack_case(ref):
    """tests/test_blocks.py:33-65: non-contiguous pool rows into one workspace."""
    k = torch.arange(3 * 700 * 2 * 4).reshape(3, 700, 2, 4).float()
    v = -k
    pool = SimpleNamespace(layer_num=3, start_layer=0, _get_key_buffer=lambda l: k[l],
                           _get_value_buffer=lambda l: v[l])
    indices = torch.randperm(650, generator=torch.Generator().manual_seed(7))[:513] + 1
    workspace = torch.empty(2 * 3 * 512 * 2 * 4)
    d = _case_dir("pack_blocks")
    tensors = dict(indices=indices.long())
    spans = [(0, 65), (0, 512), (512, 513)]
    for start, stop in spans:
        packed = ref.pack_source_block(pool, indices, start=start, stop=stop, workspace=workspace,
                                       block_tokens=512)
        tensors[f"packed_{start}_{stop}"] = packed.clone()
    _save(d, dict(spans=spans, pool_shape=[3, 700, 2, 4]), tensors)


def geometry_case(ref):
    """peer_geometry.operations outputs for a few fragmented run lists."""
    d = _case_dir("peer_geometry")
    cases = []
    g = torch.Generator().manual_seed(3)
    for tokens, heads in [(1, 2), (3, 4), (40, 2), (2048, 4), (4096, 2)]:
        # random fragmented, non-aliasing physical placement
        perm = torch.randperm(tokens * 3, generator=g)[:tokens].sort().values.tolist()
        runs, begin = [], 0
        for i in range(1, tokens + 1):
            if i == tokens or perm[i] != perm[i - 1] + 1:
                runs.append((begin, i, perm[begin]))
                begin = i
        start = tokens // 3
        stop = tokens
        ops = ref.operations(start, stop, runs, heads=heads)
        digest = hashlib.sha256(json.dumps(ops).encode()).hexdigest()
        entry = dict(start=start, stop=stop, runs=runs, heads=heads, count=len(ops), sha256=digest)
        if len(ops) <= 512:
            entry["ops"] = ops
        cases.append(entry)
    (d / "case.json").write_text(json.dumps(cases) + "\n")


def main(argv):
    if len(argv) < 2:
        raise SystemExit(__doc__)
    ref = _reference(argv[1])
    torch.set_num_threads(4)
    if len(argv) > 2 and argv[2] == "dense":  # only the dense (nv_transfer) cases
        dense_cases(ref)
        print("dense golden fixtures written to", HERE)
        return
    reference_unit_cases(ref)
    fit_cases(ref)
    pack_case(ref)
    geometry_case(ref)
    # CPU toy configuration (fp32): 4 -> 6 layers, 2 heads x 64, S=2, 1024-slot pool at a
    # seeded random permutation (128 of the config's 512 tokens, to keep the fixture small).
    random_case(ref, "cfg1_toy", seed=1, L_s=4, L_t=6, H=2, D=64, S=2, n=128, dtype=torch.float32,
                position_start=0, source_theta=1e6, target_theta=1e6, w_var=1 / 128, b_var=0.01,
                pool_rows=1024)
    # Qwen3-14B -> 32B shapes, reduced: bf16, head_dim 128, per-channel LogNormal scales,
    # TP rank 1 of 2 narrowed from a full 4-head page, large absolute positions.
    random_case(ref, "qwen_mini_bf16", seed=2, L_s=6, L_t=4, H=2, D=128, S=2, n=130,
                dtype=torch.bfloat16, position_start=1000, source_theta=1e6, target_theta=1e6,
                tp_rank=1, tp_size=2, w_var=1 / 256, lognormal=True, bf16_weights=True,
                pool_rows=4096)
    # Llama-3.1-8B -> 70B shapes, reduced: S=4 (512 x 128 maps), Llama theta.
    random_case(ref, "llama_mini_s4", seed=4, L_s=6, L_t=2, H=2, D=128, S=4, n=130,
                dtype=torch.bfloat16, position_start=16384, source_theta=5e5, target_theta=5e5,
                w_var=1 / 512, lognormal=True, bf16_weights=True, pool_rows=2048)
    # YaRN-scaled source and target RoPE with different thetas, FP32 page, head_dim 128.
    yarn = {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 32768}
    random_case(ref, "yarn_d128_f32", seed=5, L_s=4, L_t=2, H=1, D=128, S=2, n=33, dtype=torch.float32,
                position_start=40000, source_theta=1e6, target_theta=5e5, source_scaling=yarn,
                target_scaling=yarn, w_var=1 / 256)
    # S=8 (the reference's own Qwen recipe support size), bf16, compact TP shard.
    random_case(ref, "qwen_s8_compact", seed=8, L_s=10, L_t=1, H=2, D=128, S=8, n=70,
                dtype=torch.bfloat16, position_start=7, source_theta=1e6, target_theta=1e6, tp_rank=1,
                tp_size=2, source_head_offset=1, page_heads=1, w_var=1 / 1024, lognormal=True,
                bf16_weights=True)
    dense_cases(ref)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main(sys.argv)
