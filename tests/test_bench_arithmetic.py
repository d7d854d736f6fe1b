"""The arithmetic bench.py reports beside its timings, checked on the CPU:
the algorithmic bytes and flops the rooflines divide by, the parity decision
(relative Frobenius error and the max-abs bound of one BF16 ulp beyond the
reference's own rounding), and the FP32 restatement's BF16-key option, which
isolates the one rounding step the kernels add to the reference algorithm."""

from __future__ import annotations

import torch

import bench


def test_config2_algorithmic_work():
    # Qwen3-14B -> 32B handoff of 8192 tokens: 40 -> 64 layers, 8 heads, S = 2,
    # every source layer selected. Source K/V rows read once (1.342 GB), target
    # K/V rows written once (2.147 GB), weights once, two int64 slot tables.
    bytes_, flops = bench.algorithmic_work(n=8192, L_t=64, H=8, D=128, S=2, used=40)
    assert abs(bytes_ / 1e9 - 3.557) < 1e-3
    assert flops == 4 * 64 * 8 * 2 * 128 * 128 * 8192
    assert abs(flops / 1e9 - 549.76) < 0.01


def test_config4_algorithmic_work():
    # Llama-3.1-8B -> 70B, 4 x 16384 tokens, S = 4: 11.0 TFLOP.
    _, flops = bench.algorithmic_work(n=4 * 16384, L_t=80, H=8, D=128, S=4, used=32)
    assert abs(flops / 1e12 - 10.995) < 1e-3


def test_bf16_ulp_is_the_spacing_at_the_value():
    x = torch.tensor([1.0, 1.5, 8.0, 8.9, 0.25])
    assert torch.equal(bench.bf16_ulp(x), torch.tensor([2.0 ** -7, 2.0 ** -7, 2.0 ** -4, 2.0 ** -4, 2.0 ** -9]))


def test_value_parity_accepts_the_references_own_rounding_and_one_more_ulp():
    g = torch.Generator().manual_seed(3)
    f32 = torch.randn(64, 128, generator=g) * 4
    ref = f32.to(torch.bfloat16)
    ok = bench.value_parity(ref, f32)
    assert ok["ok"] and ok["max_ulps"] == 0.0
    assert ok["max_abs"] == ok["ref_bf16_max_abs"]
    # One BF16 ulp of the largest value added to one element stays within the bound.
    i = int(f32.abs().argmax())
    nudged = ref.float().flatten().clone()
    nudged[i] += float(bench.bf16_ulp(f32.abs().max()))
    assert bench.value_parity(nudged.view_as(f32), f32)["ok"]
    # Two of them do not.
    nudged[i] += float(bench.bf16_ulp(f32.abs().max()))
    assert not bench.value_parity(nudged.view_as(f32), f32)["ok"]


def test_value_parity_rejects_a_broad_error():
    g = torch.Generator().manual_seed(4)
    f32 = torch.randn(64, 128, generator=g)
    off = (f32 * 1.01).to(torch.bfloat16)  # 1 % everywhere: relative Frobenius error 1e-2
    res = bench.value_parity(off, f32)
    assert res["rel_frobenius"] > 5e-3 and not res["ok"]


def test_bf16_keys_option_changes_only_the_keys_and_only_slightly():
    L_s, L_t, H, D, S, n, theta = 3, 4, 2, 64, 2, 40, 1e6
    layers = bench.random_layers(L_s=L_s, L_t=L_t, H=H, D=D, S=S, seed=5)
    g = torch.Generator().manual_seed(6)
    block = torch.randn(2, L_s, n, H, D, generator=g).to(torch.bfloat16)
    exact = bench.reference_map_fp32(layers, block, theta=theta, position_start=7)
    rounded = bench.reference_map_fp32(layers, block, theta=theta, position_start=7, bf16_keys=True)
    assert torch.equal(exact[1], rounded[1])  # values carry no RoPE and no extra rounding
    assert not torch.equal(exact[0], rounded[0])
    rel = float((rounded[0] - exact[0]).norm() / exact[0].norm())
    assert 0 < rel < 5e-3
