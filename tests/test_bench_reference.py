"""The benchmark's restatement of the reference's path (bench.reference_routed_forward, the CPU and GPU baselines)
against the golden vectors the reference's own _routed_forward produced: the same PyTorch operations in the same
order, so on the CPU they agree to float32 (and bf16) rounding."""

import types

import numpy as np
import pytest
import torch

import bench
import layer_inputs
from oracle import quant


def run(cfg, dtype, sentinel=False):
    inp = layer_inputs.layer(**cfg)
    if sentinel:
        inp["top_k_index"][5, 1] = cfg["experts"]
        inp["top_k_index"][17, 0] = cfg["experts"]
    ex = types.SimpleNamespace(num_experts=cfg["experts"], has_gate=True, has_bias=False, is_transposed=False,
                               gate_up_proj=inp["gate_up"].to(dtype), down_proj=inp["down"].to(dtype))
    hidden = inp["hidden"].to(dtype).requires_grad_()
    weights = inp["top_k_weights"].clone().requires_grad_()
    leaves = {n: inp[n].to(dtype).requires_grad_() for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")}
    factors = {"gate_up_proj": (leaves["gate_up_lhs"], leaves["gate_up_rhs"], inp["scaling"]),
               "down_proj": (leaves["down_lhs"], leaves["down_rhs"], inp["scaling"])}
    out = bench.reference_routed_forward(ex, hidden, inp["top_k_index"], weights, factors)
    out.backward(inp["grad"].to(dtype))
    res = {"out": out.detach(), "grad_hidden": hidden.grad, "grad_weights": weights.grad}
    for n, t in leaves.items():
        res[f"grad_{n}"] = t.grad
    return {k: v.float().numpy() for k, v in res.items()}


def close(got, want, name, tol=1e-5):
    scale = max(float(np.abs(want).max()), 1e-30)
    assert np.abs(got - want).max() <= tol * scale, name


@pytest.mark.parametrize("sentinel", [False, True])
def test_restated_path_reproduces_the_reference_in_float32(golden, sentinel):
    g = golden("layer_small")
    p = "sentinel_" if sentinel else ""
    res = run(layer_inputs.SMALL, torch.float32, sentinel)
    for name, v in res.items():
        close(v, g[p + name], name)


def test_restated_path_reproduces_the_reference_at_config1(golden):
    g = golden("layer_config1")
    res = run(layer_inputs.CONFIG1, torch.float32)
    for name, v in res.items():
        close(v.reshape(-1)[:2048], g[name + "_head"], name)
        close(v.reshape(-1)[::97], g[name + "_sample"], name)


def test_restated_path_reproduces_the_reference_on_a_bf16_model(golden):
    """The reference's bf16 path (config 2's H, I and rank): the same bits, but for the rare element where a
    different summation order inside a library kernel moves a rounding."""
    g = golden("layer_bf16")
    res = run(dict(layer_inputs.QWEN3_30B, tokens=128, experts=16), torch.bfloat16)
    for name, v in res.items():
        want = g[name] if g[name].dtype == np.float32 else quant.bf16_to_f32(g[name])
        if name.startswith("grad_") and name not in ("grad_hidden", "grad_weights"):
            v = v[::5]
        assert np.mean(v != want) < 1e-3, name
        close(v, want, name, tol=2e-2)


def test_cpu_sample_policy():
    c = bench.CONFIGS["qwen3_30b"]
    assert bench.sample_tokens(c, 5.0, 25, 240.0) == 16384  # 125 s for 25 full steps: within the budget
    assert bench.sample_tokens(c, 20.0, 25, 240.0) == 4096  # 500 s: the largest power of two that fits
    assert bench.sample_tokens(c, 5.0, 3, 30.0) == 16384
    assert bench.sample_tokens(c, 100.0, 25, 240.0) == 2048  # never below 2048 tokens
    assert bench.bench_config(types.SimpleNamespace(config="qwen3_30b"), c, 1)["parallelism"] == "dp1"


def test_peak_follows_the_clock_regime():
    assert bench.pick_peak({"sm_mhz": 1965, "sm_max_mhz": 1965, "reasons": []}, 1400, 1680) == (1680, "burst")
    assert bench.pick_peak({"sm_mhz": 1500, "sm_max_mhz": 1965, "reasons": []}, 1400, 1680) == (1400, "sustained")
    assert bench.pick_peak({"sm_mhz": 1965, "sm_max_mhz": 1965, "reasons": ["sw_power_cap"]}, 1400, 1680)[1] == "sustained"
    assert bench.pick_peak({"sm_mhz": None, "sm_max_mhz": None, "reasons": []}, 1400, 1680)[1] == "sustained"
