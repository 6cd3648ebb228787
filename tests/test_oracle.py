"""The CPU oracle against the golden vectors the reference's own code produced (tests/golden/make_golden.py)."""

import numpy as np
import pytest
import torch

import layer_inputs
from oracle import grouped, layer, quant, routing


def test_tile_map_matches_the_reference_kats(golden):
    g = golden("tile_map")
    names = sorted({k.rsplit("_", 1)[0] for k in g if k.endswith("_offsets")})
    assert "kat1" in names and "kat2" in names
    for name in names:
        te, tr, tiles = routing.tile_map(g[f"{name}_offsets"], int(g[f"{name}_rows"]), int(g[f"{name}_block_m"]))
        assert tiles == int(g[f"{name}_tiles"]), name
        np.testing.assert_array_equal(te, g[f"{name}_tile_expert"], err_msg=name)
        np.testing.assert_array_equal(tr, g[f"{name}_tile_row"], err_msg=name)
    # the reference test's literal answer (tests/test_grouped.py:18-25)
    te, tr, tiles = routing.tile_map(np.cumsum([5, 0, 130, 64]), 199, 64)
    assert tiles == 5 and te[:5].tolist() == [0, 2, 2, 2, 3] and tr[:5].tolist() == [0, 5, 69, 133, 135]


@pytest.mark.parametrize("case", ["small", "config1", "e128", "zipf"])
def test_routing_matches_the_reference_sort(golden, case):
    g = golden("routing")
    experts = int(g[f"{case}_experts"])
    r = routing.route(g[f"{case}_ids"], experts)
    np.testing.assert_array_equal(r["offsets"], g[f"{case}_offsets"])
    np.testing.assert_array_equal(r["perm"], g[f"{case}_perm_stable"])
    np.testing.assert_array_equal(g[f"{case}_ids"][r["perm"]], g[f"{case}_ids_sorted"])
    # the reference's own (unstable) CPU sort: the same rows per expert, possibly in another order within one
    ref = g[f"{case}_perm_reference"]
    start = 0
    for end in list(r["offsets"]) + [ref.size]:
        assert set(ref[start:end].tolist()) == set(r["perm"][start:end].tolist())
        start = end
    np.testing.assert_array_equal(r["inverse"][r["perm"]], np.arange(ref.size))


def _layer(cfg, sentinel=False):
    inp = layer_inputs.layer(**cfg)
    if sentinel:
        inp["top_k_index"][5, 1] = cfg["experts"]
        inp["top_k_index"][17, 0] = cfg["experts"]
    factors = {"gate_up_proj": (inp["gate_up_lhs"].numpy(), inp["gate_up_rhs"].numpy(), inp["scaling"]),
               "down_proj": (inp["down_lhs"].numpy(), inp["down_rhs"].numpy(), inp["scaling"])}
    out, saved = layer.forward(inp["hidden"].numpy(), inp["top_k_index"].numpy(), inp["top_k_weights"].numpy(),
                               inp["gate_up"].numpy(), inp["down"].numpy(), factors)
    grads = layer.backward(inp["grad"].numpy(), saved, inp["gate_up"].numpy(), inp["down"].numpy(), factors)
    return out, grads


def _close(a, b, name):
    scale = max(float(np.abs(b).max()), 1e-30)
    assert np.abs(a - b).max() <= 1e-4 * scale, name


@pytest.mark.parametrize("sentinel", [False, True])
def test_layer_matches_the_reference_routed_forward(golden, sentinel):
    g = golden("layer_small")
    p = "sentinel_" if sentinel else ""
    out, grads = _layer(layer_inputs.SMALL, sentinel)
    _close(out, g[p + "out"], "out")
    _close(grads["hidden"], g[p + "grad_hidden"], "grad_hidden")
    _close(grads["top_k_weights"], g[p + "grad_weights"], "grad_weights")
    for proj in ("gate_up", "down"):
        _close(grads[proj + "_proj"][0], g[f"{p}grad_{proj}_lhs"], proj + " lhs")
        _close(grads[proj + "_proj"][1], g[f"{p}grad_{proj}_rhs"], proj + " rhs")


def test_layer_matches_the_reference_at_config1(golden):
    g = golden("layer_config1")
    out, grads = _layer(layer_inputs.CONFIG1)
    mine = {"out": out, "grad_hidden": grads["hidden"], "grad_weights": grads["top_k_weights"],
            "grad_gate_up_lhs": grads["gate_up_proj"][0], "grad_gate_up_rhs": grads["gate_up_proj"][1],
            "grad_down_lhs": grads["down_proj"][0], "grad_down_rhs": grads["down_proj"][1]}
    for name, v in mine.items():
        _close(v.reshape(-1)[:2048], g[name + "_head"], name)
        _close(v.reshape(-1)[::97], g[name + "_sample"], name)
        assert abs(np.linalg.norm(v.astype(np.float64)) - float(g[name + "_norm"])) <= 1e-4 * float(g[name + "_norm"])


def test_layer_with_bf16_intermediates_stays_within_the_references_bf16_path(golden):
    """The oracle's bf16 mode (the layer's intermediate tensors rounded to bf16 where they are stored) against the
    reference's own _routed_forward on a bf16 model (golden vectors at config 2's H, I and rank). The reference's
    bf16 path rounds more often (the base product and the adapters' change separately, then their sum), so neither
    side is the other's bits: they agree to bf16 arithmetic's noise, the layer output and input gradient
    elementwise within the north star's abs 1e-2 + rel 2e-2, every tensor within 1% of its RMS."""
    g = golden("layer_bf16")
    inp = layer_inputs.layer(**dict(layer_inputs.QWEN3_30B, tokens=128, experts=16))
    factors = {"gate_up_proj": (inp["gate_up_lhs"].numpy(), inp["gate_up_rhs"].numpy(), inp["scaling"]),
               "down_proj": (inp["down_lhs"].numpy(), inp["down_rhs"].numpy(), inp["scaling"])}
    out, saved = layer.forward(inp["hidden"].numpy(), inp["top_k_index"].numpy(), inp["top_k_weights"].numpy(),
                               inp["gate_up"].numpy(), inp["down"].numpy(), factors, bf16_intermediates=True)
    grads = layer.backward(inp["grad"].numpy(), saved, inp["gate_up"].numpy(), inp["down"].numpy(), factors)
    assert np.array_equal(out, quant.bf16(out)) and np.array_equal(grads["hidden"], quant.bf16(grads["hidden"]))
    mine = {"out": out, "grad_hidden": grads["hidden"], "grad_weights": grads["top_k_weights"],
            "grad_gate_up_lhs": grads["gate_up_proj"][0][::5], "grad_gate_up_rhs": grads["gate_up_proj"][1][::5],
            "grad_down_lhs": grads["down_proj"][0][::5], "grad_down_rhs": grads["down_proj"][1][::5]}
    for name, v in mine.items():
        ref = g[name] if g[name].dtype == np.float32 else quant.bf16_to_f32(g[name])
        err = np.abs(v - ref)
        assert np.sqrt(np.mean(err ** 2)) <= 0.01 * np.sqrt(np.mean(ref ** 2)), name
        if name in ("out", "grad_hidden"):
            assert np.all(err <= 1e-2 + 2e-2 * np.abs(ref)), name


def test_bf16_intermediates_are_rounded_where_the_reference_rounds_them():
    """The bf16 mode differs from the float32 oracle only by the roundings it states: on inputs whose products
    are exact in float32 (small integers times powers of two) every intermediate is the float32 value rounded."""
    rng = np.random.default_rng(2)
    gu = (rng.integers(-300, 300, size=(6, 8)) / 64.0).astype(np.float32)
    h = grouped.swiglu(gu, round_bf16=True)
    act = quant.bf16(grouped.silu(gu[:, :4]))
    np.testing.assert_array_equal(h, quant.bf16(act * gu[:, 4:]))
    dh = quant.bf16(rng.standard_normal((6, 4)).astype(np.float32))
    d = grouped.swiglu_backward(gu, dh, round_bf16=True)
    np.testing.assert_array_equal(d[:, 4:], quant.bf16(dh * act))
    assert np.array_equal(d, quant.bf16(d))


@pytest.mark.parametrize("prefix,is_transposed", [("n_", False), ("t_", True)])
def test_grouped_product_matches_reference_lora(golden, prefix, is_transposed):
    g = golden("grouped")
    f = {k[len(prefix):]: v for k, v in g.items() if k.startswith(prefix)}
    x, w, lhs, rhs, bias, grad = (quant.bf16_to_f32(f[n]) for n in ("x", "weight", "lhs", "rhs", "bias", "grad"))
    out = grouped.lora_forward(x, w, f["scale"], f["offsets"], is_transposed, lhs, rhs, 2.0, bias)
    _close(out, f["out"], "out")
    gx, gl, gr = grouped.lora_backward(x, grad, w, f["scale"], f["offsets"], is_transposed, lhs, rhs, 2.0)
    _close(gx, f["grad_x"], "grad_x")
    _close(gl, f["grad_lhs"], "grad_lhs")
    _close(gr, f["grad_rhs"], "grad_rhs")


def test_bf16_rounding_matches_torch():
    x = torch.randn(100000) * torch.logspace(-30, 30, 100000)
    x[:5] = torch.tensor([0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 65504.0])
    np.testing.assert_array_equal(quant.bf16_bits(x.numpy()), x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))


def test_e4m3_codes_match_torch_everywhere_in_range():
    x = torch.cat([torch.linspace(-470, 470, 200001), torch.randn(100000) * 1e-3, torch.tensor([2 ** -10, 2 ** -9 * 1.5])])
    np.testing.assert_array_equal(quant.f32_to_e4m3(x.numpy()), x.to(torch.float8_e4m3fn).view(torch.uint8).numpy())
    codes = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(quant.e4m3_to_f32(codes), ref)


@pytest.mark.parametrize("name", ["test", "big"])
def test_fp8_stack_matches_the_reference(golden, name):
    g = golden("fp8_stack")
    w = quant.bf16_to_f32(g[f"{name}_weight"])
    codes, scale = quant.quantize_stack(w)
    np.testing.assert_array_equal(scale, g[f"{name}_scale"])
    np.testing.assert_array_equal(codes, g[f"{name}_codes"])
    np.testing.assert_array_equal(quant.dequantize_stack(codes, scale), g[f"{name}_dequant"])


@pytest.mark.parametrize("name", ["even", "tail"])
def test_fp8_blocks_match_the_reference(golden, name):
    g = golden("fp8_block")
    w = quant.bf16_to_f32(g[f"{name}_weight"])
    codes, scale = quant.quantize_fp8_blocks(w, g[f"{name}_scale"].shape)
    np.testing.assert_array_equal(scale, g[f"{name}_scale"])
    np.testing.assert_array_equal(codes, g[f"{name}_codes"])
    np.testing.assert_array_equal(quant.dequantize_fp8_blocks(g[f"{name}_codes"], g[f"{name}_scale"]), g[f"{name}_dequant"])


def test_nf4_levels_follow_the_papers_construction():
    np.testing.assert_allclose(quant.nf4_levels_from_construction(), quant.NF4_LEVELS, rtol=0, atol=2e-7)
    code = quant.dynamic_map()
    assert code.size == 256 and code[-1] == 1.0 and -1.0 < code[0] < -0.99 and np.all(np.diff(code) >= 0)


def test_nf4_round_trip_stays_within_the_level_spacing():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((8, 96, 128)) * 0.02).astype(np.float32)
    state = quant.quantize_nf4(w)
    back = quant.bf16_to_f32(quant.dequantize_nf4(state))
    blocks = np.abs(w.reshape(-1, 64)).max(axis=1)
    err = np.abs(back.reshape(-1, 64) - w.reshape(-1, 64)).max(axis=1)
    assert np.all(err <= 0.21 * blocks + 1e-6)  # half the widest NF4 gap, plus absmax requantisation
    assert state["packed"].size == w.size // 2 and state["absmax"].size == w.size // 64


@pytest.mark.parametrize("prefix", ["n_", "t_"])
def test_merged_stack_matches_the_reference_merged_save(golden, prefix):
    """_save._merged_stack (_save.py:79-95): bf16 and FP8 stacks with their adapters merged, float32 and bf16
    outputs. The oracle's float32 matmul may sum the rank products in another order than torch's bmm: float32
    results agree to a few ulps, bf16 results bit for bit but for rounding-boundary cases."""
    from oracle import merge

    g = golden("merged")
    p = prefix
    lhs, rhs, s = g[p + "lhs"], g[p + "rhs"], float(g[p + "scaling"])
    w = quant.bf16_to_f32(g[p + "stack"])
    np.testing.assert_allclose(merge.merged_stack(w, lhs, rhs, s), g[p + "merged_f32"], rtol=1e-6, atol=1e-7)
    got = merge.merged_stack(w, lhs, rhs, s, "bf16")
    assert np.mean(got != g[p + "merged_bf16"]) < 1e-3
    np.testing.assert_allclose(quant.bf16_to_f32(got), quant.bf16_to_f32(g[p + "merged_bf16"]), rtol=2 ** -7)
    w8 = merge.dequantized_f32(codes=g[p + "codes"], scale=g[p + "scale"])
    np.testing.assert_array_equal(w8, g[p + "fp8_alone_f32"])
    np.testing.assert_allclose(merge.merged_stack(w8, lhs, rhs, s), g[p + "fp8_merged_f32"], rtol=1e-6, atol=1e-7)


def test_activation_quantisation_known_answers():
    """The FP8 product's x tiles (reference _grouped.py:194-197): the row's largest magnitude maps to 448, an
    all-zero row takes the 1e-12 floor, and the codes round like torch's float8_e4m3fn cast of x / scale."""
    x = np.zeros((3, 160), dtype=np.float32)
    x[0, :4] = [2.0, -1.0, 0.5, 0.1]
    x[0, 130] = 3.0          # the second tile of row 0 has its own scale
    x[2] = np.linspace(-5, 7, 160, dtype=np.float32)
    codes, scales = quant.quantize_rows(x)
    assert codes.shape == (3, 160) and scales.shape == (2, 3)
    assert scales[0, 0] == np.float32(2.0) / np.float32(448.0) and scales[1, 0] == np.float32(3.0) / np.float32(448.0)
    assert scales[0, 1] == np.float32(1e-12) / np.float32(448.0) and not codes[1].any()
    assert quant.e4m3_to_f32(codes[0, :1])[0] == 448.0 and quant.e4m3_to_f32(codes[0, 130:131])[0] == 448.0
    for r in range(3):
        for b in range(2):
            cols = slice(128 * b, min(160, 128 * (b + 1)))
            want = torch.from_numpy(x[r, cols] / scales[b, r]).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
            np.testing.assert_array_equal(codes[r, cols], want)


def test_fp8_product_is_exact_on_representable_activations():
    """Activations that are e4m3 values times a power of two (the row's largest 448 * 2^j) quantise without error,
    so the oracle's FP8 product equals the float32 product over the decoded stack."""
    rng = np.random.default_rng(4)
    levels = quant.e4m3_to_f32(np.arange(0, 0x7E, dtype=np.uint8))
    rows, k, n = 40, 256, 48
    x = rng.choice(levels, size=(rows, k)) * rng.choice([-1.0, 1.0], size=(rows, k))
    x[:, 0] = 448.0
    x[:, 128] = 448.0
    x = (x * np.exp2(rng.integers(-6, 3, size=(rows, 1)))).astype(np.float32)
    codes = rng.integers(0, 0x7E, size=(2, n, k)).astype(np.uint8)
    offsets = np.array([15, 40])
    got = grouped.fp8_product(x, codes, np.array([0.5, 2.0], dtype=np.float32), offsets, False)
    w = quant.e4m3_to_f32(codes)
    want = np.concatenate([x[:15] @ w[0].T * 0.5, x[15:] @ w[1].T * 2.0]).astype(np.float32)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-3 * np.abs(want).max())


def test_the_router_restatement_matches_transformers_router():
    """oracle.routing.router against Transformers' own Qwen3MoeTopKRouter on the CPU (the router whose outputs the
    routed layer takes): the same experts in the same order, probabilities and weights within float32 rounding."""
    import torch
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeTopKRouter

    class Config:
        num_experts_per_tok, num_experts, norm_topk_prob, hidden_size = 8, 128, True, 64

    for norm in (True, False):
        Config.norm_topk_prob = norm
        router = Qwen3MoeTopKRouter(Config())
        gen = torch.Generator().manual_seed(0)
        router.weight.data = torch.randn(router.weight.shape, generator=gen)
        h = torch.randn(512, 64, generator=gen)
        with torch.no_grad():
            probs, weights, index = router(h)
            logits = torch.nn.functional.linear(h, router.weight)
        p, w, i = routing.router(logits.numpy(), 8, norm)
        np.testing.assert_array_equal(i, index.numpy())
        np.testing.assert_allclose(p, probs.numpy(), rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(w, weights.numpy(), rtol=1e-5, atol=1e-7)
