"""The whole routed MoE-LoRA layer on the GPU (routing, gate/up with SwiGLU, down, un-permute, and the backward)
against the reference's golden vectors and the float32 oracle."""

import numpy as np
import pytest
import torch

import layer_inputs
import meepsquared_b200 as mb
from oracle import layer as olayer
from parity import as_np, assert_close, bf16_ulp

pytestmark = pytest.mark.gpu
DEV = "cuda"


class Experts(torch.nn.Module):
    """The attributes of a Transformers experts module that the routed layer reads."""

    def __init__(self, gate_up, down):
        super().__init__()
        self.num_experts = gate_up.shape[0]
        self.has_gate, self.has_bias, self.is_transposed = True, False, False
        self.gate_up_proj = torch.nn.Parameter(gate_up, requires_grad=False)
        self.down_proj = torch.nn.Parameter(down, requires_grad=False)


def run_layer(inp, sentinel=False):
    idx = inp["top_k_index"].clone()
    if sentinel:
        idx[5, 1] = inp["gate_up"].shape[0]
        idx[17, 0] = inp["gate_up"].shape[0]
    bf = lambda n: inp[n].to(DEV, torch.bfloat16)  # noqa: E731
    experts = Experts(bf("gate_up"), bf("down"))
    hidden = bf("hidden").requires_grad_()
    weights = inp["top_k_weights"].to(DEV).requires_grad_()
    leaves = {n: bf(n).requires_grad_() for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")}
    factors = {"gate_up_proj": (leaves["gate_up_lhs"], leaves["gate_up_rhs"], inp["scaling"]),
               "down_proj": (leaves["down_lhs"], leaves["down_rhs"], inp["scaling"])}
    out = mb.routed_forward(experts, hidden, idx.to(DEV), weights, factors)
    out.backward(inp["grad"].to(DEV, torch.bfloat16))
    res = {"out": out.detach(), "grad_hidden": hidden.grad, "grad_weights": weights.grad}
    for n, t in leaves.items():
        res[f"grad_{n}"] = t.grad
    return res, idx


def check_against(res, want, prefix="", scaled=False):
    """scaled: the absolute allowance follows the tensor's size (1e-2 max|want|), as the reference's own tests
    do, for shapes whose bf16 intermediates (gate/up pre-activation, h, as in the reference's path) carry
    rounding of ~1% of the tensor's scale into near-zero elements."""
    assert_close(res["out"], want[prefix + "out"], "out", scaled=scaled, rounding=want.get(prefix + "out_rounding"))
    assert_close(res["grad_hidden"], want[prefix + "grad_hidden"], "grad_hidden", scaled=scaled,
                 rounding=want.get(prefix + "grad_hidden_rounding"))
    assert_close(res["grad_weights"], want[prefix + "grad_weights"], "grad_weights", scaled=True)
    for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs"):
        assert_close(res[f"grad_{n}"], want[f"{prefix}grad_{n}"], f"grad_{n}", scaled=True)


@pytest.fixture(params=["fold", "gather", "copy"])
def routed_rows_mode(request, monkeypatch):
    """How the layer meets the routing: the un-permute's backward folded into the down stack's input gradient, the
    products also reading their rows from the token-major tensors, or gathered copies throughout."""
    monkeypatch.setenv("MEEP2B_ROUTED_ROWS", request.param)
    return request.param


@pytest.mark.parametrize("sentinel", [False, True])
def test_layer_matches_the_reference_golden_vectors(golden, sentinel, pair_mode, routed_rows_mode):
    res, _ = run_layer(layer_inputs.layer(**layer_inputs.SMALL), sentinel)
    check_against(res, golden("layer_small"), "sentinel_" if sentinel else "")


def oracle_layer(inp, idx, bf16_intermediates=False, mode="copy"):
    """The float32 oracle of the layer; bf16_intermediates: with the bf16 roundings of the reference's bf16 path
    (the gate/up output, the gate's activation and h, y, the output and their gradients), at the rounding points of
    the routed-row mode: "copy" rounds the rows' gradient g * w to bf16 as the reference's autograd does, "fold"
    and "gather" apply the routing weight to the down stack's float32 input-gradient product instead."""
    factors = {"gate_up_proj": (inp["gate_up_lhs"].numpy(), inp["gate_up_rhs"].numpy(), inp["scaling"]),
               "down_proj": (inp["down_lhs"].numpy(), inp["down_rhs"].numpy(), inp["scaling"])}
    out, saved = olayer.forward(inp["hidden"].numpy(), idx.numpy(), inp["top_k_weights"].numpy(),
                                inp["gate_up"].numpy(), inp["down"].numpy(), factors,
                                bf16_intermediates=bf16_intermediates)
    g = olayer.backward(inp["grad"].numpy(), saved, inp["gate_up"].numpy(), inp["down"].numpy(), factors,
                        round_grad_rows=bf16_intermediates and mode == "copy")
    res = {"out": out, "grad_hidden": g["hidden"], "grad_weights": g["top_k_weights"],
           "grad_gate_up_lhs": g["gate_up_proj"][0], "grad_gate_up_rhs": g["gate_up_proj"][1],
           "grad_down_lhs": g["down_proj"][0], "grad_down_rhs": g["down_proj"][1]}
    if bf16_intermediates:
        # one bf16 ulp of each stored row a token's output (w y) and input gradient (the rows' gradients) sum
        r, k = saved["route"], saved["k"]
        rows = r["inverse"].reshape(-1, k)
        live = (~r["sentinel"])[rows][:, :, None]
        res["out_rounding"] = (live * np.abs(saved["w_g"][rows])[:, :, None] * bf16_ulp(saved["y"][rows])).sum(1)
        res["grad_hidden_rounding"] = (live * bf16_ulp(g["rows"][rows])).sum(1)
    return res


def test_layer_at_config1_matches_the_oracle_and_the_reference_slices(golden):
    inp = layer_inputs.layer(**layer_inputs.CONFIG1)
    res, idx = run_layer(inp)
    check_against(res, oracle_layer(inp, idx))
    g = golden("layer_config1")
    for name in ("out", "grad_hidden"):
        assert_close(as_np(res[name]).reshape(-1)[:2048], g[name + "_head"], name + " head")


# Inputs and oracle results shared by the parametrisations of a test (both are deterministic functions of the
# config): the BASELINE-shaped stacks are large to generate and the oracle takes seconds on them.
_INPUTS, _ORACLE = {}, {}


def cached_inputs(name, cfg):
    if name not in _INPUTS:
        _INPUTS[name] = layer_inputs.layer(**cfg)
    return _INPUTS[name]


def cached_oracle(key, inp, idx, mode):
    rounding = "copy" if mode == "copy" else "fold"
    if (key, rounding) not in _ORACLE:
        _ORACLE[key, rounding] = oracle_layer(inp, idx, bf16_intermediates=True, mode=rounding)
    return _ORACLE[key, rounding]


BASELINE_SHAPES = {
    # config 2 (Qwen3-30B-A3B) with 512 tokens: 32 routed rows per expert
    "qwen3_30b": dict(layer_inputs.QWEN3_30B, tokens=512),
    # config 3 (Mixtral-8x7B) with 2048 tokens: 512 routed rows per expert, so the I=14336 products run several
    # 128- and 256-row tiles per expert
    "mixtral": dict(layer_inputs.MIXTRAL, tokens=2048),
    # config 5's shape (H=4096, I=1536, Zipf routing) with bf16 stacks and 256 tokens
    "qwen3_235b": dict(layer_inputs.QWEN3_235B_FP8, tokens=256),
}


@pytest.mark.parametrize("shape", sorted(BASELINE_SHAPES))
def test_layer_at_baseline_shapes_matches_the_oracle(shape, pair_mode, routed_rows_mode):
    """The layer at the BASELINE shapes against the oracle with the reference's bf16 intermediates, the layer's
    output and input gradient within the north star's tolerance (abs 1e-2 + rel 2e-2, elementwise) plus one bf16
    ulp of each stored row their sums add (at Mixtral's shape |y| reaches ~10, where a bf16 ulp is 0.06, and a
    token's two weighted rows can cancel); the routing weights' and the adapters' gradients (sums over H, or over
    an expert's rows) with the allowance scaled to the tensor, as the reference's own tests treat sums."""
    inp = cached_inputs(shape, BASELINE_SHAPES[shape])
    res, idx = run_layer(inp)
    check_against(res, cached_oracle(shape, inp, idx, routed_rows_mode), scaled=False)


def token_subset(inp, tokens, experts=None):
    """The layer's inputs for `tokens` only (the rows of every per-token tensor; the same stacks and adapters). With
    `experts`, the tokens' assignments to any other expert become sentinels (ids >= E), which carry nothing: the
    layer is row by row, so every routed row keeps its value and gradient, and the adapters' gradients of the
    listed experts come only from their own rows."""
    t = torch.as_tensor(np.asarray(tokens, dtype=np.int64))
    sub = dict(inp)
    for n in ("hidden", "top_k_index", "top_k_weights", "grad"):
        sub[n] = inp[n][t].clone()
    if experts is not None:
        idx = sub["top_k_index"]
        idx[~torch.isin(idx, torch.as_tensor(list(experts)))] = inp["gate_up"].shape[0]
    return sub


@pytest.mark.parametrize("mode", ["fold", "copy"])
def test_full_size_config2_layer_matches_the_oracle_on_sampled_tokens_and_experts(mode, monkeypatch):
    """BASELINE config 2 at its full size (T=16384, E=128, top-8, r=16: ~1024 routed rows per expert, so the
    products run multi-tile units and the CTA-pair gate/up forward exactly as the benchmark does), the default tile
    kernels. The oracle recomputes 256 sampled tokens (their output, input gradient and routing weights'
    gradient) and every routed row of four experts (those experts' adapter gradients) with the reference's bf16
    intermediates; output and input gradient within abs 1e-2 + rel 2e-2."""
    monkeypatch.setenv("MEEP2B_ROUTED_ROWS", mode)
    monkeypatch.delenv("MEEP2B_PAIR", raising=False)
    inp = cached_inputs("qwen3_30b_full", layer_inputs.QWEN3_30B)
    res, idx = run_layer(inp)
    tokens = np.sort(np.random.default_rng(0).choice(inp["hidden"].shape[0], 256, replace=False))
    sub = token_subset(inp, tokens)
    want = cached_oracle("qwen3_30b_full_tokens", sub, sub["top_k_index"], mode)
    t = torch.as_tensor(tokens, device=DEV)
    assert_close(res["out"][t], want["out"], "out", rounding=want["out_rounding"])
    assert_close(res["grad_hidden"][t], want["grad_hidden"], "grad_hidden", rounding=want["grad_hidden_rounding"])
    assert_close(res["grad_weights"][t], want["grad_weights"], "grad_weights", scaled=True)
    experts = [0, 41, 86, 127]
    routed = np.unique(np.nonzero(np.isin(idx.numpy(), experts))[0])
    sub_e = token_subset(inp, routed, experts)
    want_e = cached_oracle("qwen3_30b_full_experts", sub_e, sub_e["top_k_index"], mode)
    e = torch.as_tensor(experts, device=DEV)
    for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs"):
        assert_close(res[f"grad_{n}"][e], want_e[f"grad_{n}"][experts], f"grad_{n}", scaled=True)


@pytest.mark.parametrize("sentinel", [False, True])
@pytest.mark.parametrize("rank", [32, 40])
def test_layer_with_adapters_of_rank_above_16_matches_the_oracle(rank, sentinel):
    """Ranks above one fused panel's 16 (the reference pads any rank to a multiple of 16): the layer runs unfused,
    each product taking the adapters in 16-rank chunks; with sentinel ids, whose rows nothing writes or reads."""
    inp = layer_inputs.layer(**dict(layer_inputs.CONFIG1, rank=rank, alpha=2 * rank))
    res, idx = run_layer(inp, sentinel=sentinel)
    check_against(res, oracle_layer(inp, idx), scaled=True)


@pytest.mark.parametrize("mode", ["fold", "copy"])
def test_adapter_gradients_are_written_into_a_gradient_bucket_with_the_same_bits(mode, monkeypatch):
    """With the four factors in a LoRA-gradient bucket released before the step (ddp.LoraGradBucket.release), the
    layer's reductions write the adapters' gradients straight into the bucket's flat buffer and autograd adopts
    them as .grad: the same bits as without a bucket, every .grad a view of the buffer, and a second step gives
    the same bits again (nothing accumulates from the first)."""
    from meepsquared_b200 import ddp

    monkeypatch.setenv("MEEP2B_ROUTED_ROWS", mode)
    inp = layer_inputs.layer(**dict(layer_inputs.QWEN3_30B, tokens=512, experts=32))
    plain, _ = run_layer(inp)
    bf = lambda n: inp[n].to(DEV, torch.bfloat16)  # noqa: E731
    experts = Experts(bf("gate_up"), bf("down"))
    names = ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")
    leaves = {n: bf(n).requires_grad_() for n in names}
    bucket = ddp.LoraGradBucket([leaves[n] for n in names])
    factors = {"gate_up_proj": (leaves["gate_up_lhs"], leaves["gate_up_rhs"], inp["scaling"]),
               "down_proj": (leaves["down_lhs"], leaves["down_rhs"], inp["scaling"])}
    for _ in range(2):
        bucket.release()
        hidden = bf("hidden").requires_grad_()
        weights = inp["top_k_weights"].to(DEV).requires_grad_()
        out = mb.routed_forward(experts, hidden, inp["top_k_index"].to(DEV), weights, factors)
        out.backward(inp["grad"].to(DEV, torch.bfloat16))
        adopted = [leaves[n].grad.data_ptr() == v.data_ptr() for n, v in zip(names, bucket.views)]
        bucket.reduce()
        assert all(adopted), adopted
        for n in names:
            assert torch.equal(leaves[n].grad, plain[f"grad_{n}"]), n
        assert torch.equal(hidden.grad, plain["grad_hidden"])


def test_the_token_major_combine_gives_the_bits_of_the_sorted_rows(monkeypatch):
    """MEEP2B_COMBINE=token (the down product and the gate/up input gradient store their rows token-major through
    the permutation, a streaming combine sums them) against the default (rows in expert order, the un-permute):
    the same bits for the output and every gradient (float32 routing weights)."""
    inp = layer_inputs.layer(**dict(layer_inputs.QWEN3_30B, tokens=512, experts=32))
    monkeypatch.setenv("MEEP2B_COMBINE", "sorted")
    sorted_rows, _ = run_layer(inp, sentinel=True)
    monkeypatch.setenv("MEEP2B_COMBINE", "token")
    token_rows, _ = run_layer(inp, sentinel=True)
    for name, value in sorted_rows.items():
        assert torch.equal(value, token_rows[name]), name


def test_full_size_layer_step_is_finite_and_deterministic():
    """BASELINE config 2 at full size (T=16384, E=128, top-8): two runs give identical bits, all finite."""
    inp = cached_inputs("qwen3_30b_full", layer_inputs.QWEN3_30B)
    a, _ = run_layer(inp)
    b, _ = run_layer(inp)
    for k in a:
        assert torch.isfinite(a[k].float()).all(), k
        assert torch.equal(a[k], b[k]), k


def _dequantised(ex, name):
    from meepsquared_b200 import _fp8, _nf4

    w = getattr(ex, name)
    if isinstance(w, _nf4.NF4State):
        return _nf4.dequantize(w).float().cpu()
    return _fp8.dequantize(w, getattr(ex, name + "_scale_inv")).float().cpu()


def _quantised_layer(kind):
    """(the layer's inputs, an experts module with its stacks quantised as `kind`, a function running the layer
    forward and backward and returning the outputs and gradients)."""
    from meepsquared_b200 import _fp8, _nf4

    inp = layer_inputs.layer(**dict(layer_inputs.QWEN3_30B, tokens=256, experts=16))
    idx = inp["top_k_index"]
    bf = lambda n: inp[n].to(DEV, torch.bfloat16)  # noqa: E731
    experts = Experts(bf("gate_up"), bf("down"))
    if kind == "nf4":
        assert _nf4.convert_stacks(experts) == 2
        assert isinstance(experts.gate_up_proj, _nf4.NF4State)
    else:
        assert _fp8.convert_stacks(experts, block=128 if kind == "fp8_block128" else None) == 2
        assert experts.gate_up_proj.dtype == torch.float8_e4m3fn

    def run():
        hidden = bf("hidden").requires_grad_()
        weights = inp["top_k_weights"].to(DEV).requires_grad_()
        leaves = {n: bf(n).requires_grad_() for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")}
        factors = {"gate_up_proj": (leaves["gate_up_lhs"], leaves["gate_up_rhs"], inp["scaling"]),
                   "down_proj": (leaves["down_lhs"], leaves["down_rhs"], inp["scaling"])}
        out = mb.routed_forward(experts, hidden, idx.to(DEV), weights, factors)
        out.backward(inp["grad"].to(DEV, torch.bfloat16))
        res = {"out": out.detach(), "grad_hidden": hidden.grad, "grad_weights": weights.grad}
        for n, t in leaves.items():
            res[f"grad_{n}"] = t.grad
        return res

    return inp, experts, run


@pytest.mark.parametrize("kind", ["fp8_expert", "fp8_block128"])
def test_layer_with_fp8_products_stays_within_the_references_tolerance(kind, monkeypatch):
    """MEEPSQUARED_FP8_PRODUCTS=1: the routed layer's products on the FP8 tensor cores (activations and gradients
    quantised per row and 128-column tile). The reference accepts 6% of the norm for such products
    (tests/test_grouped.py:137-140); every output and gradient of the layer stays within it of the float32 layer
    over the dequantised stacks."""
    monkeypatch.setenv("MEEPSQUARED_FP8_PRODUCTS", "1")
    inp, experts, run = _quantised_layer(kind)
    res = run()
    ref_inp = dict(inp, gate_up=_dequantised(experts, "gate_up_proj"), down=_dequantised(experts, "down_proj"))
    want = oracle_layer(ref_inp, inp["top_k_index"])
    for name in ("out", "grad_hidden", "grad_weights", "grad_gate_up_lhs", "grad_gate_up_rhs", "grad_down_lhs",
                 "grad_down_rhs"):
        g, w = as_np(res[name]).astype(np.float64), np.asarray(want[name], dtype=np.float64)
        assert np.linalg.norm(g - w) <= 0.06 * np.linalg.norm(w), name
    monkeypatch.delenv("MEEPSQUARED_FP8_PRODUCTS")
    assert not torch.equal(run()["out"], res["out"])  # the switch off: the dequantised bf16 products


@pytest.mark.parametrize("dequant", ["fused", "product"])
@pytest.mark.parametrize("kind", ["nf4", "fp8_expert", "fp8_block128"])
def test_layer_with_quantised_stacks_matches_the_oracle_on_the_dequantised_weights(kind, dequant, monkeypatch):
    """QLoRA (NF4) and FP8 stacks (one scale per expert, or 128 x 128 blocks) in the routed layer, dequantised in
    the products' shared memory or to a bf16 copy per product: the layer equals the float32 computation with the
    stacks dequantised as the reference dequantises them."""
    monkeypatch.setenv("MEEP2B_DEQUANT", dequant)
    inp, experts, run = _quantised_layer(kind)
    res = run()
    idx = inp["top_k_index"]
    ref_inp = dict(inp, gate_up=_dequantised(experts, "gate_up_proj"), down=_dequantised(experts, "down_proj"))
    check_against(res, oracle_layer(ref_inp, idx), scaled=True)


@pytest.mark.parametrize("kind", ["nf4", "fp8_expert", "fp8_block128"])
def test_quantised_stacks_give_the_same_bits_fused_or_dequantised_per_product(kind, monkeypatch):
    """The fused conversion writes exactly the bf16 stack the dequantisation kernels write, so with the same
    routed-row mode and tile kernels the whole layer's outputs and gradients are identical bit for bit."""
    monkeypatch.setenv("MEEP2B_ROUTED_ROWS", "copy")
    monkeypatch.setenv("MEEP2B_PAIR", "0")
    _, _, run = _quantised_layer(kind)
    monkeypatch.setenv("MEEP2B_DEQUANT", "fused")
    fused = run()
    monkeypatch.setenv("MEEP2B_DEQUANT", "product")
    per_product = run()
    for k in fused:
        assert torch.equal(fused[k], per_product[k]), k


def test_the_layer_step_replays_from_a_cuda_graph_with_the_eager_bits():
    """Forward and backward of the routed layer captured into one CUDA graph (the library makes no host
    synchronisation, allocation or stream query while a stream is being captured) and replayed: the same outputs
    and gradients as the eager step, bit for bit."""
    inp = layer_inputs.layer(**dict(layer_inputs.QWEN3_30B, tokens=512, experts=32))
    bf = lambda n: inp[n].to(DEV, torch.bfloat16)  # noqa: E731
    experts = Experts(bf("gate_up"), bf("down"))
    hidden = bf("hidden").requires_grad_()
    weights = inp["top_k_weights"].to(DEV)
    idx = inp["top_k_index"].to(DEV)
    grad = inp["grad"].to(DEV, torch.bfloat16)
    leaves = {n: bf(n).requires_grad_() for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")}
    factors = {"gate_up_proj": (leaves["gate_up_lhs"], leaves["gate_up_rhs"], inp["scaling"]),
               "down_proj": (leaves["down_lhs"], leaves["down_rhs"], inp["scaling"])}

    def step():
        hidden.grad = None
        for t in leaves.values():
            t.grad = None
        out = mb.routed_forward(experts, hidden, idx, weights, factors)
        out.backward(grad)
        return out

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            eager_out = step().detach().clone()
    torch.cuda.current_stream().wait_stream(side)
    eager = {"grad_hidden": hidden.grad.clone(), **{n: t.grad.clone() for n, t in leaves.items()}}
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = step()
    hidden.grad.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(static_out, eager_out)
    assert torch.equal(hidden.grad, eager["grad_hidden"])
    for n, t in leaves.items():
        assert torch.equal(t.grad, eager[n]), n


def torch_routed(inp, act, gated=True):
    """A float32 torch computation of the reference's routed layer (_moe.py:70-126) per expert, with the gate
    act(first half) * second half (gated) or act(up) (ungated), its autograd gradients for the layer's inputs."""
    dev = DEV
    hidden = inp["hidden"].to(dev).requires_grad_()
    weights = inp["top_k_weights"].to(dev).requires_grad_()
    idx = inp["top_k_index"].to(dev)
    lv = {n: inp[n].to(dev).requires_grad_() for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")}
    s = inp["scaling"]
    w1 = inp["gate_up"].to(dev) if gated else inp["gate_up"][:, : inp["gate_up"].shape[1] // 2].to(dev)
    l1 = lv["gate_up_lhs"] if gated else lv["gate_up_lhs"][:, : w1.shape[1]]
    w2 = inp["down"].to(dev)
    out = torch.zeros_like(hidden)
    for e in range(w1.shape[0]):
        tok, slot = torch.where(idx == e)
        if tok.numel() == 0:
            continue
        x = hidden[tok]
        p = x @ (w1[e] + s * l1[e] @ lv["gate_up_rhs"][e]).t()
        if gated:
            g, u = p.chunk(2, dim=-1)
            h = act(g) * u
        else:
            h = act(p)
        y = h @ (w2[e] + s * lv["down_lhs"][e] @ lv["down_rhs"][e]).t()
        out = out.index_add(0, tok, y * weights[tok, slot, None])
    out.backward(inp["grad"].to(dev))
    res = {"out": out.detach(), "grad_hidden": hidden.grad, "grad_weights": weights.grad}
    for n, t in lv.items():
        res[f"grad_{n}"] = t.grad if gated or n != "gate_up_lhs" else t.grad[:, : w1.shape[1]]
    return res


def run_module(inp, experts, factors):
    hidden = inp["hidden"].to(DEV, torch.bfloat16).requires_grad_()
    weights = inp["top_k_weights"].to(DEV).requires_grad_()
    out = mb.routed_forward(experts, hidden, inp["top_k_index"].to(DEV), weights, factors)
    out.backward(inp["grad"].to(DEV, torch.bfloat16))
    res = {"out": out.detach(), "grad_hidden": hidden.grad, "grad_weights": weights.grad}
    return res


class GatedExperts(torch.nn.Module):
    """A Transformers-style experts module with an activation and, optionally, transposed stacks."""

    def __init__(self, gate_up, down, act, transposed):
        super().__init__()
        self.num_experts = gate_up.shape[0]
        self.has_gate, self.has_bias, self.is_transposed = True, False, transposed
        if transposed:
            gate_up, down = gate_up.transpose(1, 2).contiguous(), down.transpose(1, 2).contiguous()
        self.gate_up_proj = torch.nn.Parameter(gate_up, requires_grad=False)
        self.down_proj = torch.nn.Parameter(down, requires_grad=False)
        self.act_fn = act

    def _apply_gate(self, gate_up_out):
        gate, up = gate_up_out.chunk(2, dim=-1)
        return self.act_fn(gate) * up


@pytest.mark.parametrize("sentinel", [False, True])
@pytest.mark.parametrize("case", ["transposed_silu", "gelu", "ungated_gelu"])
def test_modules_the_epilogues_do_not_fuse_take_the_unfused_layer(case, sentinel):
    """Transposed stacks, another activation (the module's own gate) or an ungated up projection: the products on
    the grouped kernels, the module's gate in between, against a float32 torch computation of the reference. With
    sentinel ids (ids >= E, which the reference masks): their rows are neither written by the products nor read by
    anything after them, so the module's own gate runs over rows nobody reads and the results are unchanged."""
    inp = layer_inputs.layer(**layer_inputs.CONFIG1)
    if sentinel:
        inp["top_k_index"][5, 1] = inp["gate_up"].shape[0]
        inp["top_k_index"][17, 0] = inp["gate_up"].shape[0]
    bf = lambda n: inp[n].to(DEV, torch.bfloat16)  # noqa: E731
    s = inp["scaling"]
    transposed = case == "transposed_silu"
    act = torch.nn.SiLU() if transposed else torch.nn.GELU(approximate="tanh")
    leaves = {n: bf(n).requires_grad_() for n in ("gate_up_lhs", "gate_up_rhs", "down_lhs", "down_rhs")}
    if case == "ungated_gelu":
        inter = inp["gate_up"].shape[1] // 2
        experts = GatedExperts(bf("gate_up")[:, :inter], bf("down"), act, False)
        experts.has_gate = False
        experts.up_proj = experts.gate_up_proj
        del experts.gate_up_proj
        factors = {"up_proj": (leaves["gate_up_lhs"][:, :inter], leaves["gate_up_rhs"], s),
                   "down_proj": (leaves["down_lhs"], leaves["down_rhs"], s)}
    elif transposed:  # delta (in, out) = rhs^T lhs^T
        experts = GatedExperts(bf("gate_up"), bf("down"), act, True)
        factors = {"gate_up_proj": (leaves["gate_up_rhs"].transpose(1, 2), leaves["gate_up_lhs"].transpose(1, 2), s),
                   "down_proj": (leaves["down_rhs"].transpose(1, 2), leaves["down_lhs"].transpose(1, 2), s)}
    else:
        experts = GatedExperts(bf("gate_up"), bf("down"), act, False)
        factors = {"gate_up_proj": (leaves["gate_up_lhs"], leaves["gate_up_rhs"], s),
                   "down_proj": (leaves["down_lhs"], leaves["down_rhs"], s)}
    assert not mb._moe._default_swiglu(experts)
    got = run_module(inp, experts, factors)
    for n, t in leaves.items():
        got[f"grad_{n}"] = t.grad if t.grad is not None else torch.zeros_like(t)
    want = torch_routed(inp, act, gated=case != "ungated_gelu")
    if case == "ungated_gelu":
        got["grad_gate_up_lhs"] = got["grad_gate_up_lhs"][:, : inp["gate_up"].shape[1] // 2]
    check_against(got, {k: v.cpu().numpy() for k, v in want.items()}, scaled=True)



def test_the_unfused_gate_kernels_match_the_oracle():
    """meep2b_swiglu / meep2b_swiglu_backward (the default gate of the unfused layer) against SwiGLU with the bf16
    roundings of the fused epilogues (h = bf16(bf16(silu(g)) u), and autograd's on bf16 tensors for the backward),
    elementwise within abs 1e-2 + rel 2e-2."""
    from meepsquared_b200 import _moe
    from oracle import grouped as ogrouped

    gen = torch.Generator().manual_seed(9)
    gate_up = (torch.randn(300, 400, generator=gen) * 3).to(DEV, torch.bfloat16).requires_grad_()
    h = _moe._SwiGLU.apply(gate_up)
    grad_h = torch.randn(300, 200, generator=gen).to(DEV, torch.bfloat16)
    h.backward(grad_h)
    assert_close(h.detach(), ogrouped.swiglu(as_np(gate_up.detach()), round_bf16=True), "h")
    want = ogrouped.swiglu_backward(as_np(gate_up.detach()), as_np(grad_h), round_bf16=True)
    assert_close(gate_up.grad, want, "grad_gate_up")
