"""Routing kernels on the GPU against the oracle and the reference's golden vectors: bit-exact."""

import numpy as np
import pytest
import torch

import layer_inputs
import meepsquared_b200 as mb
from meepsquared_b200 import _moe
from oracle import routing as oroute
from parity import as_np, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("case", ["small", "config1", "e128", "zipf"])
def test_route_matches_the_golden_permutation(golden, case):
    g = golden("routing")
    experts = int(g[f"{case}_experts"])
    ids = torch.from_numpy(g[f"{case}_ids"]).to(DEV)
    r = mb.route(ids.view(-1, 1), None, experts)
    np.testing.assert_array_equal(r.perm.cpu().numpy(), g[f"{case}_perm_stable"])
    np.testing.assert_array_equal(r.offsets.cpu().numpy(), g[f"{case}_offsets"])
    np.testing.assert_array_equal(r.expert_ids_g.cpu().numpy(), np.minimum(g[f"{case}_ids_sorted"], experts - 1))
    inv = r.inverse.cpu().numpy()
    np.testing.assert_array_equal(inv[g[f"{case}_perm_stable"]], np.arange(inv.size))


@pytest.mark.parametrize("tokens,experts,k", [(16384, 128, 8), (8192, 8, 2), (32768, 128, 8), (1, 4, 2), (3, 1, 1),
                                              (5000, 1024, 4)])
def test_route_matches_the_oracle_at_config_sizes(tokens, experts, k):
    gen = torch.Generator().manual_seed(tokens + experts)
    idx, _ = layer_inputs.routing(tokens, experts, k, gen, zipf=1.1 if experts == 128 else None)
    r = mb.route(idx.to(DEV), None, experts)
    want = oroute.route(idx.numpy(), experts)
    for name in ("perm", "offsets", "inverse", "expert_ids_g"):
        np.testing.assert_array_equal(getattr(r, name).cpu().numpy(), want[name], err_msg=name)


def test_route_with_sentinels():
    ids = torch.tensor([[3, 9], [0, 4], [4, 1], [9, 2], [7, 0]], dtype=torch.int64)  # E=5: 9 and 7 are sentinels
    r = mb.route(ids.to(DEV), None, 5)
    want = oroute.route(ids.numpy(), 5)
    np.testing.assert_array_equal(r.offsets.cpu().numpy(), want["offsets"])
    valid = int(want["offsets"][-1])
    np.testing.assert_array_equal(r.perm.cpu().numpy()[:valid], want["perm"][:valid])
    assert sorted(r.perm.cpu().numpy()[valid:].tolist()) == sorted(want["perm"][valid:].tolist())


def test_tile_map_matches_the_reference_kats(golden):
    g = golden("tile_map")
    for name in sorted({k.rsplit("_", 1)[0] for k in g if k.endswith("_offsets")}):
        te, tr, tiles = mb.tile_map(torch.from_numpy(g[f"{name}_offsets"]).to(DEV), int(g[f"{name}_rows"]),
                                    int(g[f"{name}_block_m"]))
        assert tiles.item() == int(g[f"{name}_tiles"]), name
        np.testing.assert_array_equal(te.cpu().numpy(), g[f"{name}_tile_expert"], err_msg=name)
        np.testing.assert_array_equal(tr.cpu().numpy(), g[f"{name}_tile_row"], err_msg=name)


@pytest.mark.parametrize("experts", [1, 100, 1023, 1025, 10000, 16384])
@pytest.mark.parametrize("block_m", [128, 512])
def test_tile_map_matches_the_oracle_for_many_experts(experts, block_m):
    """Expert counts around the scan's 1024 threads and up to the limit (whose table takes 128 KB of shared
    memory), some experts empty, against the oracle's tile map."""
    gen = torch.Generator().manual_seed(experts + block_m)
    counts = torch.randint(0, 3 * block_m, (experts,), generator=gen)
    counts[torch.rand(experts, generator=gen) < 0.3] = 0
    offsets = torch.cumsum(counts, 0).to(torch.int32)
    rows = int(offsets[-1])
    te, tr, tiles = mb.tile_map(offsets.to(DEV), rows, block_m)
    want_e, want_r, want_n = oroute.tile_map(offsets.numpy(), rows, block_m)
    assert tiles.item() == want_n
    np.testing.assert_array_equal(te.cpu().numpy()[:want_n], want_e[:want_n])
    np.testing.assert_array_equal(tr.cpu().numpy()[:want_n], want_r[:want_n])


@pytest.mark.parametrize("hidden_dim,tokens", [(768, 3001), (2048, 3001), (4096, 1500), (8192, 300)])
def test_gather_of_many_rows_matches_the_oracle(hidden_dim, tokens):
    """Thousands of rows of 768 to 8192 columns gathered into expert order, sentinel rows zeroed, the routing
    weights gathered with them."""
    experts, k = 16, 3
    gen = torch.Generator().manual_seed(hidden_dim)
    idx = torch.stack([torch.randperm(experts + 1, generator=gen)[:k] for _ in range(tokens)])  # id 16: a sentinel
    w = torch.rand(tokens, k, generator=gen)
    hidden = torch.randn(tokens, hidden_dim, generator=gen).to(torch.bfloat16)
    r = mb.route(idx.to(DEV), w.to(DEV), experts)
    sel = mb.gather(hidden.to(DEV), r, w.to(DEV))
    want = oroute.route(idx.numpy(), experts)
    assert want["sentinel"].any()
    np.testing.assert_array_equal(as_np(sel), oroute.gather(as_np(hidden), want["perm"], k, want["sentinel"]))
    np.testing.assert_array_equal(as_np(r.weights_g), as_np(w).reshape(-1)[want["perm"]])


@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16])
def test_gather_and_unpermute_match_the_oracle(wdtype):
    cfg = dict(layer_inputs.SMALL)
    inp = layer_inputs.layer(**cfg)
    idx = inp["top_k_index"].clone()
    idx[3, 1] = cfg["experts"]  # a sentinel
    w = inp["top_k_weights"].to(wdtype)
    hidden = inp["hidden"].to(torch.bfloat16)
    r = mb.route(idx.to(DEV), w.to(DEV), cfg["experts"])
    sel = mb.gather(hidden.to(DEV), r, w.to(DEV))
    want = oroute.route(idx.numpy(), cfg["experts"])
    np.testing.assert_array_equal(as_np(sel), oroute.gather(as_np(hidden), want["perm"], cfg["top_k"], want["sentinel"]))
    np.testing.assert_array_equal(as_np(r.weights_g), as_np(w).reshape(-1)[want["perm"]])
    y = torch.randn(sel.shape, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    y_np = as_np(y)
    y_np[want["sentinel"]] = 0
    out = mb.unpermute(y.to(DEV), r, r.weights_g)
    ref = oroute.unpermute(y_np, as_np(r.weights_g), want["inverse"], cfg["tokens"], cfg["top_k"])
    # float32 weights: one bf16 rounding of a float32 sum; bf16 weights: each product rounded to bf16 first, as the
    # reference's bf16 multiply does, so the parity tolerance against float32
    if wdtype == torch.float32:
        np.testing.assert_allclose(as_np(out), ref, rtol=8e-3, atol=1e-6)
    else:
        assert_close(out, ref, "unpermute")
    grad = torch.randn(cfg["tokens"], cfg["hidden"], generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    gy, gw = _moe.unpermute_backward(grad.to(DEV), y.to(DEV), r)
    ref_gy, ref_gw = oroute.unpermute_backward(as_np(grad), y_np, as_np(r.weights_g), want["perm"], cfg["top_k"])
    ref_gy[want["sentinel"]] = 0
    ref_gw[want["sentinel"]] = 0
    assert_close(gy, ref_gy, "grad_y")
    flat = np.zeros(cfg["tokens"] * cfg["top_k"], dtype=np.float32)
    flat[want["perm"]] = ref_gw
    assert_close(as_np(gw).reshape(-1), flat, "grad_weights", scaled=True)  # a sum over the hidden size


@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16])
def test_the_token_major_combine_gives_the_bits_of_the_unpermute(wdtype):
    """Rows stored at their flat assignment (token-major, as the down product stores them through out_rows = perm)
    and summed by meep2b_combine with the router-order weights: the same bits as the un-permute of the same rows in
    expert order with the weights in expert order; sentinel assignments (never stored) count as zero."""
    cfg = dict(layer_inputs.SMALL)
    inp = layer_inputs.layer(**cfg)
    idx = inp["top_k_index"].clone()
    idx[3, 1] = cfg["experts"]  # a sentinel
    idx[7, 0] = cfg["experts"] + 5
    w = inp["top_k_weights"].to(wdtype).to(DEV)
    r = mb.route(idx.to(DEV), w, cfg["experts"])
    mb.gather(torch.zeros(cfg["tokens"], 8, dtype=torch.bfloat16, device=DEV), r, w)  # fills r.weights_g
    rows = r.perm.numel()
    y = torch.randn(rows, cfg["hidden"], generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(DEV)
    y_tok = torch.full_like(y, float("nan"))  # slots of sentinel assignments are never written
    valid = int(r.offsets[-1])
    y_tok[r.perm[:valid]] = y[:valid]
    for weights, weights_g in ((w, r.weights_g), (None, None)):
        got = _moe.combine(y_tok, r, weights)
        want = mb.unpermute(y, r, weights_g)
        assert torch.equal(got, want)


def _same_topk_up_to_ties(got_idx, want_idx, probs):
    """The selected experts agree, except where the k-th and (k+1)-th probabilities of a token are within a few
    float32 units (then either choice is a correct top-k of values that differ only by rounding)."""
    got_idx, want_idx = np.asarray(got_idx), np.asarray(want_idx)
    differ = np.nonzero((got_idx != want_idx).any(axis=1))[0]
    srt = -np.sort(-probs, axis=1)
    for t in differ:
        k = got_idx.shape[1]
        assert abs(srt[t, k - 1] - srt[t, k]) <= 4e-7 * srt[t, k - 1] or \
            abs(srt[t, :k][:-1] - srt[t, 1:k]).min() <= 4e-7 * srt[t, 0], f"token {t}"
    assert differ.size <= max(1, got_idx.shape[0] // 1000)


@pytest.mark.parametrize("logits_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("tokens,experts,k,norm", [(16384, 128, 8, True), (8192, 8, 2, True), (777, 60, 4, False),
                                                   (300, 1000, 32, True)])
def test_the_router_fused_with_the_sort_matches_the_oracle(logits_dtype, tokens, experts, k, norm):
    """route_logits: the router (softmax, top-k, renormalised weights) against the numpy restatement of
    Transformers' router, and its routing bit-exact with route() over the ids it chose (the router's pass does the
    sort's histogram)."""
    gen = torch.Generator().manual_seed(tokens + experts)
    logits = torch.randn(tokens, experts, generator=gen).to(logits_dtype)
    probs, weights, index, r = _moe.route_logits(logits.to(DEV), k, experts, norm_topk_prob=norm)
    p_ref, w_ref, i_ref = oroute.router(logits.float().numpy(), k, norm)
    np.testing.assert_allclose(as_np(probs), p_ref, rtol=2e-6, atol=1e-9)
    _same_topk_up_to_ties(as_np(index).astype(np.int64), i_ref, p_ref)
    same = (as_np(index).astype(np.int64) == i_ref).all(axis=1)
    np.testing.assert_allclose(as_np(weights)[same], w_ref[same], rtol=2e-6, atol=1e-9)
    want = mb.route(index, weights, experts)
    for name in ("perm", "expert_ids_g", "offsets", "inverse"):
        assert torch.equal(getattr(r, name), getattr(want, name)), name
    # and against torch's own softmax / topk on the GPU
    tp = torch.softmax(logits.to(DEV), dim=-1, dtype=torch.float32)
    torch.testing.assert_close(probs, tp, rtol=2e-6, atol=1e-9)


def test_the_fused_router_feeds_the_layer_with_the_bits_of_the_plain_routing():
    """routed_forward(..., routing=route_logits(...)[3]) gives the bits of routed_forward over the same ids."""
    cfg = dict(layer_inputs.SMALL)
    inp = layer_inputs.layer(**cfg)
    gen = torch.Generator().manual_seed(5)
    logits = torch.randn(cfg["tokens"], cfg["experts"], generator=gen).to(DEV)

    class Experts(torch.nn.Module):
        pass

    ex = Experts()
    ex.num_experts, ex.has_gate, ex.has_bias, ex.is_transposed = cfg["experts"], True, False, False
    ex.gate_up_proj = inp["gate_up"].to(DEV, torch.bfloat16)
    ex.down_proj = inp["down"].to(DEV, torch.bfloat16)
    fac = {"gate_up_proj": (inp["gate_up_lhs"].to(DEV, torch.bfloat16), inp["gate_up_rhs"].to(DEV, torch.bfloat16),
                            inp["scaling"]),
           "down_proj": (inp["down_lhs"].to(DEV, torch.bfloat16), inp["down_rhs"].to(DEV, torch.bfloat16),
                         inp["scaling"])}
    hidden = inp["hidden"].to(DEV, torch.bfloat16)
    _, weights, index, r = _moe.route_logits(logits, cfg["top_k"], cfg["experts"])
    a = mb.routed_forward(ex, hidden, index, weights, fac, routing=r)
    b = mb.routed_forward(ex, hidden, index, weights, fac)
    assert torch.equal(a, b)


def test_empty_routing():
    r = mb.route(torch.zeros((0, 2), dtype=torch.int64, device=DEV), None, 4)
    assert r.perm.numel() == 0 and r.offsets.cpu().tolist() == [0, 0, 0, 0]
