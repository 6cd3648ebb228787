"""The layer's fusions of the routing into the products: the gate/up product reading its x rows from the hidden
states through the routing (no gathered copy), the down stack's input gradient reading the upstream gradient's rows
with the routing weight applied (the un-permute's backward), and the adapter reductions over gathered rows."""

import numpy as np
import pytest
import torch

from meepsquared_b200 import _grouped, _lib, _moe
from oracle import grouped as ogrouped
from parity import as_np, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def routing_case(tokens, experts, k, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(experts, generator=g)[:k] for _ in range(tokens)]).to(DEV)
    w = torch.rand(tokens, k, generator=g).to(DEV)
    routing = _moe.route(idx, w, experts)
    token_rows, w32 = _moe.routed_rows(routing, w)
    return routing, token_rows, w32, w


def test_routed_rows_are_the_permutations_tokens_and_weights():
    routing, token_rows, w32, w = routing_case(300, 16, 4, 0)
    assert torch.equal(token_rows.long(), routing.perm // 4)
    assert torch.equal(w32, w.reshape(-1)[routing.perm])


@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("lora", [False, True])
def test_gathered_rows_give_the_gathered_copys_product_bit_for_bit(pair, lora, monkeypatch):
    monkeypatch.setenv("MEEP2B_PAIR", pair)
    routing, token_rows, w32, w = routing_case(1024, 8, 4, 1)
    gen = torch.Generator().manual_seed(2)
    H, I = 1024, 320
    hidden = torch.randn(1024, H, generator=gen).to(DEV, torch.bfloat16)
    stack = (torch.randn(8, 2 * I, H, generator=gen) * 0.05).to(DEV, torch.bfloat16)
    ad = None
    if lora:
        ad = _grouped._Adapters((torch.randn(8, 2 * I, 16, generator=gen) * 0.1).to(DEV, torch.bfloat16),
                                (torch.randn(8, 16, H, generator=gen) * 0.1).to(DEV, torch.bfloat16), False)
    sel = _moe.gather(hidden, routing, w)
    rows = sel.shape[0]
    gu_a = torch.empty(rows, 2 * I, device=DEV, dtype=torch.bfloat16)
    gu_b = torch.empty_like(gu_a)
    tiles = routing.tile_map()
    ha, la = _grouped._launch(hidden, stack, None, routing.offsets, True, ad, 2.0, None, lora, tiles=tiles,
                              epilogue=_lib.EPI_SWIGLU, aux=gu_a, x_rows=token_rows)
    hb, lb = _grouped._launch(sel, stack, None, routing.offsets, True, ad, 2.0, None, lora, tiles=tiles,
                              epilogue=_lib.EPI_SWIGLU, aux=gu_b)
    torch.cuda.synchronize()
    assert torch.equal(ha.view(torch.int16), hb.view(torch.int16))
    assert torch.equal(gu_a.view(torch.int16), gu_b.view(torch.int16))
    if lora:
        assert torch.equal(la.view(torch.int16), lb.view(torch.int16))


def test_the_weighted_gathered_reduction_matches_float32():
    routing, token_rows, w32, w = routing_case(512, 8, 2, 3)
    gen = torch.Generator().manual_seed(4)
    g = torch.randn(512, 384, generator=gen).to(DEV, torch.bfloat16)
    low = torch.randn(routing.perm.numel(), 16, generator=gen).to(DEV, torch.bfloat16)
    got = _grouped._reduce(g, low, routing.offsets, 2.0, g_rows=token_rows, row_scale=w32)
    rows = as_np(g)[as_np(token_rows).astype(np.int64)]
    lw = as_np(low) * as_np(w32)[:, None]
    want = ogrouped.reduce_adapter(rows, lw, as_np(routing.offsets), 2.0)
    assert_close(got, want, "reduce", scaled=True)


@pytest.mark.parametrize("n", [768, 1536, 2048])
@pytest.mark.parametrize("weighted", [False, True])
@pytest.mark.parametrize("layout", [0, 1])
def test_the_whole_row_gathered_reduction_matches_float32(n, weighted, layout):
    """The widths whose gathered reductions read whole rows per CTA (chunks of an expert's rows, the chunks' sums
    added in order): an expert with no rows, one with a few, the rest over several chunks with a ragged last one; g
    a column slice of a wider tensor (row pitch above n)."""
    tokens, experts, k = 1500, 8, 3
    gen = torch.Generator().manual_seed(5 + n)
    probs = torch.tensor([0.3, 0.2, 0.2, 0.15, 0.1, 0.05, 0.0, 0.0])
    idx = torch.multinomial(probs.expand(tokens, experts), k, replacement=False, generator=gen)
    idx[:5, 2] = 6  # five rows for expert 6, none for expert 7
    idx = idx.to(DEV)
    w = torch.rand(tokens, k, generator=gen).to(DEV)
    routing = _moe.route(idx, w, experts)
    token_rows, w32 = _moe.routed_rows(routing, w)
    counts = np.diff(np.concatenate([[0], as_np(routing.offsets)]))
    chunk = int(_lib.load().meep2b_reduce_chunk_rows())
    assert counts[7] == 0 and counts[6] == 5 and counts.max() > 2 * chunk
    wide = torch.randn(tokens, n + 64, generator=gen).to(DEV, torch.bfloat16)
    g = wide[:, :n]
    low = torch.randn(routing.perm.numel(), 16, generator=gen).to(DEV, torch.bfloat16)
    scale = w32 if weighted else None
    got = _grouped._reduce(g, low, routing.offsets, 2.0, g_rows=token_rows, row_scale=scale, layout=layout,
                           tiles=routing.tile_map())
    rows = as_np(g)[as_np(token_rows).astype(np.int64)]
    lw = as_np(low) * (as_np(w32)[:, None] if weighted else 1.0)
    want = ogrouped.reduce_adapter(rows, lw, as_np(routing.offsets), 2.0)
    if layout == 1:
        want = want.transpose(0, 2, 1)
    assert_close(got, want, f"reduce n={n}", scaled=True)
    assert not as_np(got)[7].any()
    # deterministic: the chunks' sums are added in a fixed order (the chunk map built anew here)
    again = _grouped._reduce(g, low, routing.offsets, 2.0, g_rows=token_rows, row_scale=scale, layout=layout)
    assert torch.equal(got.view(torch.int16), again.view(torch.int16))
