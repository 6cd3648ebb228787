"""The grouped product over a quantised stack, dequantised in shared memory between the TMA load and the MMA.

The converter writes exactly the bf16 stack the reference's dequantisation gives (NF4: bitsandbytes' two stages as
axolotl quantize.py:52-101 calls them; block FP8: quantize.py:131-157, blocks of ceil(rows/sr) x ceil(cols/sc) for
an (sr, sc) scale grid; per-expert FP8: the exact e4m3
values with the scale on the accumulator, _grouped.py:200-208), and the MMA reads it in the same order as a bf16
stack's: so the fused product equals, bit for bit, the product over the stack dequantised beforehand.
"""

import numpy as np
import pytest
import torch

import meepsquared_b200 as mb
from meepsquared_b200 import _fp8, _grouped, _lib, _nf4
from oracle import grouped as ogrouped
from parity import as_np, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
KINDS = ["nf4", "e4m3", "e4m3_blocks"]


def offsets_of(rows_per_expert):
    return torch.cumsum(torch.tensor(rows_per_expert, dtype=torch.int32, device=DEV), 0, dtype=torch.int32)


def quantised(kind, shape, gen):
    """(QuantStack, the same stack dequantised to bf16, the per-expert scale for the epilogue or None)."""
    w = (torch.randn(shape, generator=gen) * 0.05).to(DEV)
    if kind == "nf4":
        st = _nf4.quantize(w)
        return _grouped.QuantStack.from_nf4(st), _nf4.dequantize(st), None
    if kind == "e4m3":
        codes, scale = _fp8.quantize_stack(w)
        ones = torch.ones(shape[0], device=DEV)
        return _grouped.QuantStack.from_fp8(codes, scale), _fp8.dequantize_stack(codes, ones, torch.bfloat16), scale
    rows, cols = shape[1], shape[2]  # 128 x 128 blocks where they divide; 64-column blocks otherwise
    grid = (-(-rows // 128), cols // 128 if cols % 128 == 0 else cols // 64)
    codes, scale = _fp8.quantize_blocks(w, grid=grid)
    return _grouped.QuantStack.from_fp8(codes, scale), _fp8.dequantize_blocks(codes, scale), None


def bits(t):
    return t.contiguous().view(torch.int16)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("mode", ["fwd_plain", "fwd_swiglu", "bwd_plain", "bwd_dswiglu", "fwd_plain_pair",
                                  "fwd_swiglu_pair"])
@pytest.mark.parametrize("lora", [False, True])
def test_the_fused_dequantisation_gives_the_dequantised_stacks_product_bit_for_bit(kind, mode, lora, monkeypatch):
    # both products on one-CTA tiles, or both on CTA pairs (the forward, K-major products)
    monkeypatch.setenv("MEEP2B_PAIR", "1" if mode.endswith("_pair") else "0")
    mode = mode.replace("_pair", "")
    gen = torch.Generator().manual_seed(11 + KINDS.index(kind))
    rows_per_expert = [37, 0, 200, 129]
    experts, rows = len(rows_per_expert), sum(rows_per_expert)
    offsets = offsets_of(rows_per_expert)
    backward = mode.startswith("bwd")
    # the stored stack (E, out, in); the forward contracts over in (K-major), the backward over out (MN-major)
    out_dim, in_dim = {"fwd_plain": (448, 256), "fwd_swiglu": (448, 256), "bwd_plain": (256, 448),
                       "bwd_dswiglu": (256, 192)}[mode]
    qs, w_bf16, scale = quantised(kind, (experts, out_dim, in_dim), gen)
    assert qs is not None and qs.kind == {"nf4": _lib.NF4, "e4m3": _lib.E4M3, "e4m3_blocks": _lib.E4M3_BLOCKS}[kind]
    K, N = (out_dim, in_dim) if backward else (in_dim, out_dim)
    x = torch.randn(rows, K, generator=gen).to(DEV, torch.bfloat16)
    ad = None
    if lora:
        lhs = (torch.randn(experts, out_dim, 16, generator=gen) * 0.1).to(DEV, torch.bfloat16)
        rhs = (torch.randn(experts, 16, in_dim, generator=gen) * 0.1).to(DEV, torch.bfloat16)
        ad = _grouped._Adapters(lhs, rhs, False)
    epi = {"fwd_plain": _lib.EPI_PLAIN, "fwd_swiglu": _lib.EPI_SWIGLU, "bwd_plain": _lib.EPI_PLAIN,
           "bwd_dswiglu": _lib.EPI_DSWIGLU}[mode]
    aux_f = aux_r = None
    if epi == _lib.EPI_SWIGLU:
        aux_f = torch.empty(rows, N, device=DEV, dtype=torch.bfloat16)
        aux_r = torch.empty_like(aux_f)
    elif epi == _lib.EPI_DSWIGLU:
        aux_f = aux_r = torch.randn(rows, 2 * N, generator=gen).to(DEV, torch.bfloat16)
    fused = _grouped._launch(x, qs, scale, offsets, not backward, ad, 2.0, None, lora, backward=backward,
                             epilogue=epi, aux=aux_f)
    plain = _grouped._launch(x, w_bf16, scale, offsets, not backward, ad, 2.0, None, lora, backward=backward,
                             epilogue=epi, aux=aux_r)
    torch.cuda.synchronize()
    assert torch.equal(bits(fused[0]), bits(plain[0]))
    if lora:
        assert torch.equal(bits(fused[1]), bits(plain[1]))
    if epi == _lib.EPI_SWIGLU:
        assert torch.equal(bits(aux_f), bits(aux_r))


@pytest.mark.parametrize("kind", KINDS)
def test_fused_products_at_a_qwen3_shape_match_float32(kind):
    """gate/up forward at config 2's width (K = 2048, N = 1536) with SwiGLU and adapters, checked against the
    float32 product over the dequantised stack (the oracle), on 8 experts of ragged rows."""
    gen = torch.Generator().manual_seed(3)
    rows_per_expert = [300, 1, 0, 128, 257, 64, 500, 2]
    experts, rows = len(rows_per_expert), sum(rows_per_expert)
    offsets = offsets_of(rows_per_expert)
    qs, w_bf16, scale = quantised(kind, (experts, 1536, 2048), gen)
    x = torch.randn(rows, 2048, generator=gen).to(DEV, torch.bfloat16)
    gu = torch.empty(rows, 1536, device=DEV, dtype=torch.bfloat16)
    h, _ = _grouped._launch(x, qs, scale, offsets, True, None, 1.0, None, False, epilogue=_lib.EPI_SWIGLU, aux=gu)
    want = ogrouped.lora_forward(as_np(x), as_np(w_bf16), as_np(scale) if scale is not None else None,
                                 as_np(offsets), False)
    assert_close(gu, want, "pre-activation")


def test_stacks_without_whole_64_blocks_are_dequantised_for_the_call():
    w = torch.randn(3, 80, 96, device=DEV) * 0.05
    codes, scale = _fp8.quantize_stack(w)
    assert _grouped.QuantStack.from_fp8(codes, scale) is None
    codes_b, scale_b = _fp8.quantize_blocks(w, grid=(2, 2))  # 40 x 48 blocks
    assert _grouped.QuantStack.from_fp8(codes_b, scale_b) is None


@pytest.mark.parametrize("grid", [(7, 4), (1, 1), (4, 2)])
def test_block_grids_other_than_128_are_fused_bit_exactly(grid, monkeypatch):
    """Blocks of 64 x 64, one block per matrix, and 112 x 128 (448 rows over 4): the reference's ceil sizing."""
    monkeypatch.setenv("MEEP2B_PAIR", "0")
    gen = torch.Generator().manual_seed(sum(grid))
    offsets = offsets_of([100, 156])
    w = (torch.randn(2, 448, 256, generator=gen) * 0.05).to(DEV)
    codes, scale = _fp8.quantize_blocks(w, grid=grid)
    qs = _grouped.QuantStack.from_fp8(codes, scale)
    assert qs is not None and qs.grid == grid
    x = torch.randn(256, 256, generator=gen).to(DEV, torch.bfloat16)
    fused, _ = _grouped._launch(x, qs, None, offsets, True, None, 1.0, None, False)
    plain, _ = _grouped._launch(x, _fp8.dequantize_blocks(codes, scale), None, offsets, True, None, 1.0, None, False)
    assert torch.equal(bits(fused), bits(plain))


def test_lora_linear_with_an_fp8_stack_takes_the_fused_path_and_matches_float32():
    gen = torch.Generator().manual_seed(5)
    rows_per_expert, K, N = [37, 0, 200, 64, 1], 256, 448
    offsets = offsets_of(rows_per_expert)
    x = torch.randn(sum(rows_per_expert), K, generator=gen).to(DEV, torch.bfloat16).requires_grad_()
    w8, scale = _fp8.quantize_stack((torch.randn(5, N, K, generator=gen) * 0.05).to(DEV))
    stack, _ = _grouped._dequantized(w8, scale)
    assert isinstance(stack, _grouped.QuantStack)
    lhs = (torch.randn(5, N, 16, generator=gen) * 0.1).to(DEV, torch.bfloat16).requires_grad_()
    rhs = (torch.randn(5, 16, K, generator=gen) * 0.1).to(DEV, torch.bfloat16).requires_grad_()
    out = mb.lora_linear(x, w8, scale, offsets, False, lhs, rhs, 2.0)
    grad = torch.randn(out.shape, generator=gen).to(DEV, torch.bfloat16)
    out.backward(grad)
    from oracle import quant

    w_exact = quant.e4m3_to_f32(w8.view(torch.uint8).cpu().numpy())
    args = [as_np(t) for t in (x.detach(), scale, offsets, lhs.detach(), rhs.detach(), grad)]
    xs, sc, offs, l, r, g = args
    want = ogrouped.lora_forward(xs, w_exact, sc, offs, False, l, r, 2.0, None)
    gx, gl, gr = ogrouped.lora_backward(xs, g, w_exact, sc, offs, False, l, r, 2.0)
    assert_close(out.detach(), want, "out")
    assert_close(x.grad, gx, "grad_x")
    assert_close(lhs.grad, gl, "grad_lhs", scaled=True)
    assert_close(rhs.grad, gr, "grad_rhs", scaled=True)


def test_the_multipliers_follow_the_reference_block_sizing():
    """meep2b_quant_multipliers: NF4 absmax transposed to (experts, cols/64, rows); block scales expanded per
    64-column group with blocks of ceil(rows/sr) x ceil(cols/sc), rounded to bf16 as dequantize_fp8 rounds them."""
    gen = torch.Generator().manual_seed(9)
    w = (torch.randn(3, 448, 256, generator=gen) * 0.05).to(DEV)
    st = _nf4.quantize(w)
    mult = st.multipliers()
    want = st.absmax_f32().view(3, 448, 4).transpose(1, 2)
    assert torch.equal(mult, want)
    codes, scale = _fp8.quantize_blocks(w, grid=(4, 2))  # 112 x 128 blocks
    qs = _grouped.QuantStack.from_fp8(codes, scale)
    rows = torch.arange(448, device=DEV) // 112
    groups = (torch.arange(4, device=DEV) * 64) // 128
    expect = scale[:, rows][:, :, groups].transpose(1, 2).to(torch.bfloat16).float()
    assert torch.equal(qs.mult, expect)
