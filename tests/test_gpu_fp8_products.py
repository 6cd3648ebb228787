"""FP8 tensor-core products (products_fp8=True / MEEPSQUARED_FP8_PRODUCTS=1), the reference's X_FP8 path
(meepsquared/_grouped.py:141-146,194-197): the activations' codes and scales bit-exact with the oracle, the
products against the oracle's restatement of the same arithmetic, and against float32 within the reference's own
tolerance for the path (tests/test_grouped.py:66-79,137-140: 6% of the norm, 10% of the largest value)."""

import numpy as np
import pytest
import torch

import meepsquared_b200 as mb
from meepsquared_b200 import _fp8, _grouped
from oracle import grouped as ogrouped
from oracle import quant
from parity import as_np

pytestmark = pytest.mark.gpu
DEV = "cuda"


def offsets_of(sizes):
    return torch.cumsum(torch.tensor(sizes, dtype=torch.int32), 0, dtype=torch.int32).to(DEV)


def close_to_oracle(got, want, name, rel=1e-2):
    """The kernel's float32 sums differ from the oracle's in order only, and the output is rounded to bf16."""
    g, w = as_np(got).astype(np.float64), np.asarray(want, dtype=np.float64)
    assert g.shape == w.shape, name
    scale = max(1e-6, float(np.abs(w).max()))
    worst = float(np.abs(g - w).max())
    assert worst <= rel * scale, f"{name}: worst {worst:.4g} against {rel} * {scale:.4g}"


def within_reference_tolerance(got, want, name):
    g, w = as_np(got).astype(np.float64), as_np(want).astype(np.float64)
    assert np.abs(g - w).max() <= 0.1 * np.abs(w).max(), name
    assert np.linalg.norm(g - w) <= 0.06 * np.linalg.norm(w), name


@pytest.mark.parametrize("shape", [(300, 128), (77, 208), (513, 4096)])
def test_the_activations_are_quantized_bit_exact_with_the_oracle(shape):
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(shape, generator=gen)
    x[::7] *= 20  # rows of different sizes: the scale is per row
    x[5] = 0.0    # an all-zero row takes the 1e-12 floor
    xb = x.to(DEV, torch.bfloat16)
    codes, scales = _grouped._quantize_rows(xb)
    want_codes, want_scales = quant.quantize_rows(as_np(xb))
    np.testing.assert_array_equal(codes.cpu().numpy(), want_codes)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), want_scales.view(np.uint32))


def test_quantisation_on_rounding_midpoints_is_bit_exact():
    """Quotients on e4m3 rounding midpoints (ties to even) and next to them: the kernel's fast path (a multiply by
    the reciprocal, bracketed) hands these to the division, so the codes stay those of x / scale."""
    levels = quant.e4m3_to_f32(np.arange(0, 0x7E, dtype=np.uint8)).astype(np.float64)
    mids = (levels[1:] + levels[:-1]) / 2
    rows = []
    for scale_pow in (0, -3, 5):  # a row's largest value 448 * 2^p makes its scale 2^p: the quotients are exact
        row = np.zeros(128, dtype=np.float32)
        row[0] = 448.0 * 2.0 ** scale_pow
        picks = mids[np.linspace(0, len(mids) - 1, 127).astype(int)]
        row[1:] = (picks * 2.0 ** scale_pow * np.where(np.arange(127) % 2, -1, 1)).astype(np.float32)
        rows.append(row)
    rng = np.random.default_rng(0)
    for _ in range(61):  # odd scales: quotients near the midpoints after rounding
        row = (rng.choice(mids, 128) * rng.uniform(0.9, 1.1)).astype(np.float32)
        rows.append(row)
    x = torch.from_numpy(np.stack(rows)).to(DEV, torch.bfloat16)
    codes, scales = _grouped._quantize_rows(x)
    want_codes, want_scales = quant.quantize_rows(as_np(x))
    np.testing.assert_array_equal(codes.cpu().numpy(), want_codes)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), want_scales.view(np.uint32))


@pytest.mark.parametrize("is_transposed", [False, True])
def test_the_fp8_product_quantizes_the_activations_per_row_and_stays_close(is_transposed):
    """The reference's test_grouped.py:66-79 on the same shapes, and the oracle's arithmetic."""
    torch.manual_seed(0)
    x = torch.randn(300, 128, device=DEV, dtype=torch.bfloat16)
    x[::7] *= 20
    shape = (4, 128, 96) if is_transposed else (4, 96, 128)
    weight = (torch.randn(shape, device=DEV) * 0.05).to(torch.float8_e4m3fn)
    offsets = offsets_of([100, 0, 150, 50])
    expected = mb.reference(x, weight, offsets, is_transposed).float()
    out = mb.grouped_linear(x, weight, offsets, is_transposed, products_fp8=True).float()
    within_reference_tolerance(out, expected, "out")
    codes = weight.view(torch.uint8).cpu().numpy()
    want = ogrouped.fp8_product(as_np(x), codes, None, as_np(offsets), is_transposed)
    close_to_oracle(out, want, "out")


def adapters(experts, K, N, rank, is_transposed, gen):
    if is_transposed:
        lhs = torch.randn(experts, K, rank, generator=gen) * 0.1
        rhs = torch.randn(experts, rank, N, generator=gen) * 0.1
    else:
        lhs = torch.randn(experts, N, rank, generator=gen) * 0.1
        rhs = torch.randn(experts, rank, K, generator=gen) * 0.1
    return (lhs.to(DEV, torch.bfloat16).requires_grad_(), rhs.to(DEV, torch.bfloat16).requires_grad_())


@pytest.mark.parametrize("rank", [4, 16, 32])
@pytest.mark.parametrize("is_transposed", [False, True])
def test_the_fp8_product_with_adapters_and_its_gradients(is_transposed, rank):
    """The reference's test_grouped.py:103-143 with fp8="products": out and grad_x within 6% of float32, the
    adapters' gradients as tight as the bf16 path's; and out / grad_x against the oracle's FP8 arithmetic."""
    gen = torch.Generator().manual_seed(rank + 7 * is_transposed)
    sizes, K, N, E = [70, 0, 300, 130], 256, 384, 4
    offsets = offsets_of(sizes)
    shape = (E, K, N) if is_transposed else (E, N, K)
    w = (torch.randn(shape, generator=gen) * 0.05).to(DEV)
    weight, scale = _fp8.quantize_stack(w)
    lhs, rhs = adapters(E, K, N, rank, is_transposed, gen)
    bias = (torch.randn(E, N, generator=gen) * 0.1).to(DEV, torch.bfloat16)
    x = torch.randn(sum(sizes), K, generator=gen).to(DEV, torch.bfloat16).requires_grad_()
    scaling = 2.0
    out = mb.lora_linear(x, weight, scale, offsets, is_transposed, lhs, rhs, scaling, bias, products_fp8=True)
    grad = torch.randn(out.shape, generator=gen).to(DEV, torch.bfloat16)
    out.backward(grad)
    got = (out.detach(), x.grad.clone(), lhs.grad.clone(), rhs.grad.clone())
    x.grad = lhs.grad = rhs.grad = None

    expected_out = mb.reference_lora(x, weight, scale, offsets, is_transposed, lhs, rhs, scaling, bias)
    expected_out.backward(grad)
    expected = (expected_out.detach(), x.grad, lhs.grad, rhs.grad)
    for name, a, b in zip(("out", "grad_x", "grad_lhs", "grad_rhs"), got, expected):
        assert a.shape == b.shape, name
        if name in ("out", "grad_x"):
            assert (a.float() - b.float()).norm() <= 0.06 * b.float().norm(), name
            continue
        torch.testing.assert_close(a.float(), b.float(), atol=1e-2 * b.float().abs().max().item(), rtol=0, msg=name)

    codes = weight.view(torch.uint8).cpu().numpy()
    args = (codes, as_np(scale), as_np(offsets))
    l, r = as_np(lhs.detach()), as_np(rhs.detach())
    want = ogrouped.fp8_product(as_np(x.detach()), *args, is_transposed, l, r, scaling, as_np(bias))
    close_to_oracle(got[0], want, "out")
    want_gx = ogrouped.fp8_product(as_np(grad), *args, not is_transposed, l, r, scaling)
    close_to_oracle(got[1], want_gx, "grad_x")


@pytest.mark.parametrize("is_transposed", [False, True])
def test_a_block_scaled_stack_feeds_the_fp8_tensor_cores(is_transposed):
    """A stack with 128 x 128 block scales (the fp8 method of the north star): each k-block's partial sum takes the
    row's scale times the block's scale (rounded to bf16, as the reference's dequantisation applies it)."""
    gen = torch.Generator().manual_seed(21 + is_transposed)
    sizes, K, N, E = [200, 45, 0, 260], 384, 256, 4
    offsets = offsets_of(sizes)
    shape = (E, K, N) if is_transposed else (E, N, K)
    w = (torch.randn(shape, generator=gen) * 0.05).to(DEV)
    w[:, :128] *= 8  # blocks of different sizes
    weight, scale = _fp8.quantize_blocks(w, block=128)
    x = torch.randn(sum(sizes), K, generator=gen).to(DEV, torch.bfloat16)
    out = mb.lora_linear(x, weight, scale, offsets, is_transposed, products_fp8=True)
    deq = _fp8.dequantize(weight, scale)
    expected = mb.reference(x, deq, offsets, is_transposed).float()
    within_reference_tolerance(out, expected, "out")

    sb = quant.bf16(as_np(scale))
    if is_transposed:  # stored (E, K, N): the row blocks run along k
        block_scale = lambda e, b, c: sb[e, b, c]  # noqa: E731
    else:              # stored (E, N, K): the row blocks run along n
        block_scale = lambda e, b, c: sb[e, c, b]  # noqa: E731
    codes = weight.view(torch.uint8).cpu().numpy()
    want = ogrouped.fp8_product(as_np(x), codes, None, as_np(offsets), is_transposed, block_scale=block_scale)
    close_to_oracle(out, want, "out")


def test_fp8_products_follow_the_switch(monkeypatch):
    """MEEPSQUARED_FP8_PRODUCTS=1 turns the FP8 products on when products_fp8 is None (_grouped.py:70-80,316-320)."""
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(64, 128, generator=gen).to(DEV, torch.bfloat16)
    x[3] *= 50
    weight = (torch.randn(2, 128, 128, generator=gen) * 0.05).to(DEV).to(torch.float8_e4m3fn)
    offsets = offsets_of([30, 34])
    monkeypatch.setenv("MEEPSQUARED_FP8_PRODUCTS", "1")
    on = mb.grouped_linear(x, weight, offsets, False)
    monkeypatch.delenv("MEEPSQUARED_FP8_PRODUCTS")
    off = mb.grouped_linear(x, weight, offsets, False)
    want = ogrouped.fp8_product(as_np(x), weight.view(torch.uint8).cpu().numpy(), None, as_np(offsets), False)
    close_to_oracle(on, want, "on")
    exact = mb.reference(x, weight, offsets, False)
    torch.testing.assert_close(off.float(), exact.float(), atol=2e-2, rtol=2e-2)
    assert not torch.equal(on, off)


def test_an_empty_batch_and_sizes_the_kernel_does_not_take():
    weight = torch.zeros(2, 96, 128, device=DEV).to(torch.float8_e4m3fn)
    x = torch.zeros(0, 128, device=DEV, dtype=torch.bfloat16)
    out = mb.grouped_linear(x, weight, offsets_of([0, 0]), False, products_fp8=True)
    assert out.shape == (0, 96)
    odd = torch.zeros(2, 96, 120, device=DEV).to(torch.float8_e4m3fn)
    with pytest.raises(NotImplementedError):
        mb.grouped_linear(torch.zeros(4, 120, device=DEV, dtype=torch.bfloat16), odd, offsets_of([2, 2]), False,
                          products_fp8=True)
