"""The reference's own grouped-product test cases (meepsquared tests/test_grouped.py:34-173), run against this
package's `_grouped` module as a caller that swapped modules would run them: the same operator calls, the same
comparison functions (`reference`, `reference_lora`, exposed by this module too) and the same tolerances. The
cases are restated here, not imported: the reference repository does not travel to the GPU box. The `tile_map`
known answers of that file are checked in tests/test_oracle.py (the oracle) and tests/test_gpu_routing.py (the
GPU kernel; here tile_map runs on the GPU).
"""

import pytest
import torch

from meepsquared_b200 import _fp8
from meepsquared_b200 import _grouped as grouped

pytestmark = pytest.mark.gpu
DEV = "cuda"


def ends(counts):
    """Inclusive end of each expert's rows (int32 on the GPU), the offsets convention of the operator."""
    return torch.tensor(counts, dtype=torch.int32, device=DEV).cumsum(0, dtype=torch.int32)


def stack(experts, k, n, transposed, scale=0.05):
    shape = (experts, k, n) if transposed else (experts, n, k)
    return torch.randn(shape, device=DEV, dtype=torch.bfloat16) * scale


CASES = [([37, 0, 200, 64, 1], 96, 80), ([300] * 8, 256, 128), ([3], 2048, 1024)]


@pytest.mark.parametrize("transposed", [False, True], ids=["out-in", "in-out"])
@pytest.mark.parametrize("counts,k,n", CASES, ids=["ragged", "even", "one-expert"])
def test_grouped_linear_against_the_per_expert_loop(transposed, counts, k, n):
    torch.manual_seed(0)
    x = torch.randn(sum(counts), k, device=DEV, dtype=torch.bfloat16)
    w = stack(len(counts), k, n, transposed)
    got = grouped.grouped_linear(x, w, ends(counts), transposed)
    want = grouped.reference(x, w, ends(counts), transposed)
    torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("transposed", [False, True], ids=["out-in", "in-out"])
def test_an_fp8_stack_is_converted_to_bf16_weights(transposed):
    torch.manual_seed(0)
    x = torch.randn(70, 64, device=DEV, dtype=torch.bfloat16)
    w8 = (stack(3, 64, 48, transposed).float()).to(torch.float8_e4m3fn)
    got = grouped.grouped_linear(x, w8, ends([10, 40, 20]), transposed, products_fp8=False)
    want = grouped.reference(x, w8, ends([10, 40, 20]), transposed)
    torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("transposed", [False, True], ids=["out-in", "in-out"])
def test_fp8_products_quantise_the_rows_and_stay_within_six_percent(transposed):
    torch.manual_seed(0)
    x = torch.randn(300, 128, device=DEV, dtype=torch.bfloat16)
    x[::7] *= 20  # rows of very different magnitudes: one scale per row
    w8 = stack(4, 128, 96, transposed).float().to(torch.float8_e4m3fn)
    offsets = ends([100, 0, 150, 50])
    want = grouped.reference(x, w8, offsets, transposed).float()
    got = grouped.grouped_linear(x, w8, offsets, transposed, products_fp8=True).float()
    assert (got - want).abs().max() <= 0.1 * want.abs().max()
    assert (got - want).norm() / want.norm() < 0.06


def test_a_stack_of_the_wrong_width_is_refused_with_the_references_message():
    x = torch.randn(8, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(2, 16, 32, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="in=32"):
        grouped.grouped_linear(x, w, ends([4, 4]), is_transposed=False)


def peft_factors(experts, k, n, rank, transposed):
    """lhs (E, out, r) and rhs (E, r, in) for a stack (E, out, in); (E, in, r) and (E, r, out) when transposed."""
    first, last = (k, n) if transposed else (n, k)
    lhs = (torch.randn(experts, first, rank, device=DEV, dtype=torch.bfloat16) * 0.1).requires_grad_()
    rhs = (torch.randn(experts, rank, last, device=DEV, dtype=torch.bfloat16) * 0.1).requires_grad_()
    return lhs, rhs


@pytest.mark.parametrize("transposed", [False, True], ids=["out-in", "in-out"])
@pytest.mark.parametrize("fp8", [None, "weights", "products"])
@pytest.mark.parametrize("rank", [4, 16])
def test_lora_linear_and_its_gradients_against_the_float32_loop(transposed, fp8, rank):
    torch.manual_seed(0)
    counts, k, n = [37, 0, 200, 64, 1], 96, 80
    experts, offsets = len(counts), ends(counts)
    x = torch.randn(sum(counts), k, device=DEV, dtype=torch.bfloat16).requires_grad_()
    w = stack(experts, k, n, transposed)
    scale = None
    if fp8:
        w, scale = _fp8.quantize_stack(w)
    lhs, rhs = peft_factors(experts, k, n, rank, transposed)
    bias = torch.randn(experts, n, device=DEV, dtype=torch.bfloat16)

    out = grouped.lora_linear(x, w, scale, offsets, transposed, lhs, rhs, 2.0, bias, products_fp8=fp8 == "products")
    upstream = torch.randn_like(out)
    out.backward(upstream)
    ours = {"out": out.detach(), "x": x.grad, "lhs": lhs.grad, "rhs": rhs.grad}
    x.grad = lhs.grad = rhs.grad = None
    ref = grouped.reference_lora(x, w, scale, offsets, transposed, lhs, rhs, 2.0, bias)
    ref.backward(upstream)
    theirs = {"out": ref.detach(), "x": x.grad, "lhs": lhs.grad, "rhs": rhs.grad}
    for name in ours:
        a, b = ours[name].float(), theirs[name].float()
        assert a.shape == b.shape, name
        if fp8 == "products" and name in ("out", "x"):
            assert (a - b).norm() <= 0.06 * b.norm(), name  # e4m3 activations: ~4% of the norm
        else:
            torch.testing.assert_close(a, b, atol=1e-2 * b.abs().max().item(), rtol=0, msg=name)


def test_without_adapters_the_input_gradient_is_the_stack_summed_over_outputs():
    torch.manual_seed(0)
    offsets = ends([10, 30])
    x = torch.randn(40, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(2, 48, 64, device=DEV, dtype=torch.bfloat16) * 0.05
    out = grouped.lora_linear(x, w, None, offsets, False)
    out.sum().backward()
    torch.testing.assert_close(out.float(), grouped.reference(x.detach(), w, offsets, False).float(),
                               atol=2e-2, rtol=2e-2)
    expert_of_row = torch.repeat_interleave(torch.arange(2, device=DEV), torch.tensor([10, 30], device=DEV))
    torch.testing.assert_close(x.grad.float(), w.sum(dim=1)[expert_of_row].float(), atol=5e-2, rtol=3e-2)


def test_the_fp8_product_switch_and_the_kernel_override(monkeypatch):
    monkeypatch.delenv("MEEPSQUARED_FP8_PRODUCTS", raising=False)
    assert grouped.fp8_products(torch.device(DEV, 0)) is False
    monkeypatch.setenv("MEEPSQUARED_FP8_PRODUCTS", "1")
    assert grouped.fp8_products(torch.device(DEV, 0)) is True
    monkeypatch.setenv("MEEPSQUARED_GROUPED_KERNEL", "0")
    assert grouped.wanted(torch.device(DEV, 0)) is False
    monkeypatch.setenv("MEEPSQUARED_GROUPED_KERNEL", "1")
    assert grouped.wanted(torch.device("cpu")) is True
    monkeypatch.delenv("MEEPSQUARED_GROUPED_KERNEL")
    assert grouped.wanted(torch.device("cpu")) is False
