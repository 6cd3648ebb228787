"""The grouped product (tcgen05 GEMM) and its gradients on the GPU, against float32 computations and the reference's
golden vectors; the reference tests' cases (tests/test_grouped.py:34-157) plus the BASELINE shapes."""

import numpy as np
import pytest
import torch

import meepsquared_b200 as mb
from oracle import grouped as ogrouped
from oracle import quant
from parity import as_np, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def offsets_of(rows_per_expert, device=DEV):
    return torch.cumsum(torch.tensor(rows_per_expert, dtype=torch.int32, device=device), 0, dtype=torch.int32)


@pytest.mark.parametrize("is_transposed", [False, True])
@pytest.mark.parametrize("rows_per_expert,K,N", [
    ([37, 0, 200, 64, 1], 96, 80),
    ([300] * 8, 256, 128),
    ([3], 2048, 1024),
    ([129, 0, 0, 500, 127], 2048, 1536),
])
def test_the_kernel_matches_one_product_per_expert(is_transposed, rows_per_expert, K, N, pair_mode):
    torch.manual_seed(0)
    rows, experts = sum(rows_per_expert), len(rows_per_expert)
    x = torch.randn(rows, K, device=DEV, dtype=torch.bfloat16)
    shape = (experts, K, N) if is_transposed else (experts, N, K)
    weight = torch.randn(shape, device=DEV, dtype=torch.bfloat16) * 0.05
    offsets = offsets_of(rows_per_expert)
    out = mb.grouped_linear(x, weight, offsets, is_transposed)
    want = ogrouped.lora_forward(as_np(x), as_np(weight), None, as_np(offsets), is_transposed)
    assert_close(out, want, "out")


def test_a_stack_stored_the_other_way_is_read_in_place():
    torch.manual_seed(1)
    x = torch.randn(300, 128, device=DEV, dtype=torch.bfloat16)
    w = (torch.randn(3, 128, 96, device=DEV, dtype=torch.bfloat16) * 0.05).transpose(1, 2)  # (E, out, in) view
    offsets = offsets_of([100, 50, 150])
    assert_close(mb.grouped_linear(x, w, offsets, False),
                 ogrouped.lora_forward(as_np(x), as_np(w), None, as_np(offsets), False), "out")


def test_a_mismatched_stack_is_refused():
    x = torch.randn(8, 64, device=DEV, dtype=torch.bfloat16)
    weight = torch.randn(2, 16, 32, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="in=32"):
        mb.grouped_linear(x, weight, offsets_of([4, 4]), is_transposed=False)


def adapters(experts, K, N, rank, is_transposed, gen):
    if is_transposed:
        lhs = torch.randn(experts, K, rank, generator=gen) * 0.1
        rhs = torch.randn(experts, rank, N, generator=gen) * 0.1
    else:
        lhs = torch.randn(experts, N, rank, generator=gen) * 0.1
        rhs = torch.randn(experts, rank, K, generator=gen) * 0.1
    return lhs.to(torch.bfloat16), rhs.to(torch.bfloat16)


def run_lora(x, weight, scale, offsets, is_transposed, lhs, rhs, scaling, bias, grad):
    x = x.to(DEV).requires_grad_()
    lhs = lhs.to(DEV).requires_grad_()
    rhs = rhs.to(DEV).requires_grad_()
    out = mb.lora_linear(x, weight.to(DEV), scale.to(DEV) if scale is not None else None, offsets.to(DEV),
                         is_transposed, lhs, rhs, scaling, bias.to(DEV) if bias is not None else None)
    out.backward(grad.to(DEV))
    return out.detach(), x.grad, lhs.grad, rhs.grad


def check_lora(got, x, weight, scale, offsets, is_transposed, lhs, rhs, scaling, bias, grad):
    args = [as_np(t) if t is not None else None for t in (x, weight, scale, offsets, lhs, rhs, bias, grad)]
    x, weight, scale, offsets, lhs, rhs, bias, grad = args
    out = ogrouped.lora_forward(x, weight, scale, offsets, is_transposed, lhs, rhs, scaling, bias)
    gx, gl, gr = ogrouped.lora_backward(x, grad, weight, scale, offsets, is_transposed, lhs, rhs, scaling)
    rows = int(offsets[-1])
    # ranks above 16: each chunk past the first adds its bf16 update to the bf16 output (two more roundings), so the
    # allowance follows the tensor's size there, as the reference's own tests allow for its kernel
    chunked = lhs is not None and lhs.shape[2] > 16
    assert_close(got[0][:rows], out[:rows], "out", scaled=chunked)
    assert_close(got[1][:rows], gx[:rows], "grad_x", scaled=chunked)
    assert_close(got[2], gl, "grad_lhs", scaled=True)
    assert_close(got[3], gr, "grad_rhs", scaled=True)


@pytest.mark.parametrize("prefix,is_transposed", [("n_", False), ("t_", True)])
def test_lora_matches_the_reference_golden_vectors(golden, prefix, is_transposed, pair_mode):
    g = golden("grouped")
    f = {k[len(prefix):]: v for k, v in g.items() if k.startswith(prefix)}
    t = {n: torch.from_numpy(quant.bf16_to_f32(f[n])).to(torch.bfloat16) for n in ("x", "weight", "lhs", "rhs", "bias", "grad")}
    offsets = torch.from_numpy(f["offsets"])
    scale = torch.from_numpy(f["scale"])
    got = run_lora(t["x"], t["weight"], scale, offsets, is_transposed, t["lhs"], t["rhs"], 2.0, t["bias"], t["grad"])
    assert_close(got[0], f["out"], "out")
    assert_close(got[1], f["grad_x"], "grad_x")
    assert_close(got[2], f["grad_lhs"], "grad_lhs", scaled=True)
    assert_close(got[3], f["grad_rhs"], "grad_rhs", scaled=True)


@pytest.mark.parametrize("is_transposed", [False, True])
@pytest.mark.parametrize("rank", [4, 8, 16, 20, 32, 64])  # above 16: the fused chunk plus 16-rank chunks
@pytest.mark.parametrize("rows_per_expert,K,N", [([37, 0, 200, 64, 1], 96, 80), ([1000, 3, 0, 700], 2048, 1536),
                                                  ([513, 256], 768, 2048)])
def test_lora_forward_and_backward_match_float32(is_transposed, rank, rows_per_expert, K, N, pair_mode):
    gen = torch.Generator().manual_seed(rank + K)
    experts = len(rows_per_expert)
    offsets = torch.cumsum(torch.tensor(rows_per_expert, dtype=torch.int32), 0, dtype=torch.int32)
    x = torch.randn(sum(rows_per_expert), K, generator=gen).to(torch.bfloat16)
    shape = (experts, K, N) if is_transposed else (experts, N, K)
    weight = (torch.randn(shape, generator=gen) * 0.05).to(torch.bfloat16)
    lhs, rhs = adapters(experts, K, N, rank, is_transposed, gen)
    bias = torch.randn(experts, N, generator=gen).to(torch.bfloat16)
    grad = torch.randn(sum(rows_per_expert), N, generator=gen).to(torch.bfloat16)
    got = run_lora(x, weight, None, offsets, is_transposed, lhs, rhs, 2.0, bias, grad)
    check_lora(got, x, weight, None, offsets, is_transposed, lhs, rhs, 2.0, bias, grad)


def test_lora_with_an_fp8_stack_matches_the_dequantized_stack():
    gen = torch.Generator().manual_seed(7)
    rows_per_expert, K, N = [37, 0, 200, 64, 1], 96, 80
    offsets = torch.cumsum(torch.tensor(rows_per_expert, dtype=torch.int32), 0, dtype=torch.int32)
    x = torch.randn(sum(rows_per_expert), K, generator=gen).to(torch.bfloat16)
    weight = torch.randn(5, N, K, generator=gen) * 0.05
    w8, scale = mb._fp8.quantize_stack(weight.to(DEV))
    lhs, rhs = adapters(5, K, N, 16, False, gen)
    grad = torch.randn(sum(rows_per_expert), N, generator=gen).to(torch.bfloat16)
    got = run_lora(x, w8, scale, offsets, False, lhs, rhs, 2.0, None, grad)
    w_deq = quant.e4m3_to_f32(w8.view(torch.uint8).cpu().numpy())  # the exact e4m3 values; scale applied per expert
    check_lora(got, x, torch.from_numpy(w_deq), scale.cpu(), offsets, False, lhs, rhs, 2.0, None, grad)


def test_the_product_without_adapters_gives_the_base_and_its_input_gradient():
    torch.manual_seed(0)
    offsets = offsets_of([10, 30])
    x = torch.randn(40, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    weight = torch.randn(2, 48, 64, device=DEV, dtype=torch.bfloat16) * 0.05
    out = mb.lora_linear(x, weight, None, offsets, False)
    out.sum().backward()
    assert_close(out, ogrouped.lora_forward(as_np(x), as_np(weight), None, as_np(offsets), False), "out")
    want = np.repeat(as_np(weight).sum(axis=1), [10, 30], axis=0)
    assert_close(x.grad, want, "grad_x")


def test_qwen3_shaped_products_sampled_rows(pair_mode):
    """Full BASELINE config-2 product sizes (131072 routed rows, 128 experts): sampled rows against float32."""
    gen = torch.Generator(device=DEV).manual_seed(11)
    experts, rows, H, I = 128, 131072, 2048, 768
    counts = torch.full((experts,), rows // experts, dtype=torch.int32)
    counts[::3] += 37
    counts[1::3] -= 37
    offsets = torch.cumsum(counts, 0, dtype=torch.int32).to(DEV)
    x = torch.randn(rows, H, device=DEV, generator=gen).to(torch.bfloat16)
    w = (torch.randn(experts, 2 * I, H, device=DEV, generator=gen) * 0.02).to(torch.bfloat16)
    out = mb.grouped_linear(x, w, offsets, False)
    ends = offsets.cpu().numpy()
    sample = torch.randint(0, rows, (512,), generator=torch.Generator().manual_seed(0))
    e = np.searchsorted(ends, sample.numpy(), side="right")
    want = torch.einsum("rk,rnk->rn", x[sample.to(DEV)].float(), w[torch.from_numpy(e).to(DEV)].float())
    assert_close(out[sample.to(DEV)], want, "sampled rows")
