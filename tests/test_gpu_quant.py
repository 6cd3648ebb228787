"""Quantised stacks on the GPU: FP8 per expert and 128x128 block FP8 bit-exact with the reference's golden
vectors, NF4 double dequantisation bit-exact with the oracle."""

import numpy as np
import pytest
import torch

import meepsquared_b200 as mb
from meepsquared_b200 import _fp8, _nf4
from oracle import quant

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("name", ["test", "big"])
def test_fp8_stack_is_bit_exact_with_the_reference(golden, name):
    g = golden("fp8_stack")
    w = torch.from_numpy(g[f"{name}_weight"].view(np.int16)).view(torch.bfloat16).to(DEV)
    codes, scale = _fp8.quantize_stack(w)
    np.testing.assert_array_equal(scale.cpu().numpy(), g[f"{name}_scale"])
    np.testing.assert_array_equal(codes.view(torch.uint8).cpu().numpy(), g[f"{name}_codes"])
    np.testing.assert_array_equal(bits(_fp8.dequantize_stack(codes, scale, torch.bfloat16)), g[f"{name}_dequant"])


@pytest.mark.parametrize("name", ["even", "tail"])
def test_fp8_blocks_are_bit_exact_with_the_reference(golden, name):
    g = golden("fp8_block")
    w = torch.from_numpy(g[f"{name}_weight"].view(np.int16)).view(torch.bfloat16).to(DEV)
    codes, scale = _fp8.quantize_blocks(w, g[f"{name}_scale"].shape)
    np.testing.assert_array_equal(scale.cpu().numpy(), g[f"{name}_scale"])
    np.testing.assert_array_equal(codes.view(torch.uint8).cpu().numpy(), g[f"{name}_codes"])
    c = torch.from_numpy(g[f"{name}_codes"]).to(DEV).view(torch.float8_e4m3fn)
    np.testing.assert_array_equal(bits(_fp8.dequantize_blocks(c, torch.from_numpy(g[f"{name}_scale"]).to(DEV))),
                                  g[f"{name}_dequant"])


def test_fp8_blocks_of_a_config5_stack_match_the_oracle():
    """A stack of BASELINE config 5's down projection (a few experts of (4096, 1536), 128x128 blocks)."""
    gen = torch.Generator().manual_seed(5)
    w = (torch.randn(3, 4096, 1536, generator=gen) * 0.02).to(torch.bfloat16)
    codes, scale = _fp8.quantize_blocks(w.to(DEV))
    deq = bits(_fp8.dequantize_blocks(codes, scale))
    for e in range(3):
        c_ref, s_ref = quant.quantize_fp8_blocks(w[e].float().numpy())
        np.testing.assert_array_equal(scale[e].cpu().numpy(), s_ref)
        np.testing.assert_array_equal(codes[e].view(torch.uint8).cpu().numpy(), c_ref)
        np.testing.assert_array_equal(deq[e], quant.dequantize_fp8_blocks(c_ref, s_ref))


@pytest.mark.parametrize("shape", [(4, 96, 128), (2, 1536, 2048), (3, 64 * 5)])
def test_nf4_dequantisation_is_bit_exact_with_the_oracle(shape):
    rng = np.random.default_rng(sum(shape))
    w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    if int(np.prod(shape)) % 64:
        pytest.skip("whole blocks only")
    st = quant.quantize_nf4(w)
    state = _nf4.NF4State(torch.from_numpy(st["packed"]), torch.from_numpy(st["absmax"]),
                          torch.from_numpy(st["absmax2"]), torch.from_numpy(st["code2"]),
                          torch.tensor([st["offset"]], dtype=torch.float32), tuple(shape)).to(DEV)
    np.testing.assert_array_equal(bits(_nf4.dequantize(state)), quant.dequantize_nf4(st))


def _state_np(state):
    return {"packed": state.packed.cpu().numpy(), "absmax": state.absmax.cpu().numpy(),
            "absmax2": state.absmax2.cpu().numpy(), "code2": state.code2.cpu().numpy(),
            "offset": np.float32(state.offset.item()), "blocksize": state.blocksize,
            "blocksize2": state.blocksize2, "shape": state.shape}


@pytest.mark.parametrize("shape", [(4, 96, 128), (2, 1536, 2048)])
def test_nf4_quantisation_on_the_gpu_matches_the_oracle(shape):
    """The load-time quantiser: the same codes and absmax state as the oracle's bitsandbytes restatement, and its
    state dequantises bit-exactly as the oracle dequantises it."""
    rng = np.random.default_rng(7 + sum(shape))
    w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    state = _nf4.quantize(torch.from_numpy(w).to(DEV))
    want = quant.quantize_nf4(w)
    np.testing.assert_array_equal(state.code2.cpu().numpy(), want["code2"])
    np.testing.assert_array_equal(state.packed.cpu().numpy(), want["packed"])
    np.testing.assert_allclose(state.offset.item(), want["offset"], rtol=1e-6)
    # the offset is a mean (its last bit depends on the summation order); the codes of the centred absmax agree
    # wherever no value sits on a rounding boundary
    assert (state.absmax.cpu().numpy() == want["absmax"]).mean() > 0.999
    np.testing.assert_array_equal(bits(_nf4.dequantize(state)), quant.dequantize_nf4(_state_np(state)))


def test_fp8_dequantize_takes_either_form_of_scale():
    w = torch.randn(3, 256, 384, device=DEV) * 0.05
    c1, s1 = _fp8.quantize_stack(w)
    c2, s2 = _fp8.quantize_blocks(w)
    assert s2.shape == (3, 2, 3)
    assert torch.equal(_fp8.dequantize(c1, s1), _fp8.dequantize_stack(c1, s1, torch.bfloat16))
    assert torch.equal(_fp8.dequantize(c2, s2), _fp8.dequantize_blocks(c2, s2))
    with pytest.raises(ValueError):
        _fp8.dequantize(c2, s2[0])


@pytest.mark.parametrize("block", [None, 128])
def test_the_fp8_grouped_product_matches_the_dequantized_stack(block):
    """_fp8.grouped_product (meepsquared/_fp8.py:137-164): x against an FP8 stack and x's gradient, against float32
    over the stack as the reference dequantises it."""
    from oracle import grouped as ogrouped
    from parity import as_np, assert_close

    gen = torch.Generator().manual_seed(12)
    rows_per_expert, K, N = [37, 0, 200, 64, 1], 256, 192
    offsets = torch.cumsum(torch.tensor(rows_per_expert, dtype=torch.int32), 0, dtype=torch.int32).to("cuda")
    w = (torch.randn(5, N, K, generator=gen) * 0.05).to("cuda")
    if block is None:
        w8, scale = _fp8.quantize_stack(w)
    else:
        w8, scale = _fp8.quantize_blocks(w, block=block)
    x = torch.randn(sum(rows_per_expert), K, generator=gen).to("cuda", torch.bfloat16).requires_grad_()
    out = _fp8.grouped_product(x, w8, scale, offsets, None, False)
    grad = torch.randn(out.shape, generator=gen).to("cuda", torch.bfloat16)
    out.backward(grad)
    w_deq = as_np(_fp8.dequantize(w8, scale))
    want = ogrouped.lora_forward(as_np(x.detach()), w_deq, None, as_np(offsets), False)
    gx, _, _ = ogrouped.lora_backward(as_np(x.detach()), as_np(grad), w_deq, None, as_np(offsets), False, None, None,
                                      1.0)
    assert_close(out.detach(), want, "out", scaled=True)
    assert_close(x.grad, gx, "grad_x", scaled=True)


def test_a_backward_pass_on_a_thread_new_to_cuda_runs(tmp_path):
    """The first library call of autograd's backward thread can be a tensor-map encoding (an FP8 stack's product
    without adapters): the library makes the device's context current on that thread first. Run in a fresh process,
    where nothing else has touched CUDA on that thread."""
    import subprocess
    import sys

    script = tmp_path / "backward_thread.py"
    script.write_text(
        "import sys, torch\n"
        f"sys.path.insert(0, {repr(str(__import__('pathlib').Path(__file__).resolve().parents[1]))})\n"
        "import meepsquared_b200 as mb\n"
        "from meepsquared_b200 import _fp8\n"
        "g = torch.Generator().manual_seed(0)\n"
        "offsets = torch.tensor([37, 37, 237, 301, 302], dtype=torch.int32, device='cuda')\n"
        "w8, scale = _fp8.quantize_stack((torch.randn(5, 192, 256, generator=g) * 0.05).cuda())\n"
        "x = torch.randn(302, 256, generator=g).to('cuda', torch.bfloat16).requires_grad_()\n"
        "out = mb.lora_linear(x, w8, scale, offsets, False)\n"
        "out.backward(torch.randn(out.shape, generator=g).to('cuda', torch.bfloat16))\n"
        "torch.cuda.synchronize()\n"
        "assert torch.isfinite(x.grad.float()).all()\n"
        "print('ok')\n")
    run = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, timeout=600)
    assert run.returncode == 0 and run.stdout.strip().endswith("ok"), run.stderr[-2000:]
