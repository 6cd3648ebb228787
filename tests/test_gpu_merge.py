"""The merged save of an expert stack on the GPU (meep2b_merge_stack through _save.merged_stack) against the
reference's _save._merged_stack (_save.py:79-95: golden vectors) and the float32 oracle."""

import types

import numpy as np
import pytest
import torch

from meepsquared_b200 import _fp8, _save
from oracle import merge, quant

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16_tensor(bits):
    return torch.from_numpy(np.asarray(bits).astype(np.int16)).view(torch.bfloat16).to(DEV)


@pytest.mark.parametrize("prefix", ["n_", "t_"])
def test_merged_stacks_match_the_reference_merged_save(golden, prefix):
    g = golden("merged")
    p = prefix
    lhs = torch.from_numpy(g[p + "lhs"]).to(DEV)
    rhs = torch.from_numpy(g[p + "rhs"]).to(DEV)
    factors = (lhs, rhs, float(g[p + "scaling"]))
    experts = types.SimpleNamespace(stack=bf16_tensor(g[p + "stack"]))
    got32 = _save.merged_stack(experts, "stack", factors, torch.float32).cpu().numpy()
    np.testing.assert_allclose(got32, g[p + "merged_f32"], rtol=1e-6, atol=1e-7)
    got16 = _save.merged_stack(experts, "stack", factors, torch.bfloat16).cpu().view(torch.int16).numpy()
    got16 = got16.view(np.uint16)
    assert np.mean(got16 != g[p + "merged_bf16"]) < 1e-3  # a float32 sum order differing at a rounding boundary
    np.testing.assert_allclose(quant.bf16_to_f32(got16), quant.bf16_to_f32(g[p + "merged_bf16"]), rtol=2 ** -7)
    codes = torch.from_numpy(g[p + "codes"]).to(DEV).view(torch.float8_e4m3fn)
    experts8 = types.SimpleNamespace(stack=codes)
    setattr(experts8, "stack" + _fp8.STACK_SCALE, torch.from_numpy(g[p + "scale"]).to(DEV))
    alone = _save.merged_stack(experts8, "stack", None, torch.float32).cpu().numpy()
    np.testing.assert_array_equal(alone, g[p + "fp8_alone_f32"])  # f32(code) * scale, one rounding: exact
    got8 = _save.merged_stack(experts8, "stack", factors, torch.float32).cpu().numpy()
    np.testing.assert_allclose(got8, g[p + "fp8_merged_f32"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("rank", [1, 16, 128])
@pytest.mark.parametrize("shape", [(2, 768, 2048), (3, 37, 300)])
def test_merged_stacks_match_the_oracle_at_any_rank_and_ragged_sizes(rank, shape):
    gen = torch.Generator().manual_seed(rank + shape[1])
    E, rows, cols = shape
    w = (torch.randn(shape, generator=gen) * 0.02).to(torch.bfloat16)
    lhs = torch.randn(E, rows, rank, generator=gen) * 0.1
    rhs = torch.randn(E, rank, cols, generator=gen) * 0.1
    experts = types.SimpleNamespace(stack=w.to(DEV))
    got = _save.merged_stack(experts, "stack", (lhs.to(DEV), rhs.to(DEV), 2.0), torch.float32).cpu().numpy()
    want = merge.merged_stack(w.float().numpy(), lhs.numpy(), rhs.numpy(), 2.0)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)


def test_factors_that_do_not_make_the_stack_are_refused():
    experts = types.SimpleNamespace(stack=torch.zeros(2, 8, 16, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        _save.merged_stack(experts, "stack", (torch.zeros(2, 8, 4, device=DEV), torch.zeros(2, 4, 8, device=DEV), 1.0),
                           torch.bfloat16)
    with pytest.raises(TypeError):
        _save.merged_stack(experts, "stack", None, torch.float16)
