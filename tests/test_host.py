"""Host-side logic of the package that needs no GPU: the NF4 code book tables and the fused-product eligibility of
quantised stacks."""

import numpy as np
import torch

from meepsquared_b200 import _grouped, _lib, _nf4
from oracle import quant


def test_the_second_level_code_is_the_oracles_dynamic_map():
    np.testing.assert_array_equal(_nf4.dynamic_map(), quant.dynamic_map())


def test_the_nf4_levels_are_the_oracles():
    np.testing.assert_array_equal(np.array(_nf4.NF4_LEVELS, dtype=np.float32), quant.NF4_LEVELS)


def test_quantised_stacks_are_fused_only_with_whole_64_blocks():
    ok = torch.zeros(2, 128, 256, dtype=torch.float8_e4m3fn)
    assert _grouped.QuantStack.from_fp8(ok, torch.ones(2)).kind == _lib.E4M3
    assert _grouped.QuantStack.from_fp8(ok, torch.ones(2, 1, 2)).kind == _lib.E4M3_BLOCKS
    assert _grouped.QuantStack.from_fp8(ok, torch.ones(2, 2, 4)).grid == (2, 4)  # 64 x 64 blocks
    assert _grouped.QuantStack.from_fp8(ok, torch.ones(2, 2, 8)) is None  # 32-column blocks
    assert _grouped.QuantStack.from_fp8(torch.zeros(2, 80, 256, dtype=torch.float8_e4m3fn), torch.ones(2)) is None


def test_the_tile_kernel_choice(monkeypatch):
    """bf16 stacks on one CTA (TMA-store epilogues, 4 stages); CTA pairs for quantised stacks only NF4 K-major (at
    any k); MEEP2B_PAIR overrides."""
    monkeypatch.delenv("MEEP2B_PAIR", raising=False)
    rows, experts = 131072, 128  # 1024 rows per expert
    assert not _grouped._pair_tiles(0, rows, experts, 2048, True)
    assert not _grouped._pair_tiles(0, rows, experts, 768, True)
    assert not _grouped._pair_tiles(1, rows, experts, 2048, True)
    assert not _grouped._pair_tiles(1, rows, experts, 2048, False)
    assert _grouped._pair_tiles(0, rows, experts, 768, True, _lib.NF4)
    assert not _grouped._pair_tiles(1, rows, experts, 2048, False, _lib.NF4)
    assert not _grouped._pair_tiles(0, rows, experts, 2048, True, _lib.E4M3_BLOCKS)
    assert not _grouped._pair_tiles(0, rows, experts, 2048, True, _lib.E4M3)
    monkeypatch.setenv("MEEP2B_PAIR", "1")
    assert _grouped._pair_tiles(0, 16384, experts, 768, True, _lib.E4M3)
    assert _grouped._pair_tiles(0, rows, experts, 2048, True)
    monkeypatch.setenv("MEEP2B_PAIR", "0")
    assert not _grouped._pair_tiles(0, rows, experts, 768, True, _lib.NF4)


def test_only_the_default_silu_gate_on_a_k_major_stack_is_fused():
    """The fused layer computes Transformers' default gate with SiLU (the epilogues' SwiGLU) on a gate/up stack
    stored (experts, 2I, hidden); another activation, gating function, an ungated module or a transposed stack takes
    the unfused layer."""
    from transformers.activations import ACT2FN
    from transformers.integrations.moe import _default_apply_gate

    from meepsquared_b200 import _moe

    class Experts(torch.nn.Module):
        _apply_gate = _default_apply_gate

        def __init__(self):
            super().__init__()
            self.num_experts, self.has_gate, self.has_bias, self.is_transposed = 2, True, False, False
            self.act_fn = ACT2FN["silu"]

    experts = Experts()
    assert _moe._default_swiglu(experts)
    experts.act_fn = torch.nn.SiLU()
    assert _moe._default_swiglu(experts)
    experts.act_fn = ACT2FN["gelu"]
    assert not _moe._default_swiglu(experts)
    experts.act_fn = ACT2FN["silu"]
    experts.is_transposed = True
    assert not _moe._default_swiglu(experts)
    experts.is_transposed, experts.has_gate = False, False
    assert not _moe._default_swiglu(experts)

    class Custom(Experts):
        def _apply_gate(self, gate_up_out):
            gate, up = gate_up_out.chunk(2, dim=-1)
            return self.act_fn(gate.clamp(max=7.0)) * up

    assert not _moe._default_swiglu(Custom())


def test_fp8_products_take_per_expert_scales_and_whole_128_blocks(monkeypatch):
    """The FP8 products' stack: one scale per expert, or block scales whose blocks are whole 128 x 128 tiles (or
    one block along a dimension); sizes multiples of 16. Others are refused, as the products cannot apply them."""
    import pytest

    codes = torch.zeros(3, 256, 384, dtype=torch.float8_e4m3fn)
    st = _grouped.Fp8Stack.of(codes, torch.ones(3))
    assert st.scale is not None and st.blocks is None
    st = _grouped.Fp8Stack.of(codes, torch.full((3, 2, 3), 0.3))
    ws, br, bc = st.blocks
    assert (br, bc) == (128, 128) and ws.dtype == torch.float32
    assert float(ws[0, 0, 0]) == float(torch.tensor(0.3).to(torch.bfloat16))  # rounded to bf16, as dequantised
    assert _grouped.Fp8Stack.of(codes, torch.ones(3, 1, 1)).blocks[1:] == (256, 384)
    with pytest.raises(NotImplementedError):
        _grouped.Fp8Stack.of(codes, torch.ones(3, 4, 3))  # 64-row blocks
    with pytest.raises(NotImplementedError):
        _grouped.Fp8Stack.of(torch.zeros(3, 100, 384, dtype=torch.float8_e4m3fn), torch.ones(3))
    monkeypatch.delenv("MEEPSQUARED_FP8_PRODUCTS", raising=False)
    assert not _grouped._fp8_products_on(codes, None, torch.device("cpu"))
    assert _grouped._fp8_products_on(codes, True, torch.device("cpu"))
    assert not _grouped._fp8_products_on(torch.zeros(2, dtype=torch.bfloat16), True, torch.device("cpu"))
    monkeypatch.setenv("MEEPSQUARED_FP8_PRODUCTS", "1")
    assert _grouped._fp8_products_on(codes, None, torch.device("cpu"))
    assert not _grouped._fp8_products_on(codes, False, torch.device("cpu"))


def test_the_fp8_products_switch_reads_stacks_of_every_kind(monkeypatch):
    """The routed layer's FP8-products test reads the stacks' dtype without assuming a tensor (an NF4 stack is an
    NF4State): NF4 and bf16 modules stay on their paths with the switch on, an FP8 module follows the switch."""
    from meepsquared_b200 import _moe

    class Experts:
        pass

    nf4, bf16, fp8 = Experts(), Experts(), Experts()
    nf4.gate_up_proj = nf4.down_proj = _nf4.NF4State.__new__(_nf4.NF4State)
    bf16.gate_up_proj = bf16.down_proj = torch.zeros(2, 4, 4, dtype=torch.bfloat16)
    fp8.gate_up_proj = fp8.down_proj = torch.zeros(2, 4, 4, dtype=torch.float8_e4m3fn)
    cpu = torch.device("cpu")
    monkeypatch.setenv("MEEPSQUARED_FP8_PRODUCTS", "1")
    assert not _moe._fp8_products_layer(nf4, cpu) and not _moe._fp8_products_layer(bf16, cpu)
    assert _moe._fp8_products_layer(fp8, cpu)
    monkeypatch.delenv("MEEPSQUARED_FP8_PRODUCTS")
    assert not _moe._fp8_products_layer(fp8, cpu)
