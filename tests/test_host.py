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
