"""The merged save of an expert stack, restated in numpy (test infrastructure; see oracle/__init__.py).

``meepsquared/_save.py:79-95`` (``_merged_stack``): the stack dequantised to float32 (an FP8 stack with its
per-expert scale, ``_fp8.dequantize_stack`` with dtype float32: ``f32(code) * scale[e]``), plus
``scaling * bmm(lhs, rhs)`` with the factors of ``meepsquared/_moe.py:150-163`` (``_delta_factors``, float32, in
the stack's layout), stored in the requested dtype (bf16: round to nearest even).
"""

import numpy as np

from . import quant


def dequantized_f32(stack=None, codes=None, scale=None) -> np.ndarray:
    """The stack in float32: bf16/float32 values as they are, or FP8 codes times their expert's scale."""
    if codes is not None:
        return (quant.e4m3_to_f32(codes) * np.asarray(scale, np.float32)[:, None, None]).astype(np.float32)
    return np.asarray(stack, dtype=np.float32)


def merged_stack(weight_f32, lhs=None, rhs=None, scaling=1.0, dtype="f32") -> np.ndarray:
    """W + scaling * lhs @ rhs per expert in float32; dtype "f32" or "bf16" (bf16 bit patterns, uint16)."""
    w = np.asarray(weight_f32, dtype=np.float32)
    if lhs is not None:
        delta = np.matmul(np.asarray(lhs, np.float32), np.asarray(rhs, np.float32)).astype(np.float32)
        w = (w + np.float32(scaling) * delta).astype(np.float32)
    return quant.bf16_bits(w) if dtype == "bf16" else w
