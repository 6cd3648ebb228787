"""Parity helpers of the GPU tests: the tolerance BASELINE.json's north star states, written down once.

bf16 outputs against a float32 computation: |got - want| <= 1e-2 + 2e-2 |want| elementwise (abs 1e-2, rel 2e-2).
A layer output that sums stored bf16 rows (the weighted combine of the k rows of a token, the input gradient's sum
over them) also gets one bf16 ulp of each summed term: near cancellation the sum is far smaller than its terms, and
two computations whose float32 values straddle a bf16 rounding boundary store terms one ulp apart.
Sums over an expert's rows (the adapters' gradients) carry the bf16 rounding of their many terms, so their
absolute allowance scales with the tensor (1e-2 * max|want|, the reference tests' own rule,
tests/test_grouped.py:141-143), with rel 2e-2 on top.
"""

import numpy as np
import torch

ATOL, RTOL = 1e-2, 2e-2


def as_np(t):
    if isinstance(t, torch.Tensor):
        return t.detach().float().cpu().numpy()
    return np.asarray(t, dtype=np.float32)


def bf16_ulp(v):
    """The spacing of bf16 values at |v| (2^(e-7) for |v| in [2^e, 2^(e+1))), elementwise, float32."""
    v = np.abs(np.asarray(v, dtype=np.float32))
    _, e = np.frexp(np.maximum(v, np.float32(2.0 ** -126)))
    return np.ldexp(np.float32(1.0), e - 8).astype(np.float32)


def assert_close(got, want, name="", scaled=False, rounding=None):
    """|got - want| <= atol + RTOL |want| elementwise; atol = ATOL, or ATOL max|want| when scaled. rounding: an
    extra elementwise allowance for a sum of stored bf16 rows (one bf16 unit in the last place of each summed
    term, which two correct computations may round to either side when their float32 values straddle a rounding
    boundary), added to the north star's tolerance."""
    g, w = as_np(got), as_np(want)
    assert g.shape == w.shape, f"{name}: shape {g.shape} != {w.shape}"
    atol = ATOL * max(1.0, float(np.abs(w).max())) if scaled else ATOL
    allow = atol + RTOL * np.abs(w)
    if rounding is not None:
        allow = allow + rounding
    err = np.abs(g - w) - allow
    bad = err > 0
    if bad.any():
        i = np.unravel_index(np.argmax(err), err.shape)
        raise AssertionError(f"{name}: {int(bad.sum())} of {bad.size} outside atol {atol:.3g} rtol {RTOL}; "
                             f"worst at {i}: got {g[i]} want {w[i]}")
