"""Parity helpers of the GPU tests: the tolerance BASELINE.json's north star states, written down once.

bf16 outputs against a float32 computation: |got - want| <= 1e-2 + 2e-2 |want| elementwise (abs 1e-2, rel 2e-2).
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


def assert_close(got, want, name="", scaled=False):
    g, w = as_np(got), as_np(want)
    assert g.shape == w.shape, f"{name}: shape {g.shape} != {w.shape}"
    atol = ATOL * max(1.0, float(np.abs(w).max())) if scaled else ATOL
    err = np.abs(g - w) - (atol + RTOL * np.abs(w))
    bad = err > 0
    if bad.any():
        i = np.unravel_index(np.argmax(err), err.shape)
        raise AssertionError(f"{name}: {int(bad.sum())} of {bad.size} outside atol {atol:.3g} rtol {RTOL}; "
                             f"worst at {i}: got {g[i]} want {w[i]}")
