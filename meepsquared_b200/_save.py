"""The merged save of an expert stack on the GPU: the reference's ``_save._merged_stack`` (``_save.py:79-95``).

A merged save writes every expert's frozen weight with its adapter merged in, ``W + scaling * lhs @ rhs``,
computed in float32 and stored in the model's dtype; an FP8 stack with one scale per expert is dequantised first
(``f32(code) * scale``, as ``_fp8.dequantize_stack`` does for float32). Here one kernel
(``meep2b_merge_stack``) reads the stack once and writes the merged stack once. Stacks the reference never merges
(block-scaled FP8, NF4) are taken as the layer reads them, dequantised to bf16 by their kernels first.
"""

import torch

from . import _lib

_OUT = {torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


def _weight(experts, name):
    """(the stack as the merge kernel reads it, its dtype code, the per-expert scale or None)."""
    from . import _fp8, _nf4

    w = getattr(experts, name)
    if isinstance(w, _nf4.NF4State):
        return _nf4.dequantize(w).contiguous(), _lib.BF16, None
    w = w.detach()
    if w.dtype == torch.float8_e4m3fn:
        scale = getattr(experts, name + _fp8.STACK_SCALE)
        if scale.dim() != 1:  # a grid of block scales: the bf16 stack the layer computes with
            return _fp8.dequantize(w, scale).contiguous(), _lib.BF16, None
        return w.contiguous(), _lib.E4M3, scale.detach().float().contiguous()
    if w.dtype == torch.bfloat16:
        return w.contiguous(), _lib.BF16, None
    if w.dtype == torch.float32:
        return w.contiguous(), _lib.F32, None
    raise TypeError(f"expert stacks in bf16, float32, FP8 (e4m3) or NF4; got {w.dtype}")


def merged_stack(experts, name: str, factors, dtype: torch.dtype) -> torch.Tensor:
    """The stack `name` of an experts module with its adapter merged, in the stack's layout and `dtype`.

    factors: (lhs, rhs, scaling) with lhs @ rhs in the stack's layout, as ``_moe._delta_factors`` gives them
    (``_moe.py:150-163``), or None for the stack alone (dequantised). dtype: torch.bfloat16 or torch.float32.
    """
    if dtype not in _OUT:
        raise TypeError(f"a merged stack is stored in bf16 or float32; got {dtype}")
    w, wdt, scale = _weight(experts, name)
    if not w.is_cuda:
        raise RuntimeError("the merged save runs on a CUDA GPU (compute capability 10.0)")
    experts_n, rows, cols = w.shape
    if factors is None:
        lhs = rhs = None
        rank, scaling = 0, 1.0
    else:
        lhs, rhs, scaling = factors
        lhs = lhs.detach().to(torch.float32).contiguous()
        rhs = rhs.detach().to(torch.float32).contiguous()
        if lhs.shape[:2] != (experts_n, rows) or rhs.shape != (experts_n, lhs.shape[2], cols):
            raise ValueError(f"factors {tuple(lhs.shape)} @ {tuple(rhs.shape)} do not make a stack of "
                             f"{tuple(w.shape)}")
        rank = lhs.shape[2]
    out = torch.empty(w.shape, device=w.device, dtype=dtype)
    _lib.check(_lib.load().meep2b_merge_stack(_lib.ptr(w), wdt, _lib.ptr(scale), _lib.ptr(lhs), _lib.ptr(rhs),
                                              rank, float(scaling), experts_n, rows, cols, _lib.ptr(out),
                                              _OUT[dtype], _lib.stream_of(w)), "meep2b_merge_stack")
    return out
