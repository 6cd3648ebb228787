"""Expert stacks held as FP8 (e4m3), on the B200: the stack functions of meepsquared._fp8 and the block FP8 of the
vendored axolotl quantize module, computed by libmeep2b (csrc/quant.cu).

* ``quantize_stack`` / ``dequantize_stack``: one scale per expert (``meepsquared/_fp8.py:122-134``);
* ``quantize_blocks`` / ``dequantize_blocks``: a 2-D grid of scales per matrix, 128 x 128 blocks for sizes that are
  multiples of 128 (``meepsquared/_vendor/axolotl/quantize.py:131-157, 238-263``), here for a stack of matrices;
* ``convert_stacks``: every frozen 3-D stack of an experts module as FP8 with its scale as ``<name>_scale_inv``
  (``meepsquared/_fp8.py:167-186``).
"""

import torch
from torch import nn

from . import _lib

E4M3_MAX = 448.0
STACK_SCALE = "_scale_inv"


def _cuda(t, what):
    if not t.is_cuda:
        raise RuntimeError(f"{what} runs on a CUDA GPU; got a tensor on {t.device}")
    _lib.load()


def _src(weight):
    w = weight.detach().contiguous()
    if w.dtype == torch.bfloat16:
        return w, _lib.BF16
    if w.dtype == torch.float32:
        return w, _lib.F32
    return w.float(), _lib.F32


def quantize_stack(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """A stack (experts, ...) as e4m3 with one scale per expert: weight ~= fp8 * scale[expert]."""
    _cuda(weight, "quantize_stack")
    w, dtype = _src(weight)
    experts = w.shape[0]
    per = w[0].numel()
    codes = torch.empty(w.shape, device=w.device, dtype=torch.float8_e4m3fn)
    scale = torch.empty(experts, device=w.device, dtype=torch.float32)
    work = torch.empty(experts, device=w.device, dtype=torch.float32)
    _lib.check(_lib.load().meep2b_fp8_stack_quantize(_lib.ptr(w), dtype, experts, per, _lib.ptr(codes),
                                                     _lib.ptr(scale), _lib.ptr(work), _lib.stream_of(w)),
               "meep2b_fp8_stack_quantize")
    return codes, scale


def dequantize_stack(weight8: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """The stack back in bf16 for one product: bf16(float32(w8) * scale[expert])."""
    _cuda(weight8, "dequantize_stack")
    if dtype != torch.bfloat16:
        raise TypeError(f"dequantize_stack produces bf16, not {dtype}")
    w8 = weight8.contiguous()
    out = torch.empty(w8.shape, device=w8.device, dtype=torch.bfloat16)
    _lib.check(_lib.load().meep2b_fp8_stack_dequantize(_lib.ptr(w8), _lib.ptr(scale.float().contiguous()),
                                                       w8.shape[0], w8[0].numel(), _lib.ptr(out),
                                                       _lib.stream_of(w8)), "meep2b_fp8_stack_dequantize")
    return out


def _as_matrices(t):
    return t.reshape(-1, t.shape[-2], t.shape[-1])


def quantize_blocks(weight: torch.Tensor, grid=None, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Each (rows, cols) matrix of weight (..., rows, cols) as e4m3 with an (sr, sc) grid of float32 scales.

    grid defaults to (ceil(rows/128), ceil(cols/128)); blocks are (ceil(rows/sr), ceil(cols/sc)) as in the
    reference's quantize_fp8. Returns (codes like weight, scale_inv (..., sr, sc)).
    """
    _cuda(weight, "quantize_blocks")
    w, dtype = _src(weight)
    rows, cols = w.shape[-2], w.shape[-1]
    sr, sc = grid if grid is not None else (-(-rows // block), -(-cols // block))
    m = _as_matrices(w).shape[0]
    codes = torch.empty(w.shape, device=w.device, dtype=torch.float8_e4m3fn)
    scale = torch.empty((*w.shape[:-2], sr, sc), device=w.device, dtype=torch.float32)
    _lib.check(_lib.load().meep2b_fp8_block_quantize(_lib.ptr(w), dtype, m, rows, cols, sr, sc, _lib.ptr(codes),
                                                     _lib.ptr(scale), _lib.stream_of(w)), "meep2b_fp8_block_quantize")
    return codes, scale


def dequantize(weight8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """An FP8 stack in bf16 by the form of its scale: (E,) one per expert, (E, sr, sc) a grid of blocks."""
    if scale.dim() == 1:
        return dequantize_stack(weight8, scale, torch.bfloat16)
    if scale.dim() == weight8.dim():
        return dequantize_blocks(weight8, scale)
    raise ValueError(f"an FP8 stack of shape {tuple(weight8.shape)} takes a scale of (experts,) or "
                     f"(experts, rows/block, cols/block); got {tuple(scale.shape)}")


def dequantize_blocks(codes: torch.Tensor, scale_inv: torch.Tensor) -> torch.Tensor:
    """bf16(bf16(w8) * bf16(scale)) per block, the reference's dequantize_fp8 with dtype bf16."""
    _cuda(codes, "dequantize_blocks")
    c = codes.contiguous()
    rows, cols = c.shape[-2], c.shape[-1]
    sr, sc = scale_inv.shape[-2], scale_inv.shape[-1]
    out = torch.empty(c.shape, device=c.device, dtype=torch.bfloat16)
    _lib.check(_lib.load().meep2b_fp8_block_dequantize(_lib.ptr(c), _as_matrices(c).shape[0], rows, cols,
                                                       _lib.ptr(scale_inv.float().contiguous()), sr, sc,
                                                       _lib.ptr(out), _lib.stream_of(c)),
               "meep2b_fp8_block_dequantize")
    return out


def grouped_product(x, weight8, scale, offsets, bias, is_transposed: bool) -> torch.Tensor:
    """x against a stack held as FP8, per expert group, with x's gradient (meepsquared/_fp8.py:137-164), in x's
    dtype. The grouped kernel reads the e4m3 codes and converts them in shared memory, for the forward product and
    again for the backward one; nothing dequantised is kept. One scale per expert is applied to the accumulator; a
    grid of block scales (scale (E, sr, sc)) to the converted weights, as the routed layer reads such a stack."""
    from . import _grouped

    if scale.dim() == 1:
        out = _grouped.lora_linear(x.to(torch.bfloat16), weight8, scale, offsets, is_transposed, bias=bias,
                                   products_fp8=False)
        return out.to(x.dtype)
    stack = _grouped.QuantStack.from_fp8(weight8.detach(), scale)
    if stack is None:
        stack = dequantize_blocks(weight8.detach(), scale)
    bias = bias.detach().to(torch.bfloat16).contiguous() if bias is not None else None
    out = _grouped._LoraGroupedProduct.apply(x.to(torch.bfloat16), stack, None, offsets.to(torch.int32),
                                             is_transposed, None, None, 1.0, bias, None)
    return out.to(x.dtype)


def convert_stacks(experts, block: int | None = None) -> int:
    """Every frozen stack of an experts module held as FP8, its scale as <name>_scale_inv; returns how many.

    block=None: one scale per expert, (E,) (meepsquared/_fp8.py:170-186). block=128: a grid of 128 x 128 blocks per
    expert matrix, scale_inv (E, ceil(out/128), ceil(in/128)), as an FP8 checkpoint of block-scaled weights holds.
    """
    converted = 0
    for name, parameter in list(experts.named_parameters(recurse=False)):
        if parameter.dim() != 3 or parameter.requires_grad or not parameter.is_floating_point():
            continue
        if parameter.dtype == torch.float8_e4m3fn and hasattr(experts, name + STACK_SCALE):
            converted += 1
            continue
        if block is None:
            weight8, scale = quantize_stack(parameter.detach())
        else:
            weight8, scale = quantize_blocks(parameter.detach(), block=block)
        setattr(experts, name, nn.Parameter(weight8, requires_grad=False))
        experts.register_buffer(name + STACK_SCALE, scale)
        converted += 1
    if converted:
        experts._meepsquared_fp8 = True
    return converted
