"""NF4 expert stacks with a double-quantised absmax (QLoRA), dequantised on the B200 by libmeep2b.

The state is what bitsandbytes' ``quantize_4bit(..., quant_type="nf4", compress_statistics=True)`` keeps and what
``meepsquared/_vendor/axolotl/quantize.py:52-101`` hands to bitsandbytes' C kernels: packed codes (two per byte, the
first in the high nibble), an 8-bit absmax per block of 64 weights, a float32 absmax2 per block of 256 absmax
values, the 256-entry code2 and the float32 offset. ``dequantize`` restates that call sequence
(absmax = code2[q] * absmax2 + offset, then w = NF4[code] * absmax) in one library call.
"""

from dataclasses import dataclass

import numpy as np
import torch
from torch import nn

from . import _lib

# The 16 NormalFloat-4 levels of the QLoRA paper (Dettmers et al., 2023, appendix E), as float32.
NF4_LEVELS = (-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453, -0.28444138169288635,
              -0.18477343022823334, -0.09105003625154495, 0.0, 0.07958029955625534, 0.16093020141124725,
              0.24611230194568634, 0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
              0.7229568362236023, 1.0)


@dataclass
class NF4State:
    packed: torch.Tensor    # uint8 (n / 2,)
    absmax: torch.Tensor    # uint8 (n / blocksize,)
    absmax2: torch.Tensor   # float32 (ceil(n / blocksize / blocksize2),)
    code2: torch.Tensor     # float32 (256,)
    offset: torch.Tensor    # float32 (1,)
    shape: tuple
    blocksize: int = 64
    blocksize2: int = 256

    def to(self, device):
        return NF4State(self.packed.to(device), self.absmax.to(device), self.absmax2.to(device),
                        self.code2.to(device), self.offset.to(device), self.shape, self.blocksize, self.blocksize2)

    def multipliers(self) -> torch.Tensor:
        """absmax_f32 laid out (experts, cols/64, rows) for the fused product (computed once: the stack is frozen)."""
        cached = self.__dict__.get("_multipliers")
        if cached is None or cached.device != self.absmax.device:
            from ._grouped import QuantStack
            from . import _lib as lib

            cached = QuantStack.multipliers(lib.NF4, self.absmax_f32(), self.shape)
            self.__dict__["_multipliers"] = cached
        return cached

    def absmax_f32(self) -> torch.Tensor:
        """The first dequantisation stage, absmax as float32 per block (computed once: the stack is frozen)."""
        cached = self.__dict__.get("_absmax_f32")
        if cached is None or cached.device != self.absmax.device:
            cached = absmax_f32(self)
            self.__dict__["_absmax_f32"] = cached
        return cached


def absmax_f32(state: NF4State) -> torch.Tensor:
    """code2[absmax] * absmax2[block / blocksize2] + offset per block of the state, float32 (two roundings)."""
    if not state.packed.is_cuda:
        raise RuntimeError("NF4 dequantisation runs on a CUDA GPU")
    count = state.absmax.numel()
    out = torch.empty(count, device=state.absmax.device, dtype=torch.float32)
    _lib.check(_lib.load().meep2b_nf4_absmax(_lib.ptr(state.absmax.contiguous()),
                                             _lib.ptr(state.absmax2.float().contiguous()),
                                             _lib.ptr(state.code2.float().contiguous()),
                                             _lib.ptr(state.offset.float().reshape(1).contiguous()),
                                             state.blocksize2, count, _lib.ptr(out), _lib.stream_of(state.absmax)),
               "meep2b_nf4_absmax")
    return out


def dequantize(state: NF4State) -> torch.Tensor:
    """The weight in bf16, of state.shape; bit-exact with the two-stage bitsandbytes dequantisation."""
    if not state.packed.is_cuda:
        raise RuntimeError("NF4 dequantisation runs on a CUDA GPU")
    lib = _lib.load()
    n = 1
    for d in state.shape:
        n *= d
    absmax_out = torch.empty(state.absmax.numel(), device=state.packed.device, dtype=torch.float32)
    out = torch.empty(state.shape, device=state.packed.device, dtype=torch.bfloat16)
    _lib.check(lib.meep2b_nf4_dequantize(_lib.ptr(state.packed.contiguous()), _lib.ptr(state.absmax.contiguous()),
                                         _lib.ptr(state.absmax2.float().contiguous()),
                                         _lib.ptr(state.code2.float().contiguous()),
                                         _lib.ptr(state.offset.float().reshape(1).contiguous()), state.blocksize,
                                         state.blocksize2, n, _lib.ptr(absmax_out), _lib.ptr(out),
                                         _lib.stream_of(state.packed)), "meep2b_nf4_dequantize")
    return out


def dynamic_map() -> np.ndarray:
    """The signed 8-bit dynamic code (Dettmers et al., 2022) that holds the second-level absmax: for exponent i in
    0..6, the midpoints of an even split of [0.1, 1] into 2^i parts times 10^(i-6), both signs, plus 0 and 1;
    256 sorted float32 values (bitsandbytes' create_dynamic_map(signed=True), its code2)."""
    vals = []
    for i in range(7):
        bounds = np.linspace(0.1, 1, 2 ** i + 1, dtype=np.float32)
        mids = (bounds[:-1] + bounds[1:]) / np.float32(2.0)
        decade = np.float32(10.0 ** (i - 6))
        vals += (decade * mids).tolist() + (-decade * mids).tolist()
    vals += [0.0, 1.0]
    vals += [0.0] * (256 - len(vals))
    return np.sort(np.array(vals, dtype=np.float32))


def _nearest(values: torch.Tensor, levels: torch.Tensor) -> torch.Tensor:
    """Index of the nearest of the sorted levels; a tie takes the upper one."""
    idx = torch.searchsorted(levels, values).clamp(1, levels.numel() - 1)
    lo, hi = levels[idx - 1], levels[idx]
    return torch.where((values - lo).abs() < (hi - values).abs(), idx - 1, idx)


def quantize(weight: torch.Tensor, blocksize: int = 64, blocksize2: int = 256) -> NF4State:
    """weight as NF4 with a double-quantised absmax: the state of bitsandbytes' quantize_4bit(quant_type="nf4",
    compress_statistics=True), which the reference's QLoRA loading applies (meepsquared/models.py:334-336).

    Load-time conversion of a frozen stack, on the weight's device: blocks of `blocksize` weights of the flattened
    tensor, codes of the nearest NF4 level of w / absmax (two a byte, the first in the high nibble); the absmax
    vector less its mean (the offset) in blocks of `blocksize2`, each scaled by its largest magnitude (absmax2)
    and coded as the nearest entry of the dynamic map (code2).
    """
    w = weight.detach().float().reshape(-1)
    if w.numel() % blocksize or w.numel() % 2:
        raise ValueError(f"NF4 needs whole blocks of {blocksize} weights; got {w.numel()}")
    dev = w.device
    levels = torch.tensor(NF4_LEVELS, dtype=torch.float32, device=dev)
    blocks = w.view(-1, blocksize)
    absmax = blocks.abs().amax(dim=1)
    safe = torch.where(absmax == 0, torch.ones_like(absmax), absmax)
    codes = _nearest((blocks / safe[:, None]).reshape(-1), levels).to(torch.uint8)
    packed = (codes[0::2] << 4) | codes[1::2]
    offset = absmax.mean().reshape(1)
    centred = absmax - offset
    n2 = -(-centred.numel() // blocksize2)
    padded = torch.zeros(n2 * blocksize2, dtype=torch.float32, device=dev)
    padded[:centred.numel()] = centred
    absmax2 = padded.view(n2, blocksize2).abs().amax(dim=1)
    safe2 = torch.where(absmax2 == 0, torch.ones_like(absmax2), absmax2)
    code2 = torch.from_numpy(dynamic_map()).to(dev)
    normed = (padded.view(n2, blocksize2) / safe2[:, None]).reshape(-1)[:centred.numel()]
    absmax_q = _nearest(normed, code2).to(torch.uint8)
    return NF4State(packed.contiguous(), absmax_q.contiguous(), absmax2.contiguous(), code2, offset,
                    tuple(weight.shape), blocksize, blocksize2)


def convert_stacks(experts) -> int:
    """Every frozen 3-D stack of an experts module held as NF4 (an NF4State in place of the parameter), as QLoRA
    holds base weights; returns how many. The routed layer dequantises them for its products."""
    converted = 0
    for name, parameter in list(experts.named_parameters(recurse=False)):
        if parameter.dim() != 3 or parameter.requires_grad or not parameter.is_floating_point():
            continue
        state = quantize(parameter.detach())
        delattr(experts, name)
        setattr(experts, name, state)
        converted += 1
    return converted
