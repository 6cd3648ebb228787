"""NF4 expert stacks with a double-quantised absmax (QLoRA), dequantised on the B200 by libmeep2b.

The state is what bitsandbytes' ``quantize_4bit(..., quant_type="nf4", compress_statistics=True)`` keeps and what
``meepsquared/_vendor/axolotl/quantize.py:52-101`` hands to bitsandbytes' C kernels: packed codes (two per byte, the
first in the high nibble), an 8-bit absmax per block of 64 weights, a float32 absmax2 per block of 256 absmax
values, the 256-entry code2 and the float32 offset. ``dequantize`` restates that call sequence
(absmax = code2[q] * absmax2 + offset, then w = NF4[code] * absmax) in one library call.
"""

from dataclasses import dataclass

import torch

from . import _lib


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
