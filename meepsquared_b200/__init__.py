"""meepsquared_b200: Meep²'s grouped MoE-LoRA expert layer, B200-native (sm_100a).

Modules mirror the reference's operator API (thinkube/meepsquared):
  _grouped  lora_linear, grouped_linear, tile_map, ... (meepsquared/_grouped.py)
  _moe      route, route_logits, gather, unpermute, combine, routed_forward (meepsquared/_moe.py:_routed_forward)
  _fp8      FP8 expert stacks, per expert and block-scaled (meepsquared/_fp8.py, axolotl quantize.py)
  _nf4      NF4 double-quantised stacks                (axolotl quantize.py:52-101)
  ddp       the LoRA-gradient all-reduce of data-parallel training
  model     LoRA on every expert stack of a Transformers MoE model (meepsquared/_moe.py:apply)
The kernels live in libmeep2b.so (csrc/, include/meep2b.h), reached through ctypes (_lib).
"""

from . import _fp8, _grouped, _lib, _moe, _nf4, model  # noqa: F401
from ._grouped import (BLOCK_M, RANK_MULTIPLE, TORCH_HAS_GROUPED_MM, available, fp8_products,  # noqa: F401
                       grouped_linear, lora_linear, max_tiles, reference, reference_lora, tile_map, wanted)
from ._moe import combine, gather, route, route_logits, routed_forward, unpermute  # noqa: F401

__version__ = "0.1.0"
