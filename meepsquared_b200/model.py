"""LoRA on every routed-expert stack of a Transformers mixture-of-experts model, computed by this package's routed
layer: the model-level step of the reference's ``meepsquared._moe.apply`` (meepsquared/_moe.py:208-227), which
patches each PEFT-wrapped experts module so that its forward runs the routed layer with the adapters' factors.

The reference finds the experts modules PEFT wrapped (``target_parameters`` on ``gate_up_proj`` / ``down_proj``)
and reads each wrapper's lora_A / lora_B as PEFT lays them out (``_delta_factors``, :148-163). Here the factors
are held by the experts module itself, in PEFT's layout and with PEFT's initialisation (lora_A kaiming-uniform,
lora_B zero), so that a model without PEFT installed gets the same trainable parameters:

* ``install(model, rank, alpha)`` adds ``lora_<stack>_lhs`` (experts, out, rank) and ``lora_<stack>_rhs``
  (experts, rank, in) to every experts module (Transformers' ``gate_up_proj (E, 2I, H)`` / ``down_proj (E, H, I)``
  layout, or the transposed one) and makes its forward ``_moe.routed_forward`` with them;
* ``lora_parameters(model)`` lists them, in the order a data-parallel gradient bucket wants them (each layer's
  down-projection factors before its gate/up ones, ``ddp.LoraGradBucket`` segments).

Experts modules of Transformers versions that predate the ``has_gate`` / ``has_bias`` / ``is_transposed``
attributes (which ``_moe.routed_forward`` reads, as the reference's ``_routed_forward`` does) get them from the
module's stacks: a ``gate_up_proj`` means gated, no ``*_bias`` means unbiased, and a stack stored (experts, 2I,
hidden) is not transposed.
"""

import math
import types

import torch

from . import _moe

# What makes a module an experts module. The reference asks for ("num_experts", "has_gate", "has_bias",
# "is_transposed") (_moe.py:31), the attributes of Transformers >= 5.17; an experts module of an older Transformers
# has the stacks and the expert count, and _complete() derives the rest.
EXPERTS_ATTRIBUTES = ("num_experts", "down_proj")
STACKS = ("gate_up_proj", "up_proj", "down_proj")  # the reference's STACKS (_moe.py:34)


def experts_modules(model):
    """(name, module) of every Transformers experts module of the model."""
    for name, module in model.named_modules():
        if all(hasattr(module, a) for a in EXPERTS_ATTRIBUTES) and isinstance(getattr(module, "down_proj"),
                                                                               torch.nn.Parameter):
            yield name, module


def _complete(experts):
    """The attributes _moe.routed_forward reads, derived from the stacks where an older module lacks them."""
    if not hasattr(experts, "has_gate"):
        experts.has_gate = hasattr(experts, "gate_up_proj")
    if not hasattr(experts, "has_bias"):
        experts.has_bias = any(hasattr(experts, f"{s}_bias") for s in STACKS)
    if not hasattr(experts, "is_transposed"):
        # (E, out, in) stacks: the first projection's input (hidden) is the down projection's output
        first = experts.gate_up_proj if experts.has_gate else experts.up_proj
        experts.is_transposed = first.shape[2] != experts.down_proj.shape[1]


def _stack_dims(experts, name):
    """(in, out) of the projection a stack computes."""
    w = getattr(experts, name)
    return (w.shape[1], w.shape[2]) if experts.is_transposed else (w.shape[2], w.shape[1])


def _forward(self, hidden_states, top_k_index, top_k_weights, *args, **kwargs):
    """The experts' forward with the adapters (the reference's _moe._forward, :128-145): the routed layer."""
    if args or kwargs:
        raise NotImplementedError("the routed experts take (hidden_states, top_k_index, top_k_weights)")
    factors = {name: (getattr(self, f"lora_{name}_lhs"), getattr(self, f"lora_{name}_rhs"), self.lora_scaling)
               for name in self.lora_stacks}
    return _moe.routed_forward(self, hidden_states, top_k_index, top_k_weights, factors)


def install(model, rank: int = 16, alpha: float = 16, dtype=torch.bfloat16, generator=None) -> int:
    """LoRA of the given rank on every expert stack of the model, computed by the routed layer; returns how many
    experts modules were patched. The stacks are frozen; the factors are trainable parameters of the experts
    module (PEFT's names lora_A / lora_B map to rhs / lhs), initialised as PEFT does (lhs zero, rhs kaiming-uniform
    with a = sqrt(5), that is U(-1/sqrt(in), 1/sqrt(in)))."""
    patched = 0
    for name, experts in experts_modules(model):
        _complete(experts)
        stacks = [s for s in ("gate_up_proj", "up_proj", "down_proj") if isinstance(getattr(experts, s, None),
                                                                                    torch.nn.Parameter)]
        for s in stacks:
            getattr(experts, s).requires_grad_(False)
            fan_in, out = _stack_dims(experts, s)
            e = experts.num_experts
            device = getattr(experts, s).device
            bound = 1.0 / math.sqrt(fan_in)
            rhs = (torch.rand((e, rank, fan_in), generator=generator) * 2 - 1) * bound  # on the CPU, then moved
            lhs = torch.zeros((e, out, rank))
            experts.register_parameter(f"lora_{s}_lhs", torch.nn.Parameter(lhs.to(device, dtype)))
            experts.register_parameter(f"lora_{s}_rhs", torch.nn.Parameter(rhs.to(device, dtype)))
        experts.lora_stacks = tuple(stacks)
        experts.lora_scaling = alpha / rank
        experts.forward = types.MethodType(_forward, experts)
        patched += 1
    return patched


def lora_parameters(model):
    """The factors install() added, each layer's down-projection factors before its gate/up ones."""
    params = []
    for _, experts in experts_modules(model):
        for s in ("down_proj", "gate_up_proj", "up_proj"):
            if s in getattr(experts, "lora_stacks", ()):
                params += [getattr(experts, f"lora_{s}_lhs"), getattr(experts, f"lora_{s}_rhs")]
    return params
