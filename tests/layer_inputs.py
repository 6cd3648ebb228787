"""Seeded synthetic inputs of the routed MoE-LoRA layer, as BASELINE.json's configs describe them.

Pure PyTorch (CPU generator), so the golden-vector script, the CPU oracle tests and the GPU parity tests build
bit-identical inputs from the same seed. Routing logits ~N(0,1) -> softmax (float32) -> top-k -> renormalised
(Transformers' Qwen3MoeTopKRouter); base stacks ~N(0, 0.02) in the non-transposed layout gate_up (E, 2I, H),
down (E, H, I); LoRA A (E, r, in) kaiming-uniform(a=sqrt 5) as PEFT initialises lora_A, B (E, out, r) ~N(0, 0.01);
upstream gradient ~N(0, 1).
"""

import math

import torch


def routing(tokens, experts, top_k, generator, zipf=None):
    logits = torch.randn(tokens, experts, generator=generator)
    if zipf is not None:  # skewed popularity: logits + log p_{pi(e)}, p_j ~ j^-s, pi a seeded permutation
        order = torch.randperm(experts, generator=generator)
        p = torch.arange(1, experts + 1, dtype=torch.float32) ** (-zipf)
        logits = logits + torch.log(p / p.sum())[order]
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    weights, index = torch.topk(probs, top_k, dim=-1)
    weights = weights / weights.sum(dim=-1, keepdim=True)
    return index, weights


def kaiming_a(shape, generator):
    """PEFT's lora_A init, kaiming_uniform_(a=sqrt(5)) over fan_in = in: U(-1/sqrt(in), 1/sqrt(in))."""
    fan_in = shape[-1]
    bound = 1.0 / math.sqrt(fan_in)
    return (torch.rand(shape, generator=generator) * 2 - 1) * bound


def bf16_valued(t):
    """t rounded to the nearest bf16 value, kept as float32: the kernels read exactly these numbers."""
    return t.to(torch.bfloat16).float()


def layer(tokens, hidden, inter, experts, top_k, rank, alpha, seed=0, zipf=None):
    """All inputs of one layer step, float32 on the CPU, as a dict.

    Every tensor but the routing weights holds bf16-representable values, so a float32 computation on them is the
    exact-input reference for the bf16 kernels; the routing weights stay float32, as Transformers' router gives them.
    """
    g = torch.Generator().manual_seed(seed)
    index, weights = routing(tokens, experts, top_k, g, zipf)
    x = torch.randn(tokens, hidden, generator=g)
    gate_up = torch.randn(experts, 2 * inter, hidden, generator=g) * 0.02
    down = torch.randn(experts, hidden, inter, generator=g) * 0.02
    a1 = kaiming_a((experts, rank, hidden), g)
    b1 = torch.randn(experts, 2 * inter, rank, generator=g) * 0.01
    a2 = kaiming_a((experts, rank, inter), g)
    b2 = torch.randn(experts, hidden, rank, generator=g) * 0.01
    grad = torch.randn(tokens, hidden, generator=g)
    x, gate_up, down, a1, b1, a2, b2, grad = (bf16_valued(t) for t in (x, gate_up, down, a1, b1, a2, b2, grad))
    return {"hidden": x, "top_k_index": index, "top_k_weights": weights, "gate_up": gate_up, "down": down,
            # PEFT's factors for a stack (E, out, in): lhs = B (E, out, r), rhs = A (E, r, in)
            "gate_up_lhs": b1, "gate_up_rhs": a1, "down_lhs": b2, "down_rhs": a2,
            "scaling": alpha / rank, "grad": grad}


SMALL = dict(tokens=64, hidden=64, inter=32, experts=4, top_k=2, rank=4, alpha=8)
CONFIG1 = dict(tokens=512, hidden=256, inter=512, experts=8, top_k=2, rank=8, alpha=16)
QWEN3_30B = dict(tokens=16384, hidden=2048, inter=768, experts=128, top_k=8, rank=16, alpha=32)
MIXTRAL = dict(tokens=8192, hidden=4096, inter=14336, experts=8, top_k=2, rank=16, alpha=32)
QWEN3_235B_FP8 = dict(tokens=32768, hidden=4096, inter=1536, experts=128, top_k=8, rank=16, alpha=32, zipf=1.1)
