"""LoRA installed on every experts module of a Transformers MoE model (meepsquared_b200.model, the reference's
_moe.apply without PEFT): the parameters it adds, their layout and initialisation, and the order it lists them in
(CPU; the GPU test runs the model)."""

import torch

import meepsquared_b200 as mb


def tiny_qwen3_moe(layers=2):
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    cfg = Qwen3MoeConfig(vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
                         num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                         num_experts=8, num_experts_per_tok=2, decoder_sparse_step=1, mlp_only_layers=[],
                         norm_topk_prob=True)
    torch.manual_seed(0)
    return Qwen3MoeForCausalLM(cfg)


def test_install_adds_peft_shaped_factors_to_every_experts_module():
    model = tiny_qwen3_moe()
    assert mb.model.install(model, rank=8, alpha=16, generator=torch.Generator().manual_seed(0)) == 2
    mods = list(mb.model.experts_modules(model))
    assert len(mods) == 2
    for _, e in mods:
        # Transformers' Qwen3 layout: gate_up (E, 2I, H), down (E, H, I), gated, no bias, not transposed
        assert e.has_gate and not e.has_bias and not e.is_transposed
        assert not e.gate_up_proj.requires_grad and not e.down_proj.requires_grad
        assert tuple(e.lora_gate_up_proj_lhs.shape) == (8, 256, 8)   # (experts, out = 2I, rank)
        assert tuple(e.lora_gate_up_proj_rhs.shape) == (8, 8, 256)   # (experts, rank, in = H)
        assert tuple(e.lora_down_proj_lhs.shape) == (8, 256, 8)
        assert tuple(e.lora_down_proj_rhs.shape) == (8, 8, 128)
        assert e.lora_scaling == 2.0
        # PEFT's initialisation: lora_B (lhs) zero, lora_A (rhs) uniform within 1/sqrt(in)
        assert torch.count_nonzero(e.lora_down_proj_lhs) == 0
        assert e.lora_gate_up_proj_rhs.float().abs().max() <= 1 / 256 ** 0.5
        assert e.lora_down_proj_rhs.dtype == torch.bfloat16


def test_lora_parameters_list_each_layers_down_factors_first():
    model = tiny_qwen3_moe()
    mb.model.install(model, rank=4)
    params = mb.model.lora_parameters(model)
    mods = [e for _, e in mb.model.experts_modules(model)]
    want = []
    for e in mods:
        want += [e.lora_down_proj_lhs, e.lora_down_proj_rhs, e.lora_gate_up_proj_lhs, e.lora_gate_up_proj_rhs]
    assert [id(p) for p in params] == [id(p) for p in want]
    trainable = {id(p) for p in model.parameters() if p.requires_grad}
    assert all(id(p) in trainable for p in params)
