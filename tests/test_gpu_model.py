"""A whole Transformers MoE model with the routed layer installed on its experts (meepsquared_b200.model): its loss
and the adapters' gradients against the same model whose experts run the reference's PyTorch path (the routed
forward of meepsquared/_moe.py:70-126 on its non-kernel branch, restated in bench.py) with the same factors."""

import pytest
import torch

import meepsquared_b200 as mb
from test_model import tiny_qwen3_moe

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _reference_forward(self, hidden_states, top_k_index, top_k_weights):
    import bench

    factors = {name: (getattr(self, f"lora_{name}_lhs"), getattr(self, f"lora_{name}_rhs"), self.lora_scaling)
               for name in self.lora_stacks}
    return bench.reference_routed_forward(self, hidden_states, top_k_index, top_k_weights, factors)


def _step(model, ids):
    out = model(input_ids=ids, labels=ids)
    out.loss.backward()
    return out.loss.detach().float(), [p.grad.float().clone() for p in mb.model.lora_parameters(model)]


def test_the_model_step_matches_the_references_path():
    import types

    # one decoder layer: its router sees the same hidden states in both runs (with more layers the later routers
    # see the earlier experts' outputs, which the two paths round differently, and near-tied tokens may switch
    # experts)
    model = tiny_qwen3_moe(layers=1).to(DEV, torch.bfloat16)
    mb.model.install(model, rank=16, alpha=32, generator=torch.Generator().manual_seed(1))
    gen = torch.Generator().manual_seed(2)
    for p in mb.model.lora_parameters(model):  # non-zero lhs, so that the adapters change the output
        with torch.no_grad():
            p.copy_((torch.randn(p.shape, generator=gen) * 0.02).to(p))
    ids = torch.randint(0, 512, (2, 96), generator=gen).to(DEV)
    loss, grads = _step(model, ids)

    for p in mb.model.lora_parameters(model):
        p.grad = None
    for _, e in mb.model.experts_modules(model):
        e.forward = types.MethodType(_reference_forward, e)
    ref_loss, ref_grads = _step(model, ids)

    # Two bf16 computations of a whole model (attention, norms and the loss included) that round at different
    # points: the loss within 2%, each adapter gradient within 3% of its norm and 10% of its largest element.
    assert torch.isfinite(loss) and abs(loss.item() - ref_loss.item()) <= 2e-2 * abs(ref_loss.item())
    for i, (g, r) in enumerate(zip(grads, ref_grads)):
        assert (g - r).norm() <= 3e-2 * r.norm(), i
        torch.testing.assert_close(g, r, atol=0.1 * r.abs().max().item(), rtol=0, msg=str(i))
