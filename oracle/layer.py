"""The routed MoE-LoRA layer, forward and backward, in float32 numpy (test infrastructure).

Restates ``meepsquared/_moe.py:_routed_forward`` (:70-126) for a gated experts module (Qwen3 / Mixtral layout
``gate_up_proj (E, 2I, H)``, ``down_proj (E, H, I)``, or their transposes) with PEFT factors per stack, and the
gradients autograd gives it: hidden, top_k_weights and each adapter's lhs / rhs.

``bf16_intermediates=True`` rounds to bf16 every tensor the reference's path holds in bf16 when the model is bf16
(hidden states, stacks and factors bf16, routing weights float32), at the points where that path rounds them:

* forward: the gate/up projection's output (``project`` returns the stack's dtype, ``_moe.py:108-116``), the
  activation ``act_fn(gate)`` and ``h = act * up`` (Transformers' ``_default_apply_gate`` on bf16 tensors,
  ``_moe.py:118-119``), the down projection's output ``y`` (:122) and the layer output (``.to(hidden dtype)``,
  :126); every product accumulates in float32 and is rounded once;
* backward (autograd over the same bf16 graph): the rows' gradient ``grad_y = g * w`` (the product with the
  float32 weights is float32 and its gradient is cast back to y's dtype), the gradient of h, of the activation and
  of the up half (each bf16 multiply's gradient is bf16), the gate's gradient through SiLU, the gathered rows'
  gradient and the hidden states' gradient (summed over a token's k rows in float32, then bf16).

Everything else (the rank panel, the adapters' gradients, the routing weights' gradient) stays float32.
"""

import numpy as np

from . import grouped, routing
from .quant import bf16


def _round(v, on):
    return bf16(v) if on else v


def forward(hidden, top_k_index, top_k_weights, gate_up, down, factors, is_transposed=False,
            scales=(None, None), bf16_intermediates=False):
    """out (T, H) and the saved intermediates. factors = {"gate_up_proj": (lhs, rhs, s), "down_proj": (...)}."""
    rb = bf16_intermediates
    hidden = np.asarray(hidden, dtype=np.float32)
    tokens, k = np.asarray(top_k_index).shape
    experts = gate_up.shape[0]
    r = routing.route(top_k_index, experts)
    sel = routing.gather(hidden, r["perm"], k, r["sentinel"])
    w_g = np.asarray(top_k_weights, dtype=np.float32).reshape(-1)[r["perm"]]
    lhs1, rhs1, s1 = factors.get("gate_up_proj", (None, None, 1.0))
    lhs2, rhs2, s2 = factors.get("down_proj", (None, None, 1.0))
    gu = _round(grouped.lora_forward(sel, gate_up, scales[0], r["offsets"], is_transposed, lhs1, rhs1, s1), rb)
    h = grouped.swiglu(gu, round_bf16=rb)
    y = _round(grouped.lora_forward(h, down, scales[1], r["offsets"], is_transposed, lhs2, rhs2, s2), rb)
    y[r["sentinel"]] = 0
    out = routing.unpermute(y, w_g, r["inverse"], tokens, k, round_bf16=rb)
    saved = dict(route=r, sel=sel, w_g=w_g, gu=gu, h=h, y=y, k=k, tokens=tokens, bf16=rb)
    return out, saved


def backward(grad_out, saved, gate_up, down, factors, is_transposed=False, scales=(None, None),
             round_grad_rows=None):
    """Gradients: {"hidden", "top_k_weights", "gate_up_proj": (dlhs, drhs), "down_proj": (dlhs, drhs), "rows"}, where
    "rows" is the gradient of the gathered rows in expert order (the terms the hidden states' gradient sums).

    round_grad_rows: whether the rows' gradient g * w is rounded to bf16 before the down projection's backward, as
    autograd does over the reference's bf16 graph (the default in bf16 mode); False states a computation that
    applies the routing weight to the float32 product instead (one rounding fewer, the same function)."""
    r, k, tokens, rb = saved["route"], saved["k"], saved["tokens"], saved.get("bf16", False)
    round_gy = rb if round_grad_rows is None else round_grad_rows
    lhs1, rhs1, s1 = factors.get("gate_up_proj", (None, None, 1.0))
    lhs2, rhs2, s2 = factors.get("down_proj", (None, None, 1.0))
    grad_y, grad_wg = routing.unpermute_backward(grad_out, saved["y"], saved["w_g"], r["perm"], k)
    grad_y = _round(grad_y, round_gy)
    grad_y[r["sentinel"]] = 0
    grad_h, dl2, dr2 = grouped.lora_backward(saved["h"], grad_y, down, scales[1], r["offsets"], is_transposed,
                                             lhs2, rhs2, s2)
    grad_gu = grouped.swiglu_backward(saved["gu"], _round(grad_h, rb), round_bf16=rb)
    grad_sel, dl1, dr1 = grouped.lora_backward(saved["sel"], grad_gu, gate_up, scales[0], r["offsets"],
                                               is_transposed, lhs1, rhs1, s1)
    grad_sel = _round(grad_sel, rb)
    grad_sel[r["sentinel"]] = 0
    grad_hidden = np.zeros((tokens, grad_sel.shape[1]), dtype=np.float32)
    np.add.at(grad_hidden, r["perm"] // k, grad_sel)
    grad_w = np.zeros(tokens * k, dtype=np.float32)
    grad_w[r["perm"]] = grad_wg
    return {"hidden": _round(grad_hidden, rb), "top_k_weights": grad_w.reshape(tokens, k),
            "gate_up_proj": (dl1, dr1), "down_proj": (dl2, dr2), "rows": grad_sel}
