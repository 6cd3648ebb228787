"""The routed MoE-LoRA layer, forward and backward, in float32 numpy (test infrastructure).

Restates ``meepsquared/_moe.py:_routed_forward`` (:70-126) for a gated experts module (Qwen3 / Mixtral layout
``gate_up_proj (E, 2I, H)``, ``down_proj (E, H, I)``, or their transposes) with PEFT factors per stack, and the
gradients autograd gives it: hidden, top_k_weights and each adapter's lhs / rhs.
"""

import numpy as np

from . import grouped, routing


def forward(hidden, top_k_index, top_k_weights, gate_up, down, factors, is_transposed=False,
            scales=(None, None)):
    """out (T, H) and the saved intermediates. factors = {"gate_up_proj": (lhs, rhs, s), "down_proj": (...)}."""
    hidden = np.asarray(hidden, dtype=np.float32)
    tokens, k = np.asarray(top_k_index).shape
    experts = gate_up.shape[0]
    r = routing.route(top_k_index, experts)
    sel = routing.gather(hidden, r["perm"], k, r["sentinel"])
    w_g = np.asarray(top_k_weights, dtype=np.float32).reshape(-1)[r["perm"]]
    lhs1, rhs1, s1 = factors.get("gate_up_proj", (None, None, 1.0))
    lhs2, rhs2, s2 = factors.get("down_proj", (None, None, 1.0))
    gu = grouped.lora_forward(sel, gate_up, scales[0], r["offsets"], is_transposed, lhs1, rhs1, s1)
    h = grouped.swiglu(gu)
    y = grouped.lora_forward(h, down, scales[1], r["offsets"], is_transposed, lhs2, rhs2, s2)
    y[r["sentinel"]] = 0
    out = routing.unpermute(y, w_g, r["inverse"], tokens, k)
    saved = dict(route=r, sel=sel, w_g=w_g, gu=gu, h=h, y=y, k=k, tokens=tokens)
    return out, saved


def backward(grad_out, saved, gate_up, down, factors, is_transposed=False, scales=(None, None)):
    """Gradients: {"hidden", "top_k_weights", "gate_up_proj": (dlhs, drhs), "down_proj": (dlhs, drhs)}."""
    r, k, tokens = saved["route"], saved["k"], saved["tokens"]
    lhs1, rhs1, s1 = factors.get("gate_up_proj", (None, None, 1.0))
    lhs2, rhs2, s2 = factors.get("down_proj", (None, None, 1.0))
    grad_y, grad_wg = routing.unpermute_backward(grad_out, saved["y"], saved["w_g"], r["perm"], k)
    grad_y[r["sentinel"]] = 0
    grad_h, dl2, dr2 = grouped.lora_backward(saved["h"], grad_y, down, scales[1], r["offsets"], is_transposed,
                                             lhs2, rhs2, s2)
    grad_gu = grouped.swiglu_backward(saved["gu"], grad_h)
    grad_sel, dl1, dr1 = grouped.lora_backward(saved["sel"], grad_gu, gate_up, scales[0], r["offsets"],
                                               is_transposed, lhs1, rhs1, s1)
    grad_sel[r["sentinel"]] = 0
    grad_hidden = np.zeros((tokens, grad_sel.shape[1]), dtype=np.float32)
    np.add.at(grad_hidden, r["perm"] // k, grad_sel)
    grad_w = np.zeros(tokens * k, dtype=np.float32)
    grad_w[r["perm"]] = grad_wg
    return {"hidden": grad_hidden, "top_k_weights": grad_w.reshape(tokens, k),
            "gate_up_proj": (dl1, dr1), "down_proj": (dl2, dr2)}
