"""The grouped product with LoRA adapters and the SwiGLU gate, in float32 numpy (test infrastructure).

Follows ``meepsquared/_grouped.py``: the forward of ``reference_lora`` (:431-444), the per-expert base product of
``reference`` (:420-428), and the gradients ``_LoraGroupedProduct.backward`` returns (:385-405): the input's and
the adapters' (PEFT's lhs / rhs), none for the frozen stack, its scale, the offsets or the bias.
"""

import numpy as np

from .quant import bf16


def _segments(offsets):
    start = 0
    for e, end in enumerate(np.asarray(offsets, dtype=np.int64).tolist()):
        yield e, start, end
        start = end


def _base(weight, scale, e):
    w = np.asarray(weight[e], dtype=np.float32)
    if scale is not None:
        w = w * np.float32(scale[e])
    return w


def _factors(lhs, rhs, e, is_transposed):
    """(F1 (in, r), F2 (r, out)) with x @ delta^T (or x @ delta) = (x @ F1) @ F2."""
    l, r = np.asarray(lhs[e], dtype=np.float32), np.asarray(rhs[e], dtype=np.float32)
    return (l, r) if is_transposed else (r.T, l.T)


def lora_forward(x, weight, scale, offsets, is_transposed, lhs=None, rhs=None, scaling=1.0, bias=None):
    """Per expert y = x_e @ (W_e * scale_e)^T + s * (x_e @ F1_e) @ F2_e + bias_e (float32), the adapters applied
    as two products of rank depth as _moe._grouped_lora does (_moe.py:48-67); equal to reference_lora's
    x @ (W + s lhs @ rhs)^T (_grouped.py:431-444) up to float32 rounding. Rows past offsets[-1] come out zero.
    """
    x = np.asarray(x, dtype=np.float32)
    n = weight.shape[2] if is_transposed else weight.shape[1]
    out = np.zeros((x.shape[0], n), dtype=np.float32)
    for e, start, end in _segments(offsets):
        if end == start:
            continue
        w = _base(weight, scale, e)
        xe = x[start:end]
        y = xe @ (w if is_transposed else w.T)
        if lhs is not None:
            f1, f2 = _factors(lhs, rhs, e, is_transposed)
            y = y + np.float32(scaling) * ((xe @ f1) @ f2)
        if bias is not None:
            y = y + np.asarray(bias[e], dtype=np.float32)
        out[start:end] = y
    return out


def lora_low(x, offsets, is_transposed, lhs, rhs):
    """The rank panel x_e @ A_e^T the kernel keeps for the backward pass (_grouped.py:168,208,212-214)."""
    x = np.asarray(x, dtype=np.float32)
    rank = lhs.shape[2]
    low = np.zeros((x.shape[0], rank), dtype=np.float32)
    for e, start, end in _segments(offsets):
        a = np.asarray(lhs[e], dtype=np.float32) if is_transposed else np.asarray(rhs[e], dtype=np.float32).T
        low[start:end] = x[start:end] @ a
    return low


def lora_backward(x, grad, weight, scale, offsets, is_transposed, lhs=None, rhs=None, scaling=1.0):
    """Gradients of lora_forward: (grad_x, grad_lhs, grad_rhs), float32; grad_lhs/rhs None without adapters.

    grad_x = g @ W_e (the stack read the other way) + s (g @ F2^T) @ F1^T; dF1 = s x^T (g @ F2^T),
    dF2 = s (x @ F1)^T g, mapped back to PEFT's lhs / rhs (_grouped.py:385-405).
    """
    x = np.asarray(x, dtype=np.float32)
    g = np.asarray(grad, dtype=np.float32)
    grad_x = np.zeros_like(x)
    grad_lhs = np.zeros(lhs.shape, dtype=np.float32) if lhs is not None else None
    grad_rhs = np.zeros(rhs.shape, dtype=np.float32) if rhs is not None else None
    s = np.float32(scaling)
    for e, start, end in _segments(offsets):
        if end == start:
            continue
        w = _base(weight, scale, e)
        xe, ge = x[start:end], g[start:end]
        gx = ge @ (w.T if is_transposed else w)
        if lhs is not None:
            f1, f2 = _factors(lhs, rhs, e, is_transposed)
            g2 = ge @ f2.T                      # (rows, r)
            gx = gx + s * (g2 @ f1.T)
            d_f1 = s * (xe.T @ g2)              # (in, r)
            d_f2 = s * ((xe @ f1).T @ ge)       # (r, out)
            if is_transposed:                    # F1 = lhs, F2 = rhs
                grad_lhs[e], grad_rhs[e] = d_f1, d_f2
            else:                                # F1 = rhs^T, F2 = lhs^T
                grad_lhs[e], grad_rhs[e] = d_f2.T, d_f1.T
        grad_x[start:end] = gx
    return grad_x, grad_lhs, grad_rhs


def fp8_product(x, codes, scale, offsets, is_transposed, lhs=None, rhs=None, scaling=1.0, bias=None, block=128,
                block_scale=None):
    """The reference's FP8 product (_grouped.py:141-146,194-219 with W_FP8 and X_FP8), float32, tiles of `block`
    columns: per expert, acc = sum over k-blocks b of (x8_b @ W8_b) * xscale[b, row]; acc *= scale_e;
    acc += s * bf16(x @ F1) @ F2 (the adapters multiply the bf16 x, the panel rounded to bf16 as the kernel's
    `low`); + bias_e. codes: the e4m3 stack as stored ((E, out, in), or (E, in, out) when is_transposed).
    block_scale: None, or a function (e, b, c) -> the stack's scale of k-block b and 128-column block c (a
    block-scaled stack; then scale is None).
    """
    from .quant import e4m3_to_f32, quantize_rows

    x = np.asarray(x, dtype=np.float32)
    x8, xs = quantize_rows(x, block)
    xv = e4m3_to_f32(x8)
    n = codes.shape[2] if is_transposed else codes.shape[1]
    k = x.shape[1]
    out = np.zeros((x.shape[0], n), dtype=np.float32)
    for e, start, end in _segments(offsets):
        if end == start:
            continue
        w = e4m3_to_f32(codes[e])
        w = w if is_transposed else w.T  # (k, n)
        acc = np.zeros((end - start, n), dtype=np.float32)
        for b in range(-(-k // block)):
            ks = slice(b * block, min(k, (b + 1) * block))
            part = (xv[start:end, ks] @ w[ks]).astype(np.float32)
            factor = xs[b, start:end][:, None]
            if block_scale is not None:
                cols = np.array([block_scale(e, b, c // 128) for c in range(n)], dtype=np.float32)[None, :]
                factor = (factor * cols).astype(np.float32)
            acc = acc + part * factor
        if scale is not None:
            acc = acc * np.float32(scale[e])
        if lhs is not None:
            f1, f2 = _factors(lhs, rhs, e, is_transposed)
            acc = acc + np.float32(scaling) * (bf16(x[start:end] @ f1) @ f2)
        if bias is not None:
            acc = acc + np.asarray(bias[e], dtype=np.float32)
        out[start:end] = acc
    return out


def silu(v):
    v = np.asarray(v, dtype=np.float32)
    return (v / (np.float32(1.0) + np.exp(-v))).astype(np.float32)


def swiglu(gate_up, round_bf16=False):
    """Transformers' _default_apply_gate: gate, up = chunk(2, -1); silu(gate) * up.

    round_bf16: the gate on bf16 tensors, as PyTorch computes it there: act = bf16(silu(gate)), h = bf16(act * up).
    """
    gu = np.asarray(gate_up, dtype=np.float32)
    i = gu.shape[1] // 2
    if round_bf16:
        return bf16(bf16(silu(gu[:, :i])) * gu[:, i:])
    return silu(gu[:, :i]) * gu[:, i:]


def swiglu_backward(gate_up, grad_h, round_bf16=False):
    """d/d(gate, up) of silu(gate) * up: (dh * up * silu'(gate), dh * silu(gate)) concatenated.

    round_bf16: autograd's gradients on bf16 tensors: d_act = bf16(dh * up), d_up = bf16(dh * bf16(silu(gate))),
    d_gate = bf16(d_act * sigmoid(gate) * (1 + gate * (1 - sigmoid(gate)))) (SiLU's backward in float32, rounded).
    """
    gu = np.asarray(gate_up, dtype=np.float32)
    i = gu.shape[1] // 2
    g, u = gu[:, :i], gu[:, i:]
    sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
    dh = np.asarray(grad_h, dtype=np.float32)
    if round_bf16:
        d_act = bf16(dh * u)
        dg = bf16(d_act * sig * (np.float32(1.0) + g * (np.float32(1.0) - sig)))
        du = bf16(dh * bf16(silu(g)))
        return np.concatenate([dg, du], axis=1).astype(np.float32)
    dg = dh * u * sig * (np.float32(1.0) + g * (np.float32(1.0) - sig))
    du = dh * g * sig
    return np.concatenate([dg, du], axis=1).astype(np.float32)


def reduce_adapter(g, low, offsets, scaling):
    """_grouped._reduce (_grouped.py:233-256,362-370): out[e, n, r] = s * sum over expert e's rows of g[row, n] * low[row, r]."""
    g = np.asarray(g, dtype=np.float32)
    low = np.asarray(low, dtype=np.float32)
    offs = np.asarray(offsets)
    out = np.zeros((offs.size, g.shape[1], low.shape[1]), dtype=np.float32)
    for e, start, end in _segments(offs):
        out[e] = np.float32(scaling) * (g[start:end].T @ low[start:end])
    return out
