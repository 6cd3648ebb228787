"""Routing permutation, tile map and un-permute, restated in numpy (test infrastructure; see oracle/__init__.py)."""

import numpy as np

from .quant import bf16


def route(top_k_index, num_experts: int) -> dict:
    """The permutation of ``meepsquared/_moe.py:75-87``.

    expert_ids = top_k_index.reshape(-1); ``expert_ids_g, perm = sort(expert_ids)`` (:79) with a STABLE order
    (ties keep their flat position, which is what CUDA's radix sort gives and what the kernel defines);
    tokens_per_expert = histc over [0, E-1] (:82-83), offsets = int32 cumsum (:84); ids >= E are sentinels
    (:85-86): they sort last, are not counted, and their ids are clamped to E-1. inverse[perm[i]] = i (:124-125).
    """
    ids = np.asarray(top_k_index, dtype=np.int64).reshape(-1)
    perm = np.argsort(ids, kind="stable").astype(np.int64)
    ids_sorted = ids[perm]
    counts = np.bincount(ids[(ids >= 0) & (ids < num_experts)], minlength=num_experts)[:num_experts]
    offsets = np.cumsum(counts).astype(np.int32)
    inverse = np.empty_like(perm)
    inverse[perm] = np.arange(perm.size, dtype=np.int64)
    return {"perm": perm, "expert_ids_g": np.minimum(ids_sorted, num_experts - 1), "offsets": offsets,
            "inverse": inverse, "sentinel": ids_sorted >= num_experts}


def gather(hidden, perm, top_k: int, sentinel=None) -> np.ndarray:
    """selected = hidden[perm // k] (_moe.py:80), rows of sentinels zeroed (:87)."""
    sel = np.asarray(hidden)[np.asarray(perm) // top_k].copy()
    if sentinel is not None:
        sel[np.asarray(sentinel)] = 0
    return sel


def unpermute(y, weights_g, inverse, num_tokens: int, top_k: int, round_bf16: bool = False) -> np.ndarray:
    """_moe.py:123-126: sum over a token's k slots of y[row] * w_g[row], rows found through ``inverse``.

    With round_bf16 the result is rounded to bf16, as ``.to(hidden_states.dtype)`` does for a bf16 model.
    """
    weighted = np.asarray(y, dtype=np.float32) * np.asarray(weights_g, dtype=np.float32)[:, None]
    out = weighted[np.asarray(inverse)].reshape(num_tokens, top_k, -1).sum(axis=1, dtype=np.float32)
    return bf16(out) if round_bf16 else out


def unpermute_backward(grad_out, y, weights_g, perm, top_k: int):
    """Gradients of the un-permute: grad_y[p] = grad_out[perm[p] // k] * w_g[p], grad_w_g[p] = <grad_out[tok], y[p]>."""
    g = np.asarray(grad_out, dtype=np.float32)[np.asarray(perm) // top_k]
    grad_y = g * np.asarray(weights_g, dtype=np.float32)[:, None]
    grad_w = (g * np.asarray(y, dtype=np.float32)).sum(axis=1, dtype=np.float32)
    return grad_y, grad_w


def max_tiles(rows: int, experts: int, block_m: int = 128) -> int:
    """_grouped.max_tiles (_grouped.py:83-85): every expert's last tile may be partial."""
    return rows // block_m + experts


def tile_map(offsets, rows: int, block_m: int = 128):
    """_grouped.tile_map (_grouped.py:88-103): (tile_expert, tile_row, tiles).

    Each expert's rows are cut into ceil(rows_e / block_m) tiles; the arrays have max_tiles entries and the
    spare ones hold the last expert.
    """
    offsets = np.asarray(offsets, dtype=np.int64)
    experts = offsets.size
    starts = np.concatenate([[0], offsets[:-1]])
    per_expert = (offsets - starts + block_m - 1) // block_m
    ends = np.cumsum(per_expert)
    t = np.arange(max_tiles(rows, experts, block_m))
    tile_expert = np.minimum(np.searchsorted(ends, t, side="right"), experts - 1)
    tile_row = starts[tile_expert] + (t - (ends - per_expert)[tile_expert]) * block_m
    return tile_expert.astype(np.int32), tile_row.astype(np.int32), int(ends[-1])


def router(logits, top_k: int, norm_topk_prob: bool = True):
    """The router of Transformers' MoE blocks after its linear layer (Qwen3MoeTopKRouter.forward, transformers
    models/qwen3_moe/modeling_qwen3_moe.py): probs = softmax(logits) in float32 over the experts, the top_k largest
    in descending order (a tie to the smaller expert index), their probabilities divided by their sum when
    norm_topk_prob. Returns (probs (T, E), top_k_weights (T, k), top_k_index (T, k) int64), float32."""
    x = np.asarray(logits, dtype=np.float32)
    e = np.exp(x - x.max(axis=1, keepdims=True))
    probs = (e / e.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    order = np.argsort(-probs, axis=1, kind="stable")[:, :top_k]  # stable: equal values keep the smaller index
    top = np.take_along_axis(probs, order, axis=1)
    if norm_topk_prob:
        top = (top / top.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return probs, top, order.astype(np.int64)
