"""Number formats of the path, restated in numpy (test infrastructure; see oracle/__init__.py).

* bf16: round-to-nearest-even from float32, as PyTorch's ``.to(torch.bfloat16)``.
* e4m3 (OCP FP8 E4M3, PyTorch ``float8_e4m3fn``): decode exactly; encode with
  round-to-nearest-even, values of magnitude >= 480 (and the band rounding past
  448) give the NaN code 0x7F, as ``torch.float8_e4m3fn`` casts do.
* Per-expert FP8 stacks: ``meepsquared/_fp8.py:122-134``.
* The activations of an FP8 product, per row and tile: ``meepsquared/_grouped.py:194-197``.
* 128x128 block FP8: ``meepsquared/_vendor/axolotl/quantize.py:131-157``
  (dequantize, multiply in bf16) and ``:238-263`` (quantize, clamp to +-448).
* NF4 with double-quantised absmax: the format bitsandbytes 0.50.2 implements
  and ``quantize.py:52-101`` calls (``cdequantize_blockwise_fp32`` then
  ``+= offset`` then ``cdequantize_blockwise_bf16_nf4``).  Written from the QLoRA
  paper's definition; parity unpinned (bitsandbytes is not installed).
"""

import numpy as np

E4M3_MAX = 448.0
NF4_BLOCK = 64
ABSMAX_BLOCK = 256


# ----------------------------------------------------------------------------- bf16

def bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even; NaN stays NaN."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    b = f.view(np.uint32)
    # in uint32: no finite value (nor an infinity) overflows b + 0x8000; NaNs are set below
    rounded = ((b + (np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1)))) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def bf16_to_f32(bits) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32, exact."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16(x) -> np.ndarray:
    """x rounded to bf16 and returned as float32 (the value a bf16 tensor holds)."""
    return bf16_to_f32(bf16_bits(x))


# ----------------------------------------------------------------------------- e4m3

def e4m3_to_f32(codes) -> np.ndarray:
    """e4m3 codes (uint8) -> float32, exact. 0x7F / 0xFF are NaN; the format has no infinity."""
    c = np.asarray(codes, dtype=np.uint8).astype(np.int32)
    sign = np.where(c & 0x80, -1.0, 1.0).astype(np.float32)
    e = (c >> 3) & 0xF
    m = (c & 0x7).astype(np.float32)
    mag = np.where(e == 0, m * np.float32(2.0 ** -9), (1.0 + m / 8.0) * np.exp2(e.astype(np.float32) - 7.0))
    out = (sign * mag).astype(np.float32)
    out[(c & 0x7F) == 0x7F] = np.nan
    return out


def f32_to_e4m3(x) -> np.ndarray:
    """float32 -> e4m3 codes with round-to-nearest-even (PyTorch's float8_e4m3fn cast)."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    bits = f.view(np.uint32)
    sign = ((bits >> 24) & 0x80).astype(np.uint8)
    mag_bits = bits & 0x7FFFFFFF
    mag = mag_bits.view(np.float32)
    out = np.zeros(f.shape, dtype=np.uint8)
    # >= 480 (the first value past 448's rounding band) and NaN: the NaN code
    nan = (mag_bits >= np.uint32(1087 << 20)) | np.isnan(f)
    # below 2^-6 the result is subnormal: add 2^-6 * 2^... so that the float adder rounds at 2^-9
    small = (mag_bits < np.uint32(121 << 23)) & ~nan
    normal = ~nan & ~small
    if small.any():
        shifted = (mag[small] + np.float32(2.0 ** 14)).astype(np.float32)  # ulp of 2^14 in float32 is 2^-9
        out[small] = (shifted.view(np.uint32) - np.uint32(141 << 23)).astype(np.uint8)
    if normal.any():
        nb = mag_bits[normal].astype(np.int64)
        odd = (nb >> 20) & 1
        nb = nb - (120 << 23) + 0x7FFFF + odd  # rebias the exponent (127 -> 7), round to nearest even at bit 20
        out[normal] = ((nb >> 20) & 0xFF).astype(np.uint8)
    out[nan] = 0x7F
    return out | sign


# ----------------------------------------------------------------------------- FP8 stacks, one scale per expert

def quantize_stack(weight) -> tuple[np.ndarray, np.ndarray]:
    """_fp8.quantize_stack (_fp8.py:122-128): scale_e = max(amax_e, 1e-12) / 448, codes = e4m3(float32(w) / scale_e)."""
    w = np.asarray(weight, dtype=np.float32)
    amax = np.abs(w.reshape(w.shape[0], -1)).max(axis=1).astype(np.float32)
    scale = (np.maximum(amax, np.float32(1e-12)) / np.float32(E4M3_MAX)).astype(np.float32)
    q = (w / scale.reshape(-1, *([1] * (w.ndim - 1)))).astype(np.float32)
    return f32_to_e4m3(q), scale


def dequantize_stack(codes, scale) -> np.ndarray:
    """_fp8.dequantize_stack (_fp8.py:131-134, kernel :69-79): bf16(float32(w8) * scale_e), one rounding."""
    v = e4m3_to_f32(codes)
    s = np.asarray(scale, dtype=np.float32).reshape(-1, *([1] * (v.ndim - 1)))
    return bf16_bits((v * s).astype(np.float32))


# ----------------------------------------------------------------------------- activations of an FP8 product

def quantize_rows(x, block=128) -> tuple[np.ndarray, np.ndarray]:
    """The x tile quantisation of the reference's FP8 product (_grouped.py:194-197), tiles of `block` columns:
    per row r and block b, scale = max(max |x[r, block b]|, 1e-12) / 448 (float32), codes = e4m3(x / scale).

    Returns (codes (rows, k) uint8, scales (ceil(k/block), rows) float32: scales[b, r]).
    """
    x = np.asarray(x, dtype=np.float32)
    rows, k = x.shape
    nb = -(-k // block)
    padded = np.zeros((rows, nb * block), dtype=np.float32)
    padded[:, :k] = x
    blocks = padded.reshape(rows, nb, block)
    scale = (np.maximum(np.abs(blocks).max(axis=2), np.float32(1e-12)) / np.float32(E4M3_MAX)).astype(np.float32)
    q = (blocks / scale[:, :, None]).astype(np.float32).reshape(rows, nb * block)[:, :k]
    return f32_to_e4m3(q), np.ascontiguousarray(scale.T)


# ----------------------------------------------------------------------------- FP8 with 128x128 block scales

def quantize_fp8_blocks(weight, grid=None, block=128) -> tuple[np.ndarray, np.ndarray]:
    """quantize.quantize_fp8 (quantize.py:238-263) for a 2-D weight and a 2-D scale grid (sr, sc).

    The grid defaults to (ceil(rows/128), ceil(cols/128)); as in the reference the block is
    (ceil(rows/sr), ceil(cols/sc)), which is 128x128 when the sizes are multiples of 128.
    scale = max(amax_block, 1e-12) / 448 (float32); codes = e4m3(clamp(w / scale, +-448)).
    """
    w = np.asarray(weight, dtype=np.float32)
    rows, cols = w.shape
    sr, sc = grid if grid is not None else (-(-rows // block), -(-cols // block))
    br, bc = -(-rows // sr), -(-cols // sc)
    padded = np.zeros((sr * br, sc * bc), dtype=np.float32)
    padded[:rows, :cols] = w
    blocks = padded.reshape(sr, br, sc, bc)
    scale = (np.maximum(np.abs(blocks).max(axis=(1, 3)), np.float32(1e-12)) / np.float32(E4M3_MAX)).astype(np.float32)
    q = (blocks / scale[:, None, :, None]).astype(np.float32).reshape(padded.shape)[:rows, :cols]
    q = np.clip(q, -E4M3_MAX, E4M3_MAX).astype(np.float32)
    return f32_to_e4m3(q), scale


def dequantize_fp8_blocks(codes, scale_inv) -> np.ndarray:
    """quantize.dequantize_fp8 (quantize.py:131-157), dtype bf16: bf16(bf16(w8) * bf16(s)), multiply rounded once.

    Handles the tail-block case (:148-156) by ceil-divided block sizes; returns bf16 bits.
    """
    c = np.asarray(codes, dtype=np.uint8)
    rows, cols = c.shape
    s = bf16(np.asarray(scale_inv, dtype=np.float32))
    sr, sc = s.shape
    br, bc = -(-rows // sr), -(-cols // sc)
    expanded = np.repeat(np.repeat(s, br, axis=0), bc, axis=1)[:rows, :cols]
    w = e4m3_to_f32(c)  # e4m3 -> bf16 is exact
    return bf16_bits((w * expanded).astype(np.float32))


# ----------------------------------------------------------------------------- NF4, double-quantised absmax

# The 16 NormalFloat-4 levels of the QLoRA paper (Dettmers et al., 2023, appendix E), as float32.
# tests/test_oracle_quant.py rebuilds them from the paper's construction with scipy.
NF4_LEVELS = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0], dtype=np.float32)


def nf4_levels_from_construction() -> np.ndarray:
    """The NF4 levels from the paper's construction: normal quantiles from offset 0.9677 to 0.5, scaled to [-1, 1]."""
    from scipy.stats import norm

    offset = 0.9677083
    pos = norm.ppf(np.linspace(offset, 0.5, 9)[:-1])
    neg = -norm.ppf(np.linspace(offset, 0.5, 8)[:-1])
    v = np.sort(np.concatenate([pos, [0.0], neg]))
    return (v / v.max()).astype(np.float32)


def dynamic_map(signed=True, max_exponent_bits=7, total_bits=8) -> np.ndarray:
    """The 8-bit dynamic (exponent + fraction) code of 8-bit blockwise quantisation (Dettmers et al., 2022).

    For exponent i in 0..6 the code holds 2^i fraction levels (midpoints of an even split of [0.1, 1]) times
    10^(i-6), with both signs, plus 0 and 1: 256 sorted float32 values. Used as code2 for the absmax.
    """
    data = []
    non_sign_bits = total_bits - 1
    for i in range(max_exponent_bits):
        items = 2 ** (i + non_sign_bits - max_exponent_bits) + 1 if signed else 2 ** (i + non_sign_bits - max_exponent_bits + 1) + 1
        bounds = np.linspace(0.1, 1, items, dtype=np.float32)
        means = (bounds[:-1] + bounds[1:]) / np.float32(2.0)
        data += (np.float32(10.0 ** (-(max_exponent_bits - 1) + i)) * means).tolist()
        if signed:
            data += (-np.float32(10.0 ** (-(max_exponent_bits - 1) + i)) * means).tolist()
    data += [0.0, 1.0]
    data += [0.0] * (2 ** total_bits - len(data))
    return np.sort(np.array(data, dtype=np.float32))


def _nearest(values, levels) -> np.ndarray:
    """Index of the nearest level (levels sorted ascending); a tie takes the upper level."""
    idx = np.searchsorted(levels, values)
    idx = np.clip(idx, 1, len(levels) - 1)
    lo, hi = levels[idx - 1], levels[idx]
    return np.where(np.abs(values - lo) < np.abs(hi - values), idx - 1, idx)


def quantize_nf4(weight, blocksize=NF4_BLOCK, blocksize2=ABSMAX_BLOCK) -> dict:
    """NF4 with double quantisation (QLoRA): the state bitsandbytes' ``quantize_4bit(..., compress_statistics=True)`` keeps.

    Flattened weight in blocks of 64: absmax_b = max|w|, codes = nearest NF4 level of w / absmax_b, two codes a
    byte, the first in the high nibble. The absmax vector: offset = mean, (absmax - offset) in blocks of 256 with
    absmax2 = max|.| per block and an 8-bit index into the dynamic map (code2).
    """
    w = np.asarray(weight, dtype=np.float32).reshape(-1)
    if w.size % blocksize or w.size % 2:
        raise ValueError("the flattened weight must split into whole blocks")
    blocks = w.reshape(-1, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax == 0, np.float32(1.0), absmax)
    codes = _nearest((blocks / safe[:, None]).astype(np.float32).reshape(-1), NF4_LEVELS).astype(np.uint8)
    packed = ((codes[0::2] << 4) | codes[1::2]).astype(np.uint8)
    offset = np.float32(absmax.mean(dtype=np.float32))
    centred = (absmax - offset).astype(np.float32)
    n2 = -(-centred.size // blocksize2)
    padded = np.zeros(n2 * blocksize2, dtype=np.float32)
    padded[:centred.size] = centred
    absmax2 = np.abs(padded.reshape(n2, blocksize2)).max(axis=1).astype(np.float32)
    safe2 = np.where(absmax2 == 0, np.float32(1.0), absmax2)
    code2 = dynamic_map()
    normed = (padded.reshape(n2, blocksize2) / safe2[:, None]).astype(np.float32).reshape(-1)[:centred.size]
    absmax_q = _nearest(normed, code2).astype(np.uint8)
    return {"packed": packed, "absmax": absmax_q, "absmax2": absmax2, "code2": code2, "offset": offset,
            "blocksize": blocksize, "blocksize2": blocksize2, "shape": tuple(np.shape(weight))}


def dequantize_nf4_absmax(absmax_q, absmax2, code2, offset, blocksize2=ABSMAX_BLOCK) -> np.ndarray:
    """First stage (quantize.py:74-83): absmax_f32[i] = code2[absmax_q[i]] * absmax2[i // 256], then + offset.

    Two float32 operations, each rounded (a multiply, then the separate ``+=``): no fused multiply-add.
    """
    q = np.asarray(absmax_q, dtype=np.uint8)
    scaled = (np.asarray(code2, dtype=np.float32)[q] * np.asarray(absmax2, dtype=np.float32)[np.arange(q.size) // blocksize2])
    return (scaled.astype(np.float32) + np.float32(offset)).astype(np.float32)


def dequantize_nf4(state) -> np.ndarray:
    """Second stage (quantize.py:85-96): w = bf16(NF4[code] * absmax_f32[i // 64]) as bf16 bits, in ``shape``."""
    absmax = dequantize_nf4_absmax(state["absmax"], state["absmax2"], state["code2"], state["offset"],
                                   state["blocksize2"])
    packed = np.asarray(state["packed"], dtype=np.uint8)
    codes = np.empty(packed.size * 2, dtype=np.uint8)
    codes[0::2] = packed >> 4
    codes[1::2] = packed & 0xF
    vals = (NF4_LEVELS[codes] * absmax[np.arange(codes.size) // state["blocksize"]]).astype(np.float32)
    return bf16_bits(vals).reshape(state["shape"])
