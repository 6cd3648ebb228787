"""The experts' products with their LoRA adapters, one launch each, on a B200: the drop-in for meepsquared._grouped.

Same operator API as ``meepsquared/_grouped.py`` (``lora_linear`` :408-417, ``grouped_linear`` :348-359,
``tile_map`` :88-103, ``max_tiles`` :83-85, ``wanted`` :57-67, ``fp8_products`` :70-80, ``available``
:259-261, ``reference`` / ``reference_lora`` :420-444, the constants), same argument meaning and errors. The rows
of x are sorted by expert, offsets[e] is the end of expert e's rows (int32, on the device), and for every expert

    out_e = scale_e * x_e @ W_e^T + s * (x_e @ A_e^T) @ B_e^T + bias_e

with the stack W as (experts, out, in), or (experts, in, out) when is_transposed, addressed through its strides
(either memory order is read in place). The computation is libmeep2b's persistent tcgen05 GEMM
(csrc/grouped_gemm.cu): TMA-fed, accumulators in tensor memory, the rank panel x_e @ A_e^T computed by the same
MMA as the product, the adapter's second factor applied by one more MMA of depth 16. The backward pass is the
same kernel with the stack read the other way round and the adapters' roles swapped, plus one reduction kernel
per adapter (csrc/reduce.cu). The frozen stack gets no gradient. There is no other implementation: without the
library or a compute capability 10.0 GPU the functions raise.
"""

import os

import types

import torch

from . import _lib

BLOCK_M = 128  # rows per tile: the M of the tcgen05 MMA
RANK_MULTIPLE = 16  # the rank is padded to one MMA depth
# PyTorch has grouped matmul kernels of its own for these (the reference's constant, kept for the API)
TORCH_HAS_GROUPED_MM = (9, 10)


def available() -> bool:
    """Whether the kernels can run here: libmeep2b loads and the current CUDA GPU has compute capability 10.0."""
    if not torch.cuda.is_available() or not _lib.loaded():
        return False
    return _lib.device_ok(torch.cuda.current_device())


def wanted(device) -> bool:
    """Whether the kernels compute the experts on `device`: a compute capability 10.0 GPU with libmeep2b loaded.

    MEEPSQUARED_GROUPED_KERNEL=0 or 1 overrides the decision, as in the reference.
    """
    forced = os.environ.get("MEEPSQUARED_GROUPED_KERNEL")
    if forced in ("0", "1"):
        return forced == "1"
    if device.type != "cuda" or not torch.cuda.is_available() or not _lib.loaded():
        return False
    index = device.index if device.index is not None else torch.cuda.current_device()
    return _lib.device_ok(index)


def fp8_products(device) -> bool:
    """Whether an FP8 stack's products run on the FP8 tensor cores, activations quantized per row: off unless
    MEEPSQUARED_FP8_PRODUCTS=1, as in the reference."""
    return os.environ.get("MEEPSQUARED_FP8_PRODUCTS") == "1"


def max_tiles(rows: int, experts: int, block_m: int = BLOCK_M) -> int:
    """An upper bound on the tiles: every expert's last tile may be partial."""
    return rows // block_m + experts


def _require(t: torch.Tensor, what: str):
    if not t.is_cuda:
        raise RuntimeError(f"{what} runs on a CUDA GPU (compute capability 10.0); got a tensor on {t.device}")
    _lib.load()


def tile_map(offsets: torch.Tensor, rows: int, block_m: int = BLOCK_M):
    """(tile_expert, tile_row, tiles) for `rows` rows sorted by expert, built on the device by one kernel.

    offsets[e] is the end of expert e's rows (int32). The two int32 arrays have max_tiles entries; tiles, a 0-d
    int32 tensor on the device, says how many are real. Entries beyond that hold the last expert.
    """
    _require(offsets, "tile_map")
    offsets = offsets.to(torch.int32).contiguous()
    experts = offsets.numel()
    n = max_tiles(rows, experts, block_m)
    tile_expert = torch.empty(n, dtype=torch.int32, device=offsets.device)
    tile_row = torch.empty(n, dtype=torch.int32, device=offsets.device)
    tiles = torch.empty((), dtype=torch.int32, device=offsets.device)
    _lib.check(_lib.load().meep2b_tile_map(_lib.ptr(offsets), experts, rows, block_m, _lib.ptr(tile_expert),
                                           _lib.ptr(tile_row), _lib.ptr(tiles), _lib.stream_of(offsets)),
               "meep2b_tile_map")
    return tile_expert, tile_row, tiles


class TileMaps:
    """The tile maps of one set of offsets: built on the device on first use per tile height, then kept.

    Tiles of 128 rows feed the one-CTA kernel; tiles of 256 rows the CTA-pair kernel (stacks read K-major).
    """

    def __init__(self, offsets: torch.Tensor, rows: int):
        self.offsets, self.rows, self._maps = offsets, rows, {}

    def get(self, block_m: int):
        if block_m not in self._maps:
            self._maps[block_m] = tile_map(self.offsets, self.rows, block_m)
        return self._maps[block_m]


def _pair_tiles(b_mn: int, rows: int, experts: int, k: int, adapters: bool, quant_kind=None) -> bool:
    """Whether a product runs on CTA pairs (tiles of 256 rows). A bf16 stack runs on one CTA: with the epilogue's
    tiles going out by TMA stores from shared memory, the one-CTA kernel (4 stages, tiles of 128 rows, about half
    the padding rows at an expert's end) measures faster than the pair (6 stages) on every product of the
    BASELINE shapes (config-2 gate/up forward 817 against 860-873 us). A quantised stack (quant_kind, dequantised
    in shared memory) goes to pairs when it is NF4: each SM then converts half of the stack tile, which is what
    bounds the NF4 products (measured ~1.5x the one-CTA rate at config-2 size); e4m3 stacks stay on one CTA (the
    two forms measured alike). MN-major quantised products have no pair form. MEEP2B_PAIR=0 or 1 overrides."""
    forced = os.environ.get("MEEP2B_PAIR")
    if forced in ("0", "1"):
        return forced == "1"
    if quant_kind is not None:
        return quant_kind == _lib.NF4 and b_mn == 0 and rows >= 384 * experts
    return False


# ------------------------------------------------------------------------------------------------ layouts

def _stack_strides(weight: torch.Tensor, K: int, is_transposed: bool) -> int:
    """N of a stack addressed as (k, n); the reference's ValueErrors for a mismatch (_grouped.py:264-272)."""
    if is_transposed:
        if weight.shape[1] != K:
            raise ValueError(f"a transposed stack (experts, in, out) with in={weight.shape[1]} does not take x with {K} columns")
        return weight.shape[2]
    if weight.shape[2] != K:
        raise ValueError(f"a stack (experts, out, in) with in={weight.shape[2]} does not take x with {K} columns")
    return weight.shape[1]


def _stack_memory(weight: torch.Tensor, k_contiguous_layout: bool):
    """The stack as the kernel reads it: (tensor, b_mn).

    The product contracts over k. With b_mn=0 the kernel takes (experts, n, k) with k contiguous, with b_mn=1
    (experts, k, n) with n contiguous. `k_contiguous_layout` says whether the logical layout is (experts, n, k).
    A stack stored in the other order is read in place with the other mode; any other strides are copied.
    """
    if k_contiguous_layout:  # logical (E, n, k)
        if weight.is_contiguous():
            return weight, 0
        t = weight.transpose(1, 2)
        if t.is_contiguous():
            return t, 1
        return weight.contiguous(), 0
    if weight.is_contiguous():  # logical (E, k, n)
        return weight, 1
    t = weight.transpose(1, 2)
    if t.is_contiguous():
        return t, 0
    return weight.contiguous(), 1


def _rank_rows(factor: torch.Tensor) -> torch.Tensor:
    """(E, r, D) -> (E, 16, D) bf16 contiguous, zero rows past the rank."""
    e, r, d = factor.shape
    if r == RANK_MULTIPLE and factor.dtype == torch.bfloat16 and factor.is_contiguous():
        return factor
    return torch.nn.functional.pad(factor.to(torch.bfloat16), (0, 0, 0, RANK_MULTIPLE - r)).contiguous()  # one pass


# Zero-padded panel buffers (E, D, width) per device and shape: the padding columns are zeroed once and only the
# rank's columns are written per use. A buffer is filled and read by the same product launch, in stream order, so
# products of different layers may share it.
_PADDED = {}


def _rank_cols(factor: torch.Tensor, width: int) -> torch.Tensor:
    """(E, D, r) -> (E, D, width) bf16 contiguous, zero columns past the rank (width 16 or 64). A padded copy lives
    in a buffer shared by every product of its shape: it is valid until the next call for that shape."""
    e, d, r = factor.shape
    if r == width and factor.dtype == torch.bfloat16 and factor.is_contiguous():
        return factor
    key = (factor.device, e, d, width, r)
    buf = _PADDED.get(key)
    if buf is None:
        buf = torch.zeros((e, d, width), device=factor.device, dtype=torch.bfloat16)
        _PADDED[key] = buf
    buf[:, :, :r].copy_(factor)
    return buf


class _Adapters:
    """PEFT's factors (lhs, rhs) in the kernel's layouts, for the forward product and for the backward one.

    delta = lhs @ rhs in the layout of the stack (reference _grouped.py:285-310): for a stack (E, out, in)
    lhs is (E, out, r) and rhs (E, r, in); for (E, in, out) lhs is (E, in, r) and rhs (E, r, out).
    A product computes rows @ F1 (the rank panel, rows x r) and then panel @ F2, F1 (E, k, r) and F2 (E, r, n).
    The kernel takes F1 as its panel P and F2 as its up factor U: with b_mn=0 P is (E, 16, k) and U (E, n, 16),
    with b_mn=1 P is (E, k, 16) and U (E, 16, n); the rank is padded with zeros.
    """

    def __init__(self, lhs, rhs, is_transposed):
        self.rank = lhs.shape[2]
        if self.rank > RANK_MULTIPLE:  # larger ranks go to the products in 16-rank chunks (_rank_chunks)
            raise NotImplementedError(f"LoRA rank {self.rank}: one fused panel takes ranks up to {RANK_MULTIPLE}")
        self.lhs, self.rhs, self.is_transposed = lhs, rhs, is_transposed

    def factors(self, backward: bool):
        """(F1, F2) of the forward product or of the input-gradient product."""
        lhs, rhs = self.lhs, self.rhs
        if not self.is_transposed:  # x @ delta^T = (x @ rhs^T) @ lhs^T; g @ delta = (g @ lhs) @ rhs
            return (lhs, rhs) if backward else (rhs.transpose(1, 2), lhs.transpose(1, 2))
        # x @ delta = (x @ lhs) @ rhs; g @ delta^T = (g @ rhs^T) @ lhs^T
        return (rhs.transpose(1, 2), lhs.transpose(1, 2)) if backward else (lhs, rhs)

    def operands(self, b_mn: int, backward: bool):
        """(P, U) of one product, for the launch that follows at once (a padded P lives in a shared buffer)."""
        f1, f2 = self.factors(backward)
        if b_mn == 0:
            return _rank_rows(f1.transpose(1, 2)), _rank_cols(f2.transpose(1, 2), 16)
        return _rank_cols(f1, RANK_MULTIPLE), _rank_rows(f2)


class QuantStack:
    """A frozen stack held quantised, read by the product as it is and dequantised in shared memory.

    codes: the stored (experts, rows, cols) stack, cols contiguous: e4m3 codes (uint8 or float8_e4m3fn), or NF4
    codes packed two a byte (experts, rows, cols / 2). kind: _lib.E4M3 (the per-expert scale goes to the product
    as `scale`), _lib.NF4 or _lib.E4M3_BLOCKS; for the last two `mult` holds the multiplier of each group of 64
    consecutive weights, (experts, cols/64, rows) float32 (meep2b_quant_multipliers): the block absmax (NF4), or
    the bf16 value of the block scale, blocks of ceil(rows/sr) x ceil(cols/sc) as the reference's dequantize_fp8
    sizes them for an (sr, sc) grid.
    """

    def __init__(self, codes: torch.Tensor, kind: int, shape, mult=None, grid=(0, 0)):
        self.codes, self.kind, self.shape, self.mult, self.grid = codes, kind, tuple(shape), mult, tuple(grid)
        self.device = codes.device

    @staticmethod
    def fits(shape) -> bool:
        """Whether the fused product takes the stack: whole 64-weight blocks along both matrix dimensions."""
        return shape[1] % 64 == 0 and shape[2] % 64 == 0

    @staticmethod
    def multipliers(kind, src, shape, grid=(0, 0)) -> torch.Tensor:
        e, rows, cols = shape
        out = torch.empty((e, cols // 64, rows), device=src.device, dtype=torch.float32)
        _lib.check(_lib.load().meep2b_quant_multipliers(kind, _lib.ptr(src.float().contiguous()), e, rows, cols,
                                                        grid[0], grid[1], _lib.ptr(out), _lib.stream_of(src)),
                   "meep2b_quant_multipliers")
        return out

    @classmethod
    def from_fp8(cls, weight8: torch.Tensor, scale: torch.Tensor):
        """An FP8 stack with one scale per expert (E4M3) or a grid of block scales (E4M3_BLOCKS) whose column
        blocks are whole 64-column groups; None if the product does not take it fused."""
        if not cls.fits(weight8.shape) or not weight8.is_contiguous():
            return None
        e, rows, cols = weight8.shape
        if scale.dim() == 1:
            return cls(weight8, _lib.E4M3, weight8.shape)
        if scale.dim() == 3 and scale.shape[0] == e and 0 < scale.shape[1] <= rows and 0 < scale.shape[2] <= cols:
            grid = (int(scale.shape[1]), int(scale.shape[2]))
            if (-(-cols // grid[1])) % 64 == 0:
                if not weight8.is_cuda:
                    return cls(weight8, _lib.E4M3_BLOCKS, weight8.shape, None, grid)
                mult = cls.multipliers(_lib.E4M3_BLOCKS, scale, weight8.shape, grid)
                return cls(weight8, _lib.E4M3_BLOCKS, weight8.shape, mult, grid)
        return None

    @classmethod
    def from_nf4(cls, state):
        """An NF4 stack (blocks of 64 along its rows); None if not fused."""
        if len(state.shape) != 3 or not cls.fits(state.shape) or state.blocksize != 64:
            return None
        return cls(state.packed, _lib.NF4, state.shape, state.multipliers())


def _launch(x, weight, scale, offsets, k_contiguous_layout, adapters, scaling, bias, store_low, backward=False,
            tiles=None, epilogue=_lib.EPI_PLAIN, aux=None, out=None, x_rows=None, row_scale=None, w_grad=None,
            out_rows=None):
    """One launch of the grouped product; returns (out, low). The reference's _launch (_grouped.py:313-345).

    k_contiguous_layout: whether the stack is logically (experts, n, k) for this product. x_rows (int32): the
    product's row i is row x_rows[i] of x (the routed rows read from the token-major tensor); row_scale (float32):
    product row i scaled by row_scale[i]; w_grad (dSwiGLU, float32 (rows, ceil(N/96))): <dh_i, h_i> per 96 columns;
    out_rows (int64, plain epilogue, bf16 stacks): product row i stored at row out_rows[i] of the output.
    """
    K = x.shape[1]
    rows = x_rows.numel() if x_rows is not None else x.shape[0]
    quant = isinstance(weight, QuantStack)
    if quant:  # stored (E, rows, cols) as it is: K-major when the product contracts over its columns
        stack, b_mn = weight.codes, 0 if k_contiguous_layout else 1
        experts, N = weight.shape[0], weight.shape[1] if b_mn == 0 else weight.shape[2]
        if weight.shape[2 if b_mn == 0 else 1] != K:
            raise ValueError(f"a quantised stack {weight.shape} does not take x with {K} columns")
    else:
        stack, b_mn = _stack_memory(weight, k_contiguous_layout)
        experts, N = stack.shape[0], stack.shape[1] if b_mn == 0 else stack.shape[2]
        if weight.dtype == torch.float8_e4m3fn:
            raise NotImplementedError("an FP8 stack goes to the product as a QuantStack or dequantized")
        if weight.dtype != torch.bfloat16:
            raise TypeError(f"the grouped kernel computes in bf16: stack {weight.dtype}")
    if x.dtype != torch.bfloat16:
        raise TypeError(f"the grouped kernel computes in bf16: x {x.dtype}")
    if x.stride(1) != 1 or x.stride(0) % 8:
        x = x.contiguous()
    if epilogue == _lib.EPI_SWIGLU:
        width = N // 2
    elif epilogue == _lib.EPI_DSWIGLU:
        width = 2 * N
    else:
        width = N
    if out is None:
        out = torch.empty((rows, width), device=x.device, dtype=x.dtype)
    low = None
    if adapters is not None and store_low:
        low = torch.empty((rows, RANK_MULTIPLE), device=x.device, dtype=torch.bfloat16)
    if rows == 0:
        return out, low
    if tiles is None:
        tiles = TileMaps(offsets, rows)
    pair_ok = (x_rows is None or b_mn == 0) and (not quant or b_mn == 0)  # quantised pairs: K-major only
    block_m = 256 if pair_ok and _pair_tiles(b_mn, rows, experts, K, adapters is not None,
                                             weight.kind if quant else None) else 128
    tmap = tiles.get(block_m)
    panel = up = None
    if adapters is not None:
        panel, up = adapters.operands(b_mn, backward)
    p = _lib.Product()
    p.x, p.rows, p.k, p.ldx = x.data_ptr(), rows, K, x.stride(0)
    p.weight, p.experts, p.n, p.b_mn = stack.data_ptr(), experts, N, b_mn
    p.weight_dtype = weight.kind if quant else _lib.BF16
    p.wscale = weight.mult.data_ptr() if quant and weight.mult is not None else None
    if x_rows is not None:
        p.x_rows, p.x_src_rows = x_rows.data_ptr(), x.shape[0]
    p.row_scale = row_scale.data_ptr() if row_scale is not None else None
    if w_grad is not None:
        p.w_grad, p.w_ld = w_grad.data_ptr(), w_grad.stride(0)
    if out_rows is not None:
        if out_rows.dtype != torch.int64 or out_rows.numel() != rows:
            raise ValueError("out_rows: one int64 destination row per product row")
        p.out_rows = out_rows.data_ptr()
    p.scale = scale.data_ptr() if scale is not None else None
    p.panel = panel.data_ptr() if panel is not None else None
    p.up = up.data_ptr() if up is not None else None
    p.scaling = float(scaling)
    p.bias = bias.data_ptr() if bias is not None else None
    p.offsets = offsets.data_ptr()
    p.tile_expert, p.tile_row, p.tiles = tmap[0].data_ptr(), tmap[1].data_ptr(), tmap[2].data_ptr()
    p.max_tiles = tmap[0].numel()
    p.out, p.ldo = out.data_ptr(), out.stride(0)
    p.low = low.data_ptr() if low is not None else None
    p.epilogue = epilogue
    p.aux = aux.data_ptr() if aux is not None else None
    p.sm_limit = 0
    p.block_m = block_m
    observer = _launch_observer
    if observer is not None:
        observer.before(x)
    _lib.check(_lib.load().meep2b_grouped_product(p, _lib.stream_of(x)), "meep2b_grouped_product")
    if observer is not None:
        rank = adapters.rank if adapters is not None else 0
        observer.after(x, 2 * rows * N * K + 2 * rows * rank * (N + K))
    return out, low


# An object with before(x) / after(x, flops) called around every grouped-product launch, on the launching
# stream's side (the benchmark records CUDA events there to time the kernel inside a step); None normally.
_launch_observer = None


def set_launch_observer(observer):
    global _launch_observer
    _launch_observer = observer


class Fp8Stack:
    """An e4m3 stack whose products run on the FP8 tensor cores (the reference's X_FP8 path, _grouped.py:141-146,
    194-197): the activations are quantised per row and 128-column tile, the codes of both multiply as they are,
    and the scales are applied to the float32 partial sums.

    codes: the stored (experts, rows, cols) stack, cols contiguous. scale: (experts,) float32 (one scale per
    expert, the reference's FP8 stack), or None with `blocks` = (scales (experts, sr, sc) float32, the block
    height, the block width) for a stack with a grid of block scales whose blocks are whole 128 x 128 tiles.
    """

    def __init__(self, codes, scale=None, blocks=None):
        self.codes, self.scale, self.blocks = codes, scale, blocks
        self.shape = tuple(codes.shape)

    @classmethod
    def of(cls, weight8: torch.Tensor, scale):
        """The stack for the FP8 products; NotImplementedError for sizes the kernel does not take."""
        e, rows, cols = weight8.shape
        if rows % 16 or cols % 16:
            raise NotImplementedError(f"FP8 products need stack sizes that are multiples of 16: {tuple(weight8.shape)}")
        codes = weight8.contiguous()
        if scale is None:
            return cls(codes)
        if scale.dim() <= 1:
            return cls(codes, scale.reshape(-1).to(torch.float32).contiguous())
        if scale.dim() == 3 and scale.shape[0] == e:
            sr, sc = int(scale.shape[1]), int(scale.shape[2])
            br, bc = -(-rows // sr), -(-cols // sc)
            if (br % 128 == 0 or sr == 1) and (bc % 128 == 0 or sc == 1):
                # the scale as the reference's dequantisation applies it: rounded to bf16 (quantize.py:131-157)
                return cls(codes, None, (scale.to(torch.bfloat16).float().contiguous(), br, bc))
        raise NotImplementedError(f"FP8 products take one scale per expert or 128 x 128 block scales, not "
                                  f"{tuple(scale.shape)} over {tuple(weight8.shape)}")


def _quantize_rows(x: torch.Tensor):
    """(codes (rows, k) uint8, scales (ceil(k/128), rows) float32): x quantised per row and 128-column tile."""
    rows, k = x.shape
    codes = torch.empty((rows, k), device=x.device, dtype=torch.uint8)
    scales = torch.empty((-(-k // 128), rows), device=x.device, dtype=torch.float32)
    if rows:
        _lib.check(_lib.load().meep2b_fp8_rows_quantize(_lib.ptr(x), rows, k, x.stride(0), _lib.ptr(codes),
                                                        _lib.ptr(scales), rows, _lib.stream_of(x)),
                   "meep2b_fp8_rows_quantize")
    return codes, scales


def _launch_f8(x, stack: Fp8Stack, offsets, k_contiguous_layout, adapters, scaling, bias, store_low, backward=False,
               tiles=None):
    """The FP8 product (meep2b_grouped_product_f8); returns (out, low) as _launch does."""
    if x.dtype != torch.bfloat16:
        raise TypeError(f"the grouped kernel computes in bf16: x {x.dtype}")
    if x.stride(1) != 1 or x.stride(0) % 8:
        x = x.contiguous()
    rows, K = x.shape
    b_mn = 0 if k_contiguous_layout else 1
    experts, srows, scols = stack.shape
    N = srows if b_mn == 0 else scols
    if (scols if b_mn == 0 else srows) != K:
        raise ValueError(f"an FP8 stack {stack.shape} does not take x with {K} columns")
    if K % 16:
        raise NotImplementedError(f"FP8 products need x with a multiple of 16 columns: {K}")
    out = torch.empty((rows, N), device=x.device, dtype=x.dtype)
    if tiles is None:
        tiles = TileMaps(offsets, rows)
    low = None
    up = None
    if adapters is not None:
        panel, up = adapters.operands(0, backward)  # (E, 16, K) and (E, N, 16)
        low = _launch(x, panel, None, offsets, True, None, 1.0, None, False, tiles=tiles)[0]
    if rows == 0:
        return out, (low if store_low else None)
    codes, xscale = _quantize_rows(x)
    tmap = tiles.get(128)
    p = _lib.ProductF8()
    p.x8, p.rows, p.k, p.xscale, p.ld_xscale = codes.data_ptr(), rows, K, xscale.data_ptr(), rows
    p.weight, p.experts, p.n, p.b_mn = stack.codes.data_ptr(), experts, N, b_mn
    p.scale = stack.scale.data_ptr() if stack.scale is not None else None
    if stack.blocks is not None:
        ws, br, bc = stack.blocks
        sr, sc = ws.shape[1], ws.shape[2]
        huge = 1 << 30
        div_r, div_c = (br // 128 if sr > 1 else huge), (bc // 128 if sc > 1 else huge)
        p.wblock, p.wb_stride_e = ws.data_ptr(), sr * sc
        if b_mn == 0:  # k runs along the stored columns, n along the rows
            p.wb_stride_k, p.wb_div_k, p.wb_stride_n, p.wb_div_n = 1, div_c, sc, div_r
        else:
            p.wb_stride_k, p.wb_div_k, p.wb_stride_n, p.wb_div_n = sc, div_r, 1, div_c
    p.low = low.data_ptr() if low is not None else None
    p.up = up.data_ptr() if up is not None else None
    p.scaling = float(scaling)
    p.bias = bias.data_ptr() if bias is not None else None
    p.offsets = offsets.data_ptr()
    p.tile_expert, p.tile_row, p.tiles = tmap[0].data_ptr(), tmap[1].data_ptr(), tmap[2].data_ptr()
    p.max_tiles = tmap[0].numel()
    p.out, p.ldo = out.data_ptr(), out.stride(0)
    p.sm_limit = 0
    observer = _launch_observer
    if observer is not None:
        observer.before(x)
    _lib.check(_lib.load().meep2b_grouped_product_f8(p, _lib.stream_of(x)), "meep2b_grouped_product_f8")
    if observer is not None:
        observer.after(x, 2 * rows * N * K)
    return out, (low if store_low else None)


def _product(x, weight, scale, offsets, k_contiguous_layout, adapters, scaling, bias, store_low, backward=False,
             tiles=None):
    """One grouped product over a bf16, quantised or FP8-products stack."""
    if isinstance(weight, Fp8Stack):
        return _launch_f8(x, weight, offsets, k_contiguous_layout, adapters, scaling, bias, store_low, backward,
                          tiles)
    return _launch(x, weight, scale, offsets, k_contiguous_layout, adapters, scaling, bias, store_low, backward,
                   tiles=tiles)


# widths of g whose gathered reductions take the whole-row form (the layer's hidden and upstream-gradient rows at
# the benchmarked shapes; the kernel is built for these three)
_FULL_ROW_WIDTHS = (768, 1536, 2048)


def _reduce(g: torch.Tensor, low: torch.Tensor, offsets: torch.Tensor, scaling: float, g_rows=None,
            row_scale=None, out=None, layout=0, tiles=None) -> torch.Tensor:
    """scaling * sum over each expert's rows of g^T @ low (_grouped.py:362-370), bf16: (experts, N, 16) with
    layout 0, (experts, 16, N) with layout 1.

    g_rows (int32): row i is row g_rows[i] of g (the routed rows read where they are); row_scale (float32): row i
    weighted by row_scale[i]. out: a contiguous bf16 tensor of that shape to write into (a gradient bucket's slot).
    tiles: the offsets' TileMaps, whose chunk map the whole-row form of a gathered reduction reuses.
    """
    experts = offsets.numel()
    N = g.shape[1]
    rows = g_rows.numel() if g_rows is not None else g.shape[0]
    if g.stride(1) != 1 or g.stride(0) % 8:
        g = g.contiguous()
    shape = (experts, N, RANK_MULTIPLE) if layout == 0 else (experts, RANK_MULTIPLE, N)
    if out is None:
        out = torch.empty(shape, device=g.device, dtype=torch.bfloat16)
    elif tuple(out.shape) != shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError(f"a reduction into {tuple(out.shape)} {out.dtype}: {shape} bf16 contiguous expected")
    if rows == 0:
        return out.zero_()
    lib = _lib.load()
    if g_rows is None and row_scale is None:
        _lib.check(lib.meep2b_grouped_reduce(_lib.ptr(g), rows, N, g.stride(0), _lib.ptr(low.contiguous()),
                                             _lib.ptr(offsets), experts, float(scaling), _lib.ptr(out), layout,
                                             _lib.stream_of(g)), "meep2b_grouped_reduce")
    elif g_rows is not None and N in _FULL_ROW_WIDTHS:
        # gathered rows arrive whole, one bulk copy each (meep2b_grouped_reduce_rows_full): a CTA per chunk of an
        # expert's rows, the chunks' float32 sums added in order by a second kernel
        chunk = int(lib.meep2b_reduce_chunk_rows())
        cmap = tiles.get(chunk) if tiles is not None else tile_map(offsets, rows, chunk)
        partial = torch.empty(cmap[0].numel() * N * RANK_MULTIPLE, device=g.device, dtype=torch.float32)
        _lib.check(lib.meep2b_grouped_reduce_rows_full(
            _lib.ptr(g), _lib.ptr(g_rows), _lib.ptr(row_scale), rows, N, g.stride(0), _lib.ptr(low.contiguous()),
            _lib.ptr(offsets), experts, float(scaling), _lib.ptr(out), layout, _lib.ptr(cmap[0]), _lib.ptr(cmap[1]),
            _lib.ptr(cmap[2]), cmap[0].numel(), _lib.ptr(partial), partial.numel() * 4, _lib.stream_of(g)),
            "meep2b_grouped_reduce_rows_full")
    else:
        if g_rows is None:
            raise ValueError("a weighted reduction reads its rows through g_rows")
        _lib.check(lib.meep2b_grouped_reduce_rows(_lib.ptr(g), _lib.ptr(g_rows), _lib.ptr(row_scale), rows, N,
                                                  g.stride(0), _lib.ptr(low.contiguous()), _lib.ptr(offsets),
                                                  experts, float(scaling), _lib.ptr(out), layout,
                                                  _lib.stream_of(g)), "meep2b_grouped_reduce_rows")
    return out


def _to_lhs_rhs(grad_rows_k, grad_cols_n, adapters):
    """Map the reductions back to PEFT's factors (_grouped.py:400-405).

    grad_rows_k (E, K_fwd, 16) is the gradient of the factor read first in the forward, grad_cols_n (E, N_fwd, 16)
    of the one applied second.
    """
    rank = adapters.rank
    if adapters.is_transposed:  # first = lhs (E, in, r); second = rhs (E, r, out)
        return grad_rows_k[:, :, :rank], grad_cols_n.transpose(1, 2)[:, :rank, :]
    return grad_cols_n[:, :, :rank], grad_rows_k.transpose(1, 2)[:, :rank, :]  # lhs (E,out,r), rhs (E,r,in)


def _rank_chunks(lhs, rhs, is_transposed):
    """The adapters as rank-16 chunks (_Adapters each): delta = sum over chunks of lhs_c @ rhs_c. The reference pads
    any rank to a multiple of 16 (_grouped.py:275-282); the fused panel holds 16 ranks."""
    rank = lhs.shape[2]
    chunks = []
    for c in range(0, rank, RANK_MULTIPLE):
        lc, rc = lhs[:, :, c:c + RANK_MULTIPLE], rhs[:, c:c + RANK_MULTIPLE, :]
        pad = RANK_MULTIPLE - lc.shape[2]
        if rank > RANK_MULTIPLE and pad:  # a ragged last chunk of a large rank: zero ranks, as the reference pads
            lc, rc = torch.nn.functional.pad(lc, (0, pad)), torch.nn.functional.pad(rc, (0, 0, 0, pad))
        chunks.append(_Adapters(lc, rc, is_transposed))
    return chunks


def _low_rank_pass(x, first, second, offsets, tiles):
    """(x @ first (rows, 16) bf16, (x @ first) @ second): the two small products of one rank chunk beyond the first,
    each on the grouped kernel with the factor as its stack, (experts, 16, k) and (experts, n, 16)."""
    low = _launch(x, first.transpose(1, 2).contiguous(), None, offsets, True, None, 1.0, None, False, tiles=tiles)[0]
    delta = _launch(low, second.transpose(1, 2).contiguous(), None, offsets, True, None, 1.0, None, False,
                    tiles=tiles)[0]
    return low, delta


class _LoraGroupedProduct(torch.autograd.Function):
    """The experts' product with the adapters; gradients for x and the adapters, none for the frozen stack.

    Ranks up to 16 ride in the fused product's panel. A larger rank is split into 16-rank chunks: the first in the
    fused product, each further one as two small grouped products added to the output (an extra read of x per
    chunk), and the adapter gradients reduced chunk by chunk."""

    @staticmethod
    def forward(ctx, x, weight, scale, offsets, is_transposed, lhs, rhs, scaling, bias, products_fp8):
        chunks = _rank_chunks(lhs.detach(), rhs.detach(), is_transposed) if lhs is not None else []
        adapters = chunks[0] if chunks else None
        tiles = TileMaps(offsets, x.shape[0])
        out, low = _product(x, weight, scale, offsets, not is_transposed, adapters, scaling, bias, True, tiles=tiles)
        lows = [low] if low is not None else []
        for ad in chunks[1:]:
            first, second = ad.factors(False)
            low_c, delta = _low_rank_pass(x, first, second, offsets, tiles)
            out.add_(delta, alpha=scaling)
            lows.append(low_c)
        ctx.save_for_backward(x, offsets, *lows)
        ctx.weight = weight  # the frozen stack (a tensor or a QuantStack), read again by the backward product
        ctx.chunks, ctx.scale, ctx.is_transposed, ctx.scaling, ctx.tiles = chunks, scale, is_transposed, scaling, tiles
        ctx.rank = lhs.shape[2] if lhs is not None else 0
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, offsets, *lows = ctx.saved_tensors
        weight = ctx.weight
        chunks = ctx.chunks
        grad_out = grad_out.contiguous()
        if not chunks:
            grad_x, _ = _product(grad_out, weight, ctx.scale, offsets, ctx.is_transposed, None, 1.0, None, False,
                                 backward=True, tiles=ctx.tiles)
            return grad_x, None, None, None, None, None, None, None, None, None
        # grad_x = grad @ W (the stack read the other way) + s (grad @ B^T) @ A^T: the adapters swap roles
        grad_x, low2 = _product(grad_out, weight, ctx.scale, offsets, ctx.is_transposed, chunks[0], ctx.scaling, None,
                                True, backward=True, tiles=ctx.tiles)
        lows2 = [low2]
        for ad in chunks[1:]:
            first, second = ad.factors(True)
            low2_c, delta = _low_rank_pass(grad_out, first, second, offsets, ctx.tiles)
            grad_x.add_(delta, alpha=ctx.scaling)
            lows2.append(low2_c)
        grad_first = torch.cat([_reduce(x, l2, offsets, ctx.scaling) for l2 in lows2], dim=2)  # (E, K_fwd, R)
        grad_second = torch.cat([_reduce(grad_out, l, offsets, ctx.scaling) for l in lows], dim=2)  # (E, N_fwd, R)
        whole = types.SimpleNamespace(rank=ctx.rank, is_transposed=ctx.is_transposed)
        grad_lhs, grad_rhs = _to_lhs_rhs(grad_first, grad_second, whole)
        return grad_x, None, None, None, None, grad_lhs, grad_rhs, None, None, None


def _fp8_products_on(weight, products_fp8, device) -> bool:
    """Whether an FP8 stack's products run on the FP8 tensor cores (_grouped.py:316-320)."""
    return weight.dtype == torch.float8_e4m3fn and bool(fp8_products(device) if products_fp8 is None else products_fp8)


def _dequantized(weight, scale):
    """An FP8 stack for the products: (stack, the scale left for the kernel to apply). The codes go to the kernel
    as they are (converted exactly in shared memory, as the reference's kernel converts its FP8 tile) when the stack
    has whole 64-blocks; otherwise they are converted to bf16 here, exactly, without the scale."""
    if weight.dtype != torch.float8_e4m3fn:
        return weight, scale
    ones = torch.ones(weight.shape[0], device=weight.device, dtype=torch.float32)
    fused = QuantStack.from_fp8(weight, ones)
    if fused is not None:
        return fused, scale
    from . import _fp8

    return _fp8.dequantize_stack(weight, ones, torch.bfloat16), scale


def grouped_linear(x: torch.Tensor, weight: torch.Tensor, offsets: torch.Tensor, is_transposed: bool,
                   block_m: int = BLOCK_M, products_fp8=None) -> torch.Tensor:
    """x (rows, in) by the stack (experts, out, in), or (experts, in, out) when is_transposed, per expert group.

    offsets (experts,) int32 on the device: the end of each expert's rows. Returns (rows, out) in x's dtype. An
    FP8 stack is converted exactly, without a scale: the caller folds the scale in. The base product alone, for
    the tests and the benchmark. block_m is accepted for the reference's signature; the tile height is 128.
    """
    _require(x, "grouped_linear")
    _stack_strides(weight, x.shape[1], is_transposed)
    if _fp8_products_on(weight, products_fp8, x.device):
        return _launch_f8(x, Fp8Stack.of(weight, None), offsets.to(torch.int32), not is_transposed, None, 1.0, None,
                          False)[0]
    weight, _ = _dequantized(weight, None)
    return _launch(x, weight, None, offsets, not is_transposed, None, 1.0, None, False)[0]


def lora_linear(x, weight, scale, offsets, is_transposed: bool, lhs=None, rhs=None, scaling: float = 1.0, bias=None,
                products_fp8=None):
    """The experts' product of x with the stack, the adapters (PEFT's lhs, rhs, scaling) and the bias stack.

    scale (experts,) is the FP8 stack's per-expert scale, None for a BF16 stack. products_fp8 says whether an FP8
    stack's products run on the FP8 tensor cores; None lets fp8_products decide for the device.
    """
    _require(x, "lora_linear")
    _stack_strides(weight, x.shape[1], is_transposed)
    if _fp8_products_on(weight, products_fp8, x.device):
        weight, scale = Fp8Stack.of(weight, scale), None
    else:
        weight, scale = _dequantized(weight, scale)
    if lhs is not None and (lhs.dtype != torch.bfloat16 or rhs.dtype != torch.bfloat16):
        lhs, rhs = lhs.to(torch.bfloat16), rhs.to(torch.bfloat16)
    if bias is not None and bias.dtype != torch.bfloat16:
        bias = bias.to(torch.bfloat16)
    if scale is not None:
        scale = scale.to(torch.float32).contiguous()
    return _LoraGroupedProduct.apply(x, weight, scale, offsets.to(torch.int32), is_transposed, lhs, rhs, scaling,
                                     bias.contiguous() if bias is not None else None, products_fp8)


def reference(x: torch.Tensor, weight: torch.Tensor, offsets: torch.Tensor, is_transposed: bool) -> torch.Tensor:
    """The base product, one expert at a time, in float32, for the tests (the reference's, _grouped.py:420-428)."""
    out = torch.empty((x.shape[0], weight.shape[2] if is_transposed else weight.shape[1]), device=x.device, dtype=x.dtype)
    start = 0
    for e, end in enumerate(offsets.tolist()):
        w = weight[e].float()
        out[start:end] = (x[start:end].float() @ (w if is_transposed else w.t())).to(x.dtype)
        start = end
    return out


def reference_lora(x, weight, scale, offsets, is_transposed, lhs, rhs, scaling, bias=None):
    """The whole product with PyTorch operations, differentiable, for the tests (_grouped.py:431-444)."""
    out = []
    start = 0
    for e, end in enumerate(offsets.tolist()):
        w = weight[e].float() * (scale[e].float() if scale is not None else 1.0)
        if lhs is not None:
            w = w + scaling * (lhs[e].float() @ rhs[e].float())
        y = x[start:end].float() @ (w if is_transposed else w.t())
        if bias is not None:
            y = y + bias[e].float()
        out.append(y)
        start = end
    return torch.cat(out).to(x.dtype)
