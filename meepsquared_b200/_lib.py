"""ctypes binding of libmeep2b.so, the CUDA side of the package (include/meep2b.h).

The library is loaded from the package directory (built in place by ``meepsquared_b200.build``). Nothing here
falls back to another implementation: a missing library or a non-zero status raises.
"""

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmeep2b.so")

OK, ERR_SHAPE, ERR_DTYPE, ERR_LAUNCH, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_ALIGN, ERR_DEVICE = range(8)
F32, BF16, E4M3, NF4, E4M3_BLOCKS = 0, 1, 2, 3, 4  # enum meep2b_dtype
EPI_PLAIN, EPI_SWIGLU, EPI_DSWIGLU = 0, 1, 2

_p, _i64, _i32, _f32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_size_t


class Product(ctypes.Structure):
    """struct meep2b_product (include/meep2b.h)."""

    _fields_ = [
        ("x", _p), ("rows", _i64), ("k", _i64), ("ldx", _i64),
        ("weight", _p), ("weight_dtype", _i32), ("experts", _i32), ("n", _i64), ("b_mn", _i32),
        ("scale", _p), ("panel", _p), ("up", _p), ("scaling", _f32), ("bias", _p),
        ("offsets", _p), ("tile_expert", _p), ("tile_row", _p), ("tiles", _p), ("max_tiles", _i64),
        ("out", _p), ("ldo", _i64), ("low", _p), ("epilogue", _i32), ("aux", _p), ("sm_limit", _i32),
        ("block_m", _i32), ("wscale", _p),
        ("x_rows", _p), ("x_src_rows", _i64), ("row_scale", _p), ("w_grad", _p), ("w_ld", _i64),
        ("out_rows", _p),
    ]


class ProductF8(ctypes.Structure):
    """struct meep2b_product_f8 (include/meep2b.h)."""

    _fields_ = [
        ("x8", _p), ("rows", _i64), ("k", _i64), ("xscale", _p), ("ld_xscale", _i64),
        ("weight", _p), ("experts", _i32), ("n", _i64), ("b_mn", _i32), ("scale", _p),
        ("wblock", _p), ("wb_stride_e", _i64), ("wb_stride_k", _i64), ("wb_stride_n", _i64),
        ("wb_div_k", _i32), ("wb_div_n", _i32),
        ("low", _p), ("up", _p), ("scaling", _f32), ("bias", _p),
        ("offsets", _p), ("tile_expert", _p), ("tile_row", _p), ("tiles", _p), ("max_tiles", _i64),
        ("out", _p), ("ldo", _i64), ("sm_limit", _i32),
    ]


_SIGNATURES = {
    "meep2b_version": (ctypes.c_char_p, []),
    "meep2b_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "meep2b_device_ok": (ctypes.c_int, [ctypes.c_int]),
    "meep2b_device_error": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "meep2b_sm_count": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "meep2b_route_workspace_bytes": (_sz, [_i64, _i32]),
    "meep2b_route": (ctypes.c_int, [_p, _i64, _i32, _p, _p, _p, _p, _p, _sz, _p]),
    "meep2b_route_noalloc": (ctypes.c_int, [_p, _i64, _i32, _p, _p, _p, _p, _p]),
    "meep2b_route_logits": (ctypes.c_int, [_p, _i32, _i64, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "meep2b_routed_rows": (ctypes.c_int, [_p, _i64, _i32, _p, _i32, _p, _p, _p]),
    "meep2b_gather": (ctypes.c_int, [_p, _i64, _i64, _i32, _p, _p, _i32, _p, _i32, _p, _p, _p]),
    "meep2b_unpermute": (ctypes.c_int, [_p, _p, _p, _i32, _p, _i32, _i64, _i32, _i64, _p, _p]),
    "meep2b_combine": (ctypes.c_int, [_p, _p, _p, _i32, _p, _i32, _i64, _i32, _i64, _p, _p]),
    "meep2b_unpermute_backward": (ctypes.c_int, [_p, _p, _p, _p, _i32, _p, _i32, _i64, _i32, _i64, _p, _p, _p]),
    "meep2b_weight_grad": (ctypes.c_int, [_p, _i64, _i32, _p, _i64, _p, _i32, _p, _p]),
    "meep2b_tile_map": (ctypes.c_int, [_p, _i32, _i64, _i32, _p, _p, _p, _p]),
    "meep2b_grouped_product": (ctypes.c_int, [ctypes.POINTER(Product), _p]),
    "meep2b_grouped_reduce": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _p, _i32, _f32, _p, _i32, _p]),
    "meep2b_grouped_reduce_rows": (ctypes.c_int, [_p, _p, _p, _i64, _i64, _i64, _p, _p, _i32, _f32, _p, _i32, _p]),
    "meep2b_grouped_reduce_rows_full": (ctypes.c_int, [_p, _p, _p, _i64, _i64, _i64, _p, _p, _i32, _f32, _p, _i32,
                                                       _p, _p, _p, _i64, _p, _sz, _p]),
    "meep2b_reduce_chunk_rows": (ctypes.c_int, []),
    "meep2b_fp8_stack_quantize": (ctypes.c_int, [_p, _i32, _i32, _i64, _p, _p, _p, _p]),
    "meep2b_fp8_stack_dequantize": (ctypes.c_int, [_p, _p, _i32, _i64, _p, _p]),
    "meep2b_fp8_block_dequantize": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _i32, _i32, _p, _p]),
    "meep2b_fp8_block_quantize": (ctypes.c_int, [_p, _i32, _i64, _i64, _i64, _i32, _i32, _p, _p, _p]),
    "meep2b_nf4_absmax": (ctypes.c_int, [_p, _p, _p, _p, _i32, _i64, _p, _p]),
    "meep2b_quant_multipliers": (ctypes.c_int, [_i32, _p, _i32, _i64, _i64, _i32, _i32, _p, _p]),
    "meep2b_nf4_dequantize": (ctypes.c_int, [_p, _p, _p, _p, _p, _i32, _i32, _i64, _p, _p, _p]),
    "meep2b_merge_stack": (ctypes.c_int, [_p, _i32, _p, _p, _p, _i32, ctypes.c_float, _i64, _i64, _i64, _p, _i32,
                                          _p]),
    "meep2b_fp8_rows_quantize": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _p, _i64, _p]),
    "meep2b_grouped_product_f8": (ctypes.c_int, [ctypes.POINTER(ProductF8), _p]),
    "meep2b_swiglu": (ctypes.c_int, [_p, _i64, _i64, _p, _p]),
    "meep2b_swiglu_backward": (ctypes.c_int, [_p, _p, _i64, _i64, _p, _p]),
}

_lib = None
_load_error = None


def load():
    """The loaded library (ctypes.CDLL); RuntimeError when it is missing or does not load."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if _load_error is not None:
        raise RuntimeError(_load_error)
    if not os.path.exists(LIB_PATH):
        _load_error = (f"libmeep2b.so is not built ({LIB_PATH}); run `python -m meepsquared_b200.build` "
                       "(nvcc, sm_100a)")
        raise RuntimeError(_load_error)
    try:
        lib = ctypes.CDLL(LIB_PATH)
    except OSError as exc:
        _load_error = f"libmeep2b.so does not load: {exc}"
        raise RuntimeError(_load_error) from exc
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _lib = lib
    return lib


def loaded() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def exported_symbols():
    return sorted(_SIGNATURES)


class DeviceError(RuntimeError):
    pass


# Kernels each entry point launches per successful call (the ones this package calls on its hot path), for the
# count of the library's launches in a timed region (benchmark); `launches` accumulates them per entry point.
KERNELS_PER_CALL = {
    "meep2b_route": 3, "meep2b_route_noalloc": 3, "meep2b_route_logits": 3, "meep2b_routed_rows": 1, "meep2b_gather": 1,
    "meep2b_unpermute": 1, "meep2b_unpermute_backward": 1, "meep2b_tile_map": 1, "meep2b_grouped_product": 1,
    "meep2b_grouped_reduce": 1, "meep2b_grouped_reduce_rows": 1, "meep2b_grouped_reduce_rows_full": 2,
    "meep2b_fp8_stack_dequantize": 1,
    "meep2b_fp8_block_dequantize": 1, "meep2b_nf4_dequantize": 2, "meep2b_nf4_absmax": 1,
    "meep2b_merge_stack": 1,
    "meep2b_quant_multipliers": 1, "meep2b_fp8_rows_quantize": 1, "meep2b_grouped_product_f8": 1,
    "meep2b_swiglu": 1, "meep2b_swiglu_backward": 1, "meep2b_weight_grad": 1, "meep2b_combine": 1,
}
launches = {}


def launch_count() -> int:
    """Kernels the library launched through the calls checked so far (see KERNELS_PER_CALL)."""
    return sum(KERNELS_PER_CALL.get(k, 1) * v for k, v in launches.items())


def check(status: int, what: str):
    """Raises the reference's exception kind for a non-zero status (ValueError for sizes, ...)."""
    if status == OK:
        launches[what] = launches.get(what, 0) + 1
        return
    msg = f"{what}: {load().meep2b_status_string(status).decode()}"
    if status in (ERR_SHAPE, ERR_ALIGN):
        raise ValueError(msg)
    if status == ERR_DTYPE:
        raise TypeError(msg)
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def device_ok(index: int) -> bool:
    return load().meep2b_device_ok(index) == OK


def device_error(index: int) -> int:
    """Reads and clears the device's error word (a bounded wait of a kernel that ran out); synchronises."""
    code = ctypes.c_int(0)
    check(load().meep2b_device_error(index, ctypes.byref(code)), "meep2b_device_error")
    return code.value


_SM_COUNT = {}


def sm_count(index: int) -> int:
    if index not in _SM_COUNT:
        c = ctypes.c_int(0)
        check(load().meep2b_sm_count(index, ctypes.byref(c)), "meep2b_sm_count")
        _SM_COUNT[index] = c.value
    return _SM_COUNT[index]
