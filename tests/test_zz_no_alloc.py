"""The allocation-free routing entry point, meep2b_route_noalloc, against the allocating one.

Some callers of this library cannot allocate device memory: they own every device buffer and have no allocator to
lend (an FFI caller outside PyTorch, a serving process that reserves its memory up front), or must not call
cudaMalloc because it would synchronise the device. meep2b_route_noalloc serves them by keeping its bucket-count
table in a fixed array of device memory inside the library. This test calls both entry points through the C ABI on
the same inputs, twice in a row with different routings (the shared array keeps the previous call's contents, which
must not leak into the next result), and checks that every output is identical. It also checks that a request
beyond the array's fixed size is refused before any work. It sits in a file of its own, collected last, so that a
run that stops at the first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

import layer_inputs
from meepsquared_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _outputs(n, experts):
    return {"perm": torch.empty(n, dtype=torch.int64, device=DEV),
            "ids_g": torch.empty(n, dtype=torch.int64, device=DEV),
            "offsets": torch.empty(experts, dtype=torch.int32, device=DEV),
            "inverse": torch.empty(n, dtype=torch.int64, device=DEV)}


def _route_allocating(ids, experts):
    lib = _lib.load()
    o = _outputs(ids.numel(), experts)
    nbytes = lib.meep2b_route_workspace_bytes(ids.numel(), experts)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    _lib.check(lib.meep2b_route(_lib.ptr(ids), ids.numel(), experts, _lib.ptr(o["perm"]), _lib.ptr(o["ids_g"]),
                                _lib.ptr(o["offsets"]), _lib.ptr(o["inverse"]), _lib.ptr(ws), nbytes,
                                _lib.stream_of(ids)), "meep2b_route")
    return o


def _route_noalloc(ids, experts):
    o = _outputs(ids.numel(), experts)
    status = _lib.load().meep2b_route_noalloc(_lib.ptr(ids), ids.numel(), experts, _lib.ptr(o["perm"]),
                                              _lib.ptr(o["ids_g"]), _lib.ptr(o["offsets"]), _lib.ptr(o["inverse"]),
                                              _lib.stream_of(ids))
    return status, o


def test_the_no_alloc_route_matches_the_allocating_route_on_two_calls_in_a_row():
    cases = [(16384, 128, 8, 1.1), (8192, 8, 2, None)]  # config-2 shape (skewed), then the Mixtral shape
    for tokens, experts, k, zipf in cases:
        idx, _ = layer_inputs.routing(tokens, experts, k, torch.Generator().manual_seed(tokens), zipf)
        ids = idx.reshape(-1).to(DEV)
        want = _route_allocating(ids, experts)
        status, got = _route_noalloc(ids, experts)
        assert status == _lib.OK, _lib.load().meep2b_status_string(status)
        torch.cuda.synchronize()
        for name in want:  # integer outputs: bit-exact
            np.testing.assert_array_equal(got[name].cpu().numpy(), want[name].cpu().numpy(), err_msg=name)


def test_the_no_alloc_route_refuses_a_request_beyond_its_fixed_table():
    ids = torch.zeros(4097 * 64, dtype=torch.int64, device=DEV)  # 65 chunks x 1025 buckets > 65536 words
    status, _ = _route_noalloc(ids, 1024)
    assert status == _lib.ERR_SHAPE
