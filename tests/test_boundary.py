"""The C-ABI library and the host layer, without a GPU: it loads, exports every declared entry point, and the
host layer keeps the reference's API and refuses to run anywhere but on a CUDA GPU (no CPU fallback)."""

import os
import re
import subprocess

import pytest
import torch

import meepsquared_b200 as mb
from meepsquared_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "meep2b.h")).read()
    return sorted(set(re.findall(r"^\s*(?:const char\*|int|size_t)\s+(meep2b_\w+)\(", text, re.M)))


def test_library_builds_and_loads():
    from meepsquared_b200 import build

    build.build()
    assert _lib.loaded()
    assert _lib.load().meep2b_version().startswith(b"meep2b")


def test_every_declared_entry_point_is_exported_and_bound():
    decl = declared_symbols()
    assert len(decl) >= 17
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (meep2b_\w+)", out))
    assert set(decl) <= exported, set(decl) - exported
    assert set(decl) == set(_lib.exported_symbols())
    for name in decl:
        assert getattr(_lib.load(), name) is not None


def test_status_strings():
    lib = _lib.load()
    for code in range(8):
        assert lib.meep2b_status_string(code)
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_SHAPE, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_TIMEOUT, "x")


def test_the_reference_api_is_there():
    for name in ("lora_linear", "grouped_linear", "tile_map", "max_tiles", "wanted", "available", "fp8_products",
                 "reference", "reference_lora"):
        assert callable(getattr(mb, name))
    assert mb.BLOCK_M == 128 and mb.RANK_MULTIPLE == 16 and mb.TORCH_HAS_GROUPED_MM == (9, 10)
    assert mb.max_tiles(199, 4, 64) == 199 // 64 + 4


def test_no_cpu_fallback():
    x = torch.randn(8, 64, dtype=torch.bfloat16)
    w = torch.randn(2, 16, 64, dtype=torch.bfloat16)
    offsets = torch.tensor([4, 8], dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        mb.grouped_linear(x, w, offsets, False)
    with pytest.raises(RuntimeError, match="CUDA"):
        mb.lora_linear(x, w, None, offsets, False)
    with pytest.raises(RuntimeError, match="CUDA"):
        mb.tile_map(offsets, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        mb.route(torch.zeros(4, 2, dtype=torch.int64), None, 4)


def test_mismatched_stack_is_refused_before_anything_runs():
    x = torch.randn(8, 64, dtype=torch.bfloat16)
    w = torch.randn(2, 16, 32, dtype=torch.bfloat16)
    if torch.cuda.is_available():
        pytest.skip("covered on the GPU")
    with pytest.raises(RuntimeError):  # the device check comes first on a CPU box
        mb.grouped_linear(x, w, torch.tensor([4, 4], dtype=torch.int32), is_transposed=False)


def test_wanted_follows_the_override_and_the_device(monkeypatch):
    monkeypatch.setenv("MEEPSQUARED_GROUPED_KERNEL", "0")
    assert mb.wanted(torch.device("cuda", 0)) is False
    monkeypatch.setenv("MEEPSQUARED_GROUPED_KERNEL", "1")
    assert mb.wanted(torch.device("cpu")) is True
    monkeypatch.delenv("MEEPSQUARED_GROUPED_KERNEL")
    assert mb.wanted(torch.device("cpu")) is False


def test_fp8_products_are_off_unless_asked_for(monkeypatch):
    monkeypatch.delenv("MEEPSQUARED_FP8_PRODUCTS", raising=False)
    assert mb.fp8_products(torch.device("cuda", 0)) is False
    monkeypatch.setenv("MEEPSQUARED_FP8_PRODUCTS", "1")
    assert mb.fp8_products(torch.device("cuda", 0)) is True
