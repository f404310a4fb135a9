"""The C-ABI library loads, exports every declared entry point and rejects bad
arguments on the host -- all without a GPU (no kernel is launched here)."""

import ctypes
import re
from pathlib import Path

import pytest

from moe_dispatch._extension import SIGNATURES, load_library

HEADER = Path(__file__).resolve().parents[1] / "include" / "moe_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_entry_point():
    lib = load_library()
    names = declared_functions()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
    # The Python binding declares exactly the header's entry points.
    assert sorted(SIGNATURES) == names


def test_abi_version_and_scratch_query():
    lib = load_library()
    assert lib.moe_abi_version() == 1
    assert lib.moe_dispatch_scratch_bytes(4096, 8, 64) == (16 + 32 * 64) * 4
    assert lib.moe_dispatch_scratch_bytes(0, 2, 8) == (16 + 8) * 4
    assert lib.moe_dispatch_scratch_bytes(-1, 2, 8) == -1


@pytest.mark.parametrize(
    "call, message",
    [
        (lambda lib: lib.moe_topk_route(None, None, None, None, None, 4, 0, 1, None), "experts"),
        (lambda lib: lib.moe_topk_route(None, None, None, None, None, 4, 8, 9, None), "topk"),
        (lambda lib: lib.moe_topk_route(None, None, None, None, None, 4, 300, 2, None), "experts"),
        (lambda lib: lib.moe_route(None, None, None, None, None, None, None, 4, 17, 8, 2, None),
         "hidden"),
        (lambda lib: lib.moe_dispatch(None, 7, None, None, None, None, None, None, 1, 8, 2, 8, 2, 1,
                                      1, None, 0, None), "FP32"),
        (lambda lib: lib.moe_dispatch(None, 2, None, None, None, None, None, None, 1, 8, 2, 8, 2,
                                      200, 1, None, 0, None), "alignment"),
        (lambda lib: lib.moe_dispatch(None, 2, None, None, None, None, None, None, 4, 8, 2, 8, 5, 1,
                                      1, None, 0, None), "packed"),
        (lambda lib: lib.moe_combine(None, 2, None, None, None, 4, 8, 40, 8, None), "topk"),
        (lambda lib: lib.moe_grouped_gemm(None, None, None, None, 16, 12, 64, 2, None),
         "multiples of 8"),
        (lambda lib: lib.moe_grouped_gemm_swiglu(None, None, None, None, 16, 64, 64, 0, None),
         "experts"),
    ],
)
def test_invalid_arguments_are_rejected_on_the_host(call, message):
    lib = load_library()
    assert call(lib) == 1  # MOE_ERR_INVALID
    assert message in lib.moe_last_error().decode()


def test_status_word_requires_a_destination():
    lib = load_library()
    assert lib.moe_device_status(None, 0) == 1
    assert ctypes.c_int  # keep ctypes imported for readers of this file


def test_tile_choice_follows_rows_per_expert_and_the_override(monkeypatch):
    lib = load_library()
    lib.moe_grouped_gemm_tile.restype = ctypes.c_int32
    lib.moe_grouped_gemm_tile.argtypes = [ctypes.c_int64, ctypes.c_int32]
    monkeypatch.delenv("MOE_B200_GEMM_TILE", raising=False)
    assert lib.moe_grouped_gemm_tile(8256, 8) == 1       # Mixtral: ~1032 rows per expert
    assert lib.moe_grouped_gemm_tile(65536, 256) == 0    # 256 rows per expert
    assert lib.moe_grouped_gemm_tile(4095, 8) == 0
    assert lib.moe_grouped_gemm_tile(4096, 8) == 1
    monkeypatch.setenv("MOE_B200_GEMM_TILE", "single")
    assert lib.moe_grouped_gemm_tile(8256, 8) == 0
    monkeypatch.setenv("MOE_B200_GEMM_TILE", "pair")
    assert lib.moe_grouped_gemm_tile(16, 8) == 1
