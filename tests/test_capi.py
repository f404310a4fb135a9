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
        (lambda lib: lib.moe_swiglu(None, 5, None, None, 4, 8, None), "dtype"),
        (lambda lib: lib.moe_swiglu(None, 2, None, None, 4, 8, None), "null"),
        (lambda lib: lib.moe_dispatch_no_alloc(None, 2, None, None, None, None, None, None,
                                               1 << 20, 8, 8, 512, 1 << 23, 1, 1, None),
         "built-in array"),
        # arguments are checked before the built-in array is looked up or cleared
        (lambda lib: lib.moe_dispatch_no_alloc(None, 5, None, None, None, None, None, None,
                                               16, 8, 2, 8, 32, 1, 1, None), "FP32"),
        (lambda lib: lib.moe_ep_layout(None, 0, 8, 1, None, None, None, None), "ranks*experts"),
        (lambda lib: lib.moe_ep_layout(None, 2, 8, 0, None, None, None, None), "alignment"),
        (lambda lib: lib.moe_ep_layout(None, 2, 8, 8, None, None, None, None), "null"),
        (lambda lib: lib.moe_ep_regroup(None, 9, None, None, None, None, None, 2, 8, 64, 4, 4, 1,
                                        None), "dtype"),
        (lambda lib: lib.moe_ep_regroup(None, 2, None, None, None, None, None, 2, 8, 0, 4, 4, 1,
                                        None), "regroup shape"),
        (lambda lib: lib.moe_ep_p2p(0, None, None, None, None, 9, 0, 72, 8, 64, 16, 16, 100,
                                    None), "ranks"),
        (lambda lib: lib.moe_ep_p2p(0, None, None, None, None, 2, 2, 8, 8, 64, 16, 16, 100,
                                    None), "rank out of range"),
        (lambda lib: lib.moe_ep_p2p(7, None, None, None, None, 2, 0, 8, 8, 64, 16, 16, 100,
                                    None), "bad op"),
        (lambda lib: lib.moe_ep_p2p(0, None, None, None, None, 2, 0, 8, 8, 64, 16, 16, 100,
                                    None), "null"),
        (lambda lib: lib.moe_ep_p2p_down_return(None, None, None, None, 2, 0, 8, 64, 12, 16, 16,
                                                None), "down GEMM shape"),
        (lambda lib: lib.moe_peer_alloc(0, None, None), "peer allocation"),
        (lambda lib: lib.moe_peer_open(None, None), "null"),
        (lambda lib: lib.moe_peer_close(None), "null"),
        (lambda lib: lib.moe_peer_free(None), "null"),
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


def test_expert_parallel_region_queries_reject_bad_shapes():
    lib = load_library()
    assert lib.moe_ep_p2p_region_bytes(9, 72, 64, 16, 16) == -1      # more than 8 ranks
    assert lib.moe_ep_p2p_region_bytes(3, 8, 64, 16, 16) == -1       # experts not a multiple
    assert lib.moe_ep_p2p_region_bytes(2, 8, 12, 16, 16) == -1       # hidden not a multiple of 8
    good = lib.moe_ep_p2p_region_bytes(2, 8, 64, 16, 16)
    assert good > 0 and good % 1024 == 0
    grouped = lib.moe_ep_p2p_region_offset(2, 8, 64, 16, 16, 0)
    back = lib.moe_ep_p2p_region_offset(2, 8, 64, 16, 16, 1)
    assert 0 < grouped < back < good and grouped % 1024 == 0 and back - grouped >= 16 * 64 * 2
    assert lib.moe_ep_p2p_region_offset(2, 8, 64, 16, 16, 2) == -1
    assert lib.moe_ep_p2p_state_words(2, 8) > 0 and lib.moe_ep_p2p_state_words(3, 8) == -1
