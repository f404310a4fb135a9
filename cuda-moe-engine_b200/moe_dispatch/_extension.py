"""Binding to libmoe_b200.so, the C-ABI library of sm_100a kernels.

The reference builds a pybind module with ``load_inline`` and exposes five
functions (src/moe_dispatch/_extension.py:30-63, csrc/bindings.cpp:3-13).
``get_extension()`` returns an object with the same five functions -- same
names, argument order and meaning, RuntimeError on bad tensors -- plus the
fused stages of this engine.  The library is built ahead of time
(``csrc/build.py``); nothing is compiled at import or first use, and a
missing library is an error, never a fallback.
"""

from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

import torch

LIBRARY = Path(__file__).resolve().parent / "lib" / "libmoe_b200.so"

_DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

# name -> (restype, argtypes) of every entry point in include/moe_b200.h
_P, _I32, _I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
SIGNATURES = {
    "moe_abi_version": (ctypes.c_int, []),
    "moe_last_error": (ctypes.c_char_p, []),
    "moe_topk_route": (ctypes.c_int, [_P, _P, _P, _P, _P, _I64, _I32, _I32, _P]),
    "moe_route": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _P]),
    "moe_dispatch_scratch_bytes": (ctypes.c_int64, [_I64, _I32, _I32]),
    "moe_dispatch": (
        ctypes.c_int,
        [_P, _I32, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _I64, _I32, _I32, _P, _I64, _P],
    ),
    "moe_dispatch_no_alloc": (
        ctypes.c_int,
        [_P, _I32, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _I64, _I32, _I32, _P],
    ),
    "moe_combine": (ctypes.c_int, [_P, _I32, _P, _P, _P, _I64, _I64, _I32, _I64, _P]),
    "moe_swiglu": (ctypes.c_int, [_P, _I32, _P, _P, _I64, _I64, _P]),
    "moe_grouped_gemm_swiglu": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _I32, _P]),
    "moe_grouped_gemm": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _I32, _P]),
    "moe_grouped_gemm_tile": (ctypes.c_int32, [_I64, _I32]),
    "moe_quantize_rows_e4m3": (ctypes.c_int, [_P, _I32, _P, _P, _I64, _I64, _P]),
    "moe_grouped_gemm_swiglu_e4m3": (
        ctypes.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _P]
    ),
    "moe_grouped_gemm_e4m3": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _P]),
    "moe_ep_layout": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _P, _P, _P]),
    "moe_ep_regroup": (
        ctypes.c_int, [_P, _I32, _P, _P, _P, _P, _P, _I32, _I32, _I64, _I64, _I64, _I32, _P]
    ),
    "moe_peer_alloc": (ctypes.c_int, [_I64, _P, _P]),
    "moe_peer_open": (ctypes.c_int, [_P, _P]),
    "moe_peer_close": (ctypes.c_int, [_P]),
    "moe_peer_free": (ctypes.c_int, [_P]),
    "moe_ep_p2p_region_bytes": (ctypes.c_int64, [_I32, _I32, _I64, _I64, _I64]),
    "moe_ep_p2p_region_offset": (ctypes.c_int64, [_I32, _I32, _I64, _I64, _I64, _I32]),
    "moe_ep_p2p_state_words": (ctypes.c_int64, [_I32, _I32]),
    "moe_ep_p2p": (
        ctypes.c_int,
        [_I32, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _P],
    ),
    "moe_ep_p2p_gate_up": (
        ctypes.c_int, [_P, _P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _I64, _P]
    ),
    "moe_ep_p2p_down_return": (
        ctypes.c_int, [_P, _P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _P]
    ),
    "moe_device_status": (ctypes.c_int, [_P, _I32]),
}


@lru_cache(maxsize=1)
def load_library():
    """Load the prebuilt library and declare every entry point (no GPU needed)."""
    if not LIBRARY.exists():
        raise RuntimeError(
            f"{LIBRARY.name} is missing; build it with "
            "`python cuda-moe-engine_b200/moe_dispatch/csrc/build.py`"
        )
    lib = ctypes.CDLL(str(LIBRARY))
    for name, (restype, argtypes) in SIGNATURES.items():
        function = getattr(lib, name)
        function.restype = restype
        function.argtypes = argtypes
    return lib


def _require(condition, message):
    if not condition:
        raise RuntimeError(message)


def _check_cuda(tensor, anchor, name):
    _require(tensor.is_cuda, f"{name}: all tensors must be CUDA tensors")
    _require(tensor.is_contiguous(), f"{name}: all tensors must be contiguous")
    _require(tensor.device == anchor.device, f"{name}: device mismatch")


class Extension:
    """The reference's extension functions over the C ABI (plus fused stages)."""

    def __init__(self, lib):
        self.lib = lib
        self._scratch = {}

    # ---------------------------------------------------------------- helpers
    def _run(self, status):
        if status != 0:
            raise RuntimeError(self.lib.moe_last_error().decode())

    def _call(self, device, function, *args):
        """Launch on `device` and its current torch stream (the reference's CUDAGuard)."""
        index = device.index if device.index is not None else torch.cuda.current_device()
        if index != torch.cuda.current_device():
            with torch.cuda.device(index):
                self._run(function(*args, torch.cuda.current_stream(index).cuda_stream))
        else:
            self._run(function(*args, torch.cuda.current_stream(index).cuda_stream))

    def scratch_bytes(self, tokens, topk, experts):
        return int(self.lib.moe_dispatch_scratch_bytes(tokens, topk, experts))

    def make_scratch(self, tokens, topk, experts, device):
        """Zeroed device scratch for one dispatch workspace."""
        words = (self.scratch_bytes(tokens, topk, experts) + 3) // 4
        return torch.zeros(words, dtype=torch.int32, device=device)

    def _shared_scratch(self, tokens, topk, experts, device):
        needed = self.scratch_bytes(tokens, topk, experts)
        key = torch.device(device)
        buffer = self._scratch.get(key)
        if buffer is None or buffer.numel() * 4 < needed:
            buffer = torch.zeros((needed + 3) // 4, dtype=torch.int32, device=device)
            self._scratch[key] = buffer
        return buffer

    # ----------------------------------------- reference functions (bindings.cpp)
    def dispatch_out(self, x, ids, counts, offsets, slots, packed, inverse, vectorized, *,
                     scratch=None):
        """dispatch.cu:102-158: compact packing (alignment 1)."""
        self._dispatch(x, ids, counts, offsets, slots, packed, inverse, vectorized, 1, scratch)

    def dispatch_aligned_out(self, x, ids, counts, offsets, slots, packed, inverse, vectorized,
                             alignment, *, scratch=None):
        """dispatch.cu:218-275: each expert's span rounded up to `alignment` rows."""
        self._dispatch(x, ids, counts, offsets, slots, packed, inverse, vectorized, alignment,
                       scratch)

    def _dispatch(self, x, ids, counts, offsets, slots, packed, inverse, vectorized, alignment,
                  scratch):
        _require(x.is_cuda and x.is_contiguous(), "x must be contiguous CUDA")
        _require(x.dim() == 2 and ids.dim() == 2, "expected x[T,H], ids[T,K]")
        _require(x.dtype in _DTYPE_CODES, "only FP32, FP16, and BF16 are supported")
        _require(ids.dtype == torch.int32, "ids must be int32")
        tokens, hidden = x.shape
        topk = ids.shape[1]
        _require(ids.shape[0] == tokens and hidden > 0, "incompatible token dimensions")
        for tensor in (ids, counts, offsets, slots, packed, inverse):
            _check_cuda(tensor, x, "dispatch")
        _require(
            all(t.dtype == torch.int32 for t in (counts, offsets, slots, inverse)),
            "workspace indices must be int32",
        )
        experts = counts.numel()
        _require(
            offsets.numel() == experts + 1 and slots.numel() == tokens * topk
            and inverse.numel() == tokens * topk,
            "incorrect index workspace size",
        )
        _require(
            packed.dim() == 2 and packed.shape[1] == hidden and packed.dtype == x.dtype,
            "incorrect packed workspace",
        )
        if scratch is None:
            scratch = self._shared_scratch(tokens, topk, experts, x.device)
        else:
            _check_cuda(scratch, x, "dispatch scratch")
        self._call(
            x.device, self.lib.moe_dispatch,
            x.data_ptr(), _DTYPE_CODES[x.dtype], ids.data_ptr(), counts.data_ptr(),
            offsets.data_ptr(), slots.data_ptr(), packed.data_ptr(), inverse.data_ptr(),
            tokens, hidden, topk, experts, packed.shape[0], alignment, int(bool(vectorized)),
            scratch.data_ptr(), scratch.numel() * scratch.element_size(),
        )

    def combine_out(self, packed_output, inverse, weights, output):
        """dispatch.cu:160-192."""
        _require(packed_output.is_cuda and packed_output.is_contiguous(),
                 "expert output must be contiguous CUDA")
        _require(output.dim() == 2 and inverse.dim() == 2 and weights.dim() == 2,
                 "expected output[T,H], inverse[T,K], weights[T,K]")
        _require(packed_output.dim() == 2 and packed_output.dtype in _DTYPE_CODES,
                 "unsupported output dtype")
        for tensor in (inverse, weights, output):
            _check_cuda(tensor, packed_output, "combine")
        _require(inverse.dtype == torch.int32 and weights.dtype == torch.float32,
                 "inverse must be int32; weights must be FP32")
        tokens, hidden = output.shape
        topk = inverse.shape[1]
        _require(
            inverse.shape[0] == tokens and weights.shape == inverse.shape
            and packed_output.shape[0] >= tokens * topk and packed_output.shape[1] == hidden
            and output.dtype == packed_output.dtype,
            "shape/dtype mismatch",
        )
        self._call(
            output.device, self.lib.moe_combine,
                packed_output.data_ptr(), _DTYPE_CODES[output.dtype], inverse.data_ptr(),
            weights.data_ptr(), output.data_ptr(), tokens, hidden, topk,
                packed_output.shape[0],
        )

    def swiglu_out(self, projection, valid_rows, output):
        """dispatch.cu:294-323."""
        _require(projection.is_cuda and projection.is_contiguous(),
                 "projection must be contiguous CUDA")
        _require(
            projection.dim() == 2 and output.dim() == 2 and projection.shape[0] == output.shape[0]
            and projection.shape[1] == output.shape[1] * 2,
            "expected projection[R,2I], output[R,I]",
        )
        _check_cuda(valid_rows, projection, "swiglu")
        _check_cuda(output, projection, "swiglu")
        _require(valid_rows.dtype == torch.int32 and valid_rows.numel() == 1,
                 "valid_rows must be a single int32 CUDA value")
        _require(output.dtype == projection.dtype and projection.dtype in _DTYPE_CODES,
                 "unsupported dtype")
        self._call(
            projection.device, self.lib.moe_swiglu,
            projection.data_ptr(), _DTYPE_CODES[projection.dtype], valid_rows.data_ptr(),
            output.data_ptr(), output.shape[0], output.shape[1],
        )

    def topk_route_out(self, logits, bias, ids32, ids64, weights):
        """dispatch.cu:378-402 (limits lifted to top-k <= 32, experts <= 256)."""
        _require(
            logits.is_cuda and logits.is_contiguous() and logits.dim() == 2
            and logits.dtype == torch.float32,
            "expected FP32 CUDA logits[T,E]",
        )
        for tensor in (bias, ids32, ids64, weights):
            _check_cuda(tensor, logits, "topk_route")
        tokens, experts = logits.shape
        _require(bias.dim() == 1 and bias.numel() == experts and bias.dtype == torch.float32,
                 "expected FP32 bias[E]")
        _require(ids32.dim() == 2 and ids32.shape[0] == tokens and ids32.dtype == torch.int32,
                 "expected int32 ids[T,K]")
        _require(
            ids64.shape == ids32.shape and ids64.dtype == torch.int64
            and weights.shape == ids32.shape and weights.dtype == torch.float32,
            "expected int64 IDs and FP32 weights",
        )
        self._call(
            logits.device, self.lib.moe_topk_route,
            logits.data_ptr(), bias.data_ptr(), ids32.data_ptr(), ids64.data_ptr(),
            weights.data_ptr(), tokens, experts, ids32.shape[1],
        )

    # ------------------------------------------------------------ fused stages
    def route_out(self, x, router_weight, bias, logits, ids32, ids64, weights):
        """F.linear(x.float(), W) + topk_route_out in two kernels (layer.py:122-135)."""
        _require(x.is_cuda and x.is_contiguous() and x.dtype == torch.bfloat16 and x.dim() == 2,
                 "expected contiguous BF16 CUDA x[T,H]")
        for tensor in (router_weight, bias, logits, ids32, ids64, weights):
            _check_cuda(tensor, x, "route")
        tokens, hidden = x.shape
        experts = router_weight.shape[0]
        _require(router_weight.dtype == torch.float32 and router_weight.shape == (experts, hidden),
                 "expected FP32 router_weight[E,H]")
        _require(logits.shape == (tokens, experts) and logits.dtype == torch.float32,
                 "expected FP32 logits[T,E]")
        _require(bias.shape == (experts,) and bias.dtype == torch.float32, "expected FP32 bias[E]")
        _require(
            ids32.shape[0] == tokens and ids32.dtype == torch.int32 and ids64.shape == ids32.shape
            and ids64.dtype == torch.int64 and weights.shape == ids32.shape
            and weights.dtype == torch.float32,
            "expected ids32/ids64/weights [T,K]",
        )
        self._call(
            x.device, self.lib.moe_route,
            x.data_ptr(), router_weight.data_ptr(), bias.data_ptr(), logits.data_ptr(),
            ids32.data_ptr(), ids64.data_ptr(), weights.data_ptr(), tokens, hidden, experts,
            ids32.shape[1],
        )

    def _gemm_checks(self, a, weight, offsets, out):
        _require(a.is_cuda and a.is_contiguous() and a.dtype == torch.bfloat16 and a.dim() == 2,
                 "expected contiguous BF16 CUDA rows[R,K]")
        for tensor in (weight, offsets, out):
            _check_cuda(tensor, a, "grouped GEMM")
        _require(weight.dim() == 3 and weight.dtype == torch.bfloat16 and weight.shape[2] == a.shape[1],
                 "expected BF16 weight[E,N,K]")
        _require(offsets.dtype == torch.int32 and offsets.numel() == weight.shape[0] + 1,
                 "expected int32 offsets[E+1]")
        _require(out.dtype == torch.bfloat16 and out.dim() == 2 and out.shape[0] == a.shape[0],
                 "expected BF16 out[R,N]")

    def grouped_gemm_swiglu_out(self, packed, gate_up, offsets, activated):
        """Gate/up grouped GEMM with SwiGLU in its epilogue (layer.py:162-172)."""
        self._gemm_checks(packed, gate_up, offsets, activated)
        experts, two_i, hidden = gate_up.shape
        _require(two_i % 2 == 0 and activated.shape[1] * 2 == two_i,
                 "expected gate_up[E,2I,H] and activated[R,I]")
        self._call(
            packed.device, self.lib.moe_grouped_gemm_swiglu,
                packed.data_ptr(), gate_up.data_ptr(), offsets.data_ptr(), activated.data_ptr(),
                packed.shape[0], hidden, two_i // 2, experts,
        )

    def grouped_gemm_out(self, a, weight, offsets, out):
        """Plain grouped GEMM: out[r] = a[r] @ weight[e].T (layer.py:175-181)."""
        self._gemm_checks(a, weight, offsets, out)
        experts, n_cols, k_dim = weight.shape
        _require(out.shape[1] == n_cols, "expected out[R,N]")
        self._call(
            a.device, self.lib.moe_grouped_gemm,
            a.data_ptr(), weight.data_ptr(), offsets.data_ptr(), out.data_ptr(), a.shape[0],
            n_cols, k_dim, experts,
        )

    # --------------------------------------------------- FP8 (e4m3) experts
    def quantize_rows_e4m3(self, x, q, scale):
        """q[r] = e4m3(x[r] * 448 / amax_r), scale[r] = amax_r / 448 (include/moe_b200.h)."""
        _require(x.is_cuda and x.is_contiguous() and x.dtype == torch.bfloat16 and x.dim() == 2,
                 "expected contiguous BF16 CUDA x[R,C]")
        _check_cuda(q, x, "quantize_rows_e4m3")
        _check_cuda(scale, x, "quantize_rows_e4m3")
        _require(q.dtype == torch.float8_e4m3fn and tuple(q.shape) == tuple(x.shape),
                 "expected float8_e4m3fn q with x's shape")
        _require(scale.dtype == torch.float32 and scale.numel() == x.shape[0],
                 "expected fp32 scale[R]")
        self._call(x.device, self.lib.moe_quantize_rows_e4m3, x.data_ptr(), 2, q.data_ptr(),
                   scale.data_ptr(), x.shape[0], x.shape[1])

    def _e4m3_checks(self, a, a_scale, weight, weight_scale, offsets, out):
        _require(a.is_cuda and a.is_contiguous() and a.dtype == torch.float8_e4m3fn and a.dim() == 2,
                 "expected contiguous float8_e4m3fn CUDA rows[R,K]")
        for tensor in (a_scale, weight, weight_scale, offsets, out):
            _check_cuda(tensor, a, "e4m3 grouped GEMM")
        _require(weight.dim() == 3 and weight.dtype == torch.float8_e4m3fn
                 and weight.shape[2] == a.shape[1], "expected float8_e4m3fn weight[E,N,K]")
        _require(a_scale.dtype == torch.float32 and a_scale.numel() == a.shape[0],
                 "expected fp32 a_scale[R]")
        _require(weight_scale.dtype == torch.float32
                 and weight_scale.numel() == weight.shape[0] * weight.shape[1],
                 "expected fp32 weight_scale[E*N]")
        _require(offsets.dtype == torch.int32 and offsets.numel() == weight.shape[0] + 1,
                 "expected int32 offsets[E+1]")
        _require(out.dtype == torch.bfloat16 and out.dim() == 2 and out.shape[0] == a.shape[0],
                 "expected BF16 out[R,N]")

    def grouped_gemm_swiglu_e4m3_out(self, packed_q, packed_scale, gate_up_q, gate_up_scale,
                                     offsets, activated):
        """Gate/up grouped GEMM on e4m3 operands with SwiGLU in its epilogue."""
        self._e4m3_checks(packed_q, packed_scale, gate_up_q, gate_up_scale, offsets, activated)
        experts, two_i, hidden = gate_up_q.shape
        _require(two_i % 2 == 0 and activated.shape[1] * 2 == two_i,
                 "expected gate_up[E,2I,H] and activated[R,I]")
        self._call(packed_q.device, self.lib.moe_grouped_gemm_swiglu_e4m3, packed_q.data_ptr(),
                   packed_scale.data_ptr(), gate_up_q.data_ptr(), gate_up_scale.data_ptr(),
                   offsets.data_ptr(), activated.data_ptr(), packed_q.shape[0], hidden,
                   two_i // 2, experts)

    def grouped_gemm_e4m3_out(self, a_q, a_scale, weight_q, weight_scale, offsets, out):
        """Plain grouped GEMM on e4m3 operands: out[r] = dequantised a[r] @ weight[e].T."""
        self._e4m3_checks(a_q, a_scale, weight_q, weight_scale, offsets, out)
        experts, n_cols, k_dim = weight_q.shape
        _require(out.shape[1] == n_cols, "expected out[R,N]")
        self._call(a_q.device, self.lib.moe_grouped_gemm_e4m3, a_q.data_ptr(), a_scale.data_ptr(),
                   weight_q.data_ptr(), weight_scale.data_ptr(), offsets.data_ptr(), out.data_ptr(),
                   a_q.shape[0], n_cols, k_dim, experts)

    # ------------------------------------------------------- expert parallel
    def ep_layout(self, counts, alignment, src_start, dst_start, offsets):
        """Receive layout from counts[P, E_l] (see include/moe_b200.h, moe_ep_layout)."""
        _require(counts.is_cuda and counts.dtype == torch.int32 and counts.dim() == 2,
                 "expected int32 CUDA counts[P,E_l]")
        ranks, experts = counts.shape
        for tensor in (src_start, dst_start, offsets):
            _check_cuda(tensor, counts, "ep_layout")
        _require(src_start.numel() == ranks * experts and dst_start.numel() == ranks * experts
                 and offsets.numel() == experts + 1, "incorrect layout buffers")
        self._call(counts.device, self.lib.moe_ep_layout, counts.data_ptr(), ranks, experts,
                   alignment, src_start.data_ptr(), dst_start.data_ptr(), offsets.data_ptr())

    def ep_regroup(self, source, target, counts, src_start, dst_start, offsets, recv_rows,
                   grouping):
        """Received rows -> grouped (grouping=True) or grouped -> received order."""
        _require(source.is_cuda and source.dim() == 2 and source.dtype in _DTYPE_CODES,
                 "expected CUDA rows[R,H]")
        for tensor in (target, counts, src_start, dst_start, offsets):
            _check_cuda(tensor, source, "ep_regroup")
        _require(target.dtype == source.dtype and target.shape[1] == source.shape[1],
                 "row shape/dtype mismatch")
        ranks, experts = counts.shape
        grouped = target if grouping else source
        self._call(source.device, self.lib.moe_ep_regroup, source.data_ptr(),
                   _DTYPE_CODES[source.dtype], target.data_ptr(), counts.data_ptr(),
                   src_start.data_ptr(), dst_start.data_ptr(), offsets.data_ptr(), ranks,
                   experts, source.shape[1], recv_rows, grouped.shape[0], int(bool(grouping)))

    def grouped_gemm_tile(self, rows, experts):
        """"pair" or "single": the tile the grouped GEMMs pick for this shape."""
        return "pair" if self.lib.moe_grouped_gemm_tile(int(rows), int(experts)) else "single"

    def device_status(self, clear=False):
        """Current device's kernel status word (0 = no bounded wait ran out)."""
        code = ctypes.c_int32(0)
        self._run(self.lib.moe_device_status(ctypes.addressof(code), int(bool(clear))))
        return code.value


@lru_cache(maxsize=1)
def _extension():
    return Extension(load_library())


def get_extension():
    """The loaded CUDA operators; RuntimeError without a GPU or without the library."""
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA operators require an NVIDIA GPU.")
    return _extension()
