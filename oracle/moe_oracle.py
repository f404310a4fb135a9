"""Python face of the CPU oracle (``moe_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py``.  The product package never imports
it.  Every function takes and returns CPU torch tensors and calls the C
restatement through ctypes; the C file cites the reference line each
function restates.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "libmoe_oracle.so"

_DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    source = HERE / "moe_oracle.c"
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < source.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


def library():
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            build()
        lib = ctypes.CDLL(str(LIBRARY))
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        lib.oracle_router_logits.argtypes = [p, p, i64, i32, i32, p]
        lib.oracle_topk_softmax.argtypes = [p, p, i64, i32, i32, p, p, p]
        lib.oracle_dispatch_index.argtypes = [p, i64, i32, i32, i32, p, p, p, p]
        lib.oracle_pack.argtypes = [p, i32, p, p, p, i64, i32, i32, i64, i64, p]
        lib.oracle_combine.argtypes = [p, i32, p, p, i64, i32, i64, i64, p]
        lib.oracle_swiglu.argtypes = [p, i32, i64, i64, i64, p]
        lib.oracle_grouped_gemm_bf16.argtypes = [p, p, p, i32, i64, i64, i64, p]
        lib.oracle_moe_tokens.argtypes = [p, p, p, p, p, i64, i32, i32, i32, p]
        lib.oracle_ep_layout.argtypes = [p, i32, i32, i32, p, p, p]
        lib.oracle_ep_regroup.argtypes = [p, i32, p, p, p, p, p, i32, i32, i64, i64, i32]
        lib.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_bf16.restype = ctypes.c_uint16
        lib.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_f16.restype = ctypes.c_uint16
        lib.oracle_f32_to_e4m3.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_e4m3.restype = ctypes.c_uint8
        lib.oracle_quantize_rows_e4m3.argtypes = [p, i64, i64, p, p]
        lib.oracle_num_threads.restype = ctypes.c_int
        lib.oracle_set_num_threads.argtypes = [ctypes.c_int]
        _lib = lib
    return _lib


def _ptr(tensor):
    if tensor is None:
        return None
    assert tensor.device.type == "cpu" and tensor.is_contiguous()
    return ctypes.c_void_p(tensor.data_ptr())


def _check(status, name):
    if status != 0:
        raise RuntimeError(f"{name} failed with status {status}")


def num_threads() -> int:
    return library().oracle_num_threads()


def set_num_threads(n: int) -> None:
    library().oracle_set_num_threads(int(n))


def router_logits(x, router_weight):
    """fp32 logits with the sequential-fmaf order the CUDA router also uses."""
    x = x.contiguous()
    w = router_weight.float().contiguous()
    tokens, hidden = x.shape
    logits = torch.empty(tokens, w.shape[0], dtype=torch.float32)
    _check(
        library().oracle_router_logits(
            _ptr(x.view(torch.int16)), _ptr(w), tokens, hidden, w.shape[0], _ptr(logits)
        ),
        "oracle_router_logits",
    )
    return logits


def topk_softmax(logits, bias, topk):
    logits = logits.float().contiguous()
    tokens, experts = logits.shape
    bias = None if bias is None else bias.float().contiguous()
    ids32 = torch.empty(tokens, topk, dtype=torch.int32)
    ids64 = torch.empty(tokens, topk, dtype=torch.int64)
    weights = torch.empty(tokens, topk, dtype=torch.float32)
    _check(
        library().oracle_topk_softmax(
            _ptr(logits), _ptr(bias), tokens, experts, topk, _ptr(ids32), _ptr(ids64), _ptr(weights)
        ),
        "oracle_topk_softmax",
    )
    return ids32, ids64, weights


def route(x, router_weight, bias, topk):
    logits = router_logits(x, router_weight)
    return (logits, *topk_softmax(logits, bias, topk))


def capacity_rows(tokens, experts, topk, alignment):
    """workspace.py:30-34: rows a packed buffer needs at a given alignment."""
    n = tokens * topk
    if alignment == 1:
        return n
    return (n + experts * (alignment - 1) + 1 + alignment - 1) // alignment * alignment


def dispatch_index(ids, experts, alignment=1):
    ids = ids.to(torch.int32).contiguous()
    tokens, topk = ids.shape
    counts = torch.empty(experts, dtype=torch.int32)
    offsets = torch.empty(experts + 1, dtype=torch.int32)
    slots = torch.empty(tokens * topk, dtype=torch.int32)
    inverse = torch.empty(tokens, topk, dtype=torch.int32)
    _check(
        library().oracle_dispatch_index(
            _ptr(ids), tokens, topk, experts, alignment, _ptr(counts), _ptr(offsets), _ptr(slots),
            _ptr(inverse),
        ),
        "oracle_dispatch_index",
    )
    return counts, offsets, slots, inverse


def pack(x, inverse, counts, offsets, packed_rows):
    x = x.contiguous()
    tokens, hidden = x.shape
    topk = inverse.shape[1]
    packed = torch.full((packed_rows, hidden), float("nan"), dtype=x.dtype)
    _check(
        library().oracle_pack(
            _ptr(x), _DTYPES[x.dtype], _ptr(inverse), _ptr(counts), _ptr(offsets), tokens, topk,
            counts.numel(), hidden, packed_rows, _ptr(packed),
        ),
        "oracle_pack",
    )
    return packed


def dispatch(x, ids, experts, alignment=1, packed_rows=None):
    """Full dispatch: counts, offsets, slots, inverse and the packed rows."""
    counts, offsets, slots, inverse = dispatch_index(ids, experts, alignment)
    if packed_rows is None:
        packed_rows = capacity_rows(x.shape[0], experts, ids.shape[1], alignment)
    packed = pack(x, inverse, counts, offsets, packed_rows)
    return counts, offsets, slots, inverse, packed


def combine(expert_output, inverse, weights):
    expert_output = expert_output.contiguous()
    inverse = inverse.to(torch.int32).contiguous()
    weights = weights.float().contiguous()
    tokens, topk = inverse.shape
    hidden = expert_output.shape[1]
    output = torch.empty(tokens, hidden, dtype=expert_output.dtype)
    _check(
        library().oracle_combine(
            _ptr(expert_output), _DTYPES[expert_output.dtype], _ptr(inverse), _ptr(weights), tokens,
            topk, hidden, expert_output.shape[0], _ptr(output),
        ),
        "oracle_combine",
    )
    return output


def swiglu(projection, valid_rows=None):
    projection = projection.contiguous()
    rows, width2 = projection.shape
    width = width2 // 2
    output = torch.empty(rows, width, dtype=projection.dtype)
    valid = rows if valid_rows is None else int(valid_rows)
    _check(
        library().oracle_swiglu(
            _ptr(projection), _DTYPES[projection.dtype], rows, width, valid, _ptr(output)
        ),
        "oracle_swiglu",
    )
    return output


def grouped_gemm(a, weight, offsets, out_rows=None):
    """out[r] = bf16(a[r] @ weight[e].T) for r in expert e's [offsets[e], offsets[e+1])."""
    a = a.contiguous()
    weight = weight.contiguous()
    experts, n_cols, k_dim = weight.shape
    rows = a.shape[0] if out_rows is None else out_rows
    out = torch.zeros(rows, n_cols, dtype=torch.bfloat16)
    _check(
        library().oracle_grouped_gemm_bf16(
            _ptr(a.view(torch.int16)), _ptr(weight.view(torch.int16)),
            _ptr(offsets.to(torch.int32).contiguous()), experts, n_cols, k_dim, rows,
            _ptr(out.view(torch.int16)),
        ),
        "oracle_grouped_gemm_bf16",
    )
    return out


def moe_tokens(x, ids, weights, gate_up, down):
    """Token-major block output for the given routed tokens (layer.py:200-214)."""
    x = x.contiguous()
    ids = ids.to(torch.int32).contiguous()
    weights = weights.float().contiguous()
    tokens, hidden = x.shape
    intermediate = down.shape[2]
    output = torch.empty(tokens, hidden, dtype=torch.bfloat16)
    _check(
        library().oracle_moe_tokens(
            _ptr(x.view(torch.int16)), _ptr(ids), _ptr(weights),
            _ptr(gate_up.contiguous().view(torch.int16)), _ptr(down.contiguous().view(torch.int16)),
            tokens, hidden, intermediate, ids.shape[1], _ptr(output.view(torch.int16)),
        ),
        "oracle_moe_tokens",
    )
    return output


def ep_layout(counts, alignment):
    """Expert-parallel receive layout from counts[P, E_l] (see moe_oracle.c)."""
    counts = counts.to(torch.int32).contiguous()
    ranks, experts = counts.shape
    src_start = torch.empty(ranks, experts, dtype=torch.int32)
    dst_start = torch.empty(ranks, experts, dtype=torch.int32)
    offsets = torch.empty(experts + 1, dtype=torch.int32)
    _check(library().oracle_ep_layout(_ptr(counts), ranks, experts, alignment, _ptr(src_start),
                                      _ptr(dst_start), _ptr(offsets)), "oracle_ep_layout")
    return src_start, dst_start, offsets


def ep_regroup(rows, counts, layout, grouped_rows=None, grouping=True):
    """Received rows -> grouped (grouping) or grouped rows -> received order."""
    counts = counts.to(torch.int32).contiguous()
    src_start, dst_start, offsets = layout
    ranks, experts = counts.shape
    rows = rows.contiguous()
    if grouping:
        out_rows = int(offsets[-1]) if grouped_rows is None else grouped_rows
        out = torch.full((out_rows, rows.shape[1]), float("nan"), dtype=rows.dtype)
        capacity = out_rows
    else:
        out = torch.empty((int(counts.sum()), rows.shape[1]), dtype=rows.dtype)
        capacity = rows.shape[0]
    _check(library().oracle_ep_regroup(
        _ptr(rows), _DTYPES[rows.dtype], _ptr(out), _ptr(counts), _ptr(src_start),
        _ptr(dst_start), _ptr(offsets), ranks, experts, rows.shape[1], capacity, int(grouping),
    ), "oracle_ep_regroup")
    return out


def block_forward(x, router_weight, bias, gate_up, down, topk, alignment=8):
    """The whole block in the reference's stage order (layer.py:184-197)."""
    experts = router_weight.shape[0]
    logits, ids32, ids64, weights = route(x, router_weight, bias, topk)
    counts, offsets, slots, inverse, packed = dispatch(x, ids32, experts, alignment)
    projection = grouped_gemm(packed, gate_up, offsets)
    activated = swiglu(projection, int(offsets[-1]))
    expert_output = grouped_gemm(activated, down, offsets)
    output = combine(expert_output, inverse, weights)
    return {
        "logits": logits, "ids32": ids32, "ids64": ids64, "weights": weights, "counts": counts,
        "offsets": offsets, "slots": slots, "inverse": inverse, "packed": packed,
        "projection": projection, "activated": activated, "expert_output": expert_output,
        "output": output,
    }



def f32_to_e4m3(value: float) -> int:
    """The e4m3 byte of one fp32 value (round to nearest even, saturating)."""
    return int(library().oracle_f32_to_e4m3(float(value)))


def quantize_rows_e4m3(x):
    """Per-row e4m3 quantisation of bf16 rows x[R,C] -> (q float8_e4m3fn [R,C], scale fp32 [R])."""
    assert x.dtype == torch.bfloat16 and x.dim() == 2
    x = x.contiguous()
    q = torch.empty(x.shape, dtype=torch.uint8)
    scale = torch.empty(x.shape[0], dtype=torch.float32)
    _check(library().oracle_quantize_rows_e4m3(_ptr(x), x.shape[0], x.shape[1], _ptr(q), _ptr(scale)),
           "oracle_quantize_rows_e4m3")
    return q.view(torch.float8_e4m3fn), scale
