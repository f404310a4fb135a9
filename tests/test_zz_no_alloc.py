"""moe_dispatch_no_alloc: the dispatch entry point for callers that cannot allocate.

Serving hosts that fix their device memory at start-up and forbid allocation
afterwards, and language bindings that hold only raw device pointers, cannot
provide the scratch buffer moe_dispatch asks for.  moe_dispatch_no_alloc uses a fixed
array compiled into the library instead.  This test calls it through the C ABI
twice in a row, with different shapes, and requires its results to equal the
regular entry point's bit for bit -- the same tolerance as every other
dispatch test.  The second call would expose any state the first one left
behind in the shared array.  The file is named to be collected last.
"""

import pytest
import torch

from moe_dispatch._extension import load_library
from moe_dispatch.routing import transport_case
from moe_dispatch.workspace import CudaWorkspace

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def no_alloc_dispatch(lib, x, ids, experts, alignment, packed_rows):
    tokens, hidden = x.shape
    topk = ids.shape[1]
    counts = torch.full((experts,), -7, dtype=torch.int32, device="cuda")
    offsets = torch.full((experts + 1,), -7, dtype=torch.int32, device="cuda")
    slots = torch.full((tokens * topk,), -7, dtype=torch.int32, device="cuda")
    inverse = torch.full((tokens, topk), -7, dtype=torch.int32, device="cuda")
    packed = torch.zeros(packed_rows, hidden, dtype=x.dtype, device="cuda")
    status = lib.moe_dispatch_no_alloc(
        x.data_ptr(), DTYPE_CODES[x.dtype], ids.data_ptr(), counts.data_ptr(), offsets.data_ptr(),
        slots.data_ptr(), packed.data_ptr(), inverse.data_ptr(), tokens, hidden, topk, experts,
        packed_rows, alignment, 1, torch.cuda.current_stream().cuda_stream,
    )
    assert status == 0, lib.moe_last_error().decode()
    torch.cuda.synchronize()
    return counts, offsets, slots, inverse, packed


@pytest.mark.parametrize("first, second", [
    ((2048, 256, 64, 8, torch.float16, "uniform", 8), (777, 4096, 8, 2, torch.bfloat16, "zipf", 1)),
])
def test_no_alloc_dispatch_matches_the_regular_entry_point(first, second):
    lib = load_library()
    for tokens, hidden, experts, topk, dtype, popularity, alignment in (first, second):
        x, ids, _ = transport_case(tokens, hidden, experts, topk, dtype, popularity, seed=tokens)
        x, ids = x.cuda(), ids.cuda()
        ws = CudaWorkspace(tokens, hidden, experts, topk, dtype, alignment=alignment)
        ws.dispatch(x, ids)
        counts, offsets, slots, inverse, packed = no_alloc_dispatch(
            lib, x, ids, experts, alignment, ws.capacity_rows
        )
        assert torch.equal(counts, ws.counts)
        assert torch.equal(offsets, ws.offsets)
        assert torch.equal(slots, ws.slots)
        assert torch.equal(inverse, ws.inverse)
        used = int(ws.offsets[-1])
        assert torch.equal(packed[:used].view(torch.int16), ws.packed[:used].view(torch.int16))


def test_no_alloc_dispatch_rejects_sizes_beyond_its_array():
    lib = load_library()
    # 2^20 assignments over 128 experts need 1024 * 128 table words > 65536
    status = lib.moe_dispatch_no_alloc(
        None, 2, None, None, None, None, None, None, 1 << 17, 64, 8, 128, 1 << 20, 1, 1, None
    )
    assert status == 1
    assert "no_alloc" in lib.moe_last_error().decode()
