"""Dispatch / combine / SwiGLU parity on the GPU (reference: tests/test_gpu.py).

Counts, offsets, slots, inverse and packed rows are compared bit for bit
with the oracle's stable token-major order; combine bit for bit with the
oracle's fp32 rounding order.
"""

from pathlib import Path

import pytest
import torch

import cases
from oracle import moe_oracle as oracle
from moe_dispatch.routing import make_case, transport_case
from moe_dispatch.workspace import CudaWorkspace
from parity import assert_within_ulps

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]

# CUDA's expf and the CPU's differ by an ulp or two of fp32; after the multiply
# that is a few fp32 ulps, and at most one ulp of a 16-bit output.
SWIGLU_ULPS = {torch.float32: 16, torch.float16: 1, torch.bfloat16: 1}
SWIGLU_FRACTION = {torch.float32: 1.0, torch.float16: 0.05, torch.bfloat16: 0.05}

GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden.pt", weights_only=True)


@pytest.fixture(scope="module")
def ext():
    from moe_dispatch import get_extension

    return get_extension()


def check_against_oracle(ws, x, ids32, weights, experts, alignment, seed):
    tokens, hidden = x.shape
    topk = ids32.shape[1]
    ws.dispatch(x.cuda(), ids32.cuda())
    counts, offsets, slots, inverse, packed = oracle.dispatch(
        x.cpu(), ids32.cpu(), experts, alignment, packed_rows=ws.capacity_rows
    )
    assert torch.equal(ws.counts.cpu(), counts)
    assert torch.equal(ws.offsets.cpu(), offsets)
    assert torch.equal(ws.slots.cpu(), slots)
    assert torch.equal(ws.inverse.cpu(), inverse)
    used = int(offsets[-1])
    got = ws.packed[:used].cpu()
    want = packed[:used]
    if x.dtype == torch.float32:
        assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    else:
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    g = torch.Generator().manual_seed(seed + 501)
    canonical = torch.randn((tokens * topk, hidden), dtype=x.dtype, generator=g)
    expert_output = torch.zeros(ws.capacity_rows, hidden, dtype=x.dtype)
    expert_output[inverse.flatten().long()] = canonical
    ws.combine(expert_output.cuda(), weights.cuda())
    expected = oracle.combine(expert_output, inverse, weights)
    assert torch.equal(ws.output.cpu(), expected)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16])
@pytest.mark.parametrize("alignment", [1, 8])
@pytest.mark.parametrize("tokens", [0, 1, 33, 257])
@pytest.mark.parametrize("vectorized", [True, False])
def test_cuda_transport_empty_skew_and_partial_tiles(ext, dtype, alignment, tokens, vectorized):
    """tests/test_gpu.py:22-28 shapes (H=32, E=8, K=2, skewed), bit-exact."""
    x, i32, _, w = make_case(tokens, 32, 8, 2, dtype, "skewed", 42, device="cpu")
    ws = CudaWorkspace(tokens, 32, 8, 2, dtype, alignment=alignment, vectorized=vectorized,
                       extension=ext)
    check_against_oracle(ws, x, i32, w, 8, alignment, 42)


@pytest.mark.parametrize(
    "case", GOLDEN["transport"],
    ids=lambda c: "{shape}-{dtype}-a{alignment}".format(**c["spec"]).replace(" ", ""),
)
def test_golden_transport_cases(ext, case):
    spec = case["spec"]
    tokens, hidden, experts, topk = spec["shape"]
    x = cases.transport_x(spec)
    ws = CudaWorkspace(tokens, hidden, experts, topk, x.dtype, alignment=spec["alignment"],
                       extension=ext)
    ws.dispatch(x.cuda(), case["ids"].cuda())
    torch.testing.assert_close(ws.counts.cpu(), case["stable_counts"], rtol=0, atol=0)
    torch.testing.assert_close(ws.offsets.cpu(), case["stable_offsets"], rtol=0, atol=0)
    torch.testing.assert_close(ws.inverse.cpu(), case["stable_inverse"], rtol=0, atol=0)
    assert cases.checksum(ws.packed[: int(ws.offsets[-1])].cpu()) == case["packed_checksum"]
    check_against_oracle(ws, x, case["ids"], case["weights"], experts, spec["alignment"],
                         spec["seed"])


@pytest.mark.parametrize("popularity", ["uniform", "zipf"])
def test_transport_configuration_full_size(ext, popularity):
    """T4096 H4096 E64 top-8 fp16, uniform and Zipf(1.2) popularity, bit-exact."""
    x, ids, weights = transport_case(4096, 4096, 64, 8, torch.float16, popularity, seed=11)
    for alignment in (1, 8):
        ws = CudaWorkspace(4096, 4096, 64, 8, torch.float16, alignment=alignment, extension=ext)
        check_against_oracle(ws, x, ids, weights, 64, alignment, 11)
    if popularity == "zipf":
        assert int((ws.counts == 0).sum()) >= 0


def test_dispatch_is_deterministic_and_reusable(ext):
    x, ids, _ = transport_case(3000, 256, 64, 6, torch.bfloat16, "zipf", seed=5)
    ws = CudaWorkspace(3000, 256, 64, 6, torch.bfloat16, alignment=8, extension=ext)
    ws.dispatch(x.cuda(), ids.cuda())
    first = (ws.inverse.clone(), ws.packed.clone(), ws.offsets.clone())
    for _ in range(3):
        ws.dispatch(x.cuda(), ids.cuda())
        assert torch.equal(ws.inverse, first[0])
        assert torch.equal(ws.offsets, first[2])
        assert torch.equal(ws.packed[: int(first[2][-1])], first[1][: int(first[2][-1])])


@pytest.mark.parametrize("tokens,experts,topk", [(1, 8, 2), (3000, 8, 2), (4096, 8, 2),
                                                 (2000, 64, 4), (5000, 8, 2)])
def test_index_cluster_and_ticket_forms_agree(ext, monkeypatch, tokens, experts, topk):
    """Up to 8 index chunks (8192 assignments) the index CTAs hand their chunk
    totals to CTA 0 inside one thread-block cluster; MOE_B200_INDEX_CLUSTER=0
    keeps the completion-ticket form.  Both give the same bits, out-of-range
    counts included (3000 x 2: 6 chunks in a cluster of 8; 5000 x 2: 10
    chunks, the ticket form either way)."""
    x, ids, _ = transport_case(tokens, 64, experts, topk, torch.bfloat16, "zipf", seed=21)
    ids = ids.clone()
    ids[0, 0] = experts
    ids[tokens // 2, topk - 1] = -1
    results = {}
    for form in ("1", "0"):
        monkeypatch.setenv("MOE_B200_INDEX_CLUSTER", form)
        ws = CudaWorkspace(tokens, 64, experts, topk, torch.bfloat16, alignment=8, extension=ext)
        ws.dispatch(x.cuda(), ids.cuda())
        used = int(ws.offsets[-1])
        results[form] = (ws.counts.cpu(), ws.offsets.cpu(), ws.slots.cpu(), ws.inverse.cpu(),
                         ws.packed[:used].cpu(), ws.invalid_ids())
    for a, b in zip(results["1"], results["0"]):
        if isinstance(a, torch.Tensor):
            assert torch.equal(a, b)
        else:
            assert a == b
    assert results["1"][-1] == 2


def test_out_of_range_ids_are_skipped(ext):
    x = torch.randn(4, 16, dtype=torch.float16)
    ids = torch.tensor([[0, 9], [1, -1], [7, 2], [3, 3]], dtype=torch.int32)
    ws = CudaWorkspace(4, 16, 8, 2, torch.float16, extension=ext)
    ws.dispatch(x.cuda(), ids.cuda())
    counts, offsets, slots, inverse = oracle.dispatch_index(ids, 8, 1)
    assert torch.equal(ws.counts.cpu(), counts)
    assert torch.equal(ws.slots.cpu(), slots)
    assert torch.equal(ws.inverse.cpu(), inverse)
    assert int(ws.inverse[0, 1]) == -1 and int(ws.inverse[1, 1]) == -1
    assert ws.invalid_ids() == 2


def test_device_range_check_counts_without_host_sync(ext):
    """ops.dispatch(check_range="device"): no host check, the index kernel
    counts out-of-range ids per call (and the count resets between calls)."""
    from moe_dispatch import ops

    x, ids, _ = transport_case(2500, 128, 16, 4, torch.bfloat16, "uniform", seed=9)
    bad = ids.clone()
    bad[7, 1] = 16
    bad[1000, 0] = -3
    bad[2499, 3] = 99
    ws = CudaWorkspace(2500, 128, 16, 4, torch.bfloat16, extension=ext)
    with pytest.raises(ValueError):
        ops.dispatch(x.cuda(), bad.cuda(), 16, workspace=ws)
    batch = ops.dispatch(x.cuda(), bad.cuda(), 16, workspace=ws, check_range="device")
    assert int(batch.workspace.invalid_ids_device[0]) == 3
    with pytest.raises(ValueError, match="3 out-of-range"):
        ops.raise_on_invalid_ids(batch)
    counts, offsets, slots, inverse = oracle.dispatch_index(bad, 16, 1)
    assert torch.equal(ws.counts.cpu(), counts) and torch.equal(ws.inverse.cpu(), inverse)
    batch = ops.dispatch(x.cuda(), ids.cuda(), 16, workspace=ws, check_range="device")
    assert ws.invalid_ids() == 0
    ops.raise_on_invalid_ids(batch)
    with pytest.raises(ValueError):
        ops.dispatch(x.cuda(), ids.cuda(), 16, workspace=ws, check_range="sometimes")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16])
def test_swiglu_and_unused_rows(ext, dtype):
    """tests/test_gpu.py:31-40 of the reference, plus a check against the oracle."""
    projection = torch.randn(37, 34).to(dtype)
    output = torch.empty(37, 17, device="cuda", dtype=dtype)
    rows = torch.tensor([21], device="cuda", dtype=torch.int32)
    ext.swiglu_out(projection.cuda(), rows, output)
    expected = oracle.swiglu(projection, 21)
    assert_within_ulps(output.cpu(), expected, ulps=SWIGLU_ULPS[dtype],
                       max_fraction=SWIGLU_FRACTION[dtype], what="swiglu")
    torch.testing.assert_close(output[21:], torch.zeros_like(output[21:]), rtol=0, atol=0)


@pytest.mark.parametrize("case", GOLDEN["swiglu"], ids=lambda c: str(tuple(c["spec"].values())))
def test_swiglu_golden(ext, case):
    projection = cases.swiglu_input(case["spec"])
    rows, width = projection.shape[0], projection.shape[1] // 2
    output = torch.empty(rows, width, device="cuda", dtype=projection.dtype)
    valid = torch.tensor([rows], device="cuda", dtype=torch.int32)
    ext.swiglu_out(projection.cuda(), valid, output)
    assert_within_ulps(output.cpu(), case["output"], ulps=SWIGLU_ULPS[projection.dtype],
                       max_fraction=SWIGLU_FRACTION[projection.dtype], what="swiglu")
