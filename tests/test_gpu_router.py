"""Router parity on the GPU (reference: tests/test_gpu_router.py)."""

from pathlib import Path

import pytest
import torch

import cases
from oracle import moe_oracle as oracle

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]

GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden.pt", weights_only=True)


@pytest.fixture(scope="module")
def ext():
    from moe_dispatch import get_extension

    return get_extension()


def _route_buffers(tokens, topk):
    return (
        torch.empty(tokens, topk, device="cuda", dtype=torch.int32),
        torch.empty(tokens, topk, device="cuda", dtype=torch.int64),
        torch.empty(tokens, topk, device="cuda"),
    )


@pytest.mark.parametrize("experts", [2, 8, 16, 64])
@pytest.mark.parametrize("topk", [1, 2])
def test_fused_router_matches_independent_pytorch(ext, experts, topk):
    """tests/test_gpu_router.py:11-24 of the reference, unchanged in substance."""
    generator = torch.Generator(device="cuda").manual_seed(42)
    logits = torch.randn(257, experts, device="cuda", generator=generator)
    bias = torch.randn(experts, device="cuda", generator=generator)
    ids32, ids64, weights = _route_buffers(257, topk)
    ext.topk_route_out(logits, bias, ids32, ids64, weights)
    selected, expected_ids = torch.topk(logits + bias, topk, dim=-1)
    torch.testing.assert_close(ids64, expected_ids, rtol=0, atol=0)
    torch.testing.assert_close(ids32, expected_ids.int(), rtol=0, atol=0)
    torch.testing.assert_close(weights, selected.softmax(-1), rtol=2e-6, atol=2e-6)


def test_fused_router_ties_and_empty_tokens(ext):
    """tests/test_gpu_router.py:27-38: zero logits -> ids [0,1], weights exactly 0.5."""
    for tokens in (0, 5):
        logits = torch.zeros(tokens, 64, device="cuda")
        bias = torch.zeros(64, device="cuda")
        ids32, ids64, weights = _route_buffers(tokens, 2)
        ext.topk_route_out(logits, bias, ids32, ids64, weights)
        expected = torch.tensor([0, 1], device="cuda").expand(tokens, 2)
        torch.testing.assert_close(ids64, expected, rtol=0, atol=0)
        torch.testing.assert_close(weights, torch.full_like(weights, 0.5), rtol=0, atol=0)


@pytest.mark.parametrize("experts,topk", [(64, 6), (256, 8), (100, 7), (33, 32)])
def test_topk_beyond_reference_limits_matches_oracle(ext, experts, topk):
    generator = torch.Generator().manual_seed(experts * 7 + topk)
    logits = torch.randn(513, experts, generator=generator)
    # inject exact ties so the lowest-index rule is exercised
    logits[::5, 3] = logits[::5, 1]
    bias = torch.randn(experts, generator=generator)
    ids32, ids64, weights = _route_buffers(513, topk)
    ext.topk_route_out(logits.cuda(), bias.cuda(), ids32, ids64, weights)
    e32, e64, ew = oracle.topk_softmax(logits, bias, topk)
    torch.testing.assert_close(ids32.cpu(), e32, rtol=0, atol=0)
    torch.testing.assert_close(ids64.cpu(), e64, rtol=0, atol=0)
    torch.testing.assert_close(weights.cpu(), ew, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("case", GOLDEN["router"], ids=lambda c: str(tuple(c["spec"].values())))
def test_route_from_x_is_bit_exact_against_oracle_and_golden(ext, case):
    spec = case["spec"]
    x, w, bias = cases.router_inputs(spec)
    tokens, experts, topk = spec["tokens"], spec["experts"], spec["topk"]
    ids32, ids64, weights = _route_buffers(tokens, topk)
    logits = torch.empty(tokens, experts, device="cuda")
    ext.route_out(x.cuda(), w.cuda(), bias.cuda(), logits, ids32, ids64, weights)
    expected_logits = oracle.router_logits(x, w)
    # Same sequential fp32 FMA chain on both sides: identical bits.
    assert torch.equal(logits.cpu(), expected_logits)
    e32, _, ew = oracle.topk_softmax(expected_logits, bias, topk)
    torch.testing.assert_close(ids32.cpu(), e32, rtol=0, atol=0)
    torch.testing.assert_close(weights.cpu(), ew, rtol=2e-6, atol=2e-6)
    # And the reference's own selection (F.linear logits + torch.topk) agrees.
    torch.testing.assert_close(ids32.cpu(), case["ids"], rtol=0, atol=0)
    torch.testing.assert_close(weights.cpu(), case["weights"], rtol=2e-6, atol=2e-6)


def test_route_large_expert_parallel_shape(ext):
    """256 experts, top-8, H=7168 (the expert-parallel configuration's router)."""
    g = torch.Generator().manual_seed(2)
    tokens, hidden, experts, topk = 300, 7168, 256, 8
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16)
    w = torch.randn(experts, hidden, generator=g) * 0.02
    bias = torch.zeros(experts)
    ids32, ids64, weights = _route_buffers(tokens, topk)
    logits = torch.empty(tokens, experts, device="cuda")
    ext.route_out(x.cuda(), w.cuda(), bias.cuda(), logits, ids32, ids64, weights)
    expected_logits = oracle.router_logits(x, w)
    assert torch.equal(logits.cpu(), expected_logits)
    e32, _, _ = oracle.topk_softmax(expected_logits, bias, topk)
    assert torch.equal(ids32.cpu(), e32)
