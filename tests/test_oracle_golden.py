"""Pin the CPU oracle to golden vectors from the reference's PyTorch path.

The fixture is made by tests/golden/make_golden.py, which runs the reference
(src/moe_dispatch) itself.  Nothing here needs a GPU.
"""

from pathlib import Path

import pytest
import torch

import cases
from oracle import moe_oracle as oracle

GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden.pt", weights_only=True)


def _id(case):
    return "-".join(str(v) for v in case["spec"].values()) if "spec" in case else None


@pytest.mark.parametrize("case", GOLDEN["router"], ids=lambda c: str(tuple(c["spec"].values())))
def test_router_topk_matches_reference(case):
    spec = case["spec"]
    x, w, bias = cases.router_inputs(spec)
    assert cases.checksum(x) == case["x_checksum"]
    # Same fp32 logits in: ids exact, weights within the reference's own 2e-6
    # (tests/test_gpu_router.py:22-24).
    ids32, ids64, weights = oracle.topk_softmax(case["logits"], bias, spec["topk"])
    torch.testing.assert_close(ids32, case["ids"], rtol=0, atol=0)
    torch.testing.assert_close(ids64, case["ids"].long(), rtol=0, atol=0)
    torch.testing.assert_close(weights, case["weights"], rtol=2e-6, atol=2e-6)
    # The oracle's own summation order gives logits within fp32 rounding of
    # F.linear's; selections agree except at near-ties (none in these cases).
    logits = oracle.router_logits(x, w)
    scale = case["logits"].abs().max().clamp_min(1.0)
    assert float((logits - case["logits"]).abs().max() / scale) < 1e-5
    ids_own, _, _ = oracle.topk_softmax(logits, bias, spec["topk"])
    torch.testing.assert_close(ids_own, case["ids"], rtol=0, atol=0)


def test_router_ties_go_to_lowest_index():
    """Known answer of tests/test_gpu_router.py:27-38: zero logits -> ids [0, 1], weights 0.5."""
    for tokens in (0, 5):
        ids32, ids64, weights = oracle.topk_softmax(torch.zeros(tokens, 64), torch.zeros(64), 2)
        assert ids32.tolist() == [[0, 1]] * tokens
        assert torch.equal(weights, torch.full((tokens, 2), 0.5))


@pytest.mark.parametrize(
    "case", GOLDEN["transport"],
    ids=lambda c: "{shape}-{dtype}-a{alignment}".format(**c["spec"]).replace(" ", ""),
)
def test_dispatch_and_combine_match_reference(case):
    spec = case["spec"]
    tokens, hidden, experts, topk = spec["shape"]
    x = cases.transport_x(spec)
    assert cases.checksum(x) == case["x_checksum"]
    counts, offsets, slots, inverse, packed = oracle.dispatch(
        x, case["ids"], experts, spec["alignment"]
    )
    # counts/offsets bit-exact against both the reference as written and the
    # stable variant; the permutation bit-exact against the stable variant.
    for name in ("stable", "unstable"):
        torch.testing.assert_close(counts, case[f"{name}_counts"], rtol=0, atol=0)
        torch.testing.assert_close(offsets, case[f"{name}_offsets"], rtol=0, atol=0)
    torch.testing.assert_close(inverse, case["stable_inverse"], rtol=0, atol=0)
    # The reference as written (unstable sort) is a permutation of the same rows.
    assert sorted(case["unstable_inverse"].flatten().tolist()) == sorted(inverse.flatten().tolist())
    assert cases.checksum(packed[: int(offsets[-1])]) == case["packed_checksum"]
    # slots are within-expert ranks in token-major order.
    flat = case["ids"].flatten()
    for p in range(flat.numel()):
        assert int(slots[p]) == int((flat[:p] == flat[p]).sum())
    canonical = cases.canonical_expert_rows(tokens, topk, hidden, x.dtype, spec["seed"])
    expert_output = torch.zeros_like(packed)
    expert_output[inverse.flatten().long()] = canonical
    combined = oracle.combine(expert_output, inverse, case["weights"])
    # torch's CPU reduction over k is sequential in its vector body, which
    # covers whole blocks of 32 fp32 columns; the leftover columns of a row go
    # through a scalar path with another association order.  The oracle is
    # sequential everywhere: bit-exact on the vector columns, within one ulp of
    # the output type on the leftover ones.
    body = hidden - hidden % 32
    torch.testing.assert_close(combined[:, :body], case["combined"][:, :body], rtol=0, atol=0)
    tail = (combined[:, body:].float() - case["combined"][:, body:].float()).abs()
    ulp = {torch.float32: 2**-23, torch.float16: 2**-10, torch.bfloat16: 2**-7}[x.dtype]
    assert bool((tail <= case["combined"][:, body:].float().abs().clamp_min(2**-14) * ulp * 2).all())


@pytest.mark.parametrize("case", GOLDEN["swiglu"], ids=lambda c: str(tuple(c["spec"].values())))
def test_swiglu_matches_reference(case):
    projection = cases.swiglu_input(case["spec"])
    out = oracle.swiglu(projection)
    # Both sides round once from fp32; libm and torch's vector exp may differ
    # by an ulp of fp32, which can move at most one ulp of the output type.
    diff = (out.float() - case["output"].float()).abs()
    ulp = case["output"].float().abs().clamp_min(1e-3) * {
        torch.bfloat16: 2**-7, torch.float16: 2**-10, torch.float32: 2**-23}[out.dtype]
    assert bool((diff <= ulp).all())
    assert float((out != case["output"]).float().mean()) < 0.01


@pytest.mark.parametrize("case", GOLDEN["block"], ids=lambda c: c["spec"]["name"])
def test_block_matches_reference(case):
    spec = case["spec"]
    hidden, intermediate, experts, topk = spec["config"]
    router, gate_up, down = cases.block_weights(spec)
    assert cases.checksum(gate_up) ^ cases.checksum(down) ^ cases.checksum(router) == case[
        "weights_checksum"
    ]
    x = cases.block_input(spec)
    assert cases.checksum(x) == case["x_checksum"]
    bias = cases.block_bias(spec)
    result = oracle.block_forward(x, router, bias, gate_up, down, topk)
    torch.testing.assert_close(result["ids32"], case["ids"], rtol=0, atol=0)
    torch.testing.assert_close(result["weights"], case["route_weights"], rtol=2e-6, atol=2e-6)
    expected = case["output"].float()
    diff = (result["output"].float() - expected).abs()
    if expected.numel():
        rel_l2 = float(diff.norm() / expected.norm().clamp_min(1e-8))
        assert float(diff.max()) <= 1e-2 and rel_l2 <= 1e-3, (float(diff.max()), rel_l2)
    # The token-major evaluation agrees with the staged one.
    token_major = oracle.moe_tokens(x, result["ids32"], result["weights"], gate_up, down)
    if expected.numel():
        assert float((token_major.float() - result["output"].float()).abs().max()) <= 1e-2


GOLDEN_FULL = {c["workload"]: c for c in torch.load(
    Path(__file__).parent / "golden" / "golden_full.pt", weights_only=True)["full_size"]}


@pytest.mark.parametrize("name", list(GOLDEN_FULL))
def test_oracle_matches_reference_at_full_shapes(name):
    """The oracle against the reference's own MoEBlock(implementation="torch")
    on a token subset of each benchmark configuration (make_golden_full.py):
    routing exact, outputs within max-abs 1e-2 and relative L2 1e-3."""
    import psutil
    from moe_dispatch.routing import WORKLOADS, block_input, block_weights
    from parity import BLOCK_MAX_ABS, BLOCK_REL_L2, block_error

    w = WORKLOADS[name]
    weight_bytes = 3 * w.experts * w.hidden * w.intermediate * 2
    if psutil.virtual_memory().available < 2 * weight_bytes + (4 << 30):
        pytest.skip(f"{weight_bytes / 2**30:.1f} GiB of weights do not fit in host memory here")
    case = GOLDEN_FULL[name]
    weights, bias = block_weights(w)
    x = block_input(w)
    assert cases.checksum(x) == case["x_checksum"]
    assert (cases.checksum(weights.router) ^ cases.checksum(weights.gate_up[0])
            ^ cases.checksum(weights.down[-1])) == case["weights_checksum"]
    subset = case["tokens"]
    expected = oracle.block_forward(x[subset].contiguous(), weights.router, bias, weights.gate_up,
                                    weights.down, w.topk)
    assert torch.equal(expected["ids32"], case["ids"])
    # the two sides compute the logits in different fp32 orders (at H = 7168 they
    # differ by ~1e-5), so the softmax weights agree to that level, not to the
    # 2e-6 that identical logits give
    torch.testing.assert_close(expected["weights"], case["route_weights"], rtol=2e-5, atol=2e-5)
    max_abs, rel = block_error(expected["output"], case["output"])
    assert max_abs <= BLOCK_MAX_ABS and rel <= BLOCK_REL_L2, (max_abs, rel)


def test_oracle_e4m3_conversion_matches_torch():
    """The oracle's fp32 -> e4m3 conversion (round to nearest even, saturating)
    equals torch's float8_e4m3fn conversion everywhere inside +-448, including
    ties, subnormals and the largest finite value."""
    grid = torch.cat([
        torch.linspace(-448, 448, 20001),
        torch.logspace(-12, 2.65, 4001), -torch.logspace(-12, 2.65, 4001),
        # exact midpoints between neighbouring e4m3 values (ties go to even)
        (torch.arange(0, 126, dtype=torch.uint8).view(torch.float8_e4m3fn).float()[:-1]
         + torch.arange(1, 126, dtype=torch.uint8).view(torch.float8_e4m3fn).float()) / 2,
        torch.tensor([0.0, -0.0, 448.0, -448.0, 2.0**-9, 2.0**-10, 3 * 2.0**-10]),
    ])
    expected = grid.to(torch.float8_e4m3fn).view(torch.uint8)
    got = torch.tensor([oracle.f32_to_e4m3(float(v)) for v in grid], dtype=torch.uint8)
    assert torch.equal(got, expected)
    assert oracle.f32_to_e4m3(1000.0) == 0x7E and oracle.f32_to_e4m3(-1000.0) == 0xFE  # saturates


def test_oracle_quantize_rows_e4m3_dequantises_close():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(17, 256, generator=g).to(torch.bfloat16)
    x[4] = 0
    q, scale = oracle.quantize_rows_e4m3(x)
    assert float(scale[4]) == 1.0 and not bool(q[4].view(torch.uint8).any())
    deq = q.float() * scale[:, None]
    amax = x.float().abs().max(dim=1).values
    assert torch.allclose(q.float().abs().max(dim=1).values[amax > 0], torch.tensor(448.0))
    # e4m3 keeps 3 mantissa bits: each element within half an e4m3 step of x
    assert float(((deq - x.float()).abs() / (amax[:, None] + 1e-30)).max()) <= 2.0**-4
