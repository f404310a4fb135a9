"""Whole-block parity on the GPU (reference: tests/test_gpu.py:43-48 and the
block checks of block_benchmark.py:29-45).

Routing (ids) and dispatch are bit-exact against the oracle; block outputs
are within the north-star tolerance (max-abs 1e-2, relative L2 1e-3) of the
oracle and of the reference's own outputs stored in the golden fixture.  The
full benchmark shapes are covered by test_gpu_full_size.py.
"""

from pathlib import Path

import pytest
import torch

import cases
from oracle import moe_oracle as oracle
from moe_dispatch.layer import MoEBlock, MoEConfig, MoEWeights
from moe_dispatch.graphs import capture_forward
from parity import BLOCK_MAX_ABS, BLOCK_REL_L2, block_error

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]

GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden.pt", weights_only=True)


class DuckConfig:
    def __init__(self, hidden, intermediate, experts, topk, alignment=8):
        self.hidden, self.intermediate, self.experts, self.topk = hidden, intermediate, experts, topk
        self.alignment = alignment


def golden_block(spec, implementation="cuda_fused"):
    hidden, intermediate, experts, topk = spec["config"]
    router, gate_up, down = cases.block_weights(spec)
    block = MoEBlock(MoEConfig(hidden, intermediate, experts, topk), implementation=implementation,
                     weights=MoEWeights(router.cuda(), gate_up.cuda(), down.cuda()))
    block.routing_bias.copy_(cases.block_bias(spec))
    return block, (router, gate_up, down)


@pytest.mark.parametrize("case", GOLDEN["block"], ids=lambda c: c["spec"]["name"])
def test_block_matches_oracle_and_reference(case):
    spec = case["spec"]
    block, (router, gate_up, down) = golden_block(spec)
    x = cases.block_input(spec)
    out = block(x.cuda()).clone().cpu()
    ids32, _, weights = block.route(x.cuda())
    expected = oracle.block_forward(x, router, cases.block_bias(spec), gate_up, down,
                                    spec["config"][3])
    assert torch.equal(ids32.cpu(), expected["ids32"])
    assert torch.equal(ids32.cpu(), case["ids"])  # the reference's own selection
    torch.testing.assert_close(weights.cpu(), expected["weights"], rtol=2e-6, atol=2e-6)
    for name, ref in (("oracle", expected["output"]), ("reference", case["output"])):
        max_abs, rel = block_error(out, ref)
        assert max_abs <= BLOCK_MAX_ABS and rel <= BLOCK_REL_L2, (name, max_abs, rel)


def test_cuda_and_cuda_fused_agree_bit_for_bit():
    spec = GOLDEN["block"][0]["spec"]
    fused, _ = golden_block(spec, "cuda_fused")
    plain, _ = golden_block(spec, "cuda")
    x = cases.block_input(spec).cuda()
    assert torch.equal(fused(x).clone(), plain(x).clone())


def test_graph_replay_matches_eager():
    spec = GOLDEN["block"][0]["spec"]
    block, _ = golden_block(spec)
    x = cases.block_input(spec).cuda()
    eager = block(x).clone()
    graph, output = capture_forward(block, x)
    x.copy_(cases.block_input(spec).cuda())
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(output, eager)


def test_workspace_reuse_and_empty_batch():
    spec = GOLDEN["block"][0]["spec"]
    block, _ = golden_block(spec)
    x = cases.block_input(spec).cuda()
    first = block.workspace(x)
    block(x)
    assert block.workspace(x) is first
    empty = block(torch.empty(0, spec["config"][0], dtype=torch.bfloat16, device="cuda"))
    assert empty.shape == (0, spec["config"][0])
