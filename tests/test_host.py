"""Host-side logic that needs no GPU (reference: tests/test_api.py, test_block.py)."""

import pytest
import torch

from moe_dispatch.layer import MoEBlock, MoEConfig, make_weights
from moe_dispatch.ops import validate_inputs
from moe_dispatch.routing import WORKLOADS, block_input, block_weights, make_case, transport_case
from moe_dispatch.workspace import CudaWorkspace, capacity_rows
from oracle import moe_oracle as oracle
import cases


@pytest.mark.parametrize(
    "bad_ids", [torch.tensor([[0.0, 1.0]]), torch.tensor([[-1, 0]]), torch.tensor([[0, 8]])]
)
def test_invalid_expert_ids_are_rejected(bad_ids):
    with pytest.raises((TypeError, ValueError)):
        validate_inputs(torch.randn(1, 32), bad_ids, 8)


def test_forward_only_contract_is_explicit():
    with pytest.raises(ValueError, match="forward-only"):
        validate_inputs(torch.randn(1, 32, requires_grad=True), torch.tensor([[0, 1]]), 8)


def test_cpu_workspace_does_not_compile_cuda():
    with pytest.raises(RuntimeError, match="CUDA GPU"):
        CudaWorkspace(1, 32, 8, 2, torch.float32, device="cpu")


def test_invalid_block_shapes_fail_early():
    with pytest.raises(ValueError, match="multiples of 8"):
        MoEConfig(hidden=17)
    with pytest.raises(ValueError, match="expert/topk"):
        MoEConfig(experts=1, topk=2)
    with pytest.raises(ValueError, match="expert/topk"):
        MoEConfig(experts=300, topk=2)
    # the limits this engine lifts from the reference's (<=64 experts, top-k 1..2)
    assert MoEConfig(7168, 2048, 256, 8).topk == 8


def test_block_has_no_cpu_path():
    with pytest.raises(ValueError, match="CUDA implementations only"):
        MoEBlock(MoEConfig(32, 64, 8, 2), device="cpu", implementation="torch")
    with pytest.raises(RuntimeError, match="require CUDA"):
        MoEBlock(MoEConfig(32, 64, 8, 2), device="cpu")


@pytest.mark.parametrize("tokens,experts,topk,alignment", [(0, 8, 2, 8), (33, 8, 2, 1),
                                                          (4096, 8, 2, 8), (100, 64, 6, 16)])
def test_capacity_rows_matches_the_reference_formula(tokens, experts, topk, alignment):
    assert capacity_rows(tokens, experts, topk, alignment) == oracle.capacity_rows(
        tokens, experts, topk, alignment
    )


def test_make_weights_matches_the_golden_generator():
    spec = cases.BLOCK_CASES[0]
    hidden, intermediate, experts, topk = spec["config"]
    ours = make_weights(MoEConfig(hidden, intermediate, experts, topk), "cpu", torch.bfloat16,
                        spec["weight_seed"])
    router, gate_up, down = cases.block_weights(spec)
    assert torch.equal(ours.router, router)
    assert torch.equal(ours.gate_up, gate_up)
    assert torch.equal(ours.down, down)


def test_make_case_matches_the_golden_generator():
    spec = cases.TRANSPORT_CASES[5]
    tokens, hidden, experts, topk = spec["shape"]
    x, ids32, ids64, weights = make_case(tokens, hidden, experts, topk, cases.DTYPES[spec["dtype"]],
                                         spec["pattern"], spec["seed"], device="cpu")
    assert torch.equal(x, cases.transport_x(spec))
    assert torch.equal(ids32.long(), ids64)


@pytest.mark.parametrize("popularity", ["uniform", "zipf"])
def test_transport_ids_are_distinct_per_token(popularity):
    x, ids, weights = transport_case(64, 32, 64, 8, torch.float16, popularity, seed=3)
    assert ids.shape == (64, 8)
    for row in ids.tolist():
        assert len(set(row)) == 8 and all(0 <= e < 64 for e in row)
    torch.testing.assert_close(weights.sum(1), torch.ones(64))
    again = transport_case(64, 32, 64, 8, torch.float16, popularity, seed=3)
    assert torch.equal(ids, again[1]) and torch.equal(x, again[0])


def test_zipf_leaves_experts_cold():
    _, ids, _ = transport_case(4096, 8, 64, 8, torch.float16, "zipf", seed=1)
    counts = torch.bincount(ids.flatten().long(), minlength=64)
    assert counts.max() > 4 * counts.float().mean()


def test_block_workload_generators_are_shardable():
    w = WORKLOADS["small"]
    full, bias = block_weights(w)
    part, _ = block_weights(w, experts=3, first_expert=2)
    assert torch.equal(full.gate_up[2:5], part.gate_up)
    assert torch.equal(full.down[2:5], part.down)
    x = block_input(w)
    assert torch.equal(block_input(w, tokens=16, first_token=32), x[32:48])
    assert bias.abs().sum() == 0


def test_explicit_output_buffer_is_checked_on_the_host():
    from moe_dispatch.layer import check_out

    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    check_out(None, x)
    check_out(torch.empty_like(x), x)
    for bad in (torch.empty(5, 8, dtype=torch.bfloat16), torch.empty(4, 8),
                torch.empty(8, 4, dtype=torch.bfloat16).t()):
        with pytest.raises(ValueError):
            check_out(bad, x)


def test_host_pipeline_needs_a_cuda_block():
    from moe_dispatch.host_pipeline import HostPipeline

    class CpuBlock:
        class config:
            hidden = 8

    with pytest.raises(RuntimeError):
        HostPipeline(CpuBlock(), 4, device="cpu")
    with pytest.raises(ValueError):
        HostPipeline(CpuBlock(), 4, device="cpu", slots=1)


def test_range_check_can_be_left_to_the_device():
    x = torch.zeros(3, 8)
    ids = torch.tensor([[0], [5], [1]], dtype=torch.int32)
    with pytest.raises(ValueError):
        validate_inputs(x, ids, 4)
    validate_inputs(x, ids, 4, check_range=False)


def test_block_benchmark_cases_and_percentile_follow_the_reference():
    from moe_dispatch import block_benchmark as bb

    assert len(bb.workload_cases("smoke")) == 2
    assert len(bb.workload_cases("quick")) == 8
    assert [t for t, _, _ in bb.workload_cases("model")] == [128, 256]
    assert bb.percentile([1.0, 2.0, 3.0, 4.0, 5.0], 0.5) == 3.0
    assert bb.percentile([1.0, 2.0], 0.95) == pytest.approx(1.95)
    assert bb.percentile([], 0.5) == 0.0
    hashes = bb.source_hashes()
    assert "gemm_sm100.cu" in hashes and "layer.py" in hashes and "moe_b200.h" in hashes
    with pytest.raises(ValueError):
        bb.workload_cases("everything")
