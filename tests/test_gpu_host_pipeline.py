"""Host-buffer pipeline: batches in pinned host memory, copies overlapped with
compute.  Every output must equal the block run on the same batch on the
device, bit for bit (the pipeline only moves bytes)."""

import pytest
import torch

from moe_dispatch.host_pipeline import HostPipeline
from moe_dispatch.layer import MoEBlock, MoEConfig, MoEWeights
from moe_dispatch.routing import WORKLOADS, block_input, block_weights

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]


def make_block(name):
    w = WORKLOADS[name]
    weights, bias = block_weights(w)
    block = MoEBlock(MoEConfig(w.hidden, w.intermediate, w.experts, w.topk),
                     weights=MoEWeights(weights.router.cuda(), weights.gate_up.cuda(),
                                        weights.down.cuda()))
    block.routing_bias.copy_(bias)
    return block


@pytest.mark.parametrize("batches,slots", [(1, 2), (2, 2), (5, 2), (7, 3)])
def test_pipeline_matches_device_forward(batches, slots):
    w = WORKLOADS["small"]
    block = make_block("small")
    inputs = [block_input(w, first_token=i * w.tokens).pin_memory() for i in range(batches)]
    outputs = [torch.empty_like(inputs[0]).pin_memory() for _ in range(batches)]
    pipe = HostPipeline(block, w.tokens, slots=slots)
    pipe.run(inputs, outputs)
    for x, got in zip(inputs, outputs):
        expected = block(x.cuda()).cpu()
        assert torch.equal(got, expected)
    assert block.extension.device_status() == 0


def test_pipeline_reuses_host_buffers_and_runs_twice():
    """Outputs written to the same host buffer in order; a second run sees the
    slots' events from the first and still gives the same bits."""
    w = WORKLOADS["small"]
    block = make_block("small")
    a = block_input(w).pin_memory()
    b = block_input(w, first_token=w.tokens).pin_memory()
    out = [torch.empty_like(a).pin_memory() for _ in range(2)]
    pipe = HostPipeline(block, w.tokens)
    for _ in range(2):
        pipe.run([a, b, a, b, a], [out[0], out[1], out[0], out[1], out[0]])
        assert torch.equal(out[0], block(a.cuda()).cpu())
        assert torch.equal(out[1], block(b.cuda()).cpu())


@pytest.mark.parametrize("slots", [2, 3])
def test_graph_replayed_pipeline_matches_device_forward(slots):
    """graphs=True replays one captured forward per slot: same bits as eager."""
    w = WORKLOADS["small"]
    block = make_block("small")
    inputs = [block_input(w, first_token=i * w.tokens).pin_memory() for i in range(5)]
    outputs = [torch.empty_like(inputs[0]).pin_memory() for _ in range(5)]
    pipe = HostPipeline(block, w.tokens, slots=slots, graphs=True)
    for _ in range(2):
        pipe.run(inputs, outputs)
        for x, got in zip(inputs, outputs):
            assert torch.equal(got, block(x.cuda()).cpu())
    pipe.close()
    assert block.extension.device_status() == 0


def test_forward_out_argument():
    w = WORKLOADS["small"]
    block = make_block("small")
    x = block_input(w).cuda()
    y = torch.full_like(x, float("nan"))
    assert block(x, out=y) is y
    assert torch.equal(y, block(x))
    with pytest.raises(ValueError):
        block(x, out=torch.empty(x.shape[0] + 1, x.shape[1], dtype=x.dtype, device=x.device))
    with pytest.raises(ValueError):
        block(x, out=torch.empty_like(x, dtype=torch.float32))


def test_pipeline_rejects_bad_host_tensors():
    w = WORKLOADS["small"]
    block = make_block("small")
    pipe = HostPipeline(block, w.tokens)
    good = block_input(w).pin_memory()
    with pytest.raises(ValueError):
        pipe.run([block_input(w)], [torch.empty_like(good).pin_memory()])  # not pinned
    with pytest.raises(ValueError):
        pipe.run([good], [torch.empty(w.tokens + 1, w.hidden, dtype=good.dtype).pin_memory()])
    with pytest.raises(ValueError):
        pipe.run([good, good], [torch.empty_like(good).pin_memory()])
    with pytest.raises(ValueError):
        HostPipeline(block, w.tokens, slots=1)
