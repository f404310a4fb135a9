"""Expert-parallel kernels and block on the GPU.

The layout/regroup kernels are checked bit for bit against the oracle's
restatement.  The block with one rank must equal MoEBlock bit for bit (same
rows per expert, same kernels).  With two or more GPUs, tests/ep_worker.py runs
under torchrun and checks every rank's slice against the single-GPU block.
"""

import os
import socket
import subprocess
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist

from oracle import moe_oracle as oracle

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def ext():
    from moe_dispatch import get_extension

    return get_extension()


@pytest.mark.parametrize("ranks,experts,alignment", [(3, 5, 8), (1, 8, 8), (8, 32, 16), (2, 4, 1)])
def test_layout_and_regroup_match_oracle(ext, ranks, experts, alignment):
    g = torch.Generator().manual_seed(ranks * 100 + experts)
    counts = torch.randint(0, 40, (ranks, experts), generator=g, dtype=torch.int32)
    counts[0, 0] = 0
    hidden = 136
    layout = oracle.ep_layout(counts, alignment)
    src_start = torch.empty(ranks, experts, dtype=torch.int32, device="cuda")
    dst_start = torch.empty_like(src_start)
    offsets = torch.empty(experts + 1, dtype=torch.int32, device="cuda")
    cc = counts.cuda()
    ext.ep_layout(cc, alignment, src_start, dst_start, offsets)
    assert torch.equal(src_start.cpu(), layout[0])
    assert torch.equal(dst_start.cpu(), layout[1])
    assert torch.equal(offsets.cpu(), layout[2])
    n_recv = int(counts.sum())
    rows = torch.randn(n_recv, hidden, generator=g).to(torch.bfloat16)
    grouped_rows = int(layout[2][-1]) + 3
    grouped = torch.full((grouped_rows, hidden), 7.0, dtype=torch.bfloat16, device="cuda")
    ext.ep_regroup(rows.cuda(), grouped, cc, src_start, dst_start, offsets, n_recv, True)
    expected = oracle.ep_regroup(rows, counts, layout)
    used = int(layout[2][-1])
    assert torch.equal(grouped[:used].cpu(), expected)
    back = torch.empty(n_recv, hidden, dtype=torch.bfloat16, device="cuda")
    ext.ep_regroup(grouped, back, cc, src_start, dst_start, offsets, n_recv, False)
    assert torch.equal(back.cpu(), rows)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("backend,fused_return,micro_batches,overlap,tile",
                         [("p2p", True, 1, True, None), ("p2p", True, 1, True, "pair"),
                          ("p2p", False, 1, True, "pair"), ("p2p", False, 1, False, None),
                          ("p2p", True, 1, False, None), ("nccl", False, 1, False, None),
                          ("p2p", False, 3, False, None), ("p2p", True, 2, False, "pair")])
def test_single_rank_expert_parallel_block_equals_moeblock(monkeypatch, backend, fused_return,
                                                           micro_batches, overlap, tile):
    """tile="pair" forces the CTA-pair GEMMs (and so the pair kernel's fused
    return) where the shape would pick one-CTA tiles."""
    if tile:
        monkeypatch.setenv("MOE_B200_GEMM_TILE", tile)
    from moe_dispatch.expert_parallel import ExpertParallelMoEBlock
    from moe_dispatch.layer import MoEBlock, MoEConfig, MoEWeights
    from moe_dispatch.routing import BlockWorkload, block_input, block_weights

    if not dist.is_initialized():
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_port()}", rank=0,
                                world_size=1, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", 0))
    try:
        workload = BlockWorkload("ep1", 300, 256, 128, 16, 4, seed=9, router_std=0.02)
        weights, bias = block_weights(workload)
        cfg = MoEConfig(workload.hidden, workload.intermediate, workload.experts, workload.topk)
        x = block_input(workload).cuda()
        single = MoEBlock(cfg, weights=MoEWeights(weights.router.cuda(), weights.gate_up.cuda(),
                                                  weights.down.cuda()))
        single.routing_bias.copy_(bias)
        ep = ExpertParallelMoEBlock(cfg, weights.router, weights.gate_up, weights.down,
                                    routing_bias=bias, backend=backend,
                                    fused_return=fused_return, micro_batches=micro_batches,
                                    overlap=overlap)
        expected = single(x).clone()
        assert torch.equal(ep(x).clone(), expected)
        assert torch.equal(ep(x).clone(), expected)
        y = torch.full_like(x, float("nan"))
        assert ep(x, out=y) is y
        assert torch.equal(y, expected)
        counts = torch.bincount(single.route(x)[1].flatten(), minlength=workload.experts)
        assert torch.equal(ep.last_send_counts().long().cpu(), counts.cpu())
        if backend == "p2p":
            from moe_dispatch.graphs import capture_forward

            graph, captured = capture_forward(ep, x)  # every micro-batch stream joins the capture
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(captured, expected)
            del graph
        assert ep.extension.device_status() == 0
        ep.close()
    finally:
        dist.destroy_process_group()


def test_p2p_wait_gives_up_and_reports_instead_of_hanging():
    """A flag nobody raises: the bounded wait must end, record status 2, and
    leave the context usable (no trap, no hang)."""
    import ctypes

    from moe_dispatch.expert_parallel import PeerExchange

    ext_ = __import__("moe_dispatch").get_extension()
    if not dist.is_initialized():
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_port()}", rank=0,
                                world_size=1, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", 0))
    try:
        ex = PeerExchange(ext_.lib, None, 1, 0, 8, 64, 64, 16, torch.device("cuda", 0))
        counts = torch.zeros(8, dtype=torch.int32, device="cuda")
        ext_.device_status(clear=True)
        stream = torch.cuda.current_stream().cuda_stream

        def op(code, aux=None):
            status = ext_.lib.moe_ep_p2p(code, None, None if aux is None else aux.data_ptr(),
                                         ctypes.addressof(ex.regions), ex.state.data_ptr(), 1, 0,
                                         8, 8, 64, 64, 16, 300, stream)
            assert status == 0, ext_.lib.moe_last_error().decode()

        op(0, counts)      # count exchange with itself: completes
        op(2)              # rows flag never raised: must time out after 300 ms
        torch.cuda.synchronize()
        assert ext_.device_status(clear=True) == 2
        assert torch.ones(4, device="cuda").sum().item() == 4.0  # context still usable
        ex.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_multi_gpu_expert_parallel_matches_single_gpu():
    gpus = min(torch.cuda.device_count(), 8)
    gpus = 8 if gpus >= 8 else (4 if gpus >= 4 else 2)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", str(ROOT / "tests" / "ep_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    result = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert result.returncode == 0, result.stdout[-3000:] + result.stderr[-3000:]


def _state_index(ranks, experts):
    """Word offsets of the P2P state tables (csrc/ep_p2p.cu, state_view)."""
    local = experts // ranks
    offsets = 4 + experts
    recv_prefix = offsets + local + 1 + 3 * ranks * local
    group_rows = recv_prefix + ranks * local + 1 + 2 * ranks
    return {"epoch": 0, "offsets": offsets, "group_rows": group_rows}


@pytest.mark.parametrize("tile", ["single", "pair"])
@pytest.mark.parametrize("raised", [True, False])
def test_gate_up_with_arrival_groups(monkeypatch, tile, raised):
    """moe_ep_p2p_gate_up on one GPU with a made-up 3-rank state: rows of each
    expert come in three arrival groups (sizes include 0 and ragged ones).
    With every rows flag raised the output equals moe_grouped_gemm_swiglu on
    the same rows bit for bit, whichever tile kind runs; with one flag left
    down the bounded wait gives up (status 6) and the context stays usable."""
    import ctypes

    from moe_dispatch import get_extension
    from moe_dispatch.expert_parallel import _DeviceArray

    monkeypatch.setenv("MOE_B200_GEMM_TILE", tile)
    ext_ = get_extension()
    lib = ext_.lib
    ranks, me, experts, hidden, inter, align = 3, 1, 6, 256, 128, 8
    local = experts // ranks
    g = torch.Generator().manual_seed(5)
    # rows from each arrival group (0 = this rank, 1 = rank me-1, 2 = rank me-2)
    groups = [[300, 0, 129], [1, 256, 40]]
    spans = [(sum(c) + align - 1) // align * align for c in groups]
    offsets = torch.tensor([0, spans[0], spans[0] + spans[1]], dtype=torch.int32)
    grouped_rows = int(offsets[-1]) + 16
    back_rows = 64
    nbytes = lib.moe_ep_p2p_region_bytes(ranks, experts, hidden, grouped_rows, back_rows)
    own = ctypes.c_void_p()
    handle = (ctypes.c_char * 64)()
    assert lib.moe_peer_alloc(nbytes, ctypes.addressof(own), ctypes.addressof(handle)) == 0
    regions = (ctypes.c_void_p * ranks)(own.value, own.value, own.value)
    try:
        g_off = lib.moe_ep_p2p_region_offset(ranks, experts, hidden, grouped_rows, back_rows, 0)
        rows = torch.randn(grouped_rows, hidden, generator=g).to(torch.bfloat16)
        weights = (torch.randn(local, 2 * inter, hidden, generator=g) / hidden**0.5).to(torch.bfloat16)
        # the region is raw device memory: views of its grouped rows and flags
        grouped = torch.as_tensor(_DeviceArray(own.value + g_off, (grouped_rows, hidden), "<i2"),
                                  device="cuda").view(torch.bfloat16)
        grouped.copy_(rows)
        idx = _state_index(ranks, experts)
        state = torch.zeros(lib.moe_ep_p2p_state_words(ranks, experts), dtype=torch.int32)
        epoch = 5
        state[idx["epoch"]] = epoch
        state[idx["offsets"]:idx["offsets"] + local + 1] = offsets
        for e in range(local):
            bounds = [0]
            for c in groups[e]:
                bounds.append(bounds[-1] + c)
            base = idx["group_rows"] + e * (ranks + 1)
            state[base:base + ranks + 1] = torch.tensor(bounds, dtype=torch.int32)
        state = state.cuda()
        # rows flags (second of the three flag arrays): source s at index 8 + s
        flags = torch.full((3 * 8,), epoch, dtype=torch.int32)
        if not raised:
            flags[8 + (me - 2) % ranks] = epoch - 1  # group 2 never arrives
        flags_off = ((ranks * experts * 4 + 255) // 256) * 256  # region_layout in ep_p2p.cu
        torch.as_tensor(_DeviceArray(own.value + flags_off, (flags.numel(),), "<i4"),
                        device="cuda").copy_(flags)
        wd = weights.cuda()
        activated = torch.full((grouped_rows, inter), -1.0, dtype=torch.bfloat16, device="cuda")
        ext_.device_status(clear=True)
        status = lib.moe_ep_p2p_gate_up(wd.data_ptr(), activated.data_ptr(),
                                        ctypes.addressof(regions), state.data_ptr(), ranks, me,
                                        experts, hidden, inter, grouped_rows, back_rows, 300,
                                        torch.cuda.current_stream().cuda_stream)
        assert status == 0, lib.moe_last_error().decode()
        torch.cuda.synchronize()
        if not raised:
            assert ext_.device_status(clear=True) == 6
            assert torch.ones(4, device="cuda").sum().item() == 4.0  # context still usable
            return
        assert ext_.device_status() == 0
        expected = torch.full_like(activated, -1.0)
        ext_.grouped_gemm_swiglu_out(grouped, wd, offsets.cuda(), expected)
        used = int(offsets[-1])
        assert torch.equal(activated[:used], expected[:used])
    finally:
        torch.cuda.synchronize()
        lib.moe_peer_free(own.value)
