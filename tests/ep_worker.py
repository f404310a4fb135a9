"""Multi-GPU expert-parallel check, one process per GPU (launched by
tests/test_gpu_ep.py through torchrun when two or more GPUs are present).

Every rank builds the same weights, runs the single-GPU MoEBlock on all tokens
and the expert-parallel block on its own token slice, and requires the two to
agree bit for bit on its slice.
"""

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT / "cuda-moe-engine_b200", ROOT):
    sys.path.insert(0, str(path))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    from moe_dispatch.expert_parallel import ExpertParallelMoEBlock, expert_range
    from moe_dispatch.layer import MoEBlock, MoEConfig, MoEWeights
    from moe_dispatch.routing import BlockWorkload, block_input, block_weights

    status = 0
    # (backend, micro-batches, exchange overlapped with the gate/up GEMM, down
    # GEMM returning the rows itself)
    variants = (("p2p", 1, True, False), ("p2p", 1, True, True), ("p2p", 1, False, False),
                ("nccl", 1, False, False), ("p2p", 2, False, False), ("p2p", 3, False, True))
    cases = [(w,) + v for w in (BlockWorkload("ep_check", 512, 256, 128, 8, 2, seed=3),
                                BlockWorkload("ep_check_fine", 768, 128, 64, 64, 6, seed=4,
                                              router_std=0.02, zipf_bias=1.1))
             for v in variants]
    for workload, backend, micro_batches, overlap, fused_return in cases:
        weights, bias = block_weights(workload)
        x = block_input(workload).cuda()
        cfg = MoEConfig(workload.hidden, workload.intermediate, workload.experts, workload.topk)
        single = MoEBlock(cfg, weights=MoEWeights(weights.router.cuda(), weights.gate_up.cuda(),
                                                  weights.down.cuda()))
        single.routing_bias.copy_(bias)
        expected = single(x).clone()
        first, local_experts = expert_range(workload.experts, world, rank)
        ep = ExpertParallelMoEBlock(cfg, weights.router, weights.gate_up[first:first + local_experts],
                                    weights.down[first:first + local_experts], routing_bias=bias,
                                    backend=backend, micro_batches=micro_batches, overlap=overlap,
                                    fused_return=fused_return)
        per_rank = workload.tokens // world
        mine = x[rank * per_rank:(rank + 1) * per_rank].contiguous()
        for _ in range(2):  # reuse of the grown buffers
            out = ep(mine).clone()
        ok = torch.equal(out, expected[rank * per_rank:(rank + 1) * per_rank])
        if backend == "p2p":
            # replayed as a CUDA graph (every stream of the step joins the capture)
            from moe_dispatch.graphs import capture_forward

            graph, captured = capture_forward(ep, mine)
            for _ in range(2):
                graph.replay()
            torch.cuda.synchronize()
            ok = ok and torch.equal(captured, expected[rank * per_rank:(rank + 1) * per_rank])
            del graph
        ok = ok and ep.extension.device_status() == 0
        ep.close()
        flag = torch.tensor([0 if ok else 1], device="cuda")
        dist.all_reduce(flag)
        if rank == 0:
            print(f"{workload.name} [{backend}, {micro_batches} micro-batches, overlap {overlap}, "
                  f"fused return {fused_return}]: world {world}, mismatching ranks "
                  f"{int(flag.item())}", flush=True)
        status |= int(flag.item() != 0)
    dist.destroy_process_group()
    return status


if __name__ == "__main__":
    sys.exit(main())
