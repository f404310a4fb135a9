"""Profiling drivers (reference: src/moe_dispatch/profiling.py, block_benchmark.py:221-247).

    python -m moe_dispatch.profiling --workload mixtral --stage experts --iters 2
    python -m moe_dispatch.profiling --workload small --trace trace.json

`--stage` runs one stage of the block `--iters` times after one untimed
forward, so an ncu capture (`-k regex:<kernel> -s 1 -c 1`) sees a warm launch
of that stage's kernel and few launches before it.  `--trace` writes a Chrome
trace of a few forwards with one record_function range per stage (the
reference's MoE/router, MoE/dispatch, MoE/grouped_experts, MoE/combine).
"""

from __future__ import annotations

import argparse
from pathlib import Path

import torch

STAGES = ("router", "dispatch", "experts", "gemm1", "gemm2", "combine", "forward")


def build(workload_name, device="cuda", tokens=None, experts=None):
    """Block + input for a named workload, weights drawn on the GPU."""
    from .layer import MoEBlock, MoEConfig, MoEWeights
    from .routing import WORKLOADS

    w = WORKLOADS[workload_name]
    tokens = tokens or w.tokens
    experts = experts or w.experts
    cfg = MoEConfig(w.hidden, w.intermediate, experts, min(w.topk, experts))
    g = torch.Generator(device=device).manual_seed(1000 + w.seed)
    router = torch.randn(experts, w.hidden, device=device, generator=g) / w.hidden**0.5
    gate_up = torch.empty(experts, 2 * w.intermediate, w.hidden, device=device, dtype=torch.bfloat16)
    down = torch.empty(experts, w.hidden, w.intermediate, device=device, dtype=torch.bfloat16)
    for e in range(experts):
        gate_up[e] = (torch.randn(2 * w.intermediate, w.hidden, device=device, generator=g)
                      / w.hidden**0.5).to(torch.bfloat16)
        down[e] = (torch.randn(w.hidden, w.intermediate, device=device, generator=g)
                   / w.intermediate**0.5).to(torch.bfloat16)
    block = MoEBlock(cfg, device=device, weights=MoEWeights(router, gate_up, down))
    x = torch.randn(tokens, w.hidden, device=device, generator=g).to(torch.bfloat16)
    return block, x


@torch.inference_mode()
def run_stage(block, x, stage, iters):
    block(x)
    state = block.workspace(x)
    t = state.transport
    ext = block.extension
    ids32, ids64, weights = block.route(x)
    t.dispatch(x, ids32, ids64)
    actions = {
        "router": lambda: block.route(x),
        "dispatch": lambda: t.dispatch(x, ids32, ids64),
        "experts": lambda: block.experts_forward(state),
        "gemm1": lambda: ext.grouped_gemm_swiglu_out(t.packed, block.gate_up_weight, t.offsets,
                                                      state.activated),
        "gemm2": lambda: ext.grouped_gemm_out(state.activated, block.down_weight, t.offsets,
                                              state.expert_output),
        "combine": lambda: t.combine(state.expert_output, weights),
        "forward": lambda: block(x),
    }
    for _ in range(iters):
        actions[stage]()
    torch.cuda.synchronize()
    return ext.device_status()


@torch.inference_mode()
def export_trace(block, x, destination, repeats=3):
    state = block.workspace(x)
    for _ in range(3):
        block(x)
    torch.cuda.synchronize()
    record = torch.autograd.profiler.record_function
    with torch.profiler.profile(
        activities=[torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA],
        record_shapes=True,
    ) as profiler:
        for _ in range(repeats):
            with record("MoE/router"):
                ids32, ids64, weights = block.route(x)
            with record("MoE/dispatch"):
                state.transport.dispatch(x, ids32, ids64)
            with record("MoE/grouped_experts"):
                block.experts_forward(state)
            with record("MoE/combine"):
                state.transport.combine(state.expert_output, weights)
        torch.cuda.synchronize()
    destination = Path(destination)
    destination.parent.mkdir(parents=True, exist_ok=True)
    profiler.export_chrome_trace(str(destination))
    return destination


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--workload", default="mixtral")
    parser.add_argument("--stage", choices=STAGES, default="experts")
    parser.add_argument("--iters", type=int, default=2)
    parser.add_argument("--tokens", type=int, default=None)
    parser.add_argument("--experts", type=int, default=None)
    parser.add_argument("--trace", default=None)
    args = parser.parse_args()
    block, x = build(args.workload, tokens=args.tokens, experts=args.experts)
    if args.trace:
        print(export_trace(block, x, args.trace))
        return 0
    status = run_stage(block, x, args.stage, args.iters)
    print(f"{args.workload} {args.stage} x{args.iters}: device status {status}")
    return 0 if status == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
