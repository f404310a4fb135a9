"""Profiling drivers (reference: src/moe_dispatch/profiling.py, block_benchmark.py:221-247).

    python -m moe_dispatch.profiling --workload mixtral --stage experts --iters 2
    python -m moe_dispatch.profiling --workload small --trace trace.json
    python -m moe_dispatch.profiling --transport

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


def build(workload_name, device="cuda", tokens=None, experts=None, intermediate=None):
    """Block + input for a named workload: the workload's router and routing
    bias (so the expert loads are skewed as in the benchmark), expert weights
    and tokens drawn on the GPU."""
    from .layer import MoEBlock, MoEConfig, MoEWeights
    from .routing import WORKLOADS, block_router

    w = WORKLOADS[workload_name]
    tokens = tokens or w.tokens
    experts = experts or w.experts
    inter = intermediate or w.intermediate  # a small one keeps router captures small
    cfg = MoEConfig(w.hidden, inter, experts, min(w.topk, experts))
    g = torch.Generator(device=device).manual_seed(1000 + w.seed)
    router, bias = block_router(w)
    router, bias = router[:experts].to(device), bias[:experts]
    gate_up = torch.empty(experts, 2 * inter, w.hidden, device=device, dtype=torch.bfloat16)
    down = torch.empty(experts, w.hidden, inter, device=device, dtype=torch.bfloat16)
    for e in range(experts):
        gate_up[e] = (torch.randn(2 * inter, w.hidden, device=device, generator=g)
                      / w.hidden**0.5).to(torch.bfloat16)
        down[e] = (torch.randn(w.hidden, inter, device=device, generator=g)
                   / inter**0.5).to(torch.bfloat16)
    block = MoEBlock(cfg, device=device, weights=MoEWeights(router, gate_up, down))
    block.routing_bias.copy_(bias)
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
def transport_sweep(tokens=4096, hidden=4096, experts=64, topk=8, dtype=torch.float16,
                    repeats=20, stage=None, iters=None, verbose=True):
    """The transport-only configuration (dispatch + combine, no router or experts):
    T=4096, H=4096 fp16 rows, E=64, top-8, uniform and Zipf(1.2) expert popularity.

    One JSON line per (popularity, stage) with the median CUDA-event time of
    `repeats` launches, each after writing a 256 MB buffer so that no input is
    left in L2, and the achieved algorithmic GB/s: dispatch reads x once and
    writes n packed rows (+ ids and inverse, n*8 bytes); combine reads the n
    rows and writes x's shape (+ inverse and weights).  With `stage`
    ("dispatch" or "combine") it only runs that stage `iters` times (for ncu).
    Returns the lines as dicts.
    """
    import json
    import statistics

    from .routing import transport_case
    from .workspace import CudaWorkspace

    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    element = torch.empty((), dtype=dtype).element_size()
    lines = []
    n = tokens * topk
    algorithmic = {"dispatch": tokens * hidden * element + n * hidden * element + n * 8,
                   "combine": n * hidden * element + tokens * hidden * element + n * 8}
    for popularity in ("uniform", "zipf"):
        x, ids, weights = transport_case(tokens, hidden, experts, topk, dtype, popularity, seed=0)
        x, ids32, weights = x.cuda(), ids.to(torch.int32).cuda(), weights.float().cuda()
        ws = CudaWorkspace(tokens, hidden, experts, topk, dtype)
        ws.dispatch(x, ids32)
        expert_output = torch.randn(ws.packed.shape, device="cuda").to(dtype)
        runs = {"dispatch": lambda: ws.dispatch(x, ids32),
                "combine": lambda: ws.combine(expert_output, weights)}
        if stage is not None:
            for _ in range(iters or 1):
                runs[stage]()
            torch.cuda.synchronize()
            continue
        for name, fn in runs.items():
            samples = []
            for _ in range(repeats):
                flush.zero_()
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record()
                fn()
                end.record()
                torch.cuda.synchronize()
                samples.append(start.elapsed_time(end))
            ms = statistics.median(samples)
            lines.append({"config": "transport", "popularity": popularity, "stage": name,
                          "us": round(ms * 1e3, 2),
                          "gbs": round(algorithmic[name] / (ms / 1e3) / 1e9, 1),
                          "algorithmic_bytes": algorithmic[name]})
            if verbose:
                print(json.dumps(lines[-1]), flush=True)
        del ws, x, ids32, weights, expert_output
    return lines


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
    parser.add_argument("--intermediate", type=int, default=None,
                        help="override the expert width (router captures need no real experts)")
    parser.add_argument("--trace", default=None)
    parser.add_argument("--transport", action="store_true",
                        help="time dispatch and combine at the transport-only configuration")
    parser.add_argument("--transport-stage", choices=["dispatch", "combine"], default=None)
    args = parser.parse_args()
    if args.transport or args.transport_stage:
        transport_sweep(stage=args.transport_stage, iters=args.iters)
        return 0
    block, x = build(args.workload, tokens=args.tokens, experts=args.experts,
                     intermediate=args.intermediate)
    if args.trace:
        print(export_trace(block, x, args.trace))
        return 0
    status = run_stage(block, x, args.stage, args.iters)
    print(f"{args.workload} {args.stage} x{args.iters}: device status {status}")
    return 0 if status == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
