"""Profiling drivers (reference: src/moe_dispatch/profiling.py, block_benchmark.py:221-247).

    python -m moe_dispatch.profiling --workload mixtral --stage experts --iters 2
    python -m moe_dispatch.profiling --workload small --trace trace.json
    python -m moe_dispatch.profiling --tile-sweep

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


class ClockProbe:
    """Median SM clock (MHz) and board power (W) over a code region, read
    through NVML every 5 ms by a background thread (read-only queries)."""

    def __init__(self, device_index):
        self.index = device_index
        self.samples = []

    def __enter__(self):
        import threading

        import pynvml

        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.index).uuid)
        handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        self._stop = threading.Event()

        def sample():
            while not self._stop.is_set():
                self.samples.append((pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM),
                                     pynvml.nvmlDeviceGetPowerUsage(handle) / 1000.0))
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=sample, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join()

    def summary(self):
        import statistics

        if not self.samples:
            return None, None
        return (statistics.median(c for c, _ in self.samples),
                round(statistics.median(w for _, w in self.samples), 1))


@torch.inference_mode()
def tile_sweep(cases=(("mixtral", 4096), ("fine_grained", 16384), ("expert_parallel", 8192),
                      ("expert_parallel", 32768)), warmup=3, iters=10, sustain_s=0.4):
    """Time both grouped GEMMs with each tile kind (JSON lines).

    Besides the event time of `iters` back-to-back launches, each line carries
    the median SM clock and board power over a `sustain_s` loop of the same
    launches, and kcycles = ms x MHz, the clock-independent cost: at this
    board's power cap a kernel that keeps the tensor pipe busier draws more
    power and runs at a lower clock.
    """
    import json
    import os
    import time

    previous = os.environ.get("MOE_B200_GEMM_TILE")
    try:
        for name, tokens in cases:
            block, x = build(name, tokens=tokens)
            block(x)
            state = block.workspace(x)
            t = state.transport
            ext = block.extension
            ids32, ids64, _ = block.route(x)
            t.dispatch(x, ids32, ids64)
            counts = t.counts.float().cpu()
            cfg = block.config
            n = tokens * cfg.topk
            stages = {
                "gate_up_swiglu": (lambda: ext.grouped_gemm_swiglu_out(
                    t.packed, block.gate_up_weight, t.offsets, state.activated),
                    2 * n * cfg.hidden * 2 * cfg.intermediate),
                "down": (lambda: ext.grouped_gemm_out(
                    state.activated, block.down_weight, t.offsets, state.expert_output),
                    2 * n * cfg.intermediate * cfg.hidden),
            }
            for tile in ("single", "pair"):
                os.environ["MOE_B200_GEMM_TILE"] = tile
                for stage, (fn, flops) in stages.items():
                    for _ in range(warmup):
                        fn()
                    torch.cuda.synchronize()
                    start = torch.cuda.Event(enable_timing=True)
                    end = torch.cuda.Event(enable_timing=True)
                    start.record()
                    for _ in range(iters):
                        fn()
                    end.record()
                    torch.cuda.synchronize()
                    ms = start.elapsed_time(end) / iters
                    repeats = max(1, int(sustain_s * 1e3 / ms))
                    with ClockProbe(torch.cuda.current_device()) as probe:
                        t0 = time.perf_counter()
                        for _ in range(repeats):
                            fn()
                        torch.cuda.synchronize()
                        sustained_ms = (time.perf_counter() - t0) * 1e3 / repeats
                    mhz, watts = probe.summary()
                    print(json.dumps({"workload": name, "tokens": tokens, "tile": tile,
                                      "gemm": stage, "ms": round(ms, 4),
                                      "tflops": round(flops / ms / 1e9, 1),
                                      "sustained_ms": round(sustained_ms, 4),
                                      "sm_mhz": mhz, "watts": watts,
                                      "kcycles": round(sustained_ms * mhz, 1) if mhz else None,
                                      "rows_per_expert_mean": float(counts.mean()),
                                      "rows_per_expert_max": float(counts.max())}), flush=True)
            del block, x, state, t
            torch.cuda.empty_cache()
    finally:
        if previous is None:
            os.environ.pop("MOE_B200_GEMM_TILE", None)
        else:
            os.environ["MOE_B200_GEMM_TILE"] = previous


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
    parser.add_argument("--tile-sweep", action="store_true")
    args = parser.parse_args()
    if args.tile_sweep:
        tile_sweep()
        return 0
    block, x = build(args.workload, tokens=args.tokens, experts=args.experts)
    if args.trace:
        print(export_trace(block, x, args.trace))
        return 0
    status = run_stage(block, x, args.stage, args.iters)
    print(f"{args.workload} {args.stage} x{args.iters}: device status {status}")
    return 0 if status == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
