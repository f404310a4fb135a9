#!/usr/bin/env python
"""MoE-block benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the Mixtral-shaped block (T=4096 tokens per GPU, H=4096, I=14336,
E=8, top-2, bf16 experts, fp32 router), synthetic inputs drawn from seeded
generators.  A step is one forward of the block over one batch: router,
dispatch, gate/up GEMM with fused SwiGLU, down GEMM, combine.

  value      whole-job tokens/s with inputs resident in HBM: K replays of a
             CUDA graph of one step, CUDA events on the launching stream,
             barrier + synchronize on both sides, max over ranks.
             `value_per_gpu` is value / N.
  e2e        the same metric through the public host-buffer API
             (moe_dispatch.HostPipeline with per-slot CUDA graphs): every step
             copies its batch from pinned host memory to the GPU, runs
             block(x, out=y) and copies y back to pinned host memory; the
             copies run on two copy streams and overlap the neighbouring
             steps' compute.
  roofline   the gate/up+SwiGLU GEMM (the dominant kernel): algorithmic FLOPs
             per launch / its mean CUDA-event duration over K eager steps.
  cpu_baseline  the reference's own PyTorch path (MoEBlock(implementation=
             "torch", device="cpu"), imported from baseline/_ref) on a bounded
             token sample of the same workload with every host core, rank 0,
             N=1 only; beside it (`port`) the C restatement of that path (the
             test oracle) on the same sample.
  transport_config  the metric's second half (dispatch+combine HBM GB/s) on its
             own configuration, transport only: T=4096 H=4096 fp16, E=64, top-8,
             uniform and Zipf(1.2) popularity, each launch after an L2 flush
             (N=1 only).
  fine_grained_config  the fine-grained block (T=16384 H=2048 I=1408 E=64
             top-6, log-Zipf routing bias) on one GPU: eager and graph tokens/s,
             both GEMMs against the tensor peak, dispatch+combine GB/s (N=1).
  fp8_config the same block with e4m3 gate/up experts (an extension beyond the
             reference's bf16 path): tokens/s, the e4m3 GEMM's TFLOP/s and the
             output's relative L2 distance from the bf16 block (N=1).
  expert_parallel_config  the E=256 block (T=32768 per step, H=7168 I=2048
             top-8): at N=1 the single-GPU block; at N>1 experts sharded over
             the ranks with the tokens split (strong scaling), checked against
             the single-GPU block and timed beside it on rank 0.

With N > 1 (torchrun, one process per GPU) the block runs expert-parallel:
the E experts are sharded evenly over the N ranks (rank r owns E/N of them),
each rank routes its own T tokens (weak scaling), and token rows travel to
their experts' ranks and back over NVLink peer memory (ExpertParallelMoEBlock,
backend "p2p": no host sync, so the step is replayed as a CUDA graph; the
down GEMM's epilogue stores the result rows straight back to their ranks
(`--ep-fused-return 0` uses a separate return copy instead);
`--ep-overlap 1` sends the rows beside an arrival-ordered gate/up GEMM;
`--ep-backend nccl` uses NCCL all-to-all instead, eager, one host sync per step;
`--ep-micro-batches m` pipelines m token slices so the exchanges overlap the
previous slice's GEMMs).  Before timing, every rank runs the same tokens
through a single-GPU block holding all experts and compares the outputs bit
for bit (`ep_parity`).  `--workload expert_parallel` makes the E=256 block the
main line.  `--impl reference` times the reference's own PyTorch path on the
host cores instead (rank 0 only; the other ranks exit without work), on the
same workload config; at N=1 it adds the reference's own GPU path
(`cuda_fused` with its Triton grouped GEMM) as `reference_gpu`.
"""

from __future__ import annotations

import argparse
import importlib
import importlib.util
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from dataclasses import dataclass
from pathlib import Path

ROOT = Path(__file__).resolve().parent
REFERENCE_SITE = ROOT / "baseline" / "_ref"
REFERENCE_ALIAS = "reference_moe_dispatch"
_GPU_WORKER = "--reference-gpu-worker" in sys.argv
if _GPU_WORKER:
    # the reference's own package is `moe_dispatch`: this process sees only it
    sys.path.insert(0, str(REFERENCE_SITE))
else:
    for _p in (ROOT / "cuda-moe-engine_b200", ROOT):
        if str(_p) not in sys.path:
            sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "MoE-block tokens/s/GPU (H4096 I14336 E8 top2); dispatch+combine HBM GB/s"


def workload_config(workload, world):
    """The `config` object both arms print for the single-GPU (or replica) workload."""
    h, i = workload.hidden, workload.intermediate
    return {
        "workload": f"{workload.name}: T={workload.tokens}/GPU H={h} I={i} E={workload.experts} "
                    f"top{workload.topk}, fp32 router, bf16 experts",
        "tokens_per_gpu": workload.tokens, "hidden": h, "intermediate": i,
        "experts": workload.experts, "topk": workload.topk,
        "parallelism": "replicas" if world > 1 else "single GPU",
    }


def kernels_per_step(experts):
    """Engine kernels per forward: route (1 fused up to 32 experts, else logits + top-k),
    dispatch (index + pack), two grouped GEMMs, combine."""
    return (1 if experts <= 32 else 2) + 2 + 2 + 1


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description="MoE block benchmark")
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", default="mixtral")
    parser.add_argument("--cpu-sample-tokens", type=int, default=1024,
                        help="tokens in the CPU-baseline sample of our arm")
    parser.add_argument("--reference-sample-tokens", type=int, default=512,
                        help="tokens per step of --impl reference on the host cores")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-extra-configs", action="store_true",
                        help="skip the fine-grained and E=256 configuration legs")
    parser.add_argument("--no-reference-gpu", action="store_true",
                        help="--impl reference: skip the reference's own GPU path")
    parser.add_argument("--ep-backend", choices=["p2p", "nccl"], default=None,
                        help="expert-parallel exchange for N > 1 (default p2p up to 8 GPUs)")
    parser.add_argument("--ep-micro-batches", type=int, default=1,
                        help="p2p only: token slices pipelined so exchanges overlap the GEMMs")
    parser.add_argument("--ep-overlap", type=int, choices=[0, 1], default=None,
                        help="p2p: exchange beside the arrival-ordered gate/up GEMM (default off)")
    parser.add_argument("--ep-fused-return", type=int, choices=[0, 1], default=None,
                        help="p2p: the down GEMM returns the rows itself (default: the block's)")
    parser.add_argument("--reference-gpu-worker", action="store_true", help=argparse.SUPPRESS)
    return parser.parse_args(argv)


def dist_info():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def host_threads():
    """Host cores this process may run on (torchrun's OMP_NUM_THREADS=1 aside)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (every 20 ms) of SM clock and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self):
        self.file.flush()
        rows = [line.split(",") for line in Path(self.file.name).read_text().splitlines()]
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, value in zip(names, r[5:9]):
                if value.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data["hbm_gbs"], data["bf16_tflops"], data.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def profiled_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if any."""
    for path in sorted((ROOT / "profiles").glob("*.md")):
        match = re.search(rf"{kernel}\s+traffic_bytes_per_launch:\s*([0-9.eE+]+)", path.read_text())
        if match:
            return float(match.group(1))
    return None


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(value, world, device):
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def all_ranks_true(flag, world, device):
    if world == 1:
        return bool(flag)
    t = torch.tensor([0 if flag else 1], dtype=torch.int32, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return int(t.item()) == 0
# ----------------------------------------------------------- inputs on the GPU
def gpu_router(workload, device):
    """Router [E,H] fp32 and routing bias [E] of `workload`: N(0,1)/sqrt(H) rows
    (or N(0, router_std)), and a log-Zipf(s) bias -s*log(rank) when the
    workload asks for skewed load."""
    w = workload
    g = torch.Generator(device=device).manual_seed(1000 + w.seed)
    router = torch.randn(w.experts, w.hidden, device=device, generator=g)
    router = router * w.router_std if w.router_std > 0 else router / w.hidden ** 0.5
    bias = torch.zeros(w.experts)
    if w.zipf_bias > 0:
        rank = torch.randperm(w.experts, generator=torch.Generator().manual_seed(w.seed)).float()
        bias = -w.zipf_bias * torch.log(rank + 1.0)
    return router, bias.to(device)


def gpu_experts(workload, device, first, count):
    """Experts [first, first + count), each from its own seeded generator, so
    an expert-parallel shard holds the same bytes as the full set."""
    w = workload
    gate_up = torch.empty(count, 2 * w.intermediate, w.hidden, device=device, dtype=torch.bfloat16)
    down = torch.empty(count, w.hidden, w.intermediate, device=device, dtype=torch.bfloat16)
    for e in range(count):
        ge = torch.Generator(device=device).manual_seed(2000 + w.seed * 1000 + first + e)
        gate_up[e] = (torch.randn(2 * w.intermediate, w.hidden, device=device, generator=ge)
                      / w.hidden ** 0.5).to(torch.bfloat16)
        down[e] = (torch.randn(w.hidden, w.intermediate, device=device, generator=ge)
                   / w.intermediate ** 0.5).to(torch.bfloat16)
    return gate_up, down


def gpu_tokens(workload, device, tokens, rank=0):
    """x ~ N(0,1) bf16 [tokens, H], one generator per rank."""
    g = torch.Generator(device=device).manual_seed(3000 + workload.seed * 1000 + rank)
    return torch.randn(tokens, workload.hidden, device=device, generator=g).to(torch.bfloat16)


def build_block(workload, device, tokens=None, rank=0):
    """The single-GPU block of `workload` holding every expert, and its input."""
    from moe_dispatch.layer import MoEBlock, MoEConfig, MoEWeights

    w = workload
    router, bias = gpu_router(w, device)
    gate_up, down = gpu_experts(w, device, 0, w.experts)
    block = MoEBlock(MoEConfig(w.hidden, w.intermediate, w.experts, w.topk), device=device,
                     weights=MoEWeights(router, gate_up, down))
    block.routing_bias.copy_(bias)
    x = gpu_tokens(w, device, w.tokens if tokens is None else tokens, rank)
    return block, x


def ep_tokens_per_rank(workload, world):
    """The expert-parallel configuration fixes T per step and splits it over the
    ranks (strong scaling); the other workloads keep T tokens per GPU (weak)."""
    if workload.name == "expert_parallel":
        return workload.tokens // world, "strong"
    return workload.tokens, "weak"


def build_ep_block(workload, device, rank, world, backend=None, micro_batches=1, overlap=None,
                   fused_return=None):
    """This rank's shard of the workload: all router rows, E/world experts, its tokens."""
    from moe_dispatch.expert_parallel import ExpertParallelMoEBlock, expert_range
    from moe_dispatch.layer import MoEConfig

    w = workload
    cfg = MoEConfig(w.hidden, w.intermediate, w.experts, w.topk)
    first, local = expert_range(w.experts, world, rank)
    router, bias = gpu_router(w, device)
    gate_up, down = gpu_experts(w, device, first, local)
    if backend == "nccl" or (backend is None and world > 8):
        micro_batches = 1
    options = {}
    if fused_return is not None:
        options["fused_return"] = bool(fused_return)
    if overlap is not None and micro_batches == 1 and backend != "nccl":
        options["overlap"] = bool(overlap)
    block = ExpertParallelMoEBlock(cfg, router, gate_up, down, device=device, routing_bias=bias,
                                   backend=backend, micro_batches=micro_batches, **options)
    tokens, _ = ep_tokens_per_rank(w, world)
    return block, gpu_tokens(w, device, tokens, rank)


def ep_parity(block, x, workload, device):
    """Run this rank's tokens through a single-GPU block holding all experts and
    compare with the expert-parallel output bit for bit.  Returns (equal,
    max |difference|)."""
    full, _ = build_block(workload, device, tokens=0)
    with torch.inference_mode():
        expected = full(x).clone()
        got = block(x).clone()
    torch.cuda.synchronize()
    equal = torch.equal(got, expected)
    diff = float((got.float() - expected.float()).abs().max()) if x.shape[0] else 0.0
    del full, expected, got
    torch.cuda.empty_cache()
    return equal, diff


# ------------------------------------------------------------- timing helpers
def step_instrumented(block, x, events):
    """One forward with events around router, dispatch, both GEMMs and combine."""
    state = block.workspace(x)
    transport = state.transport
    ext = block.extension
    events["route"][0].record()
    ids32, ids64, weights = block.route(x)
    events["route"][1].record()
    events["dispatch"][0].record()
    transport.dispatch(x, ids32, ids64)
    events["dispatch"][1].record()
    events["gemm1"][0].record()
    ext.grouped_gemm_swiglu_out(transport.packed, block.gate_up_weight, transport.offsets,
                                state.activated)
    events["gemm1"][1].record()
    events["gemm2"][0].record()
    ext.grouped_gemm_out(state.activated, block.down_weight, transport.offsets,
                         state.expert_output)
    events["gemm2"][1].record()
    events["combine"][0].record()
    transport.combine(state.expert_output, weights)
    events["combine"][1].record()
    return transport.output


STAGES = ("route", "dispatch", "gemm1", "gemm2", "combine")


def time_graph(block, x, steps, warmup, world, device, clocks_index=None):
    """K replays of a CUDA graph of one forward after W eager and 3+ graph
    warm-up steps; barrier + synchronize on both sides, max over ranks.
    Returns (ms per step, clock summary or None)."""
    from moe_dispatch.graphs import capture_forward

    stream = torch.cuda.current_stream(device)
    with torch.inference_mode():
        for _ in range(warmup):
            block(x)
        torch.cuda.synchronize()
        barrier(world)
        graph, _ = capture_forward(block, x)
        for _ in range(max(warmup, 3)):
            graph.replay()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        sampler = ClockSampler(clocks_index) if clocks_index is not None else None
        if sampler:
            sampler.__enter__()
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
        if sampler:
            sampler.__exit__(None, None, None)
        barrier(world)
        total = max_over_ranks(start.elapsed_time(end), world, device)
        del graph
    return total / steps, (sampler.summary() if sampler else None)


def time_stages(block, x, steps, world, device):
    """Mean CUDA-event ms of each stage over K eager instrumented steps, and
    the eager ms per step (max over ranks)."""
    stream = torch.cuda.current_stream(device)
    with torch.inference_mode():
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        start.record(stream)
        per_step = []
        for _ in range(steps):
            events = {n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                      for n in STAGES}
            step_instrumented(block, x, events)
            per_step.append(events)
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    stage = {n: statistics.mean(e[n][0].elapsed_time(e[n][1]) for e in per_step) for n in STAGES}
    eager = max_over_ranks(start.elapsed_time(end), world, device) / steps
    return stage, eager


def time_host_pipeline(block, x, steps, world, device):
    """Per-step ms of K batches through HostPipeline (pinned host in and out,
    per-slot CUDA graphs)."""
    from moe_dispatch.host_pipeline import HostPipeline, pinned_on_device_node

    pipe = HostPipeline(block, x.shape[0], device=device, graphs=True)
    # batches pinned on the GPU's own memory node (matters with several ranks per host)
    hosts = pinned_on_device_node([x.cpu(), x.cpu() * -1], device)
    outs = pinned_on_device_node([torch.empty_like(hosts[0]) for _ in hosts], device)
    pipe.run(hosts, outs)  # warm-up: fills both slots once
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record(stream)
    pipe.run([hosts[i % 2] for i in range(steps)], [outs[i % 2] for i in range(steps)],
             synchronize=False)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    h2d, d2h = pipe.bytes_per_batch()
    pipe.close()
    return max_over_ranks(start.elapsed_time(end), world, device) / steps, h2d, d2h


@dataclass
class Traffic:
    """Algorithmic bytes and FLOPs of one forward (b = 2 bytes per bf16 element)."""

    route: float
    dispatch: float
    combine: float
    gemm1_flops: float
    gemm2_flops: float


def algorithmic(workload, tokens):
    w = workload
    n = tokens * w.topk
    h, i = w.hidden, w.intermediate
    route = tokens * h * 2 + w.experts * h * 4 + n * 16 + (tokens * w.experts * 8 if w.experts > 32 else 0)
    return Traffic(route=route,
                   dispatch=tokens * h * 2 + n * h * 2 + n * 8,
                   combine=n * h * 2 + tokens * h * 2 + n * 8,
                   gemm1_flops=2.0 * n * h * 2 * i,
                   gemm2_flops=2.0 * n * i * h)


def gemm_kernel_name(block, rows, experts, swiglu=True, arrival_groups=False):
    """The grouped GEMM kernel a launch of this shape runs, and its tile: a
    bf16 pair launch of one arrival group runs the operand-swapped pair tile
    unless MOE_B200_GEMM_SWAP=0."""
    tile = block.extension.grouped_gemm_tile(rows, experts)
    if tile.startswith("pair"):
        swapped = not arrival_groups and os.environ.get("MOE_B200_GEMM_SWAP", "1") != "0"
        base = "grouped_gemm_swap_kernel" if swapped else "grouped_gemm_pair_kernel"
        tile = "operand-swapped pair" if swapped else "pair"
    else:
        base = "grouped_gemm_kernel"
    return f"{base}<{1 if swiglu else 0}>", tile
def stage_summary(workload, tokens, stage, block, rows, tf_peak, hbm_peak):
    """Per-stage ms, both GEMMs against the tensor peak, router and
    dispatch+combine against the HBM peak."""
    a = algorithmic(workload, tokens)
    g1 = a.gemm1_flops / (stage["gemm1"] / 1e3) / 1e12
    g2 = a.gemm2_flops / (stage["gemm2"] / 1e3) / 1e12
    dc = (a.dispatch + a.combine) / ((stage["dispatch"] + stage["combine"]) / 1e3) / 1e9
    route = a.route / (stage["route"] / 1e3) / 1e9
    k1, tile = gemm_kernel_name(block, rows, workload.experts)
    return {
        "stage_ms": {"route": round(stage["route"], 4), "dispatch": round(stage["dispatch"], 4),
                     "gate_up_swiglu_gemm": round(stage["gemm1"], 4),
                     "down_gemm": round(stage["gemm2"], 4), "combine": round(stage["combine"], 4)},
        "gemm_tile": tile,
        "gate_up_tflops": round(g1, 1), "gate_up_frac_of_peak": round(g1 / tf_peak, 4),
        "down_tflops": round(g2, 1), "down_frac_of_peak": round(g2 / tf_peak, 4),
        "dispatch_combine_gbs": round(dc, 1), "dispatch_combine_frac_of_hbm": round(dc / hbm_peak, 4),
        "route_gbs": round(route, 1), "route_frac_of_hbm": round(route / hbm_peak, 4),
    }


def single_gpu_leg(workload, device, steps, warmup, tf_peak, hbm_peak):
    """One configuration on one GPU: graph-replayed and eager tokens/s and the
    stage summary; the block is freed afterwards."""
    block, x = build_block(workload, device)
    graph_ms, _ = time_graph(block, x, steps, warmup, 1, device)
    stage, eager_ms = time_stages(block, x, steps, 1, device)
    rows = block.workspace(x).transport.packed.shape[0]
    summary = stage_summary(workload, x.shape[0], stage, block, rows, tf_peak, hbm_peak)
    status = block.extension.device_status()
    tokens = x.shape[0]
    del block, x
    torch.cuda.empty_cache()
    return {
        "workload": workload_config(workload, 1)["workload"],
        "ms_per_step": round(graph_ms, 4), "tokens_per_s": round(tokens / (graph_ms / 1e3), 1),
        "eager_ms_per_step": round(eager_ms, 4),
        "eager_tokens_per_s": round(tokens / (eager_ms / 1e3), 1),
        **summary, "device_status": status,
        "timing": f"graph replay of {steps} steps; stages from {steps} eager steps (CUDA events)",
    }


def fp8_leg(workload, device, steps, warmup, tf_peak, hbm_peak):
    """The block with e4m3 gate/up experts (MoEBlock(expert_dtype="fp8_e4m3")):
    tokens/s, the e4m3 gate/up GEMM against twice the measured bf16 peak (the
    nominal e4m3 / bf16 ratio; no e4m3 peak is measured here), and its
    distance from the bf16 block on the same tokens."""
    from moe_dispatch.layer import MoEBlock, MoEConfig, MoEWeights

    block, x = build_block(workload, device)
    w = workload
    fp8 = MoEBlock(MoEConfig(w.hidden, w.intermediate, w.experts, w.topk), device=device,
                   weights=MoEWeights(block.router_weight, block.gate_up_weight, block.down_weight),
                   expert_dtype="fp8_e4m3")
    fp8.routing_bias.copy_(block.routing_bias)
    with torch.inference_mode():
        expected = block(x).clone()
        got = fp8(x).clone()
    diff = (got.float() - expected.float())
    rel = float(diff.norm() / expected.float().norm())
    del block, expected, got
    torch.cuda.empty_cache()
    graph_ms, _ = time_graph(fp8, x, steps, warmup, 1, device)
    # stage events: quantise, e4m3 gate/up GEMM, bf16 down GEMM
    state = fp8.workspace(x)
    ext = fp8.extension
    names = ("quantize", "gemm1", "gemm2")
    samples = {n: [] for n in names}
    with torch.inference_mode():
        for _ in range(steps):
            ev = {n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for n in names}
            ids32, ids64, weights = fp8.route(x)
            state.transport.dispatch(x, ids32, ids64)
            ev["quantize"][0].record()
            ext.quantize_rows_e4m3(state.transport.packed, state.packed_q, state.packed_scale)
            ev["quantize"][1].record()
            ev["gemm1"][0].record()
            ext.grouped_gemm_swiglu_e4m3_out(state.packed_q, state.packed_scale, fp8.gate_up_q,
                                             fp8.gate_up_scale, state.transport.offsets,
                                             state.activated)
            ev["gemm1"][1].record()
            ev["gemm2"][0].record()
            ext.grouped_gemm_out(state.activated, fp8.down_weight, state.transport.offsets,
                                 state.expert_output)
            ev["gemm2"][1].record()
            state.transport.combine(state.expert_output, weights)
            for n in names:
                samples[n].append(ev[n])
        torch.cuda.synchronize()
    stage = {n: statistics.mean(e[0].elapsed_time(e[1]) for e in samples[n]) for n in names}
    a = algorithmic(workload, x.shape[0])
    g1 = a.gemm1_flops / (stage["gemm1"] / 1e3) / 1e12
    status = ext.device_status()
    tokens = x.shape[0]
    del fp8, x
    torch.cuda.empty_cache()
    return {
        "workload": workload_config(workload, 1)["workload"] + "; gate/up experts e4m3",
        "dtype": "e4m3 gate/up (per-row activation, per-channel weight scales), bf16 down",
        "ms_per_step": round(graph_ms, 4), "tokens_per_s": round(tokens / (graph_ms / 1e3), 1),
        "stage_ms": {k: round(v, 4) for k, v in stage.items()},
        "gate_up_e4m3_tflops": round(g1, 1),
        "gate_up_frac_of_2x_bf16_peak": round(g1 / (2 * tf_peak), 4),
        "rel_l2_vs_bf16_block": round(rel, 5),
        "device_status": status,
    }


def run_ours(args, rank, world, local):
    from moe_dispatch.routing import WORKLOADS

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    workload = WORKLOADS[args.workload]
    hbm_peak, tf_peak, tf_sustained, peak_kind = measured_peaks()
    block, x = build_block(workload, device)
    tokens = workload.tokens

    # -- timed region: K graph replays (inputs resident in HBM)
    ms_per_step, clocks = time_graph(block, x, args.steps, args.warmup, world, device,
                                     clocks_index=local)
    value = tokens * world / (ms_per_step / 1e3)
    # -- per-kernel durations over K eager steps (same stream, CUDA events)
    stage, eager_ms = time_stages(block, x, args.steps, world, device)
    # -- end to end through the public API with host buffers
    e2e_ms, h2d_bytes, d2h_bytes = time_host_pipeline(block, x, args.steps, world, device)
    status = block.extension.device_status()

    rows = block.workspace(x).transport.packed.shape[0]
    summary = stage_summary(workload, tokens, stage, block, rows, tf_peak, hbm_peak)
    a = algorithmic(workload, tokens)
    gemm1_kernel, tile = gemm_kernel_name(block, rows, workload.experts)
    achieved = a.gemm1_flops / (stage["gemm1"] / 1e3) / 1e12
    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "value_per_gpu": round(value / world, 1),
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) tokens, N(0,1/fan_in) weights)",
        "config": {
            **workload_config(workload, world),
            "timing": "CUDA graph replay of one block forward per step",
            "l2": "inputs larger than L2 (expert weights streamed per step)",
        },
        "eager_ms_per_step": round(eager_ms, 4),
        **summary,
        "roofline": {
            "kernel": f"{gemm1_kernel} (gate/up + SwiGLU, tcgen05, {tile} tile)",
            "bound": "tensor",
            "achieved": round(achieved, 1),
            "peak": tf_peak,
            "unit": "TFLOP/s",
            "frac": round(achieved / tf_peak, 4),
            "peak_kind": f"{peak_kind} burst bf16 (cuBLAS)",
            "flops_per_launch": a.gemm1_flops,
            "traffic": profiled_traffic(gemm1_kernel),
        },
        "e2e": {
            "value": round(tokens * world / (e2e_ms / 1e3), 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": d2h_bytes,
            "path": "HostPipeline.run: pinned host batch in, block(x, out=y) replayed as a "
                    "per-slot CUDA graph, result out; copies on two copy streams overlap the "
                    "neighbouring steps' compute",
        },
        "gpu_launches": kernels_per_step(workload.experts) * args.steps,
        "clocks": clocks,
        "device_status": status,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(workload, block, x, args.cpu_sample_tokens)
    del block, x
    torch.cuda.empty_cache()
    if world == 1:
        result["transport_config"] = transport_config(hbm_peak)
        if not args.no_extra_configs:
            result["fp8_config"] = fp8_leg(workload, device, args.steps, args.warmup, tf_peak,
                                           hbm_peak)
            for key, name in (("fine_grained_config", "fine_grained"),
                              ("expert_parallel_config", "expert_parallel")):
                if name != workload.name:
                    result[key] = single_gpu_leg(WORKLOADS[name], device, args.steps,
                                                 args.warmup, tf_peak, hbm_peak)
    return result
EP_STAGES = ("exchange", "gemm1", "gemm2", "return")


def ep_kernels_per_step(block, workload):
    """This engine's kernels in one expert-parallel forward (NCCL's own kernels
    not counted): per micro-batch the route, dispatch (2), the exchange
    kernels, the two grouped GEMMs and the combine."""
    route = 1 if workload.experts <= 32 else 2
    if block.backend != "p2p":
        return route + 2 + 1 + 2 + 2 + 1  # layout, regroup x2
    per_lane = route + 2 + 1  # route, dispatch, counts
    per_lane += 2  # local + remote send (overlap), or send + wait for the rows
    per_lane += 1  # gate/up GEMM
    per_lane += 1 if block.fused_return else 2  # down GEMM (+ return copy)
    per_lane += 1 + 1  # wait for the returns, combine
    return per_lane * block.micro_batches


def ep_measure(block, x, workload, args, world, device, clocks_index=None):
    """Timed expert-parallel steps (graph replay for p2p), per-stage events over
    K eager steps, the exchange bytes and the grouped rows of this rank."""
    stream = torch.cuda.current_stream(device)
    graphed = block.backend == "p2p"
    with torch.inference_mode():
        for _ in range(max(args.warmup, 3)):
            block(x)
        torch.cuda.synchronize()
        barrier(world)
        graph = None
        if graphed:  # no host sync in the p2p step: replay it as a CUDA graph
            from moe_dispatch.graphs import capture_forward

            graph, _ = capture_forward(block, x)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        sampler = ClockSampler(clocks_index) if clocks_index is not None else None
        if sampler:
            sampler.__enter__()
        start.record(stream)
        for _ in range(args.steps):
            if graphed:
                graph.replay()
            else:
                block(x)
        end.record(stream)
        torch.cuda.synchronize()
        if sampler:
            sampler.__exit__(None, None, None)
        barrier(world)
        total_ms = max_over_ranks(start.elapsed_time(end), world, device)
        per_step = []
        barrier(world)
        torch.cuda.synchronize()
        stages = EP_STAGES + (("send",) if getattr(block, "overlap", False) else ())
        for _ in range(args.steps):
            events = {n: (torch.cuda.Event(enable_timing=True),
                          torch.cuda.Event(enable_timing=True)) for n in stages}
            block(x, events=events)
            per_step.append(events)
        torch.cuda.synchronize()
        barrier(world)
        del graph
    stage = {n: statistics.mean(e[n][0].elapsed_time(e[n][1]) for e in per_step)
             for n in stages}
    # stage events cover the first micro-batch: count its rows only
    counts = block.last_send_counts(lane=0).view(world, -1).sum(1).tolist()
    send_rows = [int(c) for c in counts]
    if block.backend == "nccl":
        send_rows, recv_rows = block.last_split_sizes
        rows = sum(recv_rows)
    else:
        rows = block.last_grouped_rows(lane=0)
    crossing = sum(v for r, v in enumerate(send_rows) if r != block.rank) * workload.hidden * 2
    stage_max = {n: max_over_ranks(v, world, device) for n, v in stage.items()}
    # with the overlap the rows cross NVLink in the side stream's "send" stage
    exchange_gbs = crossing / (stage.get("send", stage["exchange"]) / 1e3) / 1e9
    return_gbs = crossing / (stage["return"] / 1e3) / 1e9
    return {
        "ms_per_step": total_ms / args.steps, "stage": stage, "stage_max": stage_max,
        "rows": rows, "crossing": crossing,
        "exchange_gbs_min_over_ranks": -max_over_ranks(-exchange_gbs, world, device),
        "return_gbs_min_over_ranks": -max_over_ranks(-return_gbs, world, device),
        "graphed": graphed,
        "clocks": sampler.summary() if sampler else None,
    }


def ep_config_leg(workload, args, rank, world, device):
    """The E=256 block with its 32768 tokens split over the ranks (strong
    scaling): parity against the single-GPU block on every rank, the timed
    expert-parallel step, and on rank 0 the single-GPU block over all 32768
    tokens in the same run, for the strong-scaling efficiency."""
    block, x = build_ep_block(workload, device, rank, world, args.ep_backend,
                              args.ep_micro_batches, args.ep_overlap, args.ep_fused_return)
    equal, diff = ep_parity(block, x, workload, device)
    parity = all_ranks_true(equal, world, device)
    diff = max_over_ranks(diff, world, device)
    m = ep_measure(block, x, workload, args, world, device)
    status = block.extension.device_status()
    tokens = x.shape[0]
    block.close()
    del block, x
    torch.cuda.empty_cache()
    single_ms = None
    barrier(world)
    if rank == 0:
        full, xf = build_block(workload, device)
        single_ms, _ = time_graph(full, xf, args.steps, args.warmup, 1, device)
        del full, xf
        torch.cuda.empty_cache()
    barrier(world)
    ms = m["ms_per_step"]
    total_tokens = tokens * world
    out = {
        "workload": f"{workload.name}: T={workload.tokens} per step split {tokens}/GPU, "
                    f"H={workload.hidden} I={workload.intermediate} E={workload.experts} "
                    f"top{workload.topk}, experts sharded {workload.experts // world}/GPU",
        "scaling": "strong", "n_gpus": world, "exchange": "p2p" if m["graphed"] else "nccl",
        "ms_per_step": round(ms, 4), "tokens_per_s": round(total_tokens / (ms / 1e3), 1),
        "tokens_per_s_per_gpu": round(total_tokens / (ms / 1e3) / world, 1),
        "stage_ms_max_over_ranks": {k: round(v, 4) for k, v in m["stage_max"].items()},
        "exchange_gbs_min_over_ranks": round(m["exchange_gbs_min_over_ranks"], 1),
        "return_gbs_min_over_ranks": round(m["return_gbs_min_over_ranks"], 1),
        "nvlink_peak_gbs_per_direction": 900.0,
        "ep_parity": parity, "ep_parity_max_abs_diff": diff,
        "device_status": status,
    }
    if single_ms is not None:
        out["single_gpu_ms_per_step_same_run"] = round(single_ms, 4)
        out["strong_scaling_efficiency"] = round(single_ms / (world * ms), 4)
    return out


def run_expert_parallel(args, rank, world, local):
    from moe_dispatch.routing import WORKLOADS

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    workload = WORKLOADS[args.workload]
    _, tf_peak, _, peak_kind = measured_peaks()
    block, x = build_ep_block(workload, device, rank, world, args.ep_backend,
                              args.ep_micro_batches, args.ep_overlap, args.ep_fused_return)
    tokens, scaling = ep_tokens_per_rank(workload, world)
    # -- correctness first: this rank's tokens through a single-GPU block with every expert
    equal, diff = ep_parity(block, x, workload, device)
    parity = all_ranks_true(equal, world, device)
    diff = max_over_ranks(diff, world, device)
    m = ep_measure(block, x, workload, args, world, device, clocks_index=local)
    e2e_ms, h2d_bytes, d2h_bytes = time_host_pipeline(block, x, args.steps, world, device)
    status = block.extension.device_status()

    h, i = workload.hidden, workload.intermediate
    stage = m["stage"]
    gemm1_flops = 2.0 * m["rows"] * h * 2 * i
    achieved = gemm1_flops / (stage["gemm1"] / 1e3) / 1e12
    capacity = block.exchange.grouped.shape[0] if block.backend == "p2p" else m["rows"]
    # the overlapped exchange feeds gate/up through arrival groups
    gemm1_kernel, tile = gemm_kernel_name(block, capacity, workload.experts // world,
                                          arrival_groups=getattr(block, "overlap", False) and world > 1)
    ms_per_step = m["ms_per_step"]
    graphed = m["graphed"]
    launches = ep_kernels_per_step(block, workload)
    block_options = {"overlap": getattr(block, "overlap", False), "fused_return": block.fused_return}
    block.close()
    del block, x
    torch.cuda.empty_cache()
    value = tokens * world / (ms_per_step / 1e3)
    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "value_per_gpu": round(value / world, 1),
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) tokens, N(0,1/fan_in) weights)",
        "config": {
            "workload": f"{workload.name}: T={tokens}/GPU H={h} I={i} E={workload.experts} "
                        f"top{workload.topk}, experts sharded {workload.experts // world}/GPU",
            "tokens_per_gpu": tokens, "hidden": h, "intermediate": i,
            "experts": workload.experts, "topk": workload.topk,
            "parallelism": f"ep{world}",
            "exchange": "p2p" if graphed else "nccl",
            "micro_batches": args.ep_micro_batches,
            "exchange_overlapped_with_gate_up": bool(block_options["overlap"]),
            "fused_return": bool(block_options["fused_return"]),
            "timing": ("CUDA graph replay of one expert-parallel step (NVLink peer stores, no "
                       "host sync)" if graphed else
                       "eager steps (one host sync per step for the all-to-all split sizes)"),
            "l2": "inputs larger than L2 (expert weights streamed per step)",
        },
        "ep_parity": parity,
        "ep_parity_max_abs_diff": diff,
        "ep_parity_check": "every rank's tokens through a single-GPU block holding all experts, "
                           "compared bit for bit with the expert-parallel output before timing",
        "stage_ms_rank0": {k: round(v, 4) for k, v in stage.items()},
        "stage_ms_max_over_ranks": {k: round(v, 4) for k, v in m["stage_max"].items()},
        "all_to_all_bytes_out_rank0": m["crossing"],
        "exchange_gbs_min_over_ranks": round(m["exchange_gbs_min_over_ranks"], 1),
        "return_gbs_min_over_ranks": round(m["return_gbs_min_over_ranks"], 1),
        "roofline": {
            "kernel": f"{gemm1_kernel} (gate/up + SwiGLU, tcgen05, {tile} tile), rank 0",
            "bound": "tensor", "achieved": round(achieved, 1), "peak": tf_peak,
            "unit": "TFLOP/s", "frac": round(achieved / tf_peak, 4),
            "peak_kind": f"{peak_kind} burst bf16 (cuBLAS)", "flops_per_launch": gemm1_flops,
            "traffic": None,
            "traffic_note": "no ncu capture of a multi-rank run (ncu stays on one GPU)",
        },
        "e2e": {
            "value": round(tokens * world / (e2e_ms / 1e3), 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": d2h_bytes,
            "path": "HostPipeline.run: pinned host batch in, block(x, out=y) replayed as a "
                    "per-slot CUDA graph, result out; copies on two copy streams overlap the "
                    "neighbouring steps' compute",
        },
        "gpu_launches": launches * args.steps,
        "clocks": m["clocks"],
        "device_status": status,
    }
    if not args.no_extra_configs and workload.name != "expert_parallel":
        result["expert_parallel_config"] = ep_config_leg(WORKLOADS["expert_parallel"], args,
                                                         rank, world, device)
    return result
def transport_config(hbm_peak):
    """The metric's second half on its own configuration (transport only:
    T=4096, H=4096 fp16, E=64, top-8, uniform and Zipf(1.2) popularity)."""
    from moe_dispatch.profiling import transport_sweep

    lines = transport_sweep(verbose=False)
    total = {}
    for line in lines:
        entry = total.setdefault(line["popularity"], {"bytes": 0, "us": 0.0})
        entry["bytes"] += line["algorithmic_bytes"]
        entry["us"] += line["us"]
    out = {"workload": "transport only: T=4096 H=4096 fp16, E=64 top-8; each launch after "
                       "a 256 MB L2 flush, median of 20", "stages": lines}
    for popularity, entry in total.items():
        gbs = entry["bytes"] / (entry["us"] / 1e6) / 1e9
        out[f"dispatch_combine_gbs_{popularity}"] = round(gbs, 1)
        out[f"frac_of_hbm_{popularity}"] = round(gbs / hbm_peak, 4)
    out["hbm_peak_gbs"] = hbm_peak
    return out


# ------------------------------------------------- the reference on the host
def reference_package():
    """The reference's own package, installed under baseline/_ref, imported as
    `reference_moe_dispatch` so it does not shadow this engine's moe_dispatch
    (its modules import each other relatively).  None if it is not installed."""
    init = REFERENCE_SITE / "moe_dispatch" / "__init__.py"
    if not init.exists():
        return None
    if REFERENCE_ALIAS not in sys.modules:
        spec = importlib.util.spec_from_file_location(
            REFERENCE_ALIAS, init, submodule_search_locations=[str(init.parent)])
        module = importlib.util.module_from_spec(spec)
        sys.modules[REFERENCE_ALIAS] = module
        spec.loader.exec_module(module)
    return sys.modules[REFERENCE_ALIAS]


@dataclass(frozen=True)
class ReferenceShape:
    """The fields the reference's MoEBlock reads from its config; used where its
    MoEConfig rejects the shape (top-k > 2 or more than 64 experts)."""

    hidden: int
    intermediate: int
    experts: int
    topk: int
    alignment: int = 8


def reference_torch_block(workload, weights, bias):
    """The reference's MoEBlock(implementation="torch", device="cpu") holding
    `weights` (router fp32, experts bf16) with `bias` as its routing bias."""
    reference_package()
    layer = importlib.import_module(REFERENCE_ALIAS + ".layer")
    w = workload
    if w.topk <= 2 and w.experts <= 64:
        cfg = layer.MoEConfig(w.hidden, w.intermediate, w.experts, w.topk)
    else:
        cfg = ReferenceShape(w.hidden, w.intermediate, w.experts, w.topk)
    block = layer.MoEBlock(cfg, device="cpu", dtype=torch.bfloat16, implementation="torch",
                           weights=layer.MoEWeights(weights.router.float().contiguous(),
                                                    weights.gate_up, weights.down))
    block.routing_bias.copy_(bias)
    return block


def time_reference_torch(block, x):
    with torch.inference_mode():
        t0 = time.perf_counter()
        block(x)
        return time.perf_counter() - t0


def time_port(workload, weights, x, bias):
    """Seconds of the C restatement (the test oracle) over the rows of x."""
    from oracle import moe_oracle as oracle

    oracle.set_num_threads(host_threads())
    t0 = time.perf_counter()
    oracle.block_forward(x, weights.router, bias, weights.gate_up, weights.down, workload.topk)
    return time.perf_counter() - t0


def cpu_baseline(workload, block, x, sample_tokens):
    """Our arm's CPU baseline: the reference's PyTorch path and the C port on
    the first `sample_tokens` tokens of the workload, every host core."""
    from moe_dispatch.layer import MoEWeights

    threads = host_threads()
    weights = MoEWeights(block.router_weight.cpu(), block.gate_up_weight.cpu(),
                         block.down_weight.cpu())
    xs = x[:sample_tokens].cpu()
    bias = block.routing_bias.cpu()
    port_s = time_port(workload, weights, xs, bias)
    port = {"value": round(sample_tokens / port_s, 2), "unit": "tokens/s", "cores": threads,
            "kind": "port", "sample": f"{sample_tokens} tokens of the workload through the C "
                                      f"restatement of the reference's path, {port_s:.2f} s"}
    if reference_package() is None:
        return {**port, "note": "baseline/_ref (the reference's package) is not installed"}
    torch.set_num_threads(threads)
    ref_block = reference_torch_block(workload, weights, bias)
    time_reference_torch(ref_block, xs[:32])  # first-call set-up
    ref_s = time_reference_torch(ref_block, xs)
    return {"value": round(sample_tokens / ref_s, 2), "unit": "tokens/s", "cores": threads,
            "kind": "reference_torch",
            "sample": f"{sample_tokens} tokens of the workload through the reference's own "
                      f"MoEBlock(implementation='torch', device='cpu'), {ref_s:.2f} s, "
                      f"torch threads {torch.get_num_threads()}",
            "port": port}


def run_reference(args, rank, world):
    """--impl reference: the reference's own PyTorch path on the host cores,
    a bounded token sample of the workload per step."""
    from moe_dispatch.routing import WORKLOADS, block_input, block_weights

    workload = WORKLOADS[args.workload]
    threads = host_threads()
    torch.set_num_threads(threads)
    sample = args.reference_sample_tokens
    weights, bias = block_weights(workload)
    x = block_input(workload, tokens=sample)
    port_s = time_port(workload, weights, x, bias)
    port = {"value": round(sample / port_s, 2), "unit": "tokens/s", "cores": threads,
            "kind": "port", "sample": f"{sample} tokens, one pass of the C restatement"}
    if reference_package() is not None:
        block = reference_torch_block(workload, weights, bias)
        run = lambda: time_reference_torch(block, x)  # noqa: E731
        kind = "reference_torch"
        what = ("the reference's own MoEBlock(implementation='torch', device='cpu'), imported "
                "from baseline/_ref")
    else:
        run = lambda: time_port(workload, weights, x, bias)  # noqa: E731
        kind = "port"
        what = "the C restatement of the reference's path (baseline/_ref not installed)"
    for _ in range(args.warmup):
        run()
    times = [run() for _ in range(args.steps)]
    seconds = sum(times) / len(times)
    value = sample / seconds
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "impl": "reference",
        "value_per_gpu": round(value, 2),
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(seconds * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {**workload_config(workload, 1),
                   "timing": f"CPU: each step runs {sample} of the workload's tokens through "
                             f"{what}, {threads} host threads",
                   "sample_tokens_per_step": sample},
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads,
                         "kind": kind, "sample": f"{sample} tokens per step through {what}",
                         "port": port},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if world == 1 and not args.no_reference_gpu:
        result["reference_gpu"] = reference_gpu(workload, args)
    return result


def reference_gpu(workload, args):
    """The reference's own GPU path (cuda_fused with its default expert backend)
    at the full workload on GPU 0, run in a child process that imports only
    the reference's package."""
    if not (REFERENCE_SITE / "moe_dispatch").exists():
        return {"unavailable": "baseline/_ref (the reference's package) is not installed"}
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    w = workload
    shape = f"{w.tokens},{w.hidden},{w.intermediate},{w.experts},{w.topk}"
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT")}
    try:
        run = subprocess.run(
            [sys.executable, str(Path(__file__).resolve()), "--reference-gpu-worker",
             "--workload", shape, "--steps", str(args.steps), "--warmup", str(max(args.warmup, 3))],
            capture_output=True, text=True, timeout=900, env=env, cwd=str(ROOT))
    except subprocess.TimeoutExpired:
        return {"unavailable": "the reference's GPU path did not finish within 900 s"}
    lines = [line for line in run.stdout.splitlines() if line.startswith("{")]
    if run.returncode != 0 or not lines:
        tail = (run.stderr or run.stdout).strip().splitlines()[-1:] or ["no output"]
        return {"unavailable": f"the reference's GPU path exited {run.returncode}: {tail[0][:300]}"}
    return json.loads(lines[-1])


def reference_gpu_worker(args):
    """Child process of reference_gpu(): sys.path holds baseline/_ref only, so
    `moe_dispatch` is the reference's package, run through its public API."""
    from moe_dispatch.layer import MoEBlock, MoEConfig  # the reference's
    from moe_dispatch.block_benchmark import capture_forward  # the reference's

    tokens, hidden, inter, experts, topk = (int(v) for v in args.workload.split(","))
    if topk <= 2 and experts <= 64:
        cfg = MoEConfig(hidden, inter, experts, topk)
    else:
        cfg = ReferenceShape(hidden, inter, experts, topk)
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    t_build = time.perf_counter()
    block = MoEBlock(cfg, device=device, implementation="cuda_fused", seed=0)
    g = torch.Generator(device=device).manual_seed(0)
    x = torch.randn(tokens, hidden, device=device, generator=g).to(torch.bfloat16)
    stream = torch.cuda.current_stream(device)
    with torch.inference_mode():
        for _ in range(args.warmup):  # includes the extension build and GEMM compilation
            block(x)
        torch.cuda.synchronize()
        setup_s = time.perf_counter() - t_build
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            block(x)
        end.record(stream)
        torch.cuda.synchronize()
        eager_ms = start.elapsed_time(end) / args.steps
        graph = capture_forward(block, x)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
        graph_ms = start.elapsed_time(end) / args.steps
    print(json.dumps({
        "what": "the reference's MoEBlock(implementation='cuda_fused') on GPU 0, imported from "
                "baseline/_ref, its own weights (make_weights, seed 0) and N(0,1) tokens",
        "expert_backend": block.expert_backend,
        "tokens": tokens, "ms_per_step_graph": round(graph_ms, 4),
        "tokens_per_s_graph": round(tokens / (graph_ms / 1e3), 1),
        "ms_per_step_eager": round(eager_ms, 4),
        "tokens_per_s_eager": round(tokens / (eager_ms / 1e3), 1),
        "setup_s": round(setup_s, 1), "steps": args.steps,
    }), flush=True)
    return 0


def main():
    args = parse_args()
    if args.reference_gpu_worker:
        return reference_gpu_worker(args)
    rank, world, local = dist_info()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, rank, world)), flush=True)
        return 0
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    try:
        result = (run_ours if world == 1 else run_expert_parallel)(args, rank, world, local)
        if rank == 0:
            print(json.dumps(result), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
