"""Block benchmark that writes the reference's ``block_results.json`` schema.

Reference: src/moe_dispatch/block_benchmark.py:15-214 (cases, checks, stage
timing, result layout) and benchmark.py:15-45,145-164 (percentile, event
timing, hardware metadata).  The same keys and record layout, so the
reference's report tooling reads these results:

    {"kind": "moe_block_benchmark", "package_version", "hardware",
     "source_hashes", "configurations": [...], "validation": [...],
     "benchmarks": [{"case_id", "implementation", "stage",
                     "persistent_workspace_bytes", "median_us", "p95_us",
                     "min_us", "samples_us"}, ...], "method": {...}}

Implementations are this engine's two (``cuda`` and ``cuda_fused``); the
reference's third, ``torch``, is the reference's own PyTorch path and is not
part of this engine.  Each (case, implementation) is first checked against a
dense token-major evaluation of the same weights on the GPU (plain torch ops,
used only as the check and excluded from every timing) with the reference's
tolerances, and the two implementations must agree bit for bit.

    python -m moe_dispatch.block_benchmark --suite quick --graphs --output runs/block
"""

from __future__ import annotations

import argparse
from dataclasses import asdict
import hashlib
import json
import math
from pathlib import Path
import platform
import statistics
import subprocess
import time

import torch

from . import __version__
from .graphs import capture_forward
from .layer import MoEBlock, MoEConfig, make_weights

IMPLEMENTATIONS = ("cuda", "cuda_fused")
PACKAGE = Path(__file__).resolve().parent


def workload_cases(suite):
    """(tokens, config, routing pattern) per case; the reference's suites plus
    "mixtral" (the Mixtral-shaped block at 4096 tokens)."""
    if suite == "smoke":
        return [(128, MoEConfig(), pattern) for pattern in ("balanced", "skewed")]
    if suite == "model":
        config = MoEConfig(hidden=4096, intermediate=14336, experts=8, topk=2)
        return [(128, config, "balanced"), (256, config, "skewed")]
    if suite == "mixtral":
        config = MoEConfig(hidden=4096, intermediate=14336, experts=8, topk=2)
        return [(4096, config, "balanced")]
    if suite == "quick":
        return [
            (tokens, config, pattern)
            for tokens in (128, 2048)
            for config in (MoEConfig(), MoEConfig(1024, 2048, 16, 2))
            for pattern in ("balanced", "skewed")
        ]
    raise ValueError(f"unknown suite: {suite}")


def percentile(values, fraction):
    """Linear interpolation between order statistics (benchmark.py:15-22)."""
    ordered = sorted(values)
    if not ordered:
        return 0.0
    position = (len(ordered) - 1) * fraction
    low, high = math.floor(position), math.ceil(position)
    return ordered[low] + (ordered[high] - ordered[low]) * (position - low)


def measure(function, warmup, repeats):
    """CUDA-event time of each of `repeats` calls after `warmup` calls (us)."""
    for _ in range(warmup):
        function()
    torch.cuda.synchronize()
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(repeats)]
    for start, end in pairs:
        start.record()
        function()
        end.record()
    torch.cuda.synchronize()
    samples = [start.elapsed_time(end) * 1000.0 for start, end in pairs]
    return {"median_us": statistics.median(samples), "p95_us": percentile(samples, 0.95),
            "min_us": min(samples), "samples_us": samples}


def hardware_metadata():
    properties = torch.cuda.get_device_properties(0)
    try:
        smi = subprocess.check_output(
            ["nvidia-smi", "--query-gpu=name,driver_version,memory.total", "--format=csv,noheader"],
            text=True, timeout=10).strip()
    except (OSError, subprocess.SubprocessError):
        smi = "unavailable"
    return {
        "gpu": properties.name,
        "compute_capability": f"{properties.major}.{properties.minor}",
        "gpu_memory_bytes": properties.total_memory,
        "torch_version": torch.__version__,
        "torch_cuda": torch.version.cuda,
        "python": platform.python_version(),
        "nvidia_smi": smi,
        "utc_run_time": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
    }


def source_hashes():
    """sha256 of every kernel source, the C header and the package's modules."""
    paths = sorted((PACKAGE / "csrc").glob("*.cu")) + sorted((PACKAGE / "csrc").glob("*.cuh"))
    paths += sorted((PACKAGE / "csrc").glob("*.h")) + sorted(PACKAGE.glob("*.py"))
    header = PACKAGE.parents[1] / "include" / "moe_b200.h"
    if header.is_file():
        paths.append(header)
    return {path.name: hashlib.sha256(path.read_bytes()).hexdigest() for path in paths}


@torch.inference_mode()
def dense_check(block, x, ids64, weights):
    """The token-major evaluation of the reference's check (block_benchmark.py:29-45)
    on the GPU: every expert on every token routed to it, bf16 projection,
    fp32 SwiGLU with one bf16 cast, bf16 expert output, fp32 weighted sum."""
    config = block.config
    expected = torch.zeros(x.shape[0], config.hidden, device=x.device)
    for expert in range(config.experts):
        hit = (ids64 == expert)
        rows = hit.any(dim=1).nonzero().flatten()
        if rows.numel() == 0:
            continue
        projection = x[rows] @ block.gate_up_weight[expert].T
        gate = projection[:, :config.intermediate].float()
        up = projection[:, config.intermediate:].float()
        activation = (gate / (1.0 + torch.exp(-gate)) * up).to(x.dtype)
        output = activation @ block.down_weight[expert].T
        probability = (weights[rows] * hit[rows]).sum(dim=1)
        expected[rows] += output.float() * probability[:, None]
    expected = expected.to(x.dtype)
    actual = block(x).clone()
    torch.testing.assert_close(actual, expected, rtol=0.03, atol=0.03)
    difference = actual.float() - expected.float()
    relative = float(difference.norm() / expected.float().norm().clamp_min(1e-8))
    if relative > 0.02:
        raise AssertionError(f"relative L2 error {relative} exceeds BF16 tolerance .02")
    return actual, {
        "passed": True,
        "max_absolute_error": float(difference.abs().max()),
        "relative_l2_error": relative,
        "rtol": 0.03,
        "atol": 0.03,
        "relative_l2_limit": 0.02,
    }


def workspace_bytes(block, state):
    total = state.transport.workspace_bytes
    total += sum(t.numel() * t.element_size()
                 for t in (state.projection, state.activated, state.expert_output))
    total += sum(t.numel() * t.element_size()
                 for buffers in block._route_buffers.values() for t in buffers)
    return total


@torch.inference_mode()
def run_block_benchmark(suite="quick", warmup=10, repeats=40, output=Path("runs/block"),
                        graphs=False):
    if not torch.cuda.is_available():
        raise RuntimeError("the block benchmark needs an NVIDIA GPU")
    if warmup < 1 or repeats < 5:
        raise ValueError("use warmup>=1 and repeats>=5")
    configurations, records, validation = [], [], []
    for case_id, (tokens, config, pattern) in enumerate(workload_cases(suite)):
        weights = make_weights(config, "cuda", torch.bfloat16, 42 + case_id)
        generator = torch.Generator(device="cuda").manual_seed(100 + case_id)
        x = torch.randn(tokens, config.hidden, device="cuda", generator=generator).bfloat16()
        blocks = {name: MoEBlock(config, device="cuda", implementation=name, weights=weights)
                  for name in IMPLEMENTATIONS}
        for block in blocks.values():
            block.set_routing_pattern(pattern)
        ids32, ids64, probabilities = blocks["cuda_fused"].route(x)
        ids32, ids64, probabilities = ids32.clone(), ids64.clone(), probabilities.clone()
        counts = torch.bincount(ids64.flatten(), minlength=config.experts).cpu().tolist()
        configurations.append({"case_id": case_id, "tokens": tokens, **asdict(config),
                               "pattern": pattern, "dtype": "bfloat16",
                               "expert_backend": "tcgen05", "expert_counts": counts})
        outputs = {}
        names = list(IMPLEMENTATIONS)
        rotation = case_id % len(names)
        for name in names[rotation:] + names[:rotation]:
            block = blocks[name]
            outputs[name], checked = dense_check(block, x, ids64, probabilities)
            validation.append({"case_id": case_id, "implementation": name, **checked})
            state = block.workspace(x)
            state.transport.dispatch(x, ids32, ids64)
            block.experts_forward(state)
            stages = (
                ("router", lambda: block.route(x)),
                ("dispatch", lambda: state.transport.dispatch(x, ids32, ids64)),
                ("experts", lambda: block.experts_forward(state)),
                ("combine", lambda: state.transport.combine(state.expert_output, probabilities)),
                ("forward", lambda: block(x)),
            )
            held = workspace_bytes(block, state)
            for stage, function in stages:
                records.append({"case_id": case_id, "implementation": name, "stage": stage,
                                "persistent_workspace_bytes": held,
                                **measure(function, warmup, repeats)})
            if graphs:
                try:
                    graph, _ = capture_forward(block, x)
                    records.append({"case_id": case_id, "implementation": name,
                                    "stage": "forward_graph", "persistent_workspace_bytes": held,
                                    **measure(graph.replay, warmup, repeats)})
                    checked["graph_status"] = "passed"
                except RuntimeError as error:
                    checked["graph_status"] = "unsupported"
                    checked["graph_error"] = str(error)
                validation[-1].update(checked)
        identical = torch.equal(outputs["cuda"], outputs["cuda_fused"])
        for entry in validation[-len(IMPLEMENTATIONS):]:
            entry["implementations_bitwise_equal"] = identical
        if not identical:
            raise AssertionError(f"case {case_id}: cuda and cuda_fused outputs differ")
        print(f"MoE block {case_id + 1}/{len(workload_cases(suite))}: T={tokens}, "
              f"H={config.hidden}, I={config.intermediate}, E={config.experts}, {pattern}",
              flush=True)
    result = {
        "kind": "moe_block_benchmark",
        "package_version": __version__,
        "hardware": hardware_metadata(),
        "source_hashes": source_hashes(),
        "configurations": configurations,
        "validation": validation,
        "benchmarks": records,
        "method": {
            "suite": suite,
            "warmup": warmup,
            "repeats": repeats,
            "expert_backend": "tcgen05",
            "graphs_requested": graphs,
            "scope": "One synthetic MoE feedforward block: FP32 router/top-k/softmax, BF16 "
                     "grouped gate/up GEMM (tcgen05) with SwiGLU fused into its epilogue "
                     "(cuda_fused) or as a separate kernel (cuda), BF16 grouped down GEMM, "
                     "FP32 weighted combine. This is not complete language-model inference.",
            "timing": "CUDA events after warmup, one event pair per call. Per-stage medians "
                      "are measured in isolation and need not sum to the full-forward median. "
                      "Validation is excluded. Persistent buffers exclude the shared weights.",
        },
    }
    output = Path(output)
    output.mkdir(parents=True, exist_ok=True)
    path = output / "block_results.json"
    path.write_text(json.dumps(result, indent=2))
    return path


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--suite", default="quick", choices=["smoke", "quick", "model", "mixtral"])
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--repeats", type=int, default=40)
    parser.add_argument("--output", default="runs/block")
    parser.add_argument("--graphs", action="store_true")
    args = parser.parse_args()
    print(run_block_benchmark(args.suite, args.warmup, args.repeats, args.output, args.graphs))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
