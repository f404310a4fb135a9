"""The bench contract on the CPU: the reference arm's JSON line, and the
helpers the GPU arm uses (no GPU needed)."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_reference_arm_prints_one_contract_line():
    run = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "0", "--reference-sample-tokens", "8"],
        capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [line for line in run.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["steps"] == 1 and d["warmup"] == 0 and d["n_gpus"] == 1
    installed = (ROOT / "baseline" / "_ref" / "moe_dispatch").exists()
    assert d["cpu_baseline"]["kind"] == ("reference_torch" if installed else "port")
    assert d["cpu_baseline"]["cores"] == bench.host_threads()
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["port"]["value"] > 0
    assert "unavailable" in d["reference_gpu"]  # no GPU here
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    from moe_dispatch.routing import WORKLOADS

    # the same workload description as the GPU arm's line
    assert d["config"]["workload"] == bench.workload_config(WORKLOADS["mixtral"], 1)["workload"]


def test_gemm_kernel_name_follows_the_launcher(monkeypatch):
    """The roofline names the kernel the launcher runs: the operand-swapped
    pair tile for bf16 pair launches of one arrival group, unless switched off."""

    class Extension:
        def __init__(self, tile):
            self.tile = tile

        def grouped_gemm_tile(self, rows, experts):
            return self.tile

    class Block:
        def __init__(self, tile):
            self.extension = Extension(tile)

    monkeypatch.delenv("MOE_B200_GEMM_SWAP", raising=False)
    assert bench.gemm_kernel_name(Block("pair"), 8256, 8) == ("grouped_gemm_swap_kernel<1>",
                                                               "operand-swapped pair")
    assert bench.gemm_kernel_name(Block("pair"), 8256, 8, arrival_groups=True) == (
        "grouped_gemm_pair_kernel<1>", "pair")
    assert bench.gemm_kernel_name(Block("single"), 1000, 8, swiglu=False) == (
        "grouped_gemm_kernel<0>", "single")
    monkeypatch.setenv("MOE_B200_GEMM_SWAP", "0")
    assert bench.gemm_kernel_name(Block("pair"), 8256, 8)[0] == "grouped_gemm_pair_kernel<1>"


def test_kernel_count_and_committed_traffic():
    assert bench.kernels_per_step(8) == 6 and bench.kernels_per_step(256) == 7
    assert bench.profiled_traffic("grouped_gemm_pair_kernel<1>") > 1.9e9
    assert bench.profiled_traffic("grouped_gemm_swap_kernel<1>") > 1.9e9
    assert bench.profiled_traffic("no_such_kernel") is None
    hbm, tf, sustained, kind = bench.measured_peaks()
    assert hbm > 1000 and tf > 100 and kind in ("measured", "fallback")


def test_clock_summary_reads_reasons(tmp_path):
    sampler = bench.ClockSampler(0)
    sampler.file.write("0, 1965, 1965, 700.1, 0x4, Not Active, Not Active, Not Active, Active\n"
                       "0, 1900, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active\n"
                       "0, 1965, 1965, 650.0, 0x0, Not Active, Not Active, Not Active, Not Active\n")
    summary = sampler.summary()
    assert summary["sm_mhz"] == 1965.0 and summary["sm_max_mhz"] == 1965.0
    assert summary["reasons"] == ["sw_power_cap"] and summary["samples"] == 3


def test_expert_parallel_token_split():
    from moe_dispatch.routing import WORKLOADS

    assert bench.ep_tokens_per_rank(WORKLOADS["mixtral"], 4) == (4096, "weak")
    assert bench.ep_tokens_per_rank(WORKLOADS["expert_parallel"], 8) == (4096, "strong")


def test_reference_package_is_imported_beside_ours():
    """The reference's package loads under its own name and leaves this
    engine's moe_dispatch in place."""
    if not (ROOT / "baseline" / "_ref" / "moe_dispatch").exists():
        pytest.skip("baseline/_ref not installed")
    import moe_dispatch

    ref = bench.reference_package()
    assert ref.__name__ == bench.REFERENCE_ALIAS
    assert Path(ref.__file__).resolve().is_relative_to(ROOT / "baseline" / "_ref")
    assert Path(moe_dispatch.__file__).resolve().is_relative_to(ROOT / "cuda-moe-engine_b200")
