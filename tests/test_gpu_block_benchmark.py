"""block_results.json in the reference's schema (block_benchmark.py:186-210)."""

import json

import pytest
import torch

from moe_dispatch.block_benchmark import IMPLEMENTATIONS, run_block_benchmark

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]


def test_smoke_suite_writes_the_reference_schema(tmp_path):
    path = run_block_benchmark("smoke", warmup=1, repeats=5, output=tmp_path, graphs=True)
    result = json.loads(path.read_text())
    assert result["kind"] == "moe_block_benchmark"
    for key in ("package_version", "hardware", "source_hashes", "configurations", "validation",
                "benchmarks", "method"):
        assert key in result
    assert len(result["configurations"]) == 2
    assert all(v["passed"] and v["graph_status"] == "passed" and v["implementations_bitwise_equal"]
               for v in result["validation"])
    stages = {(r["case_id"], r["implementation"], r["stage"]) for r in result["benchmarks"]}
    for case in (0, 1):
        for name in IMPLEMENTATIONS:
            for stage in ("router", "dispatch", "experts", "combine", "forward", "forward_graph"):
                assert (case, name, stage) in stages
    record = result["benchmarks"][0]
    assert len(record["samples_us"]) == 5 and record["min_us"] <= record["median_us"] <= record["p95_us"]
