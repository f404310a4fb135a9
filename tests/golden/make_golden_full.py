"""Golden outputs of the reference's PyTorch path at the full benchmark shapes.

    python tests/golden/make_golden_full.py --reference-src <reference>/src

For the Mixtral (T4096 H4096 I14336 E8 top-2), fine-grained (T16384 H2048
I1408 E64 top-6, log-Zipf bias) and expert-parallel (T32768 H7168 I2048 E256
top-8) workloads it draws the weights and tokens exactly as
``moe_dispatch.routing.block_weights`` / ``block_input`` do (seeded CPU
generators), picks every `stride`-th token, and runs those tokens through the
reference's own ``MoEBlock(implementation="torch", device="cpu")``
(layer.py:70-197; top-k > 2 and more than 64 experts through a duck-typed
config, which ``MoEBlock`` accepts).  Every token is routed and computed on its
own, so the outputs of a token subset are the outputs those tokens get inside
the full batch.  The fixture stores the token indices, the reference's ids,
routing weights and bf16 outputs, and checksums of the regenerated inputs.

The reference package is imported from --reference-src under the name
``reference_moe_dispatch`` so that this engine's ``moe_dispatch`` (which
draws the inputs) stays importable beside it.
"""

from __future__ import annotations

import argparse
import importlib
import importlib.util
import sys
from dataclasses import dataclass
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "cuda-moe-engine_b200"))
sys.path.insert(0, str(HERE))
import cases  # noqa: E402

# (workload, token stride) -> 64, 128 and 64 tokens
FULL_SIZE = [("mixtral", 64), ("fine_grained", 128), ("expert_parallel", 512)]


@dataclass(frozen=True)
class DuckConfig:
    hidden: int
    intermediate: int
    experts: int
    topk: int
    alignment: int = 8


def import_reference(src: Path):
    init = src / "moe_dispatch" / "__init__.py"
    spec = importlib.util.spec_from_file_location(
        "reference_moe_dispatch", init, submodule_search_locations=[str(init.parent)])
    module = importlib.util.module_from_spec(spec)
    sys.modules["reference_moe_dispatch"] = module
    spec.loader.exec_module(module)
    return importlib.import_module("reference_moe_dispatch.layer")


def weights_checksum(weights):
    return (cases.checksum(weights.router) ^ cases.checksum(weights.gate_up[0])
            ^ cases.checksum(weights.down[-1]))


def full_size_case(layer, name, stride):
    from moe_dispatch.routing import WORKLOADS, block_input, block_weights

    w = WORKLOADS[name]
    weights, bias = block_weights(w)
    x = block_input(w)
    tokens = torch.arange(0, w.tokens, stride)
    xs = x[tokens].contiguous()
    if w.topk <= 2 and w.experts <= 64:
        config = layer.MoEConfig(w.hidden, w.intermediate, w.experts, w.topk)
    else:
        config = DuckConfig(w.hidden, w.intermediate, w.experts, w.topk)
    block = layer.MoEBlock(config, device="cpu", dtype=torch.bfloat16, implementation="torch",
                           weights=layer.MoEWeights(weights.router, weights.gate_up, weights.down))
    block.routing_bias.copy_(bias)
    with torch.inference_mode():
        output = block(xs).clone()
        ids32, _, route_weights = block.route(xs)
    return {
        "workload": name, "tokens": tokens, "x_checksum": cases.checksum(x),
        "weights_checksum": weights_checksum(weights),
        "ids": ids32.clone(), "route_weights": route_weights.clone(), "output": output,
    }


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference-src", required=True, type=Path)
    parser.add_argument("--output", type=Path, default=HERE / "golden_full.pt")
    args = parser.parse_args()
    layer = import_reference(args.reference_src.resolve())
    golden = {"torch_version": str(torch.__version__),
              "full_size": [full_size_case(layer, name, stride) for name, stride in FULL_SIZE]}
    torch.save(golden, args.output)
    print(f"wrote {args.output} ({args.output.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
