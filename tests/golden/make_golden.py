"""Generate golden vectors from the reference's own PyTorch path.

Run in a checkout that has the reference project (read-only is fine):

    python tests/golden/make_golden.py --reference-src <reference>/src

It imports ``moe_dispatch`` from that directory and runs, on the CPU, the
reference's PyTorch implementation of each stage of the hot path:

* router: ``F.linear(x.float(), W)`` then ``torch.topk`` + ``softmax``
  (layer.py:122-139);
* dispatch: ``TorchWorkspace.dispatch`` (reference.py:42-65) on inputs from
  ``routing.make_case`` (routing.py:6-17), once as written and once with
  ``torch.sort`` made stable, which defines the canonical token-major order;
* combine: ``TorchWorkspace.combine`` (reference.py:67-76) on arbitrary
  expert outputs placed as ``validation.validate_case`` does
  (validation.py:47-54);
* SwiGLU: ``experts.swiglu_reference`` (experts.py:38-41);
* whole block: ``MoEBlock(implementation="torch", device="cpu")``
  (layer.py:70-197) with ``make_weights`` (layer.py:38-59).  Configurations
  with top-k > 2 or more than 64 experts use a duck-typed config object,
  because ``MoEConfig`` rejects them while ``MoEBlock`` itself does not.

Inputs are regenerated from seeds by ``tests/golden/cases.py`` (torch CPU
generators), so the fixture stores only seeds, index outputs and result
tensors, plus a checksum of each input to detect generator drift.
"""

from __future__ import annotations

import argparse
import sys
from dataclasses import dataclass
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402


@dataclass(frozen=True)
class DuckConfig:
    hidden: int
    intermediate: int
    experts: int
    topk: int
    alignment: int = 8


class stable_sort:
    """Context manager: make torch.sort stable for the reference's dispatch."""

    def __enter__(self):
        self.original = torch.sort

        def sort(*args, **kwargs):
            kwargs.setdefault("stable", True)
            return self.original(*args, **kwargs)

        torch.sort = sort

    def __exit__(self, *exc):
        torch.sort = self.original


def router_cases(md):
    out = []
    for spec in cases.ROUTER_CASES:
        x, w, bias = cases.router_inputs(spec)
        logits = torch.nn.functional.linear(x.float(), w)  # layer.py:123
        selected, ids64 = torch.topk(logits + bias, spec["topk"], dim=-1)  # layer.py:136-137
        weights = torch.softmax(selected, dim=-1)  # layer.py:138
        out.append(
            {
                "spec": spec,
                "x_checksum": cases.checksum(x),
                "logits": logits,
                "ids": ids64.to(torch.int32),
                "weights": weights,
            }
        )
    return out


def transport_cases(md):
    from moe_dispatch.reference import TorchWorkspace
    from moe_dispatch.routing import make_case

    out = []
    for spec in cases.TRANSPORT_CASES:
        tokens, hidden, experts, topk = spec["shape"]
        dtype = cases.DTYPES[spec["dtype"]]
        x, ids32, ids64, weights = make_case(
            tokens, hidden, experts, topk, dtype, spec["pattern"], spec["seed"], device="cpu"
        )
        record = {"spec": spec, "x_checksum": cases.checksum(x), "ids": ids32, "weights": weights}
        for name, context in (("stable", stable_sort), ("unstable", None)):
            ws = TorchWorkspace(tokens, hidden, experts, topk, dtype, device="cpu",
                                alignment=spec["alignment"])
            if context is None:
                ws.dispatch(x, ids32, ids64)
            else:
                with context():
                    ws.dispatch(x, ids32, ids64)
            record[f"{name}_counts"] = ws.counts.clone()
            record[f"{name}_offsets"] = ws.offsets.clone()
            record[f"{name}_inverse"] = ws.inverse.to(torch.int32).clone()
            if name == "stable":
                record["packed_checksum"] = cases.checksum(ws.packed[: int(ws.offsets[-1])])
                canonical = cases.canonical_expert_rows(tokens, topk, hidden, dtype, spec["seed"])
                expert_output = torch.zeros_like(ws.packed)
                expert_output.index_copy_(0, ws.inverse.reshape(-1), canonical)
                ws.combine(expert_output, weights)
                record["combined"] = ws.output.clone()
        out.append(record)
    return out


def swiglu_cases(md):
    from moe_dispatch.experts import swiglu_reference

    out = []
    for spec in cases.SWIGLU_CASES:
        projection = cases.swiglu_input(spec)
        out.append({"spec": spec, "output": swiglu_reference(projection)})
    return out


def block_cases(md):
    from moe_dispatch.layer import MoEBlock, MoEConfig, make_weights

    out = []
    for spec in cases.BLOCK_CASES:
        hidden, intermediate, experts, topk = spec["config"]
        if topk in (1, 2) and experts <= 64:
            config = MoEConfig(hidden, intermediate, experts, topk)
        else:
            config = DuckConfig(hidden, intermediate, experts, topk)
        weights = make_weights(config, "cpu", torch.bfloat16, spec["weight_seed"])
        block = MoEBlock(config, device="cpu", dtype=torch.bfloat16, implementation="torch",
                         weights=weights)
        bias = cases.block_bias(spec)
        block.routing_bias.copy_(bias)
        x = cases.block_input(spec)
        with torch.inference_mode():
            output = block(x).clone()
            logits = torch.nn.functional.linear(x.float(), block.router_weight)
            ids32, ids64, route_weights = block.route(x)
        out.append(
            {
                "spec": spec,
                "x_checksum": cases.checksum(x),
                "weights_checksum": cases.checksum(weights.gate_up) ^ cases.checksum(weights.down)
                ^ cases.checksum(weights.router),
                "logits": logits,
                "ids": ids32.clone(),
                "route_weights": route_weights.clone(),
                "output": output,
            }
        )
    return out


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference-src", required=True, type=Path)
    parser.add_argument("--output", type=Path, default=HERE / "golden.pt")
    args = parser.parse_args()
    sys.path.insert(0, str(args.reference_src.resolve()))
    torch.set_num_threads(1)
    import moe_dispatch as md

    golden = {
        "torch_version": str(torch.__version__),
        "router": router_cases(md),
        "transport": transport_cases(md),
        "swiglu": swiglu_cases(md),
        "block": block_cases(md),
    }
    torch.save(golden, args.output)
    print(f"wrote {args.output} ({args.output.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
