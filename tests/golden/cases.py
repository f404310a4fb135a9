"""Seeded inputs for the golden fixtures (shared by make_golden.py and tests).

Inputs are rebuilt from seeds with torch CPU generators in the same draw
order the reference uses, so the fixture holds seeds and results only:

* transport inputs follow ``routing.make_case`` (routing.py:6-17): x first,
  then logits, from one generator;
* arbitrary expert outputs for the combine check follow
  ``validation.validate_case`` (validation.py:48-51, seed + 501);
* block weights follow ``layer.make_weights`` (layer.py:38-59): router
  ``randn/sqrt(H)`` fp32, gate_up ``randn/sqrt(H)``, down ``randn/sqrt(I)``,
  one generator, in that order.

Each fixture stores a checksum of the regenerated inputs, so a change of the
generators shows up as a checksum failure rather than a parity failure.
"""

from __future__ import annotations

import hashlib
import math

import torch

DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}

# Router: the reference's GPU router test grid (tests/test_gpu_router.py:11-24:
# experts {2,8,16,64} x topk {1,2}, T=257) plus the top-k 6/8 and 256-expert
# shapes of the fine-grained and expert-parallel configurations.
ROUTER_CASES = [
    {"tokens": 257, "hidden": 64, "experts": e, "topk": k, "seed": 42}
    for e in (2, 8, 16, 64) for k in (1, 2)
] + [
    {"tokens": 129, "hidden": 256, "experts": 64, "topk": 6, "seed": 7},
    {"tokens": 64, "hidden": 512, "experts": 256, "topk": 8, "seed": 8},
    {"tokens": 33, "hidden": 4096, "experts": 8, "topk": 2, "seed": 9},
    {"tokens": 17, "hidden": 7168, "experts": 256, "topk": 8, "seed": 10},
]

# Transport: tests/test_reference.py:8-10 shapes x dtypes x alignments, the
# larger validation.py:66-73 shapes, and top-k 6/8 shapes with 64 experts.
TRANSPORT_CASES = []
for _shape in [(0, 17, 8, 2), (1, 17, 8, 2), (7, 31, 8, 1), (33, 128, 8, 2)]:
    for _dtype in ("f32", "f16", "bf16"):
        for _alignment in (1, 8, 16):
            TRANSPORT_CASES.append(
                {"shape": _shape, "dtype": _dtype, "alignment": _alignment, "pattern": "skewed",
                 "seed": 42}
            )
for _index, _shape in enumerate([(129, 512, 16, 2), (257, 1024, 16, 2), (257, 64, 64, 8),
                                 (300, 40, 64, 6)]):
    for _alignment in (1, 8):
        TRANSPORT_CASES.append(
            {"shape": _shape, "dtype": "f16", "alignment": _alignment,
             "pattern": "balanced" if _index % 2 else "skewed", "seed": 43 + _index}
        )

SWIGLU_CASES = [{"rows": 37, "width": 17, "dtype": d, "seed": 5} for d in ("f16", "f32", "bf16")]
SWIGLU_CASES.append({"rows": 64, "width": 1024, "dtype": "bf16", "seed": 6})

# Blocks: config (hidden, intermediate, experts, topk).
BLOCK_CASES = [
    # configs[0] of the benchmark definition: T128 H512 I1024 E8 top-2, seed 0
    {"name": "small", "tokens": 128, "config": (512, 1024, 8, 2), "weight_seed": 0, "x_seed": 0,
     "bias": "zeros"},
]
for _k in (1, 2):
    for _tokens in (1, 13, 33):
        for _pattern in ("balanced", "skewed"):
            # tests/test_block.py:6-17 grid (H32 I64 E8)
            BLOCK_CASES.append(
                {"name": f"tiny_k{_k}_t{_tokens}_{_pattern}", "tokens": _tokens,
                 "config": (32, 64, 8, _k), "weight_seed": 42, "x_seed": 42, "bias": _pattern}
            )
BLOCK_CASES += [
    {"name": "fine_grained_small", "tokens": 96, "config": (64, 64, 64, 6), "weight_seed": 1,
     "x_seed": 1, "bias": "log_zipf"},
    {"name": "expert_parallel_small", "tokens": 48, "config": (64, 32, 256, 8), "weight_seed": 2,
     "x_seed": 2, "bias": "zeros"},
]


def checksum(tensor: torch.Tensor) -> int:
    data = tensor.detach().contiguous().cpu()
    if data.dtype == torch.bfloat16:
        data = data.view(torch.int16)
    digest = hashlib.sha1(data.numpy().tobytes()).digest()
    return int.from_bytes(digest[:7], "little")


def router_inputs(spec):
    g = torch.Generator().manual_seed(spec["seed"])
    x = torch.randn(spec["tokens"], spec["hidden"], generator=g).to(torch.bfloat16)
    w = torch.randn(spec["experts"], spec["hidden"], generator=g) / math.sqrt(spec["hidden"])
    bias = torch.randn(spec["experts"], generator=g)
    return x, w, bias


def transport_x(spec):
    """x as routing.make_case draws it (first draw of the seeded generator)."""
    tokens, hidden, _, _ = spec["shape"]
    g = torch.Generator().manual_seed(spec["seed"])
    return torch.randn((tokens, hidden), dtype=DTYPES[spec["dtype"]], generator=g)


def canonical_expert_rows(tokens, topk, hidden, dtype, seed):
    g = torch.Generator().manual_seed(seed + 501)
    return torch.randn((tokens * topk, hidden), dtype=dtype, generator=g)


def swiglu_input(spec):
    g = torch.Generator().manual_seed(spec["seed"])
    return torch.randn(spec["rows"], 2 * spec["width"], generator=g).to(DTYPES[spec["dtype"]])


def make_weights(hidden, intermediate, experts, seed):
    g = torch.Generator().manual_seed(seed)
    router = torch.randn(experts, hidden, generator=g) / math.sqrt(hidden)
    gate_up = (torch.randn(experts, 2 * intermediate, hidden, generator=g) / math.sqrt(hidden)).to(
        torch.bfloat16
    )
    down = (torch.randn(experts, hidden, intermediate, generator=g) / math.sqrt(intermediate)).to(
        torch.bfloat16
    )
    return router, gate_up, down


def block_weights(spec):
    hidden, intermediate, experts, _ = spec["config"]
    return make_weights(hidden, intermediate, experts, spec["weight_seed"])


def block_input(spec):
    hidden = spec["config"][0]
    g = torch.Generator().manual_seed(spec["x_seed"])
    return torch.randn(spec["tokens"], hidden, generator=g).to(torch.bfloat16)


def block_bias(spec):
    _, _, experts, topk = spec["config"]
    bias = torch.zeros(experts)
    if spec["bias"] == "skewed":  # layer.py:115-120 set_routing_pattern("skewed")
        bias[:topk] = 5.0
    elif spec["bias"] == "log_zipf":
        g = torch.Generator().manual_seed(spec["weight_seed"] + 1000)
        rank = torch.randperm(experts, generator=g).float() + 1.0
        bias = -1.1 * torch.log(rank)
    return bias
