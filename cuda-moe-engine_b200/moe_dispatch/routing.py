"""Seeded synthetic inputs, generated outside timed regions (reference: routing.py).

``make_case`` draws exactly as the reference's does (routing.py:6-17).  The
other generators build the benchmark configurations: transport ids with
uniform or Zipf expert popularity (drawn per token without replacement), and
block inputs and weights for the named block shapes.
"""

import math
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import torch


def make_case(tokens, hidden, experts, topk, dtype, pattern, seed, device="cuda"):
    generator = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((tokens, hidden), device=device, dtype=dtype, generator=generator)
    logits = torch.randn((tokens, experts), device=device, generator=generator)
    if pattern == "skewed":
        logits[:, :topk] += 5.0
    elif pattern != "balanced":
        raise ValueError(f"unknown pattern: {pattern}")
    selected_logits, ids64 = torch.topk(logits, topk, dim=-1)
    weights = torch.softmax(selected_logits, dim=-1).contiguous()
    return x, ids64.to(torch.int32).contiguous(), ids64.contiguous(), weights


def transport_case(tokens, hidden, experts, topk, dtype, popularity, seed, zipf_s=1.2):
    """Transport-only inputs on the CPU: x ~ N(0,1), ids drawn per token without
    replacement from uniform or Zipf(s) expert popularity, weights U(0,1)
    normalised per token."""
    generator = torch.Generator().manual_seed(seed)
    x = torch.randn((tokens, hidden), generator=generator).to(dtype)
    if popularity == "uniform":
        probs = torch.ones(experts)
    elif popularity == "zipf":
        rank = torch.randperm(experts, generator=generator).double() + 1.0
        probs = (1.0 / rank.pow(zipf_s)).float()
    else:
        raise ValueError(f"unknown popularity: {popularity}")
    ids = torch.multinomial(probs.expand(tokens, experts), topk, replacement=False,
                            generator=generator) if tokens else torch.empty(0, topk, dtype=torch.long)
    weights = torch.rand((tokens, topk), generator=generator)
    weights = weights / weights.sum(dim=1, keepdim=True)
    return x, ids.to(torch.int32).contiguous(), weights.float().contiguous()


@dataclass(frozen=True)
class BlockWorkload:
    """A named MoE block configuration and how its inputs are drawn."""

    name: str
    tokens: int
    hidden: int
    intermediate: int
    experts: int
    topk: int
    seed: int
    router_std: float = 0.0       # 0 -> N(0,1)/sqrt(H) (make_weights); else N(0, std)
    zipf_bias: float = 0.0        # > 0 -> per-expert logit bias -s*log(rank)


WORKLOADS = {
    "small": BlockWorkload("small", 128, 512, 1024, 8, 2, seed=0),
    "mixtral": BlockWorkload("mixtral", 4096, 4096, 14336, 8, 2, seed=0),
    "fine_grained": BlockWorkload("fine_grained", 16384, 2048, 1408, 64, 6, seed=1,
                                  router_std=0.02, zipf_bias=1.1),
    "expert_parallel": BlockWorkload("expert_parallel", 32768, 7168, 2048, 256, 8, seed=2,
                                     router_std=0.02),
}


def block_router(workload):
    """Router [E,H] fp32 and routing bias [E] of `workload` (the first draws of
    block_weights, from their own generator)."""
    w = workload
    g = torch.Generator().manual_seed(w.seed * 1_000_003 + 17)
    if w.router_std > 0:
        router = torch.randn(w.experts, w.hidden, generator=g) * w.router_std
    else:
        router = torch.randn(w.experts, w.hidden, generator=g) / math.sqrt(w.hidden)
    bias = torch.zeros(w.experts)
    if w.zipf_bias > 0:
        rank = torch.randperm(w.experts, generator=g).float() + 1.0
        bias = -w.zipf_bias * torch.log(rank)
    return router, bias


def block_weights(workload, experts=None, first_expert=0):
    """Weights of `workload` on the CPU (bf16 experts, fp32 router).

    Drawn per expert from seeded CPU generators so that any subset of experts
    (an expert-parallel shard) is generated without the rest: expert e uses
    seed (seed, e).  Router and bias come from their own generator.
    """
    from .layer import MoEWeights

    w = workload
    experts = w.experts if experts is None else experts
    router, bias = block_router(w)
    gate_up = torch.empty(experts, 2 * w.intermediate, w.hidden, dtype=torch.bfloat16)
    down = torch.empty(experts, w.hidden, w.intermediate, dtype=torch.bfloat16)

    def draw(local):
        ge = torch.Generator().manual_seed(w.seed * 1_000_003 + 1000 + first_expert + local)
        gate_up[local] = (torch.randn(2 * w.intermediate, w.hidden, generator=ge)
                          / math.sqrt(w.hidden)).to(torch.bfloat16)
        down[local] = (torch.randn(w.hidden, w.intermediate, generator=ge)
                       / math.sqrt(w.intermediate)).to(torch.bfloat16)

    # every expert has its own generator, so drawing them on several threads
    # gives the same bytes as drawing them in order
    workers = max(1, min(experts, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity")
                         else (os.cpu_count() or 1)))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        list(pool.map(draw, range(experts)))
    return MoEWeights(router, gate_up, down), bias


def block_input(workload, tokens=None, first_token=0):
    """x ~ N(0,1) bf16 rows [first_token, first_token + tokens) of the workload."""
    w = workload
    tokens = w.tokens if tokens is None else tokens
    g = torch.Generator().manual_seed(w.seed * 1_000_003 + 7)
    if first_token:
        torch.randn(first_token, w.hidden, generator=g)
    return torch.randn(tokens, w.hidden, generator=g).to(torch.bfloat16)
