"""Parity at the full benchmark shapes (Mixtral C3, fine-grained C4, E=256 C5).

Three comparisons per configuration, every one at the full token count the
benchmark uses (C5 routing on 2048 tokens):

* Routing against the reference's own logits, computed the reference's way
  (``F.linear(x.float(), W) + bias`` in fp32 on the GPU with TF32 off,
  layer.py:123,136) and a lowest-index top-k.  The fused router uses another
  fp32 summation order, so a near-tie can flip: every flip must be between
  two experts whose reference logits differ by no more than the two logit
  computations disagree on that token.  The flip count is printed.
* Routing and dispatch bit-exact against the oracle for every token, and the
  block output against the oracle and against the reference's own PyTorch
  path (``MoEBlock(implementation="torch", device="cpu")``, stored in
  tests/golden/golden_full.pt by make_golden_full.py) on a token subset.
* The block output against the reference's PyTorch path run on the GPU
  (imported from baseline/_ref, where the benchmark's reference arm installs
  the reference; skipped when it is absent) on the same token subset, within
  the north-star tolerance max-abs 1e-2 and relative L2 1e-3.

The CPU results (oracle and the reference's CPU path, 3e-4 apart at the
Mixtral shape) and the GPU results (this engine and the reference's GPU path,
2e-4 apart) differ by up to ~1.1e-3 relative L2 at the Mixtral shape: the bf16
re-rounding after each GEMM turns their different fp32 accumulation into
whole-ulp differences of the intermediates at K = 4096 and 14336.  Against the
two CPU results the relative L2 bound is therefore 1.5e-3 and the max-abs
bound two bf16 ulps of the largest output, or 1e-2 where that is larger (at
the E=256 shape, outputs near 2 differ by 0.0156 = one ulp above 2); against
the reference's GPU path both are the north-star 1e-2 and 1e-3.
"""

from pathlib import Path

import pytest
import torch

from moe_dispatch._extension import get_extension
from moe_dispatch.layer import MoEBlock, MoEConfig, MoEWeights
from moe_dispatch.routing import WORKLOADS, block_input, block_router, block_weights
from oracle import moe_oracle as oracle
from parity import BLOCK_MAX_ABS, BLOCK_REL_L2, block_error

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = {c["workload"]: c for c in torch.load(ROOT / "tests" / "golden" / "golden_full.pt",
                                               weights_only=True)["full_size"]}
ROUTE_TOKENS = {"mixtral": 4096, "fine_grained": 16384, "expert_parallel": 2048}
CPU_REL_L2 = 1.5e-3  # against the oracle and the reference's CPU path (see the module docstring)


def cpu_max_abs(expected):
    """1e-2, or two bf16 ulps of the largest |expected| where that is larger."""
    top = float(expected.float().abs().max())
    ulp = 2.0 ** (torch.floor(torch.log2(torch.tensor(top))).item() - 7) if top > 0 else 0.0
    return max(BLOCK_MAX_ABS, 2 * ulp)


def reference_logits(x, router, bias):
    """layer.py:123,136: fp32 linear (no TF32) plus the routing bias."""
    previous = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return torch.nn.functional.linear(x.float(), router) + bias
    finally:
        torch.backends.cuda.matmul.allow_tf32 = previous


def lowest_index_topk(logits, k):
    """Top-k with ties to the lower expert index (a stable descending sort)."""
    return torch.sort(logits, dim=-1, descending=True, stable=True)[1][:, :k].to(torch.int32)


@pytest.mark.parametrize("name", list(ROUTE_TOKENS))
def test_router_ids_against_the_reference_logits(name):
    w = WORKLOADS[name]
    router, bias = block_router(w)
    router, bias = router.cuda(), bias.cuda()
    x = block_input(w, tokens=ROUTE_TOKENS[name]).cuda()
    tokens = x.shape[0]
    ids32 = torch.empty(tokens, w.topk, dtype=torch.int32, device="cuda")
    ids64 = torch.empty(tokens, w.topk, dtype=torch.int64, device="cuda")
    weights = torch.empty(tokens, w.topk, dtype=torch.float32, device="cuda")
    logits = torch.empty(tokens, w.experts, dtype=torch.float32, device="cuda")
    get_extension().route_out(x, router, bias, logits, ids32, ids64, weights)
    ref = reference_logits(x, router, bias)
    ref_ids = lowest_index_topk(ref, w.topk)
    ours = logits + bias
    disagreement = (ours - ref).abs().max(dim=1).values  # per token
    assert float(disagreement.max()) < 1e-3, float(disagreement.max())
    flipped = (ids32 != ref_ids).any(dim=1).nonzero().flatten().tolist()
    for t in flipped:
        tol = 2 * float(disagreement[t]) + 4 * 2.0**-23 * float(ref[t].abs().max())
        for a, b in zip(ids32[t].tolist(), ref_ids[t].tolist()):
            gap = abs(float(ref[t, a]) - float(ref[t, b]))
            assert gap <= tol, (name, t, a, b, gap, tol)
    print(f"{name}: {len(flipped)} of {tokens} tokens differ from the reference's top-{w.topk}, "
          f"all near-ties; max logit disagreement {float(disagreement.max()):.3g}")
    same = torch.ones(tokens, dtype=torch.bool, device="cuda")
    same[flipped] = False
    expected = torch.softmax(torch.gather(ref, 1, ref_ids.long()), dim=-1)
    torch.testing.assert_close(weights[same], expected[same], rtol=2e-5, atol=2e-5)
    assert get_extension().device_status() == 0


@pytest.fixture(scope="module", params=list(GOLDEN))
def full_block(request):
    """The workload's block at full size on the GPU, its output for all tokens
    and what the CPU checks need."""
    name = request.param
    w = WORKLOADS[name]
    weights, bias = block_weights(w)
    x = block_input(w)
    case = GOLDEN[name]
    assert weights.router.shape == (w.experts, w.hidden)
    block = MoEBlock(MoEConfig(w.hidden, w.intermediate, w.experts, w.topk),
                     weights=MoEWeights(weights.router.cuda(), weights.gate_up.cuda(),
                                        weights.down.cuda()))
    block.routing_bias.copy_(bias)
    xc = x.cuda()
    out = block(xc).clone()
    ids32, _, route_w = block.route(xc)
    yield {"name": name, "workload": w, "weights": weights, "bias": bias, "x": x, "xc": xc,
           "block": block, "out": out, "ids32": ids32.clone(), "route_w": route_w.clone(),
           "logits": block.logits(xc).clone(), "case": case}
    del block
    torch.cuda.empty_cache()


def test_full_size_routing_and_dispatch_match_the_oracle(full_block):
    f = full_block
    w = f["workload"]
    logits = oracle.router_logits(f["x"], f["weights"].router)
    assert torch.equal(f["logits"].cpu(), logits)
    e32, _, ew = oracle.topk_softmax(logits, f["bias"], w.topk)
    assert torch.equal(f["ids32"].cpu(), e32)
    torch.testing.assert_close(f["route_w"].cpu(), ew, rtol=2e-6, atol=2e-6)
    state = f["block"].workspace(f["xc"])
    counts, offsets, slots, inverse = oracle.dispatch_index(e32, w.experts, 8)
    assert torch.equal(state.transport.counts.cpu(), counts)
    assert torch.equal(state.transport.offsets.cpu(), offsets)
    assert torch.equal(state.transport.inverse.cpu(), inverse)


def test_full_size_block_matches_oracle_and_reference_cpu_path(full_block):
    f = full_block
    case = f["case"]
    subset = case["tokens"]
    assert torch.equal(f["ids32"].cpu()[subset], case["ids"])  # the reference's own selection
    got = f["out"].cpu()[subset]
    weights = f["weights"]
    expected = oracle.moe_tokens(f["x"][subset], f["ids32"].cpu()[subset],
                                 f["route_w"].cpu()[subset], weights.gate_up, weights.down)
    for what, ref in (("oracle", expected), ("reference CPU path", case["output"])):
        max_abs, rel = block_error(got, ref)
        print(f"{f['name']} vs {what}: max-abs {max_abs:.4g}, rel-L2 {rel:.3g}")
        assert max_abs <= cpu_max_abs(ref) and rel <= CPU_REL_L2, (what, max_abs, rel)
    assert f["block"].extension.device_status() == 0


def reference_gpu_block(workload, weights, bias):
    """The reference's MoEBlock(implementation="torch") on the GPU, holding the
    same device tensors, with the PyTorch grouped GEMM (the Triton one if this
    torch cannot run grouped_mm here)."""
    import bench

    if bench.reference_package() is None:
        pytest.skip("baseline/_ref (the reference's package) is not installed")
    import importlib

    layer = importlib.import_module(bench.REFERENCE_ALIAS + ".layer")
    w = workload
    if w.topk <= 2 and w.experts <= 64:
        cfg = layer.MoEConfig(w.hidden, w.intermediate, w.experts, w.topk)
    else:
        cfg = bench.ReferenceShape(w.hidden, w.intermediate, w.experts, w.topk)
    blocks = {}
    for backend in ("torch", "triton"):
        try:
            block = layer.MoEBlock(cfg, device="cuda", implementation="torch",
                                   expert_backend=backend,
                                   weights=layer.MoEWeights(*weights))
        except RuntimeError:
            continue
        block.routing_bias.copy_(bias)
        blocks[backend] = block
    return blocks


def test_full_size_block_matches_the_reference_gpu_path(full_block):
    f = full_block
    w = f["workload"]
    block = f["block"]
    subset = torch.arange(0, w.tokens, max(1, w.tokens // 512))
    xs = f["xc"][subset].contiguous()
    blocks = reference_gpu_block(w, (block.router_weight, block.gate_up_weight,
                                     block.down_weight), f["bias"].cuda())
    checked = 0
    for backend, ref_block in blocks.items():
        try:
            with torch.inference_mode():
                expected = ref_block(xs).clone()
                ref_ids, _, _ = ref_block.route(xs)
        except RuntimeError as err:  # e.g. grouped_mm not built for this GPU
            print(f"{f['name']}: reference GPU path with {backend} GEMM unavailable: {err}")
            continue
        if not bool(torch.isfinite(expected).all()):
            # seen with the reference's Triton grouped GEMM at the E=256 shape on B200
            print(f"{f['name']}: the reference's GPU path with its {backend} GEMM returned "
                  "non-finite outputs; not compared")
            continue
        same = (ref_ids == f["ids32"][subset]).all(dim=1)
        got = f["out"][subset]
        max_abs, rel = block_error(got[same], expected[same])
        print(f"{f['name']} vs reference GPU path ({backend} GEMM, {int(same.sum())} of "
              f"{len(subset)} tokens with the same experts): max-abs {max_abs:.4g}, rel-L2 {rel:.3g}")
        assert int(same.sum()) >= len(subset) - 2
        assert max_abs <= BLOCK_MAX_ABS and rel <= BLOCK_REL_L2, (backend, max_abs, rel)
        checked += 1
    if not checked:
        pytest.skip("the reference's GPU path could not run here")
