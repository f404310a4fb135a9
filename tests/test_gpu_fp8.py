"""FP8 (e4m3) expert path on the GPU: quantiser and e4m3 grouped GEMMs.

The reference has no FP8 path (its experts are bf16, layer.py:97-98), so the
parity here is against this engine's own definition, restated in the oracle:

* the row quantiser is bit-exact against oracle.quantize_rows_e4m3, whose
  e4m3 conversion is pinned to torch's float8_e4m3fn conversion on the CPU;
* the e4m3 GEMMs multiply e4m3 values exactly and accumulate in fp32, so
  every output is checked against the fp64-exact product of the dequantised
  operands (q * scale) with the same fp32 accumulation allowance as the bf16
  GEMMs (parity.assert_gemm_close), for every tile kind;
* the fused SwiGLU epilogue is bit-exact against the plain e4m3 GEMM followed
  by the SwiGLU kernel.
"""

import pytest
import torch

from oracle import moe_oracle as oracle
from parity import assert_gemm_close

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]

TILES = ["single", "pair"]


@pytest.fixture(scope="module")
def ext():
    from moe_dispatch import get_extension

    return get_extension()


def quantize(ext, x):
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device="cuda")
    scale = torch.empty(x.shape[0], dtype=torch.float32, device="cuda")
    ext.quantize_rows_e4m3(x.cuda(), q, scale)
    torch.cuda.synchronize()
    return q, scale


@pytest.mark.parametrize("rows, cols", [(1, 16), (37, 64), (300, 4096), (9, 14336), (0, 32)])
def test_quantiser_matches_the_oracle_bit_for_bit(ext, rows, cols):
    g = torch.Generator().manual_seed(rows * 7 + cols)
    x = torch.randn(rows, cols, generator=g)
    if rows > 3:
        x[1] = 0.0                       # an all-zero row: scale 1, zeros
        x[2] *= 1e-30                    # tiny values (subnormal e4m3 after scaling)
        x[3, 5] = 3.0e4                  # one large value sets the row's amax
    x = x.to(torch.bfloat16)
    q, scale = quantize(ext, x)
    eq, escale = oracle.quantize_rows_e4m3(x)
    assert torch.equal(q.cpu().view(torch.uint8), eq.view(torch.uint8))
    assert torch.equal(scale.cpu(), escale)
    assert ext.device_status() == 0


def make_problem(counts, k_dim, n_rows_w, seed, alignment=8):
    g = torch.Generator().manual_seed(seed)
    experts = len(counts)
    spans = [(c + alignment - 1) // alignment * alignment for c in counts]
    offsets = torch.zeros(experts + 1, dtype=torch.int32)
    offsets[1:] = torch.cumsum(torch.tensor(spans, dtype=torch.int32), 0)
    rows = int(offsets[-1]) + 3
    a = torch.randn(rows, k_dim, generator=g).to(torch.bfloat16)
    w = (torch.randn(experts, n_rows_w, k_dim, generator=g) / k_dim**0.5).to(torch.bfloat16)
    return a, w, offsets


def dequantised(q, scale):
    return (q.cpu().float() * scale.cpu()[:, None]).double()


SHAPES = [
    ([128], 128, 256),
    ([1, 0, 200, 57], 144, 264),
    ([300, 0, 0, 129, 640], 512, 1024),
    ([700, 520], 4096, 512),
]


@pytest.mark.parametrize("tile", TILES)
@pytest.mark.parametrize("counts, k_dim, n_cols", SHAPES)
def test_e4m3_gemm_against_the_exact_product(ext, monkeypatch, tile, counts, k_dim, n_cols):
    monkeypatch.setenv("MOE_B200_GEMM_TILE", tile)
    a, w, offsets = make_problem(counts, k_dim, n_cols, seed=k_dim + n_cols)
    aq, ascale = quantize(ext, a)
    wq, wscale = quantize(ext, w.reshape(-1, k_dim))
    out = torch.full((a.shape[0], n_cols), -7.0, dtype=torch.bfloat16, device="cuda")
    ext.grouped_gemm_e4m3_out(aq, ascale, wq.view(w.shape), wscale, offsets.cuda(), out)
    torch.cuda.synchronize()
    assert ext.device_status() == 0
    a_deq = dequantised(aq, ascale)
    w_deq = dequantised(wq, wscale).view(w.shape)
    assert_gemm_close(out.cpu(), a_deq, w_deq, offsets, what=f"e4m3 {tile}")
    used = int(offsets[-1])
    assert bool((out[used:] == -7.0).all())  # rows past every span untouched


@pytest.mark.parametrize("tile", TILES)
def test_e4m3_swiglu_epilogue_matches_gemm_then_swiglu(ext, monkeypatch, tile):
    monkeypatch.setenv("MOE_B200_GEMM_TILE", tile)
    inter = 384
    a, w, offsets = make_problem([300, 17, 0, 640, 129], 1024, 2 * inter, seed=5)
    aq, ascale = quantize(ext, a)
    wq, wscale = quantize(ext, w.reshape(-1, 1024))
    wq = wq.view(w.shape)
    fused = torch.zeros(a.shape[0], inter, dtype=torch.bfloat16, device="cuda")
    ext.grouped_gemm_swiglu_e4m3_out(aq, ascale, wq, wscale, offsets.cuda(), fused)
    projection = torch.zeros(a.shape[0], 2 * inter, dtype=torch.bfloat16, device="cuda")
    ext.grouped_gemm_e4m3_out(aq, ascale, wq, wscale, offsets.cuda(), projection)
    plain = torch.zeros_like(fused)
    ext.swiglu_out(projection, offsets[-1:].cuda(), plain)
    torch.cuda.synchronize()
    used = int(offsets[-1])
    assert torch.equal(fused[:used], plain[:used])
    assert ext.device_status() == 0


# ------------------------------------------------------------------ the block
# FP8 parity policy: routing and dispatch are unchanged (they see the same
# bf16 tokens), and the block output stays within relative L2 8e-2 of the
# bf16 result.  e4m3 keeps 3 mantissa bits: rounding leaves each element
# within 2^-4 of its value (about 3.6 % RMS), a product of two such elements
# about 5 %, and a dot product of random-sign terms keeps that relative error
# (the error terms add like the products do); 5.4 % was measured at the small
# configuration.
FP8_REL_L2 = 8e-2


def fp8_block(workload, implementation="cuda_fused"):
    from moe_dispatch.layer import MoEBlock, MoEConfig, MoEWeights
    from moe_dispatch.routing import block_weights

    w = workload
    weights, bias = block_weights(w)
    cfg = MoEConfig(w.hidden, w.intermediate, w.experts, w.topk)
    gpu = MoEWeights(weights.router.cuda(), weights.gate_up.cuda(), weights.down.cuda())
    fp8 = MoEBlock(cfg, weights=gpu, implementation=implementation, expert_dtype="fp8_e4m3")
    ref = MoEBlock(cfg, weights=gpu)
    for block in (fp8, ref):
        block.routing_bias.copy_(bias)
    return fp8, ref, weights, bias


@pytest.mark.parametrize("name", ["small", "mixtral"])
def test_fp8_block_stays_close_to_bf16(name):
    from moe_dispatch.routing import WORKLOADS, block_input
    from parity import block_error

    w = WORKLOADS[name]
    fp8, ref, weights, bias = fp8_block(w)
    x = block_input(w).cuda()
    got = fp8(x).clone()
    expected = ref(x).clone()
    assert torch.equal(fp8.route(x)[0], ref.route(x)[0])
    assert torch.equal(fp8.workspace(x).transport.inverse, ref.workspace(x).transport.inverse)
    max_abs, rel = block_error(got, expected)
    print(f"{name}: e4m3 gate/up vs bf16 block: max-abs {max_abs:.4g}, rel-L2 {rel:.4g}")
    assert rel <= FP8_REL_L2, rel
    assert fp8.extension.device_status() == 0


def test_fp8_cuda_and_cuda_fused_agree_bit_for_bit():
    from moe_dispatch.routing import WORKLOADS, block_input

    w = WORKLOADS["small"]
    fused, _, _, _ = fp8_block(w, "cuda_fused")
    plain, _, _, _ = fp8_block(w, "cuda")
    x = block_input(w).cuda()
    assert torch.equal(fused(x).clone(), plain(x).clone())
