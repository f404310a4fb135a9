"""tcgen05 grouped GEMM parity on the GPU.

The kernel accumulates in fp32 on the tensor cores, the oracle in fp32 on
the CPU in another order, and both round once to bf16.  Each output is
checked against the fp64-exact product with an fp32 accumulation allowance
(parity.assert_gemm_close), and only a small fraction of elements may differ
from the oracle at all.  Where an element differs by more than an ulp it is a
cancellation case; cuBLAS gives the same bits there.  The fused SwiGLU
epilogue is checked bit for bit against the plain GEMM followed by the
SwiGLU kernel, and that kernel against the oracle on the same inputs.  Rows
outside every expert's span must be left untouched.
"""

import pytest
import torch

from oracle import moe_oracle as oracle
from parity import assert_gemm_close, assert_within_ulps

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU required"),
]

SENTINEL = -12345.0


TILES = ["single", "pair", "pair-padded"]


def use_tile(monkeypatch, kind):
    """single: the 128x256 one-CTA tile; pair: the CTA-pair tile with the
    weights as the 256-row side and each expert's rows spread evenly over
    tiles of N <= 256; pair-padded: the CTA-pair tile over 256-row blocks of
    packed rows (what fp8 and arrival groups use)."""
    monkeypatch.setenv("MOE_B200_GEMM_TILE", "single" if kind == "single" else "pair")
    monkeypatch.setenv("MOE_B200_GEMM_SWAP", "0" if kind == "pair-padded" else "1")


@pytest.fixture(autouse=True, params=TILES)
def tile(request, monkeypatch):
    """Run every test with each tile kind."""
    use_tile(monkeypatch, request.param)
    return request.param


@pytest.fixture(scope="module")
def ext():
    from moe_dispatch import get_extension

    return get_extension()


def make_problem(counts, k_dim, n_rows_w, seed, spare_rows=5, alignment=8):
    """Packed rows [R,K] with expert spans padded to `alignment`, and weights [E,N,K]."""
    g = torch.Generator().manual_seed(seed)
    experts = len(counts)
    spans = [(c + alignment - 1) // alignment * alignment for c in counts]
    offsets = torch.zeros(experts + 1, dtype=torch.int32)
    offsets[1:] = torch.cumsum(torch.tensor(spans, dtype=torch.int32), 0)
    rows = int(offsets[-1]) + spare_rows
    a = torch.randn(rows, k_dim, generator=g).to(torch.bfloat16)
    w = (torch.randn(experts, n_rows_w, k_dim, generator=g) / k_dim**0.5).to(torch.bfloat16)
    return a, w, offsets


def run_plain(ext, a, w, offsets):
    out = torch.full((a.shape[0], w.shape[1]), SENTINEL, dtype=torch.bfloat16, device="cuda")
    ext.grouped_gemm_out(a.cuda(), w.cuda(), offsets.cuda(), out)
    torch.cuda.synchronize()
    assert ext.device_status() == 0
    return out.cpu()


def run_swiglu(ext, a, w, offsets):
    out = torch.full((a.shape[0], w.shape[1] // 2), SENTINEL, dtype=torch.bfloat16, device="cuda")
    ext.grouped_gemm_swiglu_out(a.cuda(), w.cuda(), offsets.cuda(), out)
    torch.cuda.synchronize()
    assert ext.device_status() == 0
    return out.cpu()


PLAIN_SHAPES = [
    # (rows per expert, K, N)
    ([128], 64, 256),
    ([1, 0, 200, 57], 136, 264),
    ([300, 0, 0, 129, 640], 512, 1024),
    ([7] * 16, 64, 64),
    ([0, 0, 0], 128, 256),
]


@pytest.mark.parametrize("counts,k_dim,n_cols", PLAIN_SHAPES)
def test_plain_grouped_gemm_matches_oracle(ext, counts, k_dim, n_cols):
    a, w, offsets = make_problem(counts, k_dim, n_cols, seed=sum(counts) + k_dim)
    got = run_plain(ext, a, w, offsets)
    used = int(offsets[-1])
    assert_gemm_close(got, a, w, offsets, what="plain")
    expected = oracle.grouped_gemm(a, w, offsets)
    if used:
        assert float((got[:used] != expected[:used]).float().mean()) < 0.02
    # torch fp32 reference of the same op
    for e in range(len(counts)):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            ref = (a[lo:hi].float() @ w[e].float().T).to(torch.bfloat16)
            assert float((got[lo:hi] != ref).float().mean()) < 0.02
    assert bool((got[used:] == SENTINEL).all()), "rows past the last expert were written"


SWIGLU_SHAPES = [
    ([128], 64, 128),
    ([1, 0, 200, 57], 136, 136),
    ([300, 0, 0, 129, 640], 512, 384),
    ([33] * 8, 64, 64),
]


@pytest.mark.parametrize("counts,k_dim,intermediate", SWIGLU_SHAPES)
def test_swiglu_grouped_gemm_matches_oracle(ext, counts, k_dim, intermediate):
    a, w, offsets = make_problem(counts, k_dim, 2 * intermediate, seed=7 * sum(counts) + k_dim)
    got = run_swiglu(ext, a, w, offsets)
    used = int(offsets[-1])
    # the projection this kernel computes internally, from the plain kernel
    projection = run_plain(ext, a, w, offsets)
    assert_gemm_close(projection, a, w, offsets, what="projection")
    expected = oracle.swiglu(projection[:used], used)
    assert_within_ulps(got[:used], expected, ulps=1, max_fraction=0.05, what="swiglu")
    # against the oracle's own projection only rare elements may differ
    oracle_act = oracle.swiglu(oracle.grouped_gemm(a, w, offsets)[:used], used)
    assert float((got[:used] != oracle_act).float().mean()) < 0.03
    assert bool((got[used:] == SENTINEL).all()), "rows past the last expert were written"


def test_fused_and_unfused_expert_stage_agree(ext):
    """SwiGLU in the epilogue == plain GEMM to a bf16 projection + swiglu kernel."""
    a, w, offsets = make_problem([100, 260, 0, 31], 256, 2 * 256, seed=3)
    fused = run_swiglu(ext, a, w, offsets)
    projection = run_plain(ext, a, w, offsets)
    rows = torch.tensor([int(offsets[-1])], dtype=torch.int32, device="cuda")
    unfused = torch.empty(a.shape[0], 256, dtype=torch.bfloat16, device="cuda")
    ext.swiglu_out(projection.cuda(), rows, unfused)
    used = int(offsets[-1])
    assert torch.equal(fused[:used], unfused.cpu()[:used])


def test_mixtral_shapes_on_column_slices(ext):
    """H=4096, I=14336, 8 experts: the full GEMMs run; columns are spot-checked."""
    g = torch.Generator().manual_seed(0)
    counts = [150, 90, 0, 260, 33, 128, 1, 77]
    hidden, inter = 4096, 14336
    spans = [(c + 7) // 8 * 8 for c in counts]
    offsets = torch.zeros(9, dtype=torch.int32)
    offsets[1:] = torch.cumsum(torch.tensor(spans, dtype=torch.int32), 0)
    rows = int(offsets[-1])
    a = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    gate_up = (torch.randn(8, 2 * inter, hidden, generator=g) / hidden**0.5).to(torch.bfloat16)
    down = (torch.randn(8, hidden, inter, generator=g) / inter**0.5).to(torch.bfloat16)
    act = run_swiglu(ext, a, gate_up, offsets)
    out = run_plain(ext, act, down, offsets)
    cols = torch.cat([torch.arange(0, 64), torch.arange(7000, 7064), torch.arange(inter - 64, inter)])
    sub = torch.cat([gate_up[:, cols], gate_up[:, inter + cols]], dim=1).contiguous()
    projection = run_plain(ext, a, sub, offsets)
    assert_gemm_close(projection, a, sub, offsets, what="gate/up projection")
    assert_within_ulps(act[:, cols], oracle.swiglu(projection, rows), ulps=1, max_fraction=0.05,
                       what="gate/up swiglu")
    hcols = torch.cat([torch.arange(0, 64), torch.arange(hidden - 64, hidden)])
    assert_gemm_close(out[:, hcols], act, down[:, hcols].contiguous(), offsets, what="down")


@pytest.mark.parametrize("swiglu", [False, True])
def test_tile_kinds_give_identical_bits(ext, tile, monkeypatch, swiglu):
    """The launcher picks a tile kind from the problem shape, so every kind
    must produce the same bits (an expert-parallel rank sees other shapes
    than one GPU running all experts)."""
    if tile != "single":
        pytest.skip("compares all kinds once")
    # spans 304, 0, 24, 136, 640, 8 and 264: last pair tiles of 48, 24, 136,
    # 128, 8 and 8 rows
    a, w, offsets = make_problem([300, 0, 17, 129, 640, 5, 257], 448, 2 * 192, seed=11)
    results = {}
    for kind in TILES:
        use_tile(monkeypatch, kind)
        results[kind] = run_swiglu(ext, a, w, offsets) if swiglu else run_plain(ext, a, w, offsets)
    used = int(offsets[-1])
    for kind in TILES[1:]:
        assert torch.equal(results[kind][:used], results["single"][:used]), kind
