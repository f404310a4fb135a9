"""Comparison helpers shared by the parity tests."""

import torch

ULP = {torch.bfloat16: 2.0**-7, torch.float16: 2.0**-10, torch.float32: 2.0**-23}


def assert_within_ulps(actual, expected, ulps=1, max_fraction=1.0, what=""):
    """Every element within `ulps` units in the last place of the expected value,
    and at most `max_fraction` of the elements different at all."""
    actual = actual.detach().cpu()
    expected = expected.detach().cpu()
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    if actual.numel() == 0:
        return
    a, e = actual.float(), expected.float()
    # ulp at the larger of the two magnitudes: a rounding step that crosses a
    # power of two is one ulp of the upper binade
    scale = torch.clamp(torch.maximum(a.abs(), e.abs()), min=2.0**-14)
    ulp = torch.exp2(torch.floor(torch.log2(scale))) * ULP[expected.dtype]
    bad = (a - e).abs() > ulps * ulp
    assert not bool(bad.any()), (
        f"{what}: {int(bad.sum())} elements beyond {ulps} ulp; "
        f"worst |diff| {float((a - e).abs().max())}"
    )
    frac = float((a != e).float().mean())
    assert frac <= max_fraction, f"{what}: {frac:.4%} of elements differ (limit {max_fraction:.4%})"


def assert_gemm_close(got, a, w, offsets, what="gemm"):
    """A grouped GEMM with fp32 accumulation against the fp64-exact product.

    Every element must satisfy |got - exact| <= 1 ulp(bf16) + 16 * 2^-23 * sum|a*w|:
    one rounding of the bf16 output plus an fp32 accumulation allowance that
    scales with the magnitudes summed (so results that cancel to nearly zero
    are judged by absolute error, as any fp32 summation order must be).
    A missing or repeated product term (~|a*w|) is far outside this bound.
    """
    got = got.detach().cpu().float()
    used = int(offsets[-1])
    exact = torch.zeros(used, w.shape[1], dtype=torch.float64)
    absum = torch.zeros_like(exact)
    for e in range(w.shape[0]):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            exact[lo:hi] = a[lo:hi].double() @ w[e].double().T
            absum[lo:hi] = a[lo:hi].double().abs() @ w[e].double().abs().T
    g = got[:used].double()
    scale = torch.clamp(torch.maximum(g.abs(), exact.abs()), min=2.0**-14)
    ulp = torch.exp2(torch.floor(torch.log2(scale))) * 2.0**-7
    bound = ulp + 16 * 2.0**-23 * absum
    excess = (g - exact).abs() - bound
    assert not bool((excess > 0).any()), (
        f"{what}: {int((excess > 0).sum())} elements outside the bound; worst excess "
        f"{float(excess.max())}"
    )


def block_error(actual, expected):
    """(max-abs, rel-L2) of a block output against its reference."""
    a, e = actual.detach().cpu().float(), expected.detach().cpu().float()
    if e.numel() == 0:
        return 0.0, 0.0
    diff = a - e
    return float(diff.abs().max()), float(diff.norm() / e.norm().clamp_min(1e-8))


# The north-star tolerance for bf16 block outputs.
BLOCK_MAX_ABS = 1e-2
BLOCK_REL_L2 = 1e-3
