"""Numerical acceptance rules, written once and used by every parity test.

BASELINE's bar: float32 (TF32 tensor cores) within rtol 1e-3 / atol 1e-4 of a float64
run of the reference path; bfloat16 within rtol 2e-2. A bare relative bound is ill-posed
for values near zero, so bf16/fp16 also take an absolute floor of 1 % of the tensor's
largest magnitude (the reference's own bf16 rule is atol 0.05, rtol 0.03, relative
L2 <= 0.02; tests/test_parity.py:35-45 there) and a whole-tensor relative L2 bound.
float64 (generic CUDA-core kernels) must agree to 1e-9.

float32 reductions. Every output element is a sum of K products; fp32 arithmetic itself
(the reference's own fp32 path included) carries the textbook error bound of a pairwise
or blocked sum, ceil(log2 K) * 2^-24 * sum_k |a_k b_k| (Higham, "Accuracy and Stability
of Numerical Algorithms", 2nd ed., section 4.2). Where a caller supplies that sum of
magnitudes per element (``magnitude``), the float32 absolute tolerance of that element is
1e-4 plus this bound. For outputs and input gradients (K of a few thousand, magnitudes
of a few units) the bound is far below 1e-4 and the literal bar applies; for a weight
gradient summed over a million positions (c4's dW, values near 1000) it is the bar any
fp32 implementation is held to (the reference's own fp32 path misses the literal atol
there: tests/golden/c4_fp32_reference_error.json).

float32 weight gradients run on the tensor cores as split products: each operand is a
bfloat16 pair hi + lo (|x - hi - lo| <= 2^-16 |x|) and each product is the three terms
hi*hi + hi*lo + lo*hi, so a product carries at most 3 * 2^-16 of its magnitude besides
the fp32 sum (``split=True`` adds that term). This is more accurate than the single TF32
product (2^-11 per operand) that BASELINE allows for float32 on the tensor cores.
"""

from __future__ import annotations

import math

import torch

RULES = {
    torch.float64: {"rtol": 1e-9, "atol": 1e-9, "rel_l2": 1e-10},
    torch.float32: {"rtol": 1e-3, "atol": 1e-4, "rel_l2": 1e-4},
    torch.bfloat16: {"rtol": 2e-2, "atol_frac": 1e-2, "rel_l2": 1e-2},
    torch.float16: {"rtol": 5e-3, "atol_frac": 2e-3, "rel_l2": 2e-3},
}

FP32_UNIT_ROUNDOFF = 2.0**-24


SPLIT_PRODUCT_ERROR = 3 * 2.0**-16


def fp32_sum_bound(magnitude: torch.Tensor, terms: int, split: bool = False) -> torch.Tensor:
    """Pairwise-summation error bound of fp32 sums of `terms` products whose absolute
    values add up to `magnitude` (elementwise), plus the per-product error of bfloat16
    hi/lo split products when `split`."""
    unit = math.ceil(math.log2(max(terms, 2))) * FP32_UNIT_ROUNDOFF
    if split:
        unit += SPLIT_PRODUCT_ERROR
    return unit * magnitude


def relative_l2(actual: torch.Tensor, expected: torch.Tensor) -> float:
    a = actual.detach().to(torch.float64)
    e = expected.detach().to(torch.float64).to(a.device)
    return float((a - e).norm() / e.norm().clamp_min(1e-30))


def violations(actual, expected, dtype, magnitude=None, terms=None, split=False):
    """(count, worst error / allowed error, index of the worst element, allowed there) of
    `actual` against the float64 `expected` under the elementwise rule of `dtype`."""
    rule = RULES[dtype]
    a = actual.detach().to(torch.float64)
    e = expected.detach().to(torch.float64).to(a.device)
    atol = rule.get("atol", 0.0)
    if "atol_frac" in rule:
        atol = rule["atol_frac"] * float(e.abs().max())
    allowed = atol + rule["rtol"] * e.abs()
    if magnitude is not None and dtype == torch.float32:
        allowed = allowed + fp32_sum_bound(magnitude.to(a.device, torch.float64), terms, split)
    ratio = (a - e).abs() / allowed
    worst = int(ratio.argmax())
    return (int((ratio > 1).sum()), float(ratio.reshape(-1)[worst]), worst,
            float(allowed.reshape(-1)[worst]))


def assert_matches(actual: torch.Tensor, expected: torch.Tensor, dtype: torch.dtype, what="",
                   magnitude: torch.Tensor | None = None, terms: int | None = None,
                   split: bool = False):
    """Elementwise and relative-L2 agreement of `actual` (any device/dtype) with the
    float64 `expected`, under the rule of `dtype` (for float32 with the per-element
    summation bound when `magnitude` and `terms` are given)."""
    a = actual.detach().to(torch.float64)
    e = expected.detach().to(torch.float64).to(a.device)
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} != {tuple(e.shape)}"
    if e.numel() == 0:
        return
    count, ratio, index, allowed = violations(a, e, dtype, magnitude, terms, split)
    assert count == 0, (
        f"{what}: {count} of {e.numel()} elements outside the {dtype} bar; worst at flat "
        f"index {index}: got {float(a.reshape(-1)[index]):.9g}, expected "
        f"{float(e.reshape(-1)[index]):.9g}, error {ratio:.3g}x the allowed {allowed:.3g}")
    error = relative_l2(a, e)
    limit = RULES[dtype]["rel_l2"]
    assert error <= limit, f"{what}: relative L2 error {error:.3e} > {limit}"


def conv_magnitudes(x, w, dy, stride, padding, dilation, groups, tap=False):
    """Per-element sums of |products| of the forward output, input gradient and weight
    gradient (the same convolutions on absolute values) and their term counts, for the
    float32 summation bound. `tap` selects the oracle's tap-by-tap functions, which run
    on the tensors' device (full-size checks on the GPU)."""
    from oracle import convnd_oracle as oracle

    ax, aw, ady = x.abs(), w.abs(), dy.abs()
    rank = x.ndim - 2
    taps = math.prod(w.shape[2:])
    positions = x.shape[0] * math.prod(dy.shape[2:])
    if tap:
        y = oracle.tap_reference(ax, aw, None, stride, padding, dilation, groups)
        dx = oracle.tap_dgrad(ady, aw, tuple(x.shape[2:]), stride, padding, dilation, groups)
        dw = oracle.tap_wgrad(ady, ax, tuple(w.shape[2:]), stride, padding, dilation, groups)
    else:
        y = oracle.forward(ax, aw, None, stride, padding, dilation, groups)
        dx, dw, _ = oracle.backward(ady, ax, aw, stride, padding, dilation, groups,
                                    mask=(True, True, False))
    db = ady.to(torch.float64).sum(dim=(0, *range(2, 2 + rank)))
    # the weight gradient's float32 products are always bf16 hi/lo split products
    return {"y": (y, w.shape[1] * taps, False), "dx": (dx, (w.shape[0] // groups) * taps, False),
            "dw": (dw, positions, True), "db": (db, positions, False)}


def assert_conv_matches(got, expected, dtype, what, magnitudes=None):
    """assert_matches over a dict of {y, dx, dw, db} tensors (None entries skipped), with
    the float32 summation bound of `magnitudes` (from conv_magnitudes) when given."""
    for name, value in got.items():
        if value is None or expected.get(name) is None:
            continue
        magnitude, terms, split = (magnitudes or {}).get(name, (None, None, False))
        assert_matches(value, expected[name], dtype, f"{what} {name}", magnitude, terms, split)
