"""Numerical acceptance rules, written once and used by every parity test.

BASELINE's bar: float32 (TF32 tensor cores) within rtol 1e-3 / atol 1e-4 of a float64
run of the reference path; bfloat16 within rtol 2e-2. The float32 absolute floor is
1e-4 times the tensor's largest magnitude when that exceeds 1 (so c1/c4-scale tensors
get exactly atol 1e-4, while a weight gradient summed over thousands of positions, with
values near 60, is not held to 1e-4 absolute — below fp32's own rounding there). A bare
relative bound is ill-posed for values near zero, so bf16/fp16 also take an absolute
floor of 1 % of the tensor's largest magnitude (the reference's own bf16 rule is
atol 0.05, rtol 0.03, relative L2 <= 0.02; tests/test_parity.py:35-45 there) and a
whole-tensor relative L2 bound. float64 (generic CUDA-core kernels) must agree to 1e-9.
"""

from __future__ import annotations

import torch

RULES = {
    torch.float64: {"rtol": 1e-9, "atol": 1e-9, "rel_l2": 1e-10},
    torch.float32: {"rtol": 1e-3, "atol": 1e-4, "atol_scaled": True, "rel_l2": 1e-4},
    torch.bfloat16: {"rtol": 2e-2, "atol_frac": 1e-2, "rel_l2": 1e-2},
    torch.float16: {"rtol": 5e-3, "atol_frac": 2e-3, "rel_l2": 2e-3},
}


def relative_l2(actual: torch.Tensor, expected: torch.Tensor) -> float:
    a = actual.detach().to(torch.float64).cpu()
    e = expected.detach().to(torch.float64).cpu()
    return float((a - e).norm() / e.norm().clamp_min(1e-30))


def assert_matches(actual: torch.Tensor, expected: torch.Tensor, dtype: torch.dtype, what=""):
    """Elementwise and relative-L2 agreement of `actual` (any device/dtype) with the
    float64 `expected`, under the rule of `dtype`."""
    rule = RULES[dtype]
    a = actual.detach().to(torch.float64).cpu()
    e = expected.detach().to(torch.float64).cpu()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} != {tuple(e.shape)}"
    if e.numel() == 0:
        return
    atol = rule.get("atol", 0.0)
    if rule.get("atol_scaled"):
        atol *= max(1.0, float(e.abs().max()))
    if "atol_frac" in rule:
        atol = rule["atol_frac"] * float(e.abs().max())
    torch.testing.assert_close(a, e, rtol=rule["rtol"], atol=atol, msg=lambda m: f"{what}: {m}")
    error = relative_l2(a, e)
    assert error <= rule["rel_l2"], f"{what}: relative L2 error {error:.3e} > {rule['rel_l2']}"
