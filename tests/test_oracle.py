"""The oracle is pinned before it is trusted: both float64 restatements must reproduce
the reference's own outputs (golden fixtures made by running the reference's
backend='torch' in float64, tests/golden/make_golden.py), and must agree with each other
on generated geometries. CPU only."""

from __future__ import annotations

import itertools

import pytest
import torch

from oracle import convnd_oracle as oracle

CASES = [
    "c1", "c2r", "c3r", "c4r", "c5l1r", "c5l2r", "c5l3r", "tiled4d", "full5d", "full6d",
    "strided_bf16",
]


def _geometry(record):
    c = record["config"]
    return c["stride"], c["padding"], c["dilation"], c["groups"]


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_golden(name, golden):
    record = golden(name)
    stride, padding, dilation, groups = _geometry(record)
    y = oracle.forward(record["x"], record["weight"], record["bias"], stride, padding, dilation, groups)
    torch.testing.assert_close(y, record["y"], rtol=1e-10, atol=1e-10)
    dx, dw, db = oracle.backward(record["grad"], record["x"], record["weight"], stride, padding,
                                 dilation, groups)
    torch.testing.assert_close(dx, record["dx"], rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(dw, record["dw"], rtol=1e-10, atol=1e-10)
    if record["db"] is not None:
        torch.testing.assert_close(db, record["db"], rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("name", ["c1", "c5l2r", "tiled4d", "full5d", "strided_bf16"])
def test_tap_reference_matches_reference_golden(name, golden):
    record = golden(name)
    stride, padding, dilation, groups = _geometry(record)
    y = oracle.tap_reference(record["x"], record["weight"], record["bias"], stride, padding,
                             dilation, groups)
    torch.testing.assert_close(y, record["y"], rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("name", ["c1", "c4r", "c5l1r", "c5l2r", "tiled4d", "full5d",
                                  "strided_bf16"])
def test_tap_adjoints_match_reference_golden(name, golden):
    """tap_dgrad / tap_wgrad (used by the full-size GPU checks) reproduce the reference's
    own input and weight gradients."""
    record = golden(name)
    stride, padding, dilation, groups = _geometry(record)
    x, w, dy = record["x"], record["weight"], record["grad"]
    dx = oracle.tap_dgrad(dy, w, tuple(x.shape[2:]), stride, padding, dilation, groups)
    torch.testing.assert_close(dx, record["dx"], rtol=1e-10, atol=1e-10)
    dw = oracle.tap_wgrad(dy, x, tuple(w.shape[2:]), stride, padding, dilation, groups)
    torch.testing.assert_close(dw, record["dw"], rtol=1e-10, atol=1e-10)


def _geometries():
    """Deterministic sweep in the spirit of the reference's Hypothesis geometry test
    (tests/test_correctness_properties.py:14-91): ranks 1-5, groups 1-2, kernel 1-3,
    stride/dilation 1-2, padding 0-2."""
    generator = torch.Generator().manual_seed(604)
    out = []
    for rank, groups in itertools.product(range(1, 6), (1, 2)):
        for _ in range(3):
            pick = lambda lo, hi: int(torch.randint(lo, hi + 1, (1,), generator=generator))
            kernel = tuple(pick(1, 3) for _ in range(rank))
            dilation = tuple(pick(1, 2) for _ in range(rank))
            padding = tuple(pick(0, 2) for _ in range(rank))
            stride = tuple(pick(1, 2) for _ in range(rank))
            spatial = tuple(max(pick(3, 5), d * (k - 1) + 1 - 2 * p)
                            for k, d, p in zip(kernel, dilation, padding))
            out.append((rank, groups, kernel, dilation, padding, stride, spatial))
    return out


@pytest.mark.parametrize("geometry", _geometries())
def test_restatements_agree(geometry):
    rank, groups, kernel, dilation, padding, stride, spatial = geometry
    generator = torch.Generator().manual_seed(rank * 31 + groups)
    x = torch.randn((2, 2 * groups, *spatial), generator=generator, dtype=torch.float64)
    w = torch.randn((2 * groups, 2, *kernel), generator=generator, dtype=torch.float64)
    b = torch.randn(2 * groups, generator=generator, dtype=torch.float64)
    y = oracle.forward(x, w, b, stride, padding, dilation, groups)
    y_tap = oracle.tap_reference(x, w, b, stride, padding, dilation, groups)
    torch.testing.assert_close(y, y_tap, rtol=1e-10, atol=1e-10)
    # Backward against autograd of the independent restatement.
    dy = torch.randn(y.shape, generator=generator, dtype=torch.float64)
    xr, wr, br = (t.clone().requires_grad_() for t in (x, w, b))
    expected = torch.autograd.grad(oracle_tap_graph(xr, wr, br, stride, padding, dilation, groups),
                                   (xr, wr, br), dy)
    got = oracle.backward(dy, x, w, stride, padding, dilation, groups)
    for g, e in zip(got, expected, strict=True):
        torch.testing.assert_close(g, e, rtol=1e-10, atol=1e-10)


def oracle_tap_graph(x, w, b, stride, padding, dilation, groups):
    """Differentiable tap-by-tap convolution (same maths as oracle.tap_reference)."""
    rank = x.ndim - 2
    padded = torch.nn.functional.pad(x, tuple(v for p in reversed(padding) for v in (p, p)))
    out = oracle.output_shape(x.shape[2:], w.shape[2:], stride, padding, dilation)
    total = None
    for tap in itertools.product(*(range(k) for k in w.shape[2:])):
        slices = tuple(slice(t * d, t * d + size * s, s)
                       for t, d, size, s in zip(tap, dilation, out, stride))
        patch = padded[(slice(None), slice(None), *slices)].reshape(
            x.shape[0], groups, x.shape[1] // groups, -1)
        coefficient = w[(slice(None), slice(None), *tap)].reshape(
            groups, w.shape[0] // groups, x.shape[1] // groups)
        term = torch.einsum("goc,bgcp->bgop", coefficient, patch)
        total = term if total is None else total + term
    return total.reshape(x.shape[0], w.shape[0], *out) + b.reshape(1, -1, *((1,) * rank))


def test_sampled_forward_matches_full_oracle(golden):
    record = golden("strided_bf16")
    stride, padding, dilation, groups = _geometry(record)
    y = record["y"]
    generator = torch.Generator().manual_seed(5)
    points = []
    for _ in range(40):
        n = int(torch.randint(0, y.shape[0], (1,), generator=generator))
        co = int(torch.randint(0, y.shape[1], (1,), generator=generator))
        coords = tuple(int(torch.randint(0, s, (1,), generator=generator)) for s in y.shape[2:])
        points.append((n, co, coords))
    values = oracle.sampled_forward(record["x"], record["weight"], record["bias"], stride,
                                    padding, dilation, groups, points)
    expected = torch.stack([y[(n, co, *coords)] for n, co, coords in points])
    torch.testing.assert_close(values, expected, rtol=1e-10, atol=1e-10)


def test_known_answer_huge_stride_and_padding():
    """Reference test_convnd.py:347-356: all-padding windows give the bias."""
    x = torch.randn(1, 2, 1, 2, 2, 2, dtype=torch.float64)
    w = torch.randn(3, 2, 1, 1, 1, 1, dtype=torch.float64)
    b = torch.randn(3, dtype=torch.float64)
    out = oracle.output_shape(x.shape[2:], w.shape[2:], (2**35, 1, 1, 1), (2**34, 0, 0, 0),
                              (1, 1, 1, 1))
    assert out == (2, 2, 2, 2)


def test_compiled_reference_matches_golden():
    """The reference's own native CPU path (compiled from its sources into oracle/_ref by
    oracle/build_ref.py) reproduces the golden vectors; run in a subprocess because it
    registers CPU kernels for the same operators as the B200 package."""
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    if not (root / "oracle" / "_ref" / "libtorch_convnd_ref_cpu.so").exists():
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    result = subprocess.run(
        [sys.executable, str(root / "tests" / "_ref_check.py"), "c1", "c2r", "c5l1r", "c5l2r",
         "tiled4d", "full5d"], capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stderr[-2000:]
    worst = float(result.stdout.strip().split("=")[-1])
    assert worst < 1e-12


@pytest.mark.parametrize(
    ("shape", "cout", "kernel", "stride", "padding", "dilation", "groups"),
    [((2, 4, 7, 6, 5), 6, (3, 2, 3), (1, 2, 1), (1, 1, 2), (1, 1, 2), 2),
     ((1, 2, 9, 8), 3, (3, 3), (2, 2), (1, 0), (1, 2), 1),
     ((2, 3, 5, 4, 4, 3), 2, (2, 3, 1, 3), (1, 1, 2, 1), (0, 1, 0, 2), (2, 1, 1, 1), 1)],
)
def test_sampled_oracle_matches_full_oracle(shape, cout, kernel, stride, padding, dilation,
                                            groups):
    """The point samplers used by the full-size GPU checks agree with the full fp64
    oracle at every point of small strided, dilated and grouped problems."""
    generator = torch.Generator().manual_seed(11)
    x = torch.randn(shape, generator=generator, dtype=torch.float64)
    w = torch.randn((cout, shape[1] // groups, *kernel), generator=generator,
                    dtype=torch.float64)
    b = torch.randn(cout, generator=generator, dtype=torch.float64)
    y = oracle.forward(x, w, b, stride, padding, dilation, groups)
    dy = torch.randn(y.shape, generator=generator, dtype=torch.float64)
    dx, dw, _ = oracle.backward(dy, x, w, stride, padding, dilation, groups)
    out_points = [(n, c, idx) for n in range(shape[0]) for c in range(cout)
                  for idx in itertools.product(*map(range, y.shape[2:]))]
    in_points = [(n, c, idx) for n in range(shape[0]) for c in range(shape[1])
                 for idx in itertools.product(*map(range, shape[2:]))]
    entries = [(co, cl, t) for co in range(cout) for cl in range(shape[1] // groups)
               for t in itertools.product(*map(range, kernel))]
    sy = oracle.sampled_forward(x, w, b, stride, padding, dilation, groups, out_points)
    sdx = oracle.sampled_dgrad(dy, w, shape[2:], stride, padding, dilation, groups, in_points)
    sdw = oracle.sampled_wgrad(dy, x, kernel, stride, padding, dilation, groups, entries)
    torch.testing.assert_close(sy, torch.stack([y[n, c][i] for n, c, i in out_points]),
                               rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(sdx, torch.stack([dx[n, c][i] for n, c, i in in_points]),
                               rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(sdw, torch.stack([dw[co, cl][t] for co, cl, t in entries]),
                               rtol=1e-12, atol=1e-12)
