"""GPU parity of the B200 kernels against the reference's outputs and the fp64 oracle.

Every comparison calls the product path (torch_convnd on CUDA: the native shim and the
C-ABI library) and checks it against (a) golden fixtures made by running the reference
itself in float64, and (b) the float64 CPU oracle on further seeded geometries. The
tolerances are the rules in tests/tolerances.py.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import torch_convnd
from oracle import convnd_oracle as oracle
from tolerances import assert_conv_matches, assert_matches, conv_magnitudes
from torch_convnd import _native, conv_nd

pytestmark = pytest.mark.gpu

GOLDEN_CASES = [
    "c1", "c2r", "c3r", "c4r", "c5l1r", "c5l2r", "c5l3r", "tiled4d", "full5d", "full6d",
    "strided_bf16",
]


def _run(x, w, b, dy, stride, padding, dilation, groups, mask=(True, True, True)):
    """Forward through conv_nd and backward through autograd, on the current device."""
    x = x.detach().clone().requires_grad_(mask[0])
    w = w.detach().clone().requires_grad_(mask[1])
    b = None if b is None else b.detach().clone().requires_grad_(mask[2])
    y = conv_nd(x, w, b, stride, padding, dilation, groups, backend="native")
    inputs = [t for t in (x, w, b) if t is not None and t.requires_grad]
    grads = torch.autograd.grad(y, inputs, dy) if inputs else ()
    it = iter(grads)
    dx = next(it) if mask[0] else None
    dw = next(it) if mask[1] else None
    db = next(it) if (b is not None and mask[2]) else None
    return y, dx, dw, db


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_golden_case(name, golden):
    record = golden(name)
    c = record["config"]
    dtype = record["x"].dtype
    cuda = lambda t: None if t is None else t.cuda()
    y, dx, dw, db = _run(cuda(record["x"]), cuda(record["weight"]), cuda(record["bias"]),
                         cuda(record["grad"]), c["stride"], c["padding"], c["dilation"],
                         c["groups"])
    torch.cuda.synchronize()
    torch_convnd.device_status()
    assert y.dtype == dtype
    magnitudes = None
    if dtype == torch.float32:
        magnitudes = conv_magnitudes(record["x"], record["weight"], record["grad"],
                                     c["stride"], c["padding"], c["dilation"], c["groups"])
    assert_conv_matches({"y": y, "dx": dx, "dw": dw, "db": db}, record, dtype, name, magnitudes)


def _problem_mask(x, w, stride, padding, dilation, groups):
    """cnd_fast_path_mask for a geometry (bit 0 fwd, bit 1 dgrad, bit 2 wgrad)."""
    library = _native.core()

    class Problem(ctypes.Structure):
        _fields_ = [("rank", ctypes.c_int32), ("dtype", ctypes.c_int32),
                    ("fp32_mode", ctypes.c_int32), ("reserved", ctypes.c_int32)] + [
            (n, ctypes.c_int64) for n in ("batch", "channels", "output_channels", "groups",
                                          "input_volume", "output_volume", "kernel_volume")] + [
            (n, ctypes.c_int64 * 62)
            for n in ("input", "output", "kernel", "stride", "padding", "dilation")]

    codes = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2, torch.float64: 3}
    arr = lambda v: (ctypes.c_int64 * len(v))(*v)
    problem = Problem()
    rank = x.ndim - 2
    assert library.cnd_problem_init(ctypes.byref(problem), rank, arr(list(x.shape)),
                                    arr(list(w.shape)), arr(stride), arr(padding), arr(dilation),
                                    ctypes.c_int64(groups), codes[x.dtype]) == 0
    return library.cnd_fast_path_mask(ctypes.byref(problem))


@pytest.mark.parametrize(
    ("name", "expected"),
    [("c2r", 7), ("c3r", 7), ("c4r", 7), ("c5l1r", 7), ("c5l2r", 7), ("c5l3r", 7), ("c1", 7),
     ("strided_bf16", 7)],
)
def test_configs_run_on_tensor_cores(name, expected, golden):
    """The BASELINE configurations take the tcgen05 path for every pass, strided input
    gradients included (phase sub-convolutions; c5's first layer never requests one in
    training, but a strided layer with an input gradient no longer leaves the fast path)."""
    record = golden(name)
    c = record["config"]
    mask = _problem_mask(record["x"], record["weight"], c["stride"], c["padding"], c["dilation"],
                         c["groups"])
    assert mask & expected == expected


def _sweep():
    cases = []
    # (rank, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups)
    cases.append((4, 2, 32, 64, (6, 5, 7, 9), (3, 3, 3, 3), (1,) * 4, (1,) * 4, (1,) * 4, 1))
    cases.append((4, 3, 16, 16, (5, 6, 4, 11), (3, 1, 2, 3), (1,) * 4, (1, 0, 1, 1), (1,) * 4, 1))
    cases.append((4, 2, 64, 48, (4, 4, 5, 6), (2, 2, 2, 2), (1,) * 4, (0, 1, 1, 0), (1, 1, 2, 1), 1))
    cases.append((4, 2, 20, 24, (5, 5, 5, 5), (3, 3, 3, 3), (1,) * 4, (1,) * 4, (1,) * 4, 2))
    cases.append((4, 2, 16, 32, (9, 8, 8, 10), (3, 3, 3, 3), (2,) * 4, (1,) * 4, (1,) * 4, 1))
    cases.append((5, 1, 16, 32, (5, 4, 6, 5, 7), (3,) * 5, (1,) * 5, (1,) * 5, (1,) * 5, 1))
    cases.append((6, 1, 8, 16, (3, 4, 3, 4, 5, 4), (3,) * 6, (1,) * 6, (1,) * 6, (1,) * 6, 1))
    cases.append((3, 2, 128, 32, (6, 7, 9), (3, 3, 3), (1,) * 3, (1,) * 3, (1,) * 3, 1))
    cases.append((2, 2, 32, 16, (13, 17), (3, 5), (1, 1), (1, 2), (1, 1), 1))
    cases.append((1, 2, 16, 16, (40,), (5,), (1,), (2,), (1,), 1))
    cases.append((7, 1, 16, 16, (3, 2, 3, 2, 3, 2, 4), (2,) * 7, (1,) * 7, (1,) * 7, (1,) * 7, 1))
    cases.append((4, 2, 8, 8, (4, 4, 4, 4), (3,) * 4, (1,) * 4, (3, 0, 2, 1), (1, 1, 1, 1), 1))
    # thin groups, run dense with block-diagonal weights
    cases.append((4, 2, 16, 16, (5, 6, 4, 7), (3, 3, 1, 1), (1,) * 4, (2, 2, 0, 0), (2, 2, 1, 1),
                  4))
    cases.append((4, 2, 32, 32, (4, 5, 4, 6), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 32))
    cases.append((5, 1, 24, 12, (4, 4, 3, 5, 4), (2, 3, 3, 2, 3), (1,) * 5, (1,) * 5, (1,) * 5, 3))
    cases.append((4, 2, 16, 32, (7, 6, 8, 9), (3,) * 4, (2,) * 4, (1,) * 4, (1,) * 4, 2))
    # unit axes (extent 1, kernel 1, no padding) dropped as the reference's
    # without_unit_axes does, and runs of pointwise axes merged into one
    cases.append((5, 2, 16, 32, (1, 6, 1, 7, 5), (1, 3, 1, 3, 1), (1,) * 5, (0, 1, 0, 1, 0),
                  (1,) * 5, 1))
    cases.append((4, 2, 32, 32, (9, 10, 4, 6), (3, 3, 1, 1), (1,) * 4, (2, 2, 0, 0),
                  (2, 2, 1, 1), 4))
    cases.append((6, 1, 16, 16, (1, 1, 1, 1, 1, 1), (1,) * 6, (1,) * 6, (0,) * 6, (1,) * 6, 1))
    # a0 taps at dilation 2 folded over output planes of one parity (odd a0 extent)
    cases.append((4, 2, 16, 32, (9, 6, 5, 7), (3,) * 4, (1,) * 4, (2, 1, 1, 1), (2, 1, 1, 1), 1))
    # strided input gradients as phase sub-convolutions: mixed strides and paddings,
    # dilation sharing a factor with the stride, and a kernel-1 stride-2 axis whose odd
    # positions receive no tap (zeroed residue classes)
    cases.append((4, 1, 16, 32, (7, 8, 6, 9), (3,) * 4, (2, 1, 2, 1), (0, 1, 2, 1),
                  (1, 1, 1, 2), 1))
    cases.append((3, 2, 16, 16, (9, 10, 11), (3, 2, 1), (2, 3, 2), (1, 0, 0), (2, 1, 1), 1))
    cases.append((4, 2, 32, 16, (8, 7, 9, 6), (3, 3, 2, 3), (2, 2, 1, 1), (1, 1, 0, 1),
                  (1, 1, 1, 1), 2))
    return cases


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("case", _sweep(), ids=lambda c: f"r{c[0]}_{c[2]}x{c[3]}_g{c[9]}")
def test_geometry_sweep_against_oracle(case, dtype):
    rank, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups = case
    generator = torch.Generator().manual_seed(hash(case) % (2**31))
    x = torch.randn((batch, cin, *spatial), generator=generator).to(dtype)
    w = (torch.randn((cout, cin // groups, *kernel), generator=generator) * 0.1).to(dtype)
    b = torch.randn(cout, generator=generator).to(dtype)
    y_ref = oracle.forward(x, w, b, stride, padding, dilation, groups)
    dy = torch.randn(y_ref.shape, generator=generator).to(dtype)
    dx_ref, dw_ref, db_ref = oracle.backward(dy, x, w, stride, padding, dilation, groups)
    y, dx, dw, db = _run(x.cuda(), w.cuda(), b.cuda(), dy.cuda(), stride, padding, dilation,
                         groups)
    torch.cuda.synchronize()
    torch_convnd.device_status()
    magnitudes = None
    if dtype == torch.float32:
        magnitudes = conv_magnitudes(x, w, dy, stride, padding, dilation, groups)
    assert_conv_matches({"y": y, "dx": dx, "dw": dw, "db": db},
                        {"y": y_ref, "dx": dx_ref, "dw": dw_ref, "db": db_ref}, dtype, "sweep",
                        magnitudes)


# 12 slices along box axis 0 and enough work per slice for 6-tile folded super tiles
# (the c3 forward plan); tests/test_full_size.py pins that plan on the CPU.
SIX_TILE_CASE = (4, 4, 16, 32, (10, 12, 12, 12), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 1)


def test_six_tile_folded_super_tiles_match_oracle():
    rank, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups = SIX_TILE_CASE
    generator = torch.Generator().manual_seed(66)
    x = torch.randn((batch, cin, *spatial), generator=generator).bfloat16()
    w = (torch.randn((cout, cin, *kernel), generator=generator) * 0.1).bfloat16()
    b = torch.randn(cout, generator=generator).bfloat16()
    y_ref = oracle.forward(x, w, b, stride, padding, dilation, groups)
    dy = torch.randn(y_ref.shape, generator=generator).bfloat16()
    dx_ref, dw_ref, db_ref = oracle.backward(dy, x, w, stride, padding, dilation, groups)
    y, dx, dw, db = _run(x.cuda(), w.cuda(), b.cuda(), dy.cuda(), stride, padding, dilation,
                         groups)
    torch.cuda.synchronize()
    torch_convnd.device_status()
    for got, ref, what in ((y, y_ref, "y"), (dx, dx_ref, "dx"), (dw, dw_ref, "dw"),
                           (db, db_ref, "db")):
        assert_matches(got, ref, torch.bfloat16, what)


@pytest.mark.parametrize("rank", [4, 5, 6, 7, 8])
def test_float64_ranks_match_tap_reference(rank):
    """Reference tests/test_convnd.py:98-116 on the generic CUDA-core kernels."""
    generator = torch.Generator().manual_seed(44 + rank)
    x = torch.randn((1, 4, *((3,) * rank)), generator=generator, dtype=torch.float64)
    w = torch.randn((4, 2, *((2,) * rank)), generator=generator, dtype=torch.float64)
    b = torch.randn(4, generator=generator, dtype=torch.float64)
    stride = (2,) + (1,) * (rank - 1)
    padding = (0, 1) + (0,) * (rank - 2)
    dilation = (1,) * rank
    y_ref = oracle.tap_reference(x, w, b, stride, padding, dilation, 2)
    dy = torch.randn(y_ref.shape, generator=generator, dtype=torch.float64)
    refs = oracle.backward(dy, x, w, stride, padding, dilation, 2)
    y, dx, dw, db = _run(x.cuda(), w.cuda(), b.cuda(), dy.cuda(), stride, padding, dilation, 2)
    assert_matches(y, y_ref, torch.float64, "y")
    for got, ref in zip((dx, dw, db), refs, strict=True):
        assert_matches(got, ref, torch.float64, "grad")


def test_gradcheck_and_gradgradcheck_float64():
    """Reference tests/test_convnd.py:144-156 and :303-309."""
    x = torch.randn(1, 2, 2, 2, 2, 3, device="cuda", dtype=torch.float64, requires_grad=True)
    w = torch.randn(2, 2, 2, 1, 2, 2, device="cuda", dtype=torch.float64, requires_grad=True)
    b = torch.randn(2, device="cuda", dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(
        lambda x, w, b: conv_nd(x, w, b, padding=(1, 0, 0, 1), stride=(1, 1, 1, 2)),
        (x, w, b), fast_mode=True)
    x2 = torch.randn(1, 1, 2, 2, 2, 2, device="cuda", dtype=torch.float64, requires_grad=True)
    w2 = torch.randn(1, 1, 2, 1, 1, 1, device="cuda", dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradgradcheck(lambda x, w: conv_nd(x, w), (x2, w2), fast_mode=True)


def test_large_integer_metadata_known_answer():
    """Reference tests/test_convnd.py:347-356: huge stride/padding give the bias."""
    x = torch.randn(1, 2, 1, 2, 2, 2, device="cuda", dtype=torch.float64, requires_grad=True)
    w = torch.randn(3, 2, 1, 1, 1, 1, device="cuda", dtype=torch.float64, requires_grad=True)
    b = torch.randn(3, device="cuda", dtype=torch.float64, requires_grad=True)
    y = conv_nd(x, w, b, padding=(2**34, 0, 0, 0), stride=(2**35, 1, 1, 1))
    torch.testing.assert_close(y, b.reshape(1, 3, 1, 1, 1, 1).expand(1, 3, 2, 2, 2, 2))
    gx, gw, gb = torch.autograd.grad(y.sum(), (x, w, b))
    assert torch.count_nonzero(gx) == 0 and torch.count_nonzero(gw) == 0
    torch.testing.assert_close(gb, torch.full_like(gb, 16.0))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_deterministic_on_a_side_stream(dtype):
    """Bitwise-repeatable gradients on a non-default stream (reference
    tests/test_convnd.py:235-257); the B200 kernels use no atomics."""
    generator = torch.Generator().manual_seed(7)
    x = torch.randn(2, 16, 6, 5, 6, 7, generator=generator).to(dtype).cuda()
    w = (torch.randn(32, 16, 3, 3, 3, 3, generator=generator) * 0.1).to(dtype).cuda()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        results = []
        for _ in range(2):
            xi = x.clone().requires_grad_()
            wi = w.clone().requires_grad_()
            out = conv_nd(xi, wi, padding=1)
            results.append((out, *torch.autograd.grad(out.float().square().sum(), (xi, wi))))
    stream.synchronize()
    for first, second in zip(*results, strict=True):
        assert torch.equal(first, second)
    expected = oracle.forward(x.cpu(), w.cpu(), None, (1,) * 4, (1,) * 4, (1,) * 4, 1)
    assert_matches(results[0][0], expected, dtype, "side-stream y")


def test_empty_batch():
    """Reference tests/test_convnd.py:191-201."""
    layer = torch_convnd.Conv4d(2, 4, 2, device="cuda")
    x = torch.empty(0, 2, 3, 3, 3, 3, device="cuda", requires_grad=True)
    y = layer(x)
    assert y.shape == (0, 4, 2, 2, 2, 2)
    y.sum().backward()
    assert x.grad.shape == x.shape
    assert torch.count_nonzero(layer.weight.grad) == 0
    assert torch.count_nonzero(layer.bias.grad) == 0


def test_autocast_casts_to_bf16():
    generator = torch.Generator().manual_seed(3)
    x = torch.randn(2, 16, 5, 5, 5, 5, generator=generator)
    w = torch.randn(32, 16, 3, 3, 3, 3, generator=generator) * 0.1
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = conv_nd(x.cuda(), w.cuda(), padding=1)
    assert y.dtype == torch.bfloat16
    expected = oracle.forward(x.bfloat16(), w.bfloat16(), None, (1,) * 4, (1,) * 4, (1,) * 4, 1)
    assert_matches(y, expected, torch.bfloat16, "autocast y")


def test_opcheck_on_cuda():
    x = torch.randn(1, 2, 3, 3, 3, 3, device="cuda", requires_grad=True)
    w = torch.randn(4, 2, 2, 2, 2, 2, device="cuda", requires_grad=True)
    b = torch.randn(4, device="cuda", requires_grad=True)
    results = torch.library.opcheck(torch.ops.torch_convnd.conv_nd.default,
                                    (x, w, b, [1] * 4, [0] * 4, [1] * 4, 1, 65536))
    assert all(value == "SUCCESS" for value in results.values())


def test_module_trains_and_round_trips():
    torch.manual_seed(901)
    layer = torch_convnd.Conv4d(16, 32, 3, padding=1, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(2, 16, 4, 4, 4, 4, device="cuda", dtype=torch.bfloat16)
    optimizer = torch.optim.SGD(layer.parameters(), lr=0.01)
    before = layer.weight.detach().clone()
    layer(x).float().square().mean().backward()
    optimizer.step()
    assert not torch.equal(layer.weight, before)
    restored = torch_convnd.ConvNd(16, 32, 3, dimensions=4, padding=1, device="cuda",
                                   dtype=torch.bfloat16)
    restored.load_state_dict(layer.state_dict())
    torch.testing.assert_close(restored(x), layer(x))


def test_fp32_precision_modes():
    generator = torch.Generator().manual_seed(11)
    x = torch.randn(1, 8, 4, 4, 4, 4, 4, 4, generator=generator)
    w = torch.randn(16, 8, 3, 3, 3, 3, 3, 3, generator=generator) * (1 / 5832**0.5)
    expected = oracle.forward(x, w, None, (1,) * 6, (1,) * 6, (1,) * 6, 1)
    errors, rel = {}, {}
    try:
        for mode in ("3xtf32", "tf32", "ieee"):
            torch_convnd.set_fp32_precision(mode)
            y = conv_nd(x.cuda(), w.cuda(), padding=1).double().cpu()
            errors[mode] = float((y - expected).abs().max())
            rel[mode] = float((y - expected).norm() / expected.norm())
    finally:
        torch_convnd.set_fp32_precision("3xtf32")
    # BASELINE's float32 bar is rtol 1e-3 / atol 1e-4 against float64; 3xTF32 lands two
    # orders of magnitude inside it, one TF32 product per term does not.
    assert rel["3xtf32"] < 2e-5 and errors["3xtf32"] < 1e-3
    assert rel["ieee"] < 1e-6
    assert 1e-5 < rel["tf32"] < 2e-3


def test_native_kernels_are_launched():
    torch_convnd.launch_count(reset=True)
    x = torch.randn(2, 32, 4, 4, 4, 8, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(64, 32, 3, 3, 3, 3, device="cuda", dtype=torch.bfloat16)
    conv_nd(x, w, padding=1)
    assert torch_convnd.launch_count() >= 3  # pack x, pack w, tcgen05 pass


def test_bounded_wait_reports_timeout_and_context_survives():
    """A producer that never issues a load makes the MMA thread's bounded wait expire:
    the kernel returns, the host reads CND_ERR_TIMEOUT, and the context keeps working."""
    library = _native.core()
    status = library.cnd_debug_stall_test(50, None)
    assert status == -5, library.cnd_last_error()
    assert b"bounded wait expired" in library.cnd_last_error()
    x = torch.randn(1, 16, 4, 4, 4, 8, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(16, 16, 1, 1, 1, 1, device="cuda", dtype=torch.bfloat16)
    y = conv_nd(x, w)
    expected = oracle.forward(x.cpu(), w.cpu(), None, (1,) * 4, (0,) * 4, (1,) * 4, 1)
    assert_matches(y, expected, torch.bfloat16, "after-timeout y")
    torch_convnd.device_status()
