"""The BASELINE configurations at their full sizes, on the GPU, checked whole.

Every element of y, dx, dW and db of c2, c3, c4 and c5's three layers is compared with
the oracle's float64 tap-by-tap restatement (tap_reference / tap_dgrad / tap_wgrad, the
reference tests' formula and its adjoints, pinned to the reference's own goldens in
tests/test_oracle.py), evaluated in float64 on the same GPU as a checker. The float32
case (c4) uses BASELINE's literal bar, rtol 1e-3 / atol 1e-4, plus each element's fp32
summation bound (tests/tolerances.py); the report line printed per tensor gives the
worst element against the literal bar alone as well. These shapes run the same kernel
plans as bench.py (folded passes, the halo weight-gradient kernel with its split plans,
staged TMA-store epilogues), which the small parity cases do not reach.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import torch_convnd
from oracle import convnd_oracle as oracle
from tolerances import assert_matches, conv_magnitudes, relative_l2, violations
from torch_convnd import _native, configs
from torch_convnd.functional import conv_nd

CASES = {
    "c2": configs.C2,
    "c3": configs.C3,
    "c4": configs.C4,
    "c5l1": configs.C5_LAYERS[0],
    "c5l2": configs.C5_LAYERS[1],
    "c5l3": configs.C5_LAYERS[2],
}


def _plan_summary(cfg):
    library = _native.core()

    class Problem(ctypes.Structure):
        _fields_ = [("rank", ctypes.c_int32), ("dtype", ctypes.c_int32),
                    ("fp32_mode", ctypes.c_int32), ("reserved", ctypes.c_int32)] + [
            (n, ctypes.c_int64) for n in ("batch", "channels", "output_channels", "groups",
                                          "input_volume", "output_volume", "kernel_volume")] + [
            (n, ctypes.c_int64 * 62)
            for n in ("input", "output", "kernel", "stride", "padding", "dilation")]

    arr = lambda v: (ctypes.c_int64 * len(v))(*v)
    code = {torch.bfloat16: 1, torch.float32: 2}[cfg.dtype]
    problem = Problem()
    assert library.cnd_problem_init(
        ctypes.byref(problem), cfg.rank, arr([cfg.batch, cfg.in_channels, *cfg.spatial]),
        arr([cfg.out_channels, cfg.in_channels // cfg.groups, *cfg.kernel]), arr(cfg.stride),
        arr(cfg.padding), arr(cfg.dilation), ctypes.c_int64(cfg.groups), code) == 0
    buffer = ctypes.create_string_buffer(4096)
    library.cnd_plan_summary(ctypes.byref(problem), buffer, 4096)
    return buffer.value.decode()


def test_c2_plan_uses_the_folded_tma_store_path():
    """The c2 forward and dgrad plans are the folded ones with staged TMA stores, so the
    c2 case below checks those kernels at the benchmark's shapes (planning needs no GPU:
    without one the planner assumes the B200's 148 SMs)."""
    summary = _plan_summary(configs.C2)
    for line in summary.splitlines():
        if line.startswith(("forward", "dgrad")):
            assert "fold=1" in line and "tma_store=1" in line, line


def test_six_tile_case_uses_six_tile_super_tiles():
    """The small GPU parity case SIX_TILE_CASE plans 6-tile folded super tiles for its
    forward (as c3's forward does) and the a2 fold for its dgrad (as c3's dgrad does), so
    the GPU test checks those kernels."""
    from types import SimpleNamespace

    from test_gpu_parity import SIX_TILE_CASE

    rank, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups = SIX_TILE_CASE
    cfg = SimpleNamespace(rank=rank, batch=batch, in_channels=cin, out_channels=cout,
                          spatial=spatial, kernel=kernel, stride=stride, padding=padding,
                          dilation=dilation, groups=groups, dtype=torch.bfloat16)
    summary = _plan_summary(cfg)
    for line in summary.splitlines():
        if line.startswith("forward"):
            assert "x6 " in line and "fold=1" in line, line
        if line.startswith("dgrad"):  # 16 channels: the a2 taps fold into N as well
            assert "fold=1" in line and "k2f=3" in line, line


def test_pointwise_axes_are_merged_and_unit_axes_dropped():
    """c5's k = (3,3,1,1) layer plans its forward and dgrad on [16,16,64] (the two
    pointwise axes merged); a problem with extent-1 kernel-1 axes plans without them
    (the reference's without_unit_axes, csrc/convnd.h:32-48)."""
    from types import SimpleNamespace

    summary = _plan_summary(configs.C5_LAYERS[1])
    for line in summary.splitlines():
        if line.startswith(("forward", "dgrad")):
            assert "axes [16,16,64]" in line, line
    unit = SimpleNamespace(rank=5, batch=2, in_channels=16, out_channels=32,
                           spatial=(1, 6, 1, 7, 5), kernel=(1, 3, 1, 3, 1), stride=(1,) * 5,
                           padding=(0, 1, 0, 1, 0), dilation=(1,) * 5, groups=1,
                           dtype=torch.bfloat16)
    assert "forward: axes [6,7,5]" in _plan_summary(unit)


def test_thin_passes_fold_the_a2_taps():
    """Passes over 16 padded output channels (c3's dgrad, c4's forward and dgrad) fold the
    a2 taps into N with the a0 taps (k2f=3), so the full-size cases check that epilogue."""
    for cfg, passes in ((configs.C3, ("dgrad",)), (configs.C4, ("forward", "dgrad"))):
        for line in _plan_summary(cfg).splitlines():
            if line.startswith(passes):
                assert "k2f=3" in line, line


def test_strided_dgrad_runs_as_phase_sub_convolutions():
    """A stride-2 Conv4d (c5's first layer with an input gradient) plans its dgrad as the
    16 residue classes of dx positions, each a stride-1 tcgen05 pass."""
    summary = _plan_summary(configs.C5_LAYERS[0])
    assert "dgrad: 16 phase sub-convolutions" in summary, summary
    assert "generic" not in summary, summary


def test_thin_grouped_layer_runs_dense():
    """c5's grouped layer (4 groups of 8 channels) runs as one dense problem with
    block-diagonal weights; its full-size case below checks that plan."""
    summary = _plan_summary(configs.C5_LAYERS[1])
    assert "groups: 4 run dense" in summary, summary
    assert "groups:" not in _plan_summary(configs.C2)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CASES))
def test_full_size_config_matches_oracle_whole(name):
    cfg = CASES[name]
    inputs = configs.make_inputs(cfg, device="cuda")
    geometry = (cfg.stride, cfg.padding, cfg.dilation, cfg.groups)
    x = inputs.x.clone().requires_grad_(cfg.input_grad)
    w = inputs.weight.clone().requires_grad_()
    b = inputs.bias.clone().requires_grad_()
    y = conv_nd(x, w, b, *geometry, backend="native")
    wanted = [t for t in (x, w, b) if t.requires_grad]
    grads = list(torch.autograd.grad(y, wanted, inputs.grad))
    torch.cuda.synchronize()
    torch_convnd.device_status()
    got = {"y": y.detach(), "dx": grads.pop(0) if cfg.input_grad else None,
           "dw": grads[0], "db": grads[1]}
    del x, w, b, y, grads

    xs, ws, dy = inputs.x, inputs.weight, inputs.grad
    expected = {"y": oracle.tap_reference(xs, ws, inputs.bias, *geometry)}
    if cfg.input_grad:
        expected["dx"] = oracle.tap_dgrad(dy, ws, cfg.spatial, *geometry)
    expected["dw"] = oracle.tap_wgrad(dy, xs, cfg.kernel, *geometry)
    expected["db"] = dy.to(torch.float64).sum(dim=(0, *range(2, 2 + cfg.rank)))
    magnitudes = {}
    if cfg.dtype == torch.float32:
        magnitudes = conv_magnitudes(xs, ws, dy, *geometry, tap=True)
    for key, value in got.items():
        if value is None:
            continue
        literal = violations(value, expected[key], cfg.dtype)
        print(f"{name} {key}: rel-L2 {relative_l2(value, expected[key]):.3e}, "
              f"max |expected| {float(expected[key].abs().max()):.4g}, literal-bar "
              f"violations {literal[0]} of {value.numel()} (worst {literal[1]:.3g}x allowed)")
        magnitude, terms, split = magnitudes.get(key, (None, None, False))
        assert_matches(value, expected[key], cfg.dtype, f"{name} {key}", magnitude, terms,
                       split)
