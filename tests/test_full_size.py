"""The BASELINE configurations at their full sizes, on the GPU.

The full fp64 oracle would take minutes per configuration on the host, so these checks
use size-independent samples instead: exact float64 values from the oracle's point
samplers at seeded random output points (y), input points (dx) and weight entries (dW),
always including the corner positions where padding matters, plus the whole bias
gradient. The samples are compared under the dtype's tolerance rule. These shapes run
the same kernel plans as bench.py (for c2 the a0-tap fold and the staged TMA-store
epilogue), which the small parity cases do not reach.
"""

from __future__ import annotations

import ctypes
import itertools
import random

import pytest
import torch

import torch_convnd
from oracle import convnd_oracle as oracle
from tolerances import assert_matches
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


def _points(generator, leading, extents, count):
    """`count` random (index, channel, coordinates) points plus the two corners."""
    batch, channels = leading
    points = [(0, 0, tuple(0 for _ in extents)),
              (batch - 1, channels - 1, tuple(e - 1 for e in extents))]
    for _ in range(count):
        points.append((generator.randrange(batch), generator.randrange(channels),
                       tuple(generator.randrange(e) for e in extents)))
    return points


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
    forward and dgrad (as c3's forward does), so the GPU test checks those kernels."""
    from types import SimpleNamespace

    from test_gpu_parity import SIX_TILE_CASE

    rank, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups = SIX_TILE_CASE
    cfg = SimpleNamespace(rank=rank, batch=batch, in_channels=cin, out_channels=cout,
                          spatial=spatial, kernel=kernel, stride=stride, padding=padding,
                          dilation=dilation, groups=groups, dtype=torch.bfloat16)
    summary = _plan_summary(cfg)
    for line in summary.splitlines():
        if line.startswith(("forward", "dgrad")):
            assert "x6 " in line and "fold=1" in line, line


def test_thin_grouped_layer_runs_dense():
    """c5's grouped layer (4 groups of 8 channels) runs as one dense problem with
    block-diagonal weights; its full-size case below checks that plan."""
    summary = _plan_summary(configs.C5_LAYERS[1])
    assert "groups: 4 run dense" in summary, summary
    assert "groups:" not in _plan_summary(configs.C2)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CASES))
def test_full_size_config_matches_sampled_oracle(name):
    cfg = CASES[name]
    inputs = configs.make_inputs(cfg)
    geometry = (cfg.stride, cfg.padding, cfg.dilation, cfg.groups)
    x = inputs.x.cuda().requires_grad_(cfg.input_grad)
    w = inputs.weight.cuda().requires_grad_()
    b = inputs.bias.cuda().requires_grad_()
    y = conv_nd(x, w, b, *geometry, backend="native")
    wanted = [t for t in (x, w, b) if t.requires_grad]
    grads = torch.autograd.grad(y, wanted, inputs.grad.cuda())
    torch.cuda.synchronize()
    torch_convnd.device_status()
    grads = [g.cpu() for g in grads]
    dx = grads.pop(0) if cfg.input_grad else None
    dw, db = grads
    y = y.detach().cpu()
    del x, w, b

    generator = random.Random(hash(name) % (2**31))
    xs, ws, dy = inputs.x, inputs.weight, inputs.grad
    out_points = _points(generator, (cfg.batch, cfg.out_channels), cfg.output, 256)
    expected = oracle.sampled_forward(xs, ws, inputs.bias, *geometry, out_points)
    got = torch.stack([y[n, c][idx] for n, c, idx in out_points])
    assert_matches(got, expected, cfg.dtype, f"{name} y samples")

    if dx is not None:
        in_points = _points(generator, (cfg.batch, cfg.in_channels), cfg.spatial, 256)
        expected = oracle.sampled_dgrad(dy, ws, cfg.spatial, *geometry, in_points)
        got = torch.stack([dx[n, c][idx] for n, c, idx in in_points])
        assert_matches(got, expected, cfg.dtype, f"{name} dx samples")

    taps = list(itertools.product(*(range(k) for k in cfg.kernel)))
    cin_g = cfg.in_channels // cfg.groups
    entries = [(0, 0, taps[0]), (cfg.out_channels - 1, cin_g - 1, taps[-1])]
    for _ in range(48):
        entries.append((generator.randrange(cfg.out_channels), generator.randrange(cin_g),
                        taps[generator.randrange(len(taps))]))
    expected = oracle.sampled_wgrad(dy, xs, cfg.kernel, *geometry, entries)
    got = torch.stack([dw[co, cl][t] for co, cl, t in entries])
    assert_matches(got, expected, cfg.dtype, f"{name} dW samples")

    spatial_dims = tuple(range(2, 2 + cfg.rank))
    expected_db = dy.to(torch.float64).sum(dim=(0, *spatial_dims))
    assert_matches(db, expected_db, cfg.dtype, f"{name} db")
