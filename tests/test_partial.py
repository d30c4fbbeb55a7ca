"""Partial convolution (NVIDIA's partialconv, the reference's partial_conv_nd,
conv_nd(padding_mode="partial") and PartialConvNd): the output rescales each window's
valid samples by window size over valid count, and the update mask marks windows with a
valid sample. The float64 restatement below builds that formula on the oracle's
convolution (data and counting convolutions alike)."""

from __future__ import annotations

import itertools
import math

import pytest
import torch

from oracle import convnd_oracle as oracle
from tolerances import assert_matches
from torch_convnd import PartialConvNd, PartialConvOutput, conv_nd, partial_conv_nd
from torch_convnd._partial import _axis_counts


def test_axis_counts_match_brute_force_tap_counts():
    for size, kernel, stride, dilation, left, right in itertools.product(
            (1, 4, 7), (1, 2, 3), (1, 2), (1, 2, 3), (0, 1, 3), (0, 2)):
        windows = (size + left + right - dilation * (kernel - 1) - 1) // stride + 1
        if windows <= 0:
            continue
        expected = [sum(0 <= w * stride - left + t * dilation < size for t in range(kernel))
                    for w in range(windows)]
        got = _axis_counts(size, kernel, stride, dilation, left, right, torch.float64, "cpu")
        assert got.tolist() == expected, (size, kernel, stride, dilation, left, right)


def test_shapes_and_contract_errors_on_meta():
    x = torch.empty(2, 4, 5, 6, 7, 8, device="meta")
    w = torch.empty(8, 4, 3, 3, 3, 3, device="meta")
    b = torch.empty(8, device="meta")
    out, update = partial_conv_nd(x, w, b, padding=1, mask=torch.empty(2, 1, 5, 6, 7, 8,
                                                                        device="meta"))
    assert out.shape == (2, 8, 5, 6, 7, 8) and update.shape == (2, 1, 5, 6, 7, 8)
    grouped = partial_conv_nd(x, torch.empty(8, 2, 3, 3, 3, 3, device="meta"), b, padding=1,
                              groups=2, mask=torch.empty(1, 4, 5, 6, 7, 8, device="meta"),
                              multi_channel=True)
    assert isinstance(grouped, PartialConvOutput) and grouped.mask.shape == (2, 8, 5, 6, 7, 8)
    assert conv_nd(x, w, b, padding=1, padding_mode="partial").shape == (2, 8, 5, 6, 7, 8)
    assert partial_conv_nd(x[0], w, b, padding=1).output.shape == (8, 5, 6, 7, 8)
    with pytest.raises(ValueError, match="already rescales"):
        partial_conv_nd(x, w, padding_mode="partial")
    with pytest.raises(ValueError, match="dimensions"):
        partial_conv_nd(x, w, mask=torch.empty(2, 1, 5, 6, 7, device="meta"))
    with pytest.raises(ValueError, match="1 channel"):
        partial_conv_nd(x, w, mask=torch.empty(2, 4, 5, 6, 7, 8, device="meta"))
    with pytest.raises(ValueError, match="batch"):
        partial_conv_nd(x, w, mask=torch.empty(3, 1, 5, 6, 7, 8, device="meta"))
    with pytest.raises(ValueError, match="broadcast"):
        partial_conv_nd(x, w, mask=torch.empty(2, 1, 5, 6, 7, 3, device="meta"))
    with pytest.raises(TypeError, match="bool"):
        partial_conv_nd(x, w, multi_channel=1)
    with pytest.raises(ValueError, match="already rescales"):
        PartialConvNd(4, 8, 3, dimensions=4, padding_mode="partial")
    with pytest.raises(NotImplementedError, match="TorchScript"):
        torch.jit.script(PartialConvNd(4, 8, 3, dimensions=4))


def _reference(x, w, b, mask, stride, padding, dilation, groups, multi_channel):
    """float64 partial convolution on the oracle's convolution."""
    x, w = x.double(), w.double()
    rank = w.ndim - 2
    channels, per_group = x.shape[1], x.shape[1] // groups
    if mask is None:
        mask = torch.ones((1, 1, *x.shape[2:]), dtype=torch.float64)
    mask = mask.double()
    width = channels if multi_channel else 1
    valid = mask.expand(mask.shape[0], width, *x.shape[2:])
    if multi_channel:
        valid = valid.reshape(mask.shape[0], groups, per_group, *x.shape[2:]).sum(2)
    window = math.prod(w.shape[2:]) * (per_group if multi_channel else 1)
    ones = torch.ones((valid.shape[1], 1, *w.shape[2:]), dtype=torch.float64)
    counts = oracle.forward(valid.contiguous(), ones, None, stride, padding, dilation,
                            valid.shape[1])
    data = oracle.forward(x * mask, w, None, stride, padding, dilation, groups)
    update = counts.clamp(0, 1)
    ratio = update * window / counts.clamp_min(1e-300)
    if ratio.shape[1] > 1:
        ratio = ratio.repeat_interleave(w.shape[0] // groups, 1)
        update = update.repeat_interleave(w.shape[0] // groups, 1)
    out = data * ratio
    if b is not None:
        out = (out + b.double().reshape((1, -1) + (1,) * rank)) * update
    return out, update


CASES = [
    # dtype, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups, mask, multi
    (torch.float32, 2, 8, 16, (5, 6, 4, 5), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 1, "holes",
     False),
    (torch.bfloat16, 2, 16, 32, (6, 5, 7, 6), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 1,
     "holes", False),
    # padding 3 around 3-tap kernels: corner windows lie wholly in the padding (update 0)
    (torch.float32, 2, 8, 16, (5, 6, 4, 5), (3,) * 4, (1,) * 4, (3, 1, 2, 3), (1,) * 4, 1, None,
     False),
    (torch.bfloat16, 1, 16, 16, (6, 7, 5), (3, 3, 3), (2, 1, 1), (1, 2, 1), (1, 2, 1), 2,
     "holes", True),
    (torch.float32, 2, 8, 8, (4, 5, 6, 4, 5), (3, 1, 3, 2, 3), (1,) * 5, (1, 0, 1, 1, 1),
     (1,) * 5, 2, "fraction", True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{str(c[0])[6:]}_r{len(c[4])}_{c[10]}_"
                         f"{'multi' if c[11] else 'single'}")
def test_partial_convolution_matches_the_float64_formula(case):
    dtype, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups, kind, multi = case
    generator = torch.Generator().manual_seed(41)
    x = torch.randn((batch, cin, *spatial), generator=generator).to(dtype)
    w = (torch.randn((cout, cin // groups, *kernel), generator=generator) * 0.1).to(dtype)
    b = torch.randn(cout, generator=generator).to(dtype)
    mask = None
    if kind is not None:
        channels = cin if multi else 1
        mask = (torch.rand((batch, channels, *spatial), generator=generator) > 0.35).float()
        if kind == "fraction":
            mask = mask * torch.rand(mask.shape, generator=generator)
    expected, expected_update = _reference(x, w, b, mask, stride, padding, dilation, groups,
                                           multi)
    out, update = partial_conv_nd(x.cuda(), w.cuda(), b.cuda(), stride, padding, dilation,
                                  groups, mask=None if mask is None else mask.cuda(),
                                  multi_channel=multi)
    assert out.dtype == dtype and out.shape == expected.shape
    assert_matches(out, expected, dtype, "partial output")
    torch.testing.assert_close(update.double().cpu(), expected_update.expand(update.shape),
                               rtol=0, atol=0)


@pytest.mark.gpu
def test_padding_mode_partial_and_the_module_train():
    torch.manual_seed(12)
    x = torch.randn(2, 8, 6, 5, 6, 5, device="cuda", requires_grad=True)
    w = torch.randn(16, 8, 3, 3, 3, 3, device="cuda") * 0.1
    b = torch.randn(16, device="cuda")
    direct = conv_nd(x, w, b, padding=1, padding_mode="partial")
    output, _ = partial_conv_nd(x, w, b, padding=1)
    torch.testing.assert_close(direct, output, rtol=0, atol=0)
    layer = PartialConvNd(8, 16, 3, padding=1, dimensions=4, device="cuda", return_mask=True)
    mask = (torch.rand(2, 1, 6, 5, 6, 5, device="cuda") > 0.3).float()
    result = layer(x, mask_in=mask)
    result.output.square().mean().backward()
    assert x.grad is not None and layer.weight.grad is not None and layer.bias.grad is not None
    assert torch.equal(result.mask, result.mask.clamp(0, 1))
    assert layer(x, mask, return_mask=False).shape == result.output.shape
