"""Channels-last activations: read in place, propagated to outputs and input gradients.

A channels-last input ([N, C, d...] stored as [N, d..., C]) is what the tensor-core passes
use as their packed operand when its rows have the kernels' width, so the operators take
it without a layout pass and return channels-last outputs; every other case (other
dtypes, padded channel counts, grouped layers, the generic kernels) reads and writes the
same layout through its own index arithmetic. The results must equal the channels-first
path's, and the layout must survive a whole network (c5's three layers with GELU).
"""

from __future__ import annotations

import pytest
import torch

import torch_convnd
from oracle import convnd_oracle as oracle
from tolerances import assert_conv_matches, conv_magnitudes
from torch_convnd import channels_last, conv_nd, is_channels_last


def test_channels_last_helper_and_fake_strides():
    x = torch.randn(2, 16, 3, 4, 5, 6)
    cl = channels_last(x)
    assert is_channels_last(cl) and torch.equal(cl, x)
    assert cl.permute(0, 2, 3, 4, 5, 1).is_contiguous()
    assert not is_channels_last(x) and channels_last(cl) is cl
    meta = cl.to("meta")
    w = torch.empty(8, 16, 3, 3, 3, 3, device="meta")
    y = torch.ops.torch_convnd.conv_nd(meta, w, None, [1] * 4, [1] * 4, [1] * 4, 1, 1 << 20)
    assert is_channels_last(y) and y.shape == (2, 8, 3, 4, 5, 6)
    dx, dw, _ = torch.ops.torch_convnd.conv_nd_backward(
        y, meta, w, [1] * 4, [1] * 4, [1] * 4, 1, 1 << 20, [True, True, False])
    assert is_channels_last(dx) and dw.is_contiguous()
    y = torch.ops.torch_convnd.conv_nd(x.to("meta"), w, None, [1] * 4, [1] * 4, [1] * 4, 1,
                                       1 << 20)
    assert y.is_contiguous()


CASES = [
    # dtype, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups
    (torch.bfloat16, 2, 32, 64, (6, 5, 7, 8), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 1),
    (torch.bfloat16, 2, 16, 32, (9, 8, 8, 10), (3,) * 4, (2,) * 4, (1,) * 4, (1,) * 4, 1),
    (torch.bfloat16, 2, 32, 32, (9, 10, 4, 6), (3, 3, 1, 1), (1,) * 4, (2, 2, 0, 0),
     (2, 2, 1, 1), 4),
    (torch.bfloat16, 2, 32, 8, (5, 6, 4, 4), (1,) * 4, (1,) * 4, (0,) * 4, (1,) * 4, 1),
    (torch.bfloat16, 2, 24, 40, (5, 4, 6, 5), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 1),
    (torch.float16, 1, 16, 16, (4, 5, 4, 5, 4), (3,) * 5, (1,) * 5, (1,) * 5, (1,) * 5, 1),
    (torch.float32, 1, 8, 16, (4, 5, 4, 4, 5), (3,) * 5, (1,) * 5, (1,) * 5, (1,) * 5, 1),
    (torch.float64, 1, 4, 6, (3, 4, 5, 3), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 2),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{str(c[0])[6:]}_{c[2]}x{c[3]}_s{c[6][0]}")
def test_channels_last_matches_channels_first(case):
    dtype, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups = case
    generator = torch.Generator().manual_seed(17)
    x = torch.randn((batch, cin, *spatial), generator=generator).to(dtype)
    w = (torch.randn((cout, cin // groups, *kernel), generator=generator) * 0.1).to(dtype)
    b = torch.randn(cout, generator=generator).to(dtype)
    y_ref = oracle.forward(x, w, b, stride, padding, dilation, groups)
    dy = torch.randn(y_ref.shape, generator=generator).to(dtype)
    expected = dict(zip(("dx", "dw", "db"),
                        oracle.backward(dy, x, w, stride, padding, dilation, groups)))
    expected["y"] = y_ref
    magnitudes = None
    if dtype == torch.float32:
        magnitudes = conv_magnitudes(x, w, dy, stride, padding, dilation, groups)

    def run(x_dev, dy_dev):
        xr = x_dev.requires_grad_()
        wr = w.cuda().requires_grad_()
        br = b.cuda().requires_grad_()
        y = conv_nd(xr, wr, br, stride, padding, dilation, groups)
        dx, dw, db = torch.autograd.grad(y, (xr, wr, br), dy_dev)
        return {"y": y.detach(), "dx": dx, "dw": dw, "db": db}

    first = run(x.cuda(), dy.cuda())
    last = run(channels_last(x.cuda()), channels_last(dy.cuda()))
    torch.cuda.synchronize()
    torch_convnd.device_status()
    assert is_channels_last(last["y"]) and is_channels_last(last["dx"])
    assert first["y"].is_contiguous() and first["dx"].is_contiguous()
    assert_conv_matches(last, expected, dtype, "channels-last", magnitudes)
    # same kernels and operands in both layouts: bitwise equal outputs and gradients
    for key in ("y", "dx", "dw"):
        assert torch.equal(last[key], first[key]), key


@pytest.mark.gpu
def test_c5_network_keeps_channels_last_end_to_end():
    """Reduced c5 network: every activation and input gradient stays channels-last, and
    parameter gradients equal the channels-first run's."""
    from torch_convnd import configs

    torch.manual_seed(4)
    layers = [layer.with_batch(2) for layer in configs.C5_LAYERS]
    params = []
    for layer in layers:
        w = (torch.randn(layer.out_channels, layer.in_channels // layer.groups,
                         *layer.kernel) * 0.1).bfloat16().cuda()
        params.append((w, torch.randn(layer.out_channels).bfloat16().cuda()))
    x = torch.randn(2, 16, 16, 16, 8, 8).bfloat16().cuda()
    target = torch.randn(2, 8, 8, 8, 4, 4).bfloat16().cuda()

    def step(inp):
        tensors = [(w.clone().requires_grad_(), b.clone().requires_grad_()) for w, b in params]
        h, seen = inp, []
        for index, (layer, (w, b)) in enumerate(zip(layers, tensors)):
            h = conv_nd(h, w, b, layer.stride, layer.padding, layer.dilation, layer.groups)
            seen.append(is_channels_last(h))
            if index + 1 < len(layers):
                h = torch.nn.functional.gelu(h)
                seen.append(is_channels_last(h))
        torch.nn.functional.mse_loss(h, target).backward()
        return seen, [t.grad for pair in tensors for t in pair]

    seen_last, grads_last = step(channels_last(x))
    seen_first, grads_first = step(x)
    assert all(seen_last) and not any(seen_first)
    for got, want in zip(grads_last, grads_first):
        torch.testing.assert_close(got, want, rtol=2e-2, atol=1e-2 * float(want.abs().max()))
