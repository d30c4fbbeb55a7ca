"""Convolution with a fused GELU (an extension of the reference's API, used by the c5
training step): the forward epilogue applies bias and GELU to the fp32 accumulators and
also stores the pre-activation; the backward multiplies the incoming gradient by the GELU
derivative while packing it. The float64 reference is the oracle's convolution composed
with an exact GELU and its derivative."""

from __future__ import annotations

import math

import pytest
import torch

import torch_convnd
from oracle import convnd_oracle as oracle
from tolerances import assert_conv_matches, assert_matches, conv_magnitudes
from torch_convnd import ConvNd, channels_last, conv_nd, is_channels_last


def _gelu(v):
    return 0.5 * v * (1.0 + torch.erf(v / math.sqrt(2.0)))


def _gelu_grad(v):
    return 0.5 * (1.0 + torch.erf(v / math.sqrt(2.0))) + v * torch.exp(-0.5 * v * v) / math.sqrt(
        2.0 * math.pi)


def test_fused_activation_schemas_and_fake_shapes():
    forward = str(torch.ops.torch_convnd.conv_nd_act.default._schema)
    assert forward.endswith("int workspace_bytes, str activation) -> (Tensor, Tensor)")
    x = channels_last(torch.empty(2, 16, 4, 5, 6, 7)).to("meta")
    w = torch.empty(8, 16, 3, 3, 3, 3, device="meta")
    y, pre = torch.ops.torch_convnd.conv_nd_act(x, w, None, [1] * 4, [1] * 4, [1] * 4, 1,
                                                1 << 20, "gelu")
    assert y.shape == pre.shape == (2, 8, 4, 5, 6, 7)
    assert is_channels_last(y) and is_channels_last(pre)
    with pytest.raises(ValueError, match="activation"):
        ConvNd(2, 2, 1, dimensions=4, activation="relu")
    with pytest.raises(ValueError, match="activation"):
        conv_nd(torch.randn(1, 2, 2, 2, 2, 2), torch.randn(2, 2, 1, 1, 1, 1), activation="tanh")
    with pytest.raises(NotImplementedError, match="TorchScript"):
        torch.jit.script(ConvNd(2, 2, 1, dimensions=4, activation="gelu"))


def test_backward_runs_the_fused_operator_when_the_pre_activation_is_unused():
    """Autograd must not hand the unused pre-activation output a materialised zero
    gradient: that would route every backward through eager GELU-backward and add ops."""
    from torch.utils._python_dispatch import TorchDispatchMode

    class OpLog(TorchDispatchMode):
        def __init__(self):
            super().__init__()
            self.ops = []

        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            self.ops.append(str(func))
            return func(*args, **(kwargs or {}))

    x = channels_last(torch.empty(2, 16, 4, 5, 6, 7)).to("meta").requires_grad_()
    w = torch.empty(8, 16, 3, 3, 3, 3, device="meta", requires_grad=True)
    b = torch.empty(8, device="meta", requires_grad=True)
    geometry = ([1] * 4, [1] * 4, [1] * 4, 1, 1 << 20)
    y, _ = torch.ops.torch_convnd.conv_nd_act(x, w, b, *geometry, "gelu")
    with OpLog() as log:
        y.sum().backward()
    convs = [op for op in log.ops if "torch_convnd" in op or "gelu" in op]
    assert convs == ["torch_convnd.conv_nd_act_backward.default"]
    assert not any("zeros" in op or "fill" in op for op in log.ops)
    # a gradient that does reach the pre-activation takes the eager sum instead
    y, pre = torch.ops.torch_convnd.conv_nd_act(x, w, b, *geometry, "gelu")
    with OpLog() as log:
        (y.sum() + pre.sum()).backward()
    assert "torch_convnd.conv_nd_backward.default" in log.ops
    assert "aten.gelu_backward.default" in log.ops


CASES = [
    # dtype, layout, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups
    (torch.bfloat16, "first", 2, 32, 32, (6, 5, 7, 8), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 1),
    (torch.bfloat16, "last", 2, 32, 32, (6, 5, 7, 8), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 1),
    (torch.bfloat16, "last", 2, 16, 32, (9, 8, 8, 10), (3,) * 4, (2,) * 4, (1,) * 4, (1,) * 4, 1),
    (torch.bfloat16, "last", 2, 32, 32, (9, 10, 4, 6), (3, 3, 1, 1), (1,) * 4, (2, 2, 0, 0),
     (2, 2, 1, 1), 4),
    (torch.float16, "first", 1, 16, 16, (4, 5, 4, 5, 4), (3,) * 5, (1,) * 5, (1,) * 5, (1,) * 5, 1),
    (torch.float32, "first", 1, 8, 16, (4, 5, 4, 4, 5), (3,) * 5, (1,) * 5, (1,) * 5, (1,) * 5, 1),
    (torch.float64, "last", 1, 4, 6, (3, 4, 5, 3), (3,) * 4, (1,) * 4, (1,) * 4, (1,) * 4, 2),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES,
                         ids=lambda c: f"{str(c[0])[6:]}_{c[1]}_{c[3]}x{c[4]}_s{c[7][0]}_g{c[10]}")
def test_fused_gelu_matches_oracle(case):
    dtype, layout, batch, cin, cout, spatial, kernel, stride, padding, dilation, groups = case
    generator = torch.Generator().manual_seed(23)
    x = torch.randn((batch, cin, *spatial), generator=generator).to(dtype)
    w = (torch.randn((cout, cin // groups, *kernel), generator=generator) * 0.1).to(dtype)
    b = torch.randn(cout, generator=generator).to(dtype)
    z = oracle.forward(x, w, b, stride, padding, dilation, groups)
    dy = torch.randn(z.shape, generator=generator).to(dtype)
    dz = dy.double() * _gelu_grad(z)
    dx_ref, dw_ref, db_ref = oracle.backward(dz, x, w, stride, padding, dilation, groups)
    expected = {"y": _gelu(z), "dx": dx_ref, "dw": dw_ref, "db": db_ref}

    put = (lambda t: channels_last(t.cuda())) if layout == "last" else (lambda t: t.cuda())
    xc = put(x).requires_grad_()
    wc = w.cuda().requires_grad_()
    bc = b.cuda().requires_grad_()
    y, pre = torch.ops.torch_convnd.conv_nd_act(xc, wc, bc, list(stride), list(padding),
                                                list(dilation), groups, 1 << 26, "gelu")
    dx, dw, db = torch.autograd.grad(y, (xc, wc, bc), put(dy))
    torch.cuda.synchronize()
    torch_convnd.device_status()
    if layout == "last":
        assert is_channels_last(y) and is_channels_last(pre) and is_channels_last(dx)
    magnitudes = None
    if dtype == torch.float32:
        magnitudes = conv_magnitudes(x, w, dz.to(dtype), stride, padding, dilation, groups)
    assert_matches(pre, z, dtype, "pre-activation")
    assert_conv_matches({"y": y, "dx": dx, "dw": dw, "db": db}, expected, dtype, "fused gelu",
                        magnitudes)


@pytest.mark.gpu
def test_fused_gelu_module_trains_like_the_separate_layers():
    """A ConvNd with activation='gelu' gives the parameter gradients of ConvNd then GELU."""
    torch.manual_seed(9)
    fused = ConvNd(16, 32, 3, stride=2, padding=1, dimensions=4, device="cuda",
                   dtype=torch.bfloat16, activation="gelu")
    plain = ConvNd(16, 32, 3, stride=2, padding=1, dimensions=4, device="cuda",
                   dtype=torch.bfloat16)
    plain.load_state_dict(fused.state_dict())
    x = channels_last(torch.randn(2, 16, 12, 10, 8, 8, device="cuda", dtype=torch.bfloat16))
    target = torch.randn(2, 32, 6, 5, 4, 4, device="cuda", dtype=torch.bfloat16)
    torch.nn.functional.mse_loss(fused(x), target).backward()
    torch.nn.functional.mse_loss(torch.nn.functional.gelu(plain(x)), target).backward()
    for name, p in fused.named_parameters():
        q = dict(plain.named_parameters())[name]
        torch.testing.assert_close(p.grad, q.grad, rtol=2e-2,
                                   atol=1e-2 * float(q.grad.abs().max()), msg=name)
