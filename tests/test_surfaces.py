"""Operator surfaces beyond the eager call: vmap, compatible_conv_nd (the entry point of
scripted graphs), TorchScript and ONNX export (the reference's _autograd.py:93-149,
_dispatch.py:160-181, _script.py and onnx.py). CPU tests check shapes on meta tensors and
the contracts; GPU tests compare numbers with the eager native operator."""

from __future__ import annotations

import io

import pytest
import torch

import torch_convnd
from torch_convnd import Conv4d, ConvNd, conv_nd

GEOMETRY = ([1, 1, 1, 1], [1, 1, 1, 1], [1, 1, 1, 1])


def _conv(x, w, b=None, groups=1):
    return torch.ops.torch_convnd.conv_nd(x, w, b, *GEOMETRY, groups, 1 << 20)


def test_compatible_schema_is_the_reference_contract():
    schema = str(torch.ops.torch_convnd.compatible_conv_nd.default._schema)
    assert schema == (
        "torch_convnd::compatible_conv_nd(Tensor input, Tensor weight, Tensor? bias, "
        "int[] stride, int[] padding, int[] dilation, int groups, int workspace_bytes, "
        "str backend) -> Tensor")
    x = torch.empty(2, 3, 5, 5, 5, 5, device="meta")
    w = torch.empty(4, 3, 3, 3, 3, 3, device="meta")
    y = torch.ops.torch_convnd.compatible_conv_nd(x, w, None, *GEOMETRY, 1, 1 << 20, "auto")
    assert y.shape == (2, 4, 5, 5, 5, 5)
    with pytest.raises(ValueError, match="not part of the B200 build"):
        torch.ops.torch_convnd.compatible_conv_nd(x, w, None, *GEOMETRY, 1, 1 << 20, "torch")


@pytest.mark.parametrize("mapped", ["input", "weight", "all", "empty"])
def test_vmap_shapes_on_meta(mapped):
    x = torch.empty(5, 2, 6, 4, 4, 4, 4, device="meta")
    w = torch.empty(5, 8, 3, 3, 3, 3, 3, device="meta")
    b = torch.empty(5, 8, device="meta")
    if mapped == "input":
        y = torch.func.vmap(lambda x: _conv(x, w[0], b[0], groups=2))(x)
    elif mapped == "weight":
        y = torch.func.vmap(lambda w: _conv(x[0], w, None, groups=2))(w)
    elif mapped == "all":
        y = torch.func.vmap(lambda x, w, b: _conv(x, w, b, groups=2))(x, w, b)
    else:
        y = torch.func.vmap(lambda x, w: _conv(x, w, None, groups=2))(x[:0], w[:0])
    assert y.shape == ((0 if mapped == "empty" else 5), 2, 8, 4, 4, 4, 4)


def test_module_scripts_to_the_compatible_operator():
    layer = Conv4d(3, 4, 3, padding="same", padding_mode="reflect", bias=True)
    scripted = torch.jit.script(layer)
    assert "compatible_conv_nd" in scripted.graph.str() or "compatible_conv_nd" in str(
        scripted.inlined_graph)
    assert scripted.weight.data_ptr() == layer.weight.data_ptr()


def test_onnx_export_needs_the_onnx_package():
    """Without the optional onnx package the exporter says what to install (the
    reference's export_onnx does the same, onnx.py:143-150)."""
    try:
        import onnx  # noqa: F401
    except ImportError:
        with pytest.raises(ImportError, match="onnx"):
            torch_convnd.export_onnx(Conv4d(2, 2, 1), (torch.randn(1, 2, 2, 2, 2, 2),), None)
    else:
        pytest.skip("onnx is installed; the GPU test exports a model")


# ------------------------------------------------------------------------------------
# GPU: numbers against the eager operator
# ------------------------------------------------------------------------------------

@pytest.mark.gpu
def test_vmap_matches_a_loop_of_native_calls():
    generator = torch.Generator().manual_seed(3)
    x = torch.randn(3, 2, 16, 5, 4, 6, 5, generator=generator).bfloat16().cuda()
    w = (torch.randn(3, 32, 8, 3, 3, 3, 3, generator=generator) * 0.1).bfloat16().cuda()
    b = torch.randn(3, 32, generator=generator).bfloat16().cuda()
    cases = {
        "input": (torch.func.vmap(lambda x: _conv(x, w[0], b[0], groups=2))(x),
                  [_conv(x[i], w[0], b[0], groups=2) for i in range(3)]),
        "weight": (torch.func.vmap(lambda w, b: _conv(x[0], w, b, groups=2))(w, b),
                   [_conv(x[0], w[i], b[i], groups=2) for i in range(3)]),
        "all": (torch.func.vmap(lambda x, w, b: _conv(x, w, b, groups=2))(x, w, b),
                [_conv(x[i], w[i], b[i], groups=2) for i in range(3)]),
    }
    for name, (batched, loop) in cases.items():
        # the grouped fold runs other tile plans: compare within bf16 rounding of the output
        torch.testing.assert_close(batched, torch.stack(loop), rtol=2e-2, atol=2e-2, msg=name)


@pytest.mark.gpu
def test_scripted_module_matches_eager_forward_and_backward():
    torch.manual_seed(5)
    layer = ConvNd(8, 16, 3, padding=1, dimensions=4, device="cuda")
    scripted = torch.jit.script(layer)
    x = torch.randn(2, 8, 5, 6, 4, 5, device="cuda", requires_grad=True)
    eager = layer(x)
    (gx_eager,) = torch.autograd.grad(eager.square().sum(), x)
    out = scripted(x)
    (gx_script,) = torch.autograd.grad(out.square().sum(), x)
    torch.testing.assert_close(out, eager, rtol=0, atol=0)
    torch.testing.assert_close(gx_script, gx_eager, rtol=0, atol=0)


@pytest.mark.gpu
def test_compatible_operator_runs_native_with_autograd():
    torch.manual_seed(6)
    x = torch.randn(1, 4, 5, 5, 5, 5, device="cuda", requires_grad=True)
    w = torch.randn(8, 4, 3, 3, 3, 3, device="cuda", requires_grad=True)
    y = torch.ops.torch_convnd.compatible_conv_nd(x, w, None, *GEOMETRY, 1, 1 << 20, "native")
    torch.testing.assert_close(y, conv_nd(x, w, padding=1), rtol=0, atol=0)
    gx, gw = torch.autograd.grad(y.sum(), (x, w))
    assert gx.shape == x.shape and gw.shape == w.shape


@pytest.mark.gpu
def test_onnx_export_writes_standard_conv_nodes():
    onnx = pytest.importorskip("onnx")
    torch.manual_seed(7)
    layer = Conv4d(4, 8, 3, stride=(1, 2, 1, 1), padding=1, dilation=(1, 1, 2, 1),
                   device="cuda")
    x = torch.randn(1, 4, 6, 6, 6, 6, device="cuda")
    buffer = io.BytesIO()
    torch_convnd.export_onnx(layer, (x,), buffer, input_names=["x"])
    model = onnx.load_from_string(buffer.getvalue())
    convs = [node for node in model.graph.node if node.op_type == "Conv"]
    assert len(convs) == 1
    attributes = {a.name: list(a.ints) if a.ints else a.i for a in convs[0].attribute}
    assert attributes["strides"] == [1, 2, 1, 1]
    assert attributes["pads"] == [1, 1, 1, 1, 1, 1, 1, 1]
    assert attributes["dilations"] == [1, 1, 2, 1]
    assert attributes["group"] == 1
