"""ONNX export of models built on the torch_convnd operators, as standard ONNX Conv nodes.

ONNX's Conv is N-dimensional, so conv_nd and compatible_conv_nd translate one to one:
strides, symmetric pads (begin and end per axis), dilations and group. Like the
reference's exporter (onnx.py:143-184) this needs the optional ``onnx`` package; the
TorchScript-based exporter (``dynamo=False``) uses registered symbolic functions, the
Dynamo exporter (``dynamo=True``) a translation table built with ``onnxscript``.
Running the exported graph for a given rank and dtype depends on the ONNX runtime.
"""

from __future__ import annotations

import functools

import torch


def _conv_symbolic(graph, input, weight, bias, stride, padding, dilation, groups,
                   workspace_bytes, backend=None):
    from torch.onnx import symbolic_helper

    operands = [input, weight]
    if not symbolic_helper._is_none(bias):
        operands.append(bias)
    return graph.op("Conv", *operands, strides_i=stride, pads_i=[*padding, *padding],
                    dilations_i=dilation, group_i=groups)


@functools.cache
def _register_symbolics(opset_version: int) -> None:
    from torch.onnx import register_custom_op_symbolic, symbolic_helper

    native = symbolic_helper.parse_args("v", "v", "v", "is", "is", "is", "i", "i")(
        _conv_symbolic)
    compatible = symbolic_helper.parse_args("v", "v", "v", "is", "is", "is", "i", "i", "s")(
        _conv_symbolic)
    register_custom_op_symbolic("torch_convnd::conv_nd", native, opset_version)
    register_custom_op_symbolic("torch_convnd::compatible_conv_nd", compatible, opset_version)


def _translation_table():
    from onnxscript import opset18 as op

    def conv(input, weight, bias, stride, padding, dilation, groups, workspace_bytes,
             backend=None):
        attributes = {"strides": stride, "pads": [*padding, *padding], "dilations": dilation,
                      "group": groups}
        if bias is None:
            return op.Conv(input, weight, **attributes)
        return op.Conv(input, weight, bias, **attributes)

    return {torch.ops.torch_convnd.conv_nd.default: conv,
            torch.ops.torch_convnd.compatible_conv_nd.default: conv}


def export_onnx(model, args, path=None, *, opset_version: int = 18, dynamo: bool = False,
                **kwargs):
    """Export `model` with torch.onnx.export, its N-D convolutions as ONNX Conv nodes.

    Other keyword arguments (``input_names``, ``dynamic_axes`` ...) go to
    ``torch.onnx.export``. bfloat16 Conv needs opset 22 in ONNX; complex tensors are
    outside the Conv schema.
    """
    try:
        import onnx  # noqa: F401
    except ImportError as error:
        raise ImportError("ONNX export needs the 'onnx' package") from error
    tensors = (args,) if isinstance(args, torch.Tensor) else tuple(args)
    if isinstance(model, torch.nn.Module):
        tensors = (*tensors, *model.parameters())
    if any(isinstance(t, torch.Tensor) and t.is_complex() for t in tensors):
        raise ValueError("ONNX Conv accepts real tensors only")
    if opset_version < 22 and any(
        isinstance(t, torch.Tensor) and t.dtype == torch.bfloat16 for t in tensors
    ):
        raise ValueError("bfloat16 ONNX Conv needs opset 22 or newer")
    if dynamo:
        try:
            import onnxscript  # noqa: F401
        except ImportError as error:
            raise ImportError("the Dynamo ONNX exporter needs the 'onnxscript' package") from error
        table = _translation_table()
        table.update(kwargs.pop("custom_translation_table", {}))
        kwargs["custom_translation_table"] = table
    else:
        _register_symbolics(opset_version)
    return torch.onnx.export(model, args, path, opset_version=opset_version, dynamo=dynamo,
                             **kwargs)
