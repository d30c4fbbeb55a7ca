"""Schema definitions of the torch_convnd operators.

The two schemas are the reference's operator contract, character for character
(``src/torch_convnd/_operators.py:47-56``), because they are the drop-in boundary: code
and compiled graphs that call ``torch.ops.torch_convnd.conv_nd`` keep working. The CUDA,
AutocastCUDA and CPU kernels come from the native shim (``_lib/_C.so``); until it is
loaded, a CompositeExplicitAutograd kernel loads it on the first real call.
"""

from __future__ import annotations

import threading

import torch

_LIBRARY = None
_LOCK = threading.Lock()

CONV_ND_SCHEMA = (
    "conv_nd(Tensor input, Tensor weight, Tensor? bias, int[] stride, int[] padding, "
    "int[] dilation, int groups, int workspace_bytes) -> Tensor"
)
CONV_ND_BACKWARD_SCHEMA = (
    "conv_nd_backward(Tensor grad_output, Tensor input, Tensor weight, int[] stride, "
    "int[] padding, int[] dilation, int groups, int workspace_bytes, "
    "bool[3] output_mask) -> (Tensor?, Tensor?, Tensor?)"
)


def _first_call_forward(input, weight, bias, stride, padding, dilation, groups, workspace_bytes):
    from ._native import load_native

    load_native()
    return torch.ops.torch_convnd.conv_nd.default(
        input, weight, bias, stride, padding, dilation, groups, workspace_bytes
    )


def _first_call_backward(
    grad_output, input, weight, stride, padding, dilation, groups, workspace_bytes, output_mask
):
    from ._native import load_native

    load_native()
    return torch.ops.torch_convnd.conv_nd_backward.default(
        grad_output, input, weight, stride, padding, dilation, groups, workspace_bytes, output_mask
    )


def ensure_native_definitions() -> None:
    """Define the schemas, fake kernels and autograd formulas once per process."""
    global _LIBRARY
    with _LOCK:
        if _LIBRARY is not None:
            return
        library = torch.library.Library("torch_convnd", "DEF")
        library.define(CONV_ND_SCHEMA)
        library.define(CONV_ND_BACKWARD_SCHEMA)
        library.impl("conv_nd", _first_call_forward, "CompositeExplicitAutograd")
        library.impl("conv_nd_backward", _first_call_backward, "CompositeExplicitAutograd")
        from ._autograd import register_training

        register_training()
        _LIBRARY = library
