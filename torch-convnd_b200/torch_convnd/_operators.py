"""Schema definitions of the torch_convnd operators.

The schemas are the reference's operator contract, character for character
(``src/torch_convnd/_operators.py:47-56``; ``compatible_conv_nd``, the entry point of
scripted graphs, ``_dispatch.py:176-180``), because they are the drop-in boundary: code
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


COMPATIBLE_CONV_ND_SCHEMA = (
    "compatible_conv_nd(Tensor input, Tensor weight, Tensor? bias, int[] stride, "
    "int[] padding, int[] dilation, int groups, int workspace_bytes, str backend) -> Tensor"
)


# Convolution with a fused activation (no reference counterpart): (activation(y), y) for
# y = conv + bias, and its backward from the gradient of activation(y) and y.
CONV_ND_ACT_SCHEMA = (
    "conv_nd_act(Tensor input, Tensor weight, Tensor? bias, int[] stride, int[] padding, "
    "int[] dilation, int groups, int workspace_bytes, str activation) -> (Tensor, Tensor)"
)
CONV_ND_ACT_BACKWARD_SCHEMA = (
    "conv_nd_act_backward(Tensor grad_output, Tensor pre_activation, Tensor input, "
    "Tensor weight, int[] stride, int[] padding, int[] dilation, int groups, "
    "int workspace_bytes, str activation, bool[3] output_mask) -> (Tensor?, Tensor?, Tensor?)"
)


def _first_call(name):
    def run(*args):
        from ._native import load_native

        load_native()
        return getattr(torch.ops.torch_convnd, name).default(*args)

    return run


def _compatible_conv_nd(input, weight, bias, stride, padding, dilation, groups, workspace_bytes,
                        backend):
    """The entry point of scripted graphs (reference _dispatch.py:160-181): a composite
    over conv_nd, so autograd, autocast and vmap reach the native operator's own rules.
    `backend` follows conv_nd's policy: 'auto' and 'native' run the B200 kernels and the
    portable 'torch' decomposition is refused."""
    if backend not in ("auto", "native"):
        if backend == "torch":
            raise ValueError(
                "backend='torch' (the reference's portable decomposition) is not part of "
                "the B200 build; use backend='native' or 'auto'")
        raise ValueError(f"Invalid backend {backend!r}; expected 'auto', 'native' or 'torch'")
    return torch.ops.torch_convnd.conv_nd.default(
        input, weight, bias, stride, padding, dilation, groups, workspace_bytes)


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
        library.define(COMPATIBLE_CONV_ND_SCHEMA)
        library.impl("compatible_conv_nd", _compatible_conv_nd, "CompositeImplicitAutograd")
        library.define(CONV_ND_ACT_SCHEMA)
        library.define(CONV_ND_ACT_BACKWARD_SCHEMA)
        library.impl("conv_nd_act", _first_call("conv_nd_act"), "CompositeExplicitAutograd")
        library.impl("conv_nd_act_backward", _first_call("conv_nd_act_backward"),
                     "CompositeExplicitAutograd")
        from ._autograd import register_training

        register_training()
        _LIBRARY = library
