"""Functional N-dimensional convolution on the B200 native backend.

``conv_nd`` keeps the reference's public signature and argument checks
(``src/torch_convnd/functional.py:65-185``): batched or unbatched inputs, int/sequence
geometry, ``'same'``/``'valid'`` padding, zero/reflect/replicate/circular padding modes,
autocast. Symmetric zero padding reaches the kernels as implicit padding; any other
padding is applied on the device first. Every rank, including 1-3, runs the native
operator; there is no vendor or portable fallback in this build.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor

from ._geometry import DEFAULT_WORKSPACE_BYTES, _tuple, has_rank
from ._padding import apply_padding, padding_pairs

BACKENDS = ("auto", "native", "torch")
_PADDING_MODES = ("zeros", "reflect", "replicate", "circular", "partial")
_CASTABLE = (torch.float16, torch.bfloat16, torch.float32)


def _autocast_enabled(device_type: str) -> bool:
    return device_type in ("cpu", "cuda") and torch.is_autocast_enabled(device_type)


def _check_options(padding_mode: str, workspace_bytes: int, backend: str) -> None:
    if backend not in BACKENDS:
        raise ValueError(f"Invalid backend {backend!r}; expected 'auto', 'native' or 'torch'")
    if backend == "torch":
        raise ValueError(
            "backend='torch' (the reference's portable decomposition) is not part of the "
            "B200 build; use backend='native' or 'auto'"
        )
    if workspace_bytes <= 0:
        raise ValueError("workspace_bytes must be positive")
    if padding_mode not in _PADDING_MODES:
        raise ValueError(f"Invalid padding_mode {padding_mode!r}")


def _check_arguments(input, weight, stride, padding, dilation, groups) -> bool:
    """Geometry, device and dtype checks of a batched input; returns whether autocast
    applies (the reference's _check_arguments, functional.py:144-168)."""
    if min(*stride, *dilation) <= 0 or (not isinstance(padding, str) and min(padding) < 0):
        raise RuntimeError("stride and dilation must be positive; padding must be nonnegative")
    if groups <= 0:
        raise RuntimeError("groups must be positive")
    if (
        input.shape[1] <= 0
        or weight.shape[0] <= 0
        or input.shape[1] % groups
        or weight.shape[0] % groups
        or weight.shape[1] != input.shape[1] // groups
    ):
        raise RuntimeError("input/weight channels must match and be divisible by groups")
    if any(size <= 0 for size in (*input.shape[2:], *weight.shape[2:])):
        raise RuntimeError("spatial and kernel dimensions must be positive")
    if input.device != weight.device:
        raise RuntimeError("input and weight must have the same device and dtype")
    amp = _autocast_enabled(input.device.type)
    if input.dtype != weight.dtype and not (
        amp and input.dtype in _CASTABLE and weight.dtype in _CASTABLE
    ):
        raise RuntimeError("input and weight must have the same device and dtype")
    return amp


def _check_bias(input, weight, bias, amp: bool) -> None:
    if bias is not None and (
        bias.ndim != 1
        or bias.shape[0] != weight.shape[0]
        or bias.device != input.device
        or (
            bias.dtype != input.dtype
            and not (amp and bias.dtype in _CASTABLE and input.dtype in _CASTABLE)
        )
    ):
        raise RuntimeError("bias must match output channels, device and dtype")


def conv_nd(
    input: Tensor,
    weight: Tensor,
    bias: Tensor | None = None,
    stride: int | Sequence[int] = 1,
    padding: str | int | Sequence[int] = 0,
    dilation: int | Sequence[int] = 1,
    groups: int = 1,
    *,
    padding_mode: str = "zeros",
    workspace_bytes: int = DEFAULT_WORKSPACE_BYTES,
    backend: str = "auto",
    activation: str | None = None,
) -> Tensor:
    """Dense N-dimensional convolution with Conv2d/Conv3d-style semantics.

    ``weight`` is ``[out_channels, in_channels / groups, k_0, ..., k_{r-1}]`` and
    ``input`` is ``[N, in_channels, d_0, ..., d_{r-1}]`` (or unbatched without N).
    ``backend`` accepts ``'auto'`` and ``'native'`` (both run the B200 kernels).
    ``workspace_bytes`` is validated with the reference's rule; the kernels need no
    patch buffer. ``activation='gelu'`` (an extension of the reference's API) returns
    ``gelu(conv + bias)`` from the convolution's own epilogue, and its backward multiplies
    by the GELU derivative while packing the gradient: no separate activation passes.
    """
    rank = weight.ndim - 2
    if not 1 <= rank <= 62:
        raise ValueError("weight must have output/input channels and 1-62 spatial dimensions")
    if not has_rank(input.ndim, rank):
        raise ValueError(f"expected {rank + 1} unbatched or {rank + 2} batched dimensions")
    unbatched = input.ndim == rank + 1
    if unbatched:
        input = input.unsqueeze(0)
    stride = _tuple(stride, rank, "stride")
    dilation = _tuple(dilation, rank, "dilation")
    padding = padding if isinstance(padding, str) else _tuple(padding, rank, "padding")
    _check_options(padding_mode, workspace_bytes, backend)
    if padding_mode == "partial":
        # zero padding rescaled as a mask-free partial convolution (the reference's
        # functional.py:107-122)
        if activation is not None:
            raise ValueError("a fused activation does not combine with padding_mode='partial'")
        from ._partial import partial_conv

        output, _ = partial_conv(
            input, weight, bias, stride, padding, dilation, groups, mask=None,
            multi_channel=False, padding_mode="zeros", workspace_bytes=workspace_bytes,
            backend=backend, need_update=False)
        return output.squeeze(0) if unbatched else output
    amp = _check_arguments(input, weight, stride, padding, dilation, groups)
    _check_bias(input, weight, bias, amp)
    pairs = padding_pairs(padding, weight.shape[2:], stride, dilation)
    if padding_mode != "zeros" or any(left != right for left, right in pairs):
        input = apply_padding(input, pairs, padding_mode)
        implicit = (0,) * rank
    else:
        implicit = tuple(left for left, _ in pairs)
    from ._native import is_loaded, load_native

    if not is_loaded():
        load_native()
    if activation is None:
        output = torch.ops.torch_convnd.conv_nd.default(
            input, weight, bias, list(stride), list(implicit), list(dilation), groups,
            workspace_bytes)
    elif activation == "gelu":
        output, _ = torch.ops.torch_convnd.conv_nd_act.default(
            input, weight, bias, list(stride), list(implicit), list(dilation), groups,
            workspace_bytes, activation)
    else:
        raise ValueError(f"Invalid activation {activation!r}; expected None or 'gelu'")
    return output.squeeze(0) if unbatched else output
