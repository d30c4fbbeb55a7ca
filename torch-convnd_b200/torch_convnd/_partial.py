"""NVIDIA's partial convolution (Liu et al., 2018) over the native operator.

Behaviour of the reference's ``partial_conv_nd``, ``conv_nd(..., padding_mode="partial")``
and ``PartialConvNd`` (``src/torch_convnd/functional.py:188-258,444-560``,
``modules.py:218-320``): each output sums the valid samples of its window and is rescaled
by the window size over the valid count::

    count  = sum(mask over the window and, with multi_channel, the group's channels)
    update = clamp(count, 0, 1)
    output = conv(input * mask) * window / count * update           # without bias
    output = (conv(input * mask) * window / count * update + bias) * update

The data convolution and, with a mask, the count convolution (an all-ones depthwise
kernel over the detached mask, in float32 or float64 outside autocast, so counts stay
exact) both run the native operator. Without a mask and with zero padding the counts are
products of per-axis counts of in-bounds taps, computed on the device with no
convolution; without padding (or with a copying padding mode) every window is full and
the result is an ordinary convolution.
"""

from __future__ import annotations

import contextlib
import math
from collections.abc import Sequence
from typing import NamedTuple

import torch
from torch import Tensor

from ._geometry import DEFAULT_WORKSPACE_BYTES, _tuple, has_rank
from ._padding import padding_pairs


class PartialConvOutput(NamedTuple):
    """A partial convolution's output and its update mask, the next layer's input mask."""

    output: Tensor
    mask: Tensor


def _axis_counts(size, kernel, stride, dilation, left, right, dtype, device):
    """In-bounds taps of each output window along one zero-padded axis."""
    windows = (size + left + right - dilation * (kernel - 1) - 1) // stride + 1
    origin = torch.arange(windows, device=device) * stride - left
    first = (-torch.div(origin, dilation, rounding_mode="floor")).clamp_min(0)
    last = torch.div(size - 1 - origin, dilation, rounding_mode="floor").clamp_max(kernel - 1)
    return (last - first + 1).clamp_min(0).to(dtype)


def _mask_free_counts(spatial, kernel, stride, dilation, pairs, dtype, device):
    """Counts of an all-valid zero-padded input: products of the per-axis counts."""
    rank = len(spatial)
    counts = torch.ones((1, 1) + (1,) * rank, dtype=dtype, device=device)
    for axis, (size, taps, step, spacing, (left, right)) in enumerate(
        zip(spatial, kernel, stride, dilation, pairs)
    ):
        vector = _axis_counts(size, taps, step, spacing, left, right, dtype, device)
        shape = (1, 1) + (1,) * axis + (-1,) + (1,) * (rank - axis - 1)
        counts = counts * vector.reshape(shape)
    return counts


def _check_mask(input: Tensor, mask: Tensor, rank: int) -> None:
    if mask.ndim != input.ndim:
        raise ValueError(f"mask must have the input's {input.ndim} dimensions")
    if mask.dtype.is_complex:
        raise ValueError("mask must be real")
    if mask.device != input.device:
        raise ValueError("mask must be on the input's device")
    batch = 1 if input.ndim == rank + 1 else input.shape[0]
    if input.ndim == rank + 2 and mask.shape[0] not in (1, batch):
        raise ValueError(f"mask batch must be 1 or {batch}")
    for size, wanted in zip(mask.shape[-rank:], input.shape[-rank:]):
        if size != 1 and size != wanted:
            raise ValueError(
                f"mask spatial shape {tuple(mask.shape[-rank:])} must equal or broadcast "
                f"to the input's {tuple(input.shape[-rank:])}")


def partial_conv(
    input: Tensor,
    weight: Tensor,
    bias: Tensor | None,
    stride,
    padding,
    dilation,
    groups: int,
    *,
    mask: Tensor | None,
    multi_channel: bool,
    padding_mode: str,
    workspace_bytes: int,
    backend: str,
    need_update: bool,
) -> tuple[Tensor, Tensor | None]:
    """The partial convolution; ``need_update=False`` skips building the update mask."""
    from .functional import conv_nd

    rank = weight.ndim - 2
    if not 1 <= rank <= 62:
        raise ValueError("weight must have output/input channels and 1-62 spatial dimensions")
    if not has_rank(input.ndim, rank):
        raise ValueError(f"expected {rank + 1} unbatched or {rank + 2} batched dimensions")
    if not isinstance(multi_channel, bool):
        raise TypeError("multi_channel must be a bool")
    if padding_mode == "partial":
        raise ValueError("partial convolution already rescales zero padding; use 'zeros'")
    if mask is not None:
        _check_mask(input, mask, rank)
    unbatched = input.ndim == rank + 1
    if unbatched:
        input = input.unsqueeze(0)
        mask = None if mask is None else mask.unsqueeze(0)
    channels, spatial = input.shape[1], tuple(input.shape[2:])
    if groups <= 0 or channels % groups or weight.shape[0] % groups:
        raise RuntimeError("input/weight channels must match and be divisible by groups")
    kernel = tuple(int(size) for size in weight.shape[2:])
    steps, spacings = _tuple(stride, rank, "stride"), _tuple(dilation, rank, "dilation")
    pads = padding if isinstance(padding, str) else _tuple(padding, rank, "padding")
    pairs = padding_pairs(pads, kernel, steps, spacings)
    exact = torch.float64 if input.dtype == torch.float64 else torch.float32
    per_group = channels // groups
    out_channels = weight.shape[0]
    options = {"padding_mode": padding_mode, "workspace_bytes": workspace_bytes,
                "backend": backend}

    def finish(output, update):
        if unbatched:
            return output.squeeze(0), None if update is None else update.squeeze(0)
        return output, update

    if mask is None:
        if padding_mode != "zeros" or not any(left or right for left, right in pairs):
            # every tap reads a real or copied sample: an ordinary convolution
            output = conv_nd(input, weight, bias, steps, pads, spacings, groups, **options)
            update = None
            if need_update:
                width = out_channels if multi_channel else 1
                ones = torch.ones((), dtype=output.dtype, device=output.device)
                update = ones.expand(output.shape[0], width, *output.shape[2:])
            return finish(output, update)
        window = math.prod(kernel)
        data = input
        counts = None  # after the data convolution, which validates the geometry
    else:
        width = channels if multi_channel else 1
        if mask.shape[1] not in (1, width):
            raise ValueError(
                f"mask must have 1 or {channels} channels" if multi_channel else
                "mask must have 1 channel; use multi_channel=True for per-channel masks")
        data = input * mask.to(input.dtype)
        valid = mask.detach().to(exact).expand(mask.shape[0], width, *spatial)
        if multi_channel:
            # each output channel counts its own group's input channels
            valid = valid.reshape(mask.shape[0], groups, per_group, *spatial).sum(2)
        window = math.prod(kernel) * (per_group if multi_channel else 1)
    output = conv_nd(data, weight, None, steps, pads, spacings, groups, **options)
    if mask is None:
        counts = _mask_free_counts(spatial, kernel, steps, spacings, pairs, exact,
                                   input.device)
    else:
        count_channels = valid.shape[1]
        ones = torch.ones((count_channels, 1, *kernel), dtype=exact, device=input.device)
        device_type = input.device.type
        outside_amp = (torch.autocast(device_type=device_type, enabled=False)
                       if device_type in ("cpu", "cuda") else contextlib.nullcontext())
        with outside_amp:
            counts = conv_nd(valid.contiguous(), ones, None, steps, pads, spacings,
                             count_channels, **options)
    produced = output.dtype
    level = produced
    if produced == torch.float16 and window > torch.finfo(torch.float16).max:
        level = torch.float32  # the ratio would overflow float16: rescale in float32
        output = output.float()
    update = counts.clamp(0, 1)
    ratio = (update * window / counts.clamp_min(torch.finfo(counts.dtype).tiny)).to(level)
    update = update.to(level)
    batch = output.shape[0]
    if update.shape[1] > 1:
        # per-group counts: scale each group's output channels by its group's ratio
        shaped = output.reshape(batch, groups, out_channels // groups, *output.shape[2:])
        output = (shaped * ratio.unsqueeze(2)).reshape(output.shape)
        update = update.unsqueeze(2).expand(update.shape[0], groups, out_channels // groups,
                                            *update.shape[2:])
        update = update.reshape(update.shape[0], out_channels, *update.shape[3:])
    else:
        output = output * ratio
    if bias is not None:
        view = (1, -1) + (1,) * rank
        output = (output + bias.to(output.dtype).reshape(view)) * update
    output = output.to(produced)
    if not need_update:
        return finish(output, None)
    width = out_channels if multi_channel else 1
    if update.shape[1] != width:
        update = update.expand(update.shape[0], width, *update.shape[2:])
    if update.shape[0] != batch:
        update = update.expand(batch, *update.shape[1:])
    return finish(output, update)


def partial_conv_nd(
    input: Tensor,
    weight: Tensor,
    bias: Tensor | None = None,
    stride: int | Sequence[int] = 1,
    padding: str | int | Sequence[int] = 0,
    dilation: int | Sequence[int] = 1,
    groups: int = 1,
    *,
    mask: Tensor | None = None,
    multi_channel: bool = False,
    padding_mode: str = "zeros",
    workspace_bytes: int = DEFAULT_WORKSPACE_BYTES,
    backend: str = "auto",
) -> PartialConvOutput:
    """Apply NVIDIA's partial convolution; return the output and its update mask.

    ``mask`` (1 valid, 0 hole; fractional values follow the formula) has the input's
    number of dimensions; one channel shared by every input channel, or with
    ``multi_channel`` one per input channel (or one, broadcast) counted per group; its
    batch and spatial sizes equal the input's or are 1. It is padded like the input.
    ``mask=None`` means every sample is valid, so zero padding gives partial-convolution
    padding. No gradient flows through the counts. The update mask has one channel, or
    ``out_channels`` with ``multi_channel``; it may be a broadcast view.
    """
    if padding_mode == "partial":
        raise ValueError("partial_conv_nd already rescales zero padding; use padding_mode='zeros'")
    output, update = partial_conv(
        input, weight, bias, stride, padding, dilation, groups, mask=mask,
        multi_channel=multi_channel, padding_mode=padding_mode,
        workspace_bytes=workspace_bytes, backend=backend, need_update=True)
    return PartialConvOutput(output, update)
