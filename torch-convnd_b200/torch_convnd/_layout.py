"""Channels-last activations for any spatial rank.

PyTorch names channels-last memory formats only for 4-D and 5-D tensors; the same
layout exists for every rank as strides: a logical [N, C, d0, ..., d_{r-1}] tensor stored
as [N, d0, ..., d_{r-1}, C]. The native operators read such inputs in place and return
outputs (and input gradients) in the same layout, so a network whose first input is
channels-last keeps every activation channels-last, with no layout pass between layers
(the rule matches the shim's is_channels_last / empty_activation in csrc/shim.cpp).
"""

from __future__ import annotations

import torch


def is_channels_last(tensor: torch.Tensor) -> bool:
    """Dense channels-last strides, and not also contiguous (then it is channels-first)."""
    if tensor.dim() < 3 or tensor.is_contiguous():
        return False
    expected = 1
    if tensor.shape[1] != 1 and tensor.stride(1) != expected:
        return False
    expected *= tensor.shape[1]
    for axis in range(tensor.dim() - 1, 1, -1):
        if tensor.shape[axis] != 1 and tensor.stride(axis) != expected:
            return False
        expected *= tensor.shape[axis]
    return tensor.shape[0] == 1 or tensor.stride(0) == expected


def _order(dim: int):
    return (0, *range(2, dim), 1), (0, dim - 1, *range(1, dim - 1))


def channels_last(tensor: torch.Tensor) -> torch.Tensor:
    """`tensor` with channels-last strides (a copy unless it already has them)."""
    if is_channels_last(tensor):
        return tensor
    store, view = _order(tensor.dim())
    return tensor.permute(store).contiguous().permute(view)


def empty_activation(shape, channels_last_layout: bool, like: torch.Tensor) -> torch.Tensor:
    """New tensor of logical shape [N, C, spatial...], channels-last when asked."""
    if not channels_last_layout:
        return like.new_empty(shape)
    store, view = _order(len(shape))
    stored = [shape[i] for i in store]
    return like.new_empty(stored).permute(view)
