"""Padding semantics: ``'same'``/``'valid'`` strings and non-zero padding modes.

Symmetric zero padding is passed to the kernels as implicit padding (TMA reads
out-of-range coordinates as zero). Asymmetric padding and the reflect / replicate /
circular modes are materialised on the device first, as the reference does
(``src/torch_convnd/_padding.py:9-51``, ``functional.py:171-185``).
"""

from __future__ import annotations

import torch
from torch.nn import functional as F


def padding_pairs(padding, kernel, stride, dilation):
    """Resolve integer or string padding to per-axis (left, right) pairs."""
    if isinstance(padding, str):
        if padding not in ("same", "valid"):
            raise ValueError(f"Invalid padding string {padding!r}; expected 'same' or 'valid'")
        if padding == "same" and any(step != 1 for step in stride):
            raise ValueError("padding='same' is not supported for strided convolutions")
        pairs = []
        for size, dil in zip(kernel, dilation, strict=True):
            total = (size - 1) * dil if padding == "same" else 0
            pairs.append((total // 2, total - total // 2))
        return tuple(pairs)
    return tuple((pad, pad) for pad in padding)


def _edge_indices(size: int, left: int, right: int, mode: str, device) -> torch.Tensor:
    coordinates = torch.arange(-left, size + right, device=device)
    if mode == "replicate":
        return coordinates.clamp(0, size - 1)
    if mode == "circular":
        return coordinates.remainder(size)
    # reflect: mirror about the first and last sample without repeating them
    mirrored = coordinates.abs()
    return torch.where(mirrored >= size, 2 * (size - 1) - mirrored, mirrored)


def apply_padding(input: torch.Tensor, pairs, mode: str) -> torch.Tensor:
    """Pad every spatial axis of a batched channels-first tensor."""
    if not any(left or right for left, right in pairs):
        return input
    if mode == "zeros":
        return F.pad(input, tuple(v for pair in reversed(pairs) for v in pair))
    for axis, (left, right) in enumerate(pairs, start=2):
        if not (left or right):
            continue
        size = input.shape[axis]
        if mode == "reflect" and (left >= size or right >= size):
            raise RuntimeError("Reflection padding must be less than the input dimension")
        if mode == "circular" and (left > size or right > size):
            raise RuntimeError("Padding value causes wrapping around more than once")
        input = input.index_select(axis, _edge_indices(size, left, right, mode, input.device))
    return input
