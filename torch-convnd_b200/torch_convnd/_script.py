"""TorchScript form of ConvNd.

``torch.jit.script(ConvNd(...))`` scripts this module instead (``ConvNd`` hands it over
in ``__prepare_scriptable__``, as the reference's does, modules.py:137-155). It holds
the same parameters and geometry in TorchScript's restricted syntax, applies explicit
padding with ``F.pad`` / ``index_select`` as the eager path does, and calls
``torch_convnd::compatible_conv_nd``, so a scripted graph runs the native operator with
its autograd formulas. Mirrors the reference's ScriptableConvNd (_script.py:10-114).
"""

from __future__ import annotations

from typing import List, Optional  # noqa: UP035 (TorchScript wants typing generics)

import torch
from torch import Tensor, nn
from torch.nn import functional as F


class ScriptableConvNd(nn.Module):
    __constants__ = ["dimensions", "stride", "dilation", "groups", "workspace_bytes", "mode",
                     "left", "right", "native_padding", "explicit_padding", "reverse_padding",
                     "backend"]

    def __init__(self, layer):
        super().__init__()
        self.weight = layer.weight
        if layer.bias is None:
            self.register_parameter("bias", None)
        else:
            self.bias = layer.bias
        self.dimensions: int = layer.dimensions
        self.stride: List[int] = list(layer.stride)  # noqa: UP006
        self.dilation: List[int] = list(layer.dilation)  # noqa: UP006
        self.groups: int = layer.groups
        self.workspace_bytes: int = layer.workspace_bytes
        self.mode: str = layer.padding_mode
        self.backend: str = layer.backend
        reverse = [int(v) for v in layer._reversed_padding_repeated_twice]
        self.reverse_padding: List[int] = reverse  # noqa: UP006
        # reverse holds (left, right) pairs from the last axis to the first
        self.left: List[int] = [reverse[2 * (self.dimensions - 1 - a)]  # noqa: UP006
                                for a in range(self.dimensions)]
        self.right: List[int] = [reverse[2 * (self.dimensions - 1 - a) + 1]  # noqa: UP006
                                 for a in range(self.dimensions)]
        self.explicit_padding: bool = self.mode != "zeros" or self.left != self.right
        self.native_padding: List[int] = (  # noqa: UP006
            [0] * self.dimensions if self.explicit_padding else list(self.left))

    def _pad(self, input: Tensor) -> Tensor:
        if not self.explicit_padding:
            return input
        if self.mode == "zeros":
            return F.pad(input, self.reverse_padding)
        for axis in range(self.dimensions):
            left = self.left[axis]
            right = self.right[axis]
            if left != 0 or right != 0:
                size = input.size(axis + 2)
                if self.mode == "reflect" and (left >= size or right >= size):
                    raise RuntimeError("Reflection padding must be less than the input dimension")
                if self.mode == "circular" and (left > size or right > size):
                    raise RuntimeError("Padding value causes wrapping around more than once")
                coordinates = torch.arange(-left, size + right, device=input.device)
                if self.mode == "replicate":
                    indices = coordinates.clamp(0, size - 1)
                elif self.mode == "circular":
                    indices = coordinates.remainder(size)
                else:
                    indices = coordinates.abs()
                    indices = torch.where(indices >= size, 2 * (size - 1) - indices, indices)
                input = input.index_select(axis + 2, indices)
        return input

    def forward(self, input: Tensor) -> Tensor:
        unbatched = input.dim() == self.dimensions + 1
        if unbatched:
            input = input.unsqueeze(0)
        elif input.dim() != self.dimensions + 2:
            raise ValueError("Incorrect input rank")
        bias: Optional[Tensor] = self.bias  # noqa: UP045
        output = torch.ops.torch_convnd.compatible_conv_nd(
            self._pad(input), self.weight, bias, self.stride, self.native_padding,
            self.dilation, self.groups, self.workspace_bytes, self.backend)
        return output.squeeze(0) if unbatched else output
