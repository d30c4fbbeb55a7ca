"""Trainable convolution modules with PyTorch-compatible constructors.

``ConvNd`` and the fixed-rank ``Conv1d``..``Conv4d`` keep the reference's constructor,
validation messages, parameter names (``weight``, ``bias``) and initialisation
(``src/torch_convnd/modules.py:21-216``), so state dicts move between the two packages.
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch
from torch import Tensor, nn

from ._geometry import DEFAULT_WORKSPACE_BYTES, _tuple, has_rank
from ._padding import padding_pairs
from ._partial import PartialConvOutput, partial_conv
from .functional import _PADDING_MODES, conv_nd


class ConvNd(nn.Module):
    """Trainable dense N-dimensional convolution (``dimensions`` spatial axes)."""

    def __init__(
        self,
        in_channels: int,
        out_channels: int,
        kernel_size: int | Sequence[int],
        stride: int | Sequence[int] = 1,
        padding: str | int | Sequence[int] = 0,
        dilation: int | Sequence[int] = 1,
        groups: int = 1,
        bias: bool = True,
        padding_mode: str = "zeros",
        device=None,
        dtype=None,
        *,
        dimensions: int,
        workspace_bytes: int = DEFAULT_WORKSPACE_BYTES,
        backend: str = "auto",
        activation: str | None = None,
    ):
        super().__init__()
        if not isinstance(dimensions, int) or isinstance(dimensions, bool) or not 1 <= dimensions <= 62:
            raise ValueError("dimensions must be an integer from 1 to 62")
        self.dimensions = dimensions
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = _tuple(kernel_size, dimensions, "kernel_size")
        self.stride = _tuple(stride, dimensions, "stride")
        self.padding = padding if isinstance(padding, str) else _tuple(padding, dimensions, "padding")
        self.dilation = _tuple(dilation, dimensions, "dilation")
        self.groups = groups
        self.padding_mode = padding_mode
        self.transposed = False
        self.output_padding = (0,) * dimensions
        self.workspace_bytes = workspace_bytes
        if activation not in (None, "gelu"):
            raise ValueError(f"Invalid activation {activation!r}; expected None or 'gelu'")
        self.activation = activation
        if backend not in ("auto", "native", "torch"):
            raise ValueError(f"Invalid backend {backend!r}")
        self.backend = backend
        if groups <= 0 or in_channels <= 0 or out_channels <= 0:
            raise ValueError("channels and groups must be positive")
        if in_channels % groups or out_channels % groups:
            raise ValueError("channels must be divisible by groups")
        if min(*self.kernel_size, *self.stride, *self.dilation) <= 0 or (
            not isinstance(self.padding, str) and min(self.padding) < 0
        ):
            raise ValueError("kernel, stride and dilation must be positive; padding nonnegative")
        if padding_mode not in _PADDING_MODES:
            raise ValueError(f"Invalid padding_mode {padding_mode!r}")
        pairs = padding_pairs(self.padding, self.kernel_size, self.stride, self.dilation)
        self._reversed_padding_repeated_twice = [v for pair in reversed(pairs) for v in pair]
        if workspace_bytes <= 0:
            raise ValueError("workspace_bytes must be positive")
        factory = {"device": device, "dtype": dtype}
        self.weight = nn.Parameter(
            torch.empty(out_channels, in_channels // groups, *self.kernel_size, **factory)
        )
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels, **factory))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        """PyTorch's convolution initialisation: kaiming-uniform(a=sqrt(5)) weights and
        U(-1/sqrt(fan_in), 1/sqrt(fan_in)) bias."""
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in = self.in_channels // self.groups * math.prod(self.kernel_size)
            bound = 1 / math.sqrt(fan_in)
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, input: Tensor) -> Tensor:
        if not has_rank(input.ndim, self.dimensions):
            raise ValueError(
                f"expected {self.dimensions + 1} unbatched or {self.dimensions + 2} batched "
                f"dimensions, got {input.ndim}"
            )
        return conv_nd(
            input,
            self.weight,
            self.bias,
            self.stride,
            self.padding,
            self.dilation,
            self.groups,
            padding_mode=self.padding_mode,
            workspace_bytes=self.workspace_bytes,
            backend=self.backend,
            activation=self.activation,
        )

    def __prepare_scriptable__(self):
        """torch.jit.script hook: script the TorchScript form, which calls the native
        operator through torch_convnd::compatible_conv_nd (reference modules.py:137-155)."""
        if self.activation is not None:
            raise NotImplementedError("a fused activation does not support TorchScript")
        if self.padding_mode == "partial":
            raise NotImplementedError(
                "padding_mode='partial' does not support TorchScript; use eager execution")
        from ._script import ScriptableConvNd

        return ScriptableConvNd(self)

    def extra_repr(self) -> str:
        return (
            f"{self.in_channels}, {self.out_channels}, kernel_size={self.kernel_size}, "
            f"dimensions={self.dimensions}, stride={self.stride}, padding={self.padding}, "
            f"dilation={self.dilation}, groups={self.groups}, bias={self.bias is not None}, "
            f"padding_mode={self.padding_mode!r}, backend={self.backend!r}"
            + (f", activation={self.activation!r}" if self.activation else "")
        )


class _FixedConvNd(ConvNd):
    _spatial_dimensions = 0

    def __init__(
        self,
        in_channels,
        out_channels,
        kernel_size,
        stride=1,
        padding=0,
        dilation=1,
        groups=1,
        bias=True,
        padding_mode="zeros",
        device=None,
        dtype=None,
        *,
        workspace_bytes=DEFAULT_WORKSPACE_BYTES,
        backend="auto",
    ):
        super().__init__(
            in_channels,
            out_channels,
            kernel_size,
            stride,
            padding,
            dilation,
            groups,
            bias,
            padding_mode,
            device,
            dtype,
            dimensions=self._spatial_dimensions,
            workspace_bytes=workspace_bytes,
            backend=backend,
        )


class Conv1d(_FixedConvNd):
    """Dense 1-D convolution with the torch.nn.Conv1d constructor."""

    _spatial_dimensions = 1


class Conv2d(_FixedConvNd):
    """Dense 2-D convolution with the torch.nn.Conv2d constructor."""

    _spatial_dimensions = 2


class Conv3d(_FixedConvNd):
    """Dense 3-D convolution with the torch.nn.Conv3d constructor."""

    _spatial_dimensions = 3


class Conv4d(_FixedConvNd):
    """Dense 4-D convolution (for example x, y, z and time)."""

    _spatial_dimensions = 4


class PartialConvNd(ConvNd):
    """NVIDIA's partial convolution at any spatial rank, with ConvNd's parameters (the
    reference's PartialConvNd, modules.py:218-320).

    ``forward(input, mask=None)`` convolves only valid samples and rescales each window by
    its valid fraction (``torch_convnd.partial_conv_nd`` states the formula and the mask
    contract). ``multi_channel`` (fixed per layer) takes one mask channel per input
    channel; ``return_mask`` sets whether calls also return the update mask as
    ``PartialConvOutput(output, mask)``, and each call can override it. State dicts match
    ConvNd's.
    """

    def __init__(
        self,
        in_channels: int,
        out_channels: int,
        kernel_size: int | Sequence[int],
        stride: int | Sequence[int] = 1,
        padding: str | int | Sequence[int] = 0,
        dilation: int | Sequence[int] = 1,
        groups: int = 1,
        bias: bool = True,
        padding_mode: str = "zeros",
        device=None,
        dtype=None,
        *,
        dimensions: int,
        workspace_bytes: int = DEFAULT_WORKSPACE_BYTES,
        backend: str = "auto",
        multi_channel: bool = False,
        return_mask: bool = False,
    ):
        super().__init__(in_channels, out_channels, kernel_size, stride, padding, dilation,
                         groups, bias, padding_mode, device, dtype, dimensions=dimensions,
                         workspace_bytes=workspace_bytes, backend=backend)
        if not isinstance(multi_channel, bool) or not isinstance(return_mask, bool):
            raise TypeError("multi_channel and return_mask must be bools")
        if padding_mode == "partial":
            raise ValueError(
                "PartialConvNd already rescales zero padding; use padding_mode='zeros'")
        self.multi_channel = multi_channel
        self.return_mask = return_mask

    def forward(  # type: ignore[override]
        self,
        input: Tensor,
        mask: Tensor | None = None,
        mask_in: Tensor | None = None,
        return_mask: bool | None = None,
    ) -> Tensor | PartialConvOutput:
        """Convolve the valid samples; with ``return_mask`` also return the update mask.
        ``mask_in`` is NVIDIA's keyword for ``mask``."""
        if mask_in is not None:
            if mask is not None:
                raise TypeError("pass mask or mask_in, not both")
            mask = mask_in
        if return_mask is None:
            return_mask = self.return_mask
        elif not isinstance(return_mask, bool):
            raise TypeError("return_mask must be a bool or None")
        if not has_rank(input.ndim, self.dimensions):
            raise ValueError(
                f"expected {self.dimensions + 1} unbatched or {self.dimensions + 2} batched "
                f"dimensions, got {input.ndim}"
            )
        output, update = partial_conv(
            input, self.weight, self.bias, self.stride, self.padding, self.dilation,
            self.groups, mask=mask, multi_channel=self.multi_channel,
            padding_mode=self.padding_mode, workspace_bytes=self.workspace_bytes,
            backend=self.backend, need_update=return_mask)
        if not return_mask:
            return output
        return PartialConvOutput(output, update)

    def __prepare_scriptable__(self):
        raise NotImplementedError("PartialConvNd does not support TorchScript; use eager execution")
