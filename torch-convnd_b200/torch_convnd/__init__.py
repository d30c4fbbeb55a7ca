"""torch_convnd, B200 build: dense N-D convolution on hand-written sm_100a kernels.

A drop-in for the native backend of lyehe/torch-convnd 0.5.0: the same
``torch_convnd::conv_nd`` / ``conv_nd_backward`` operators, the ``ConvNd`` /
``Conv1d``..``Conv4d`` modules and the ``conv_nd`` function. Importing the package
defines the operator schemas and loads the prebuilt native libraries when they exist; it
never compiles anything.
"""

from ._geometry import DEFAULT_WORKSPACE_BYTES
from ._layout import channels_last, is_channels_last
from ._native import (
    device_status,
    launch_count,
    load_native,
    native_unavailable_reason,
    set_fp32_precision,
)
from ._operators import ensure_native_definitions
from ._partial import PartialConvOutput, partial_conv_nd
from .functional import conv_nd
from .modules import Conv1d, Conv2d, Conv3d, Conv4d, ConvNd, PartialConvNd
from .onnx import export_onnx

__version__ = "0.5.0+b200.1"

ensure_native_definitions()
if native_unavailable_reason() is None:
    load_native()

__all__ = [
    "DEFAULT_WORKSPACE_BYTES",
    "Conv1d",
    "Conv2d",
    "Conv3d",
    "Conv4d",
    "ConvNd",
    "PartialConvNd",
    "PartialConvOutput",
    "channels_last",
    "conv_nd",
    "device_status",
    "ensure_native_definitions",
    "export_onnx",
    "is_channels_last",
    "launch_count",
    "load_native",
    "native_unavailable_reason",
    "partial_conv_nd",
    "set_fp32_precision",
    "__version__",
]
