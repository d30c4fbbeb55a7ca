"""Host-side contract checks (CPU only): operator schemas, fake kernels, argument errors
with the reference's messages, module API, and the C-ABI library's exports."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

import torch_convnd
from torch_convnd import Conv4d, ConvNd, conv_nd
from torch_convnd import _native

ROOT = Path(__file__).resolve().parent.parent


def test_schemas_are_the_reference_contract():
    forward = str(torch.ops.torch_convnd.conv_nd.default._schema)
    backward = str(torch.ops.torch_convnd.conv_nd_backward.default._schema)
    assert forward == (
        "torch_convnd::conv_nd(Tensor input, Tensor weight, Tensor? bias, int[] stride, "
        "int[] padding, int[] dilation, int groups, int workspace_bytes) -> Tensor"
    )
    assert backward == (
        "torch_convnd::conv_nd_backward(Tensor grad_output, Tensor input, Tensor weight, "
        "int[] stride, int[] padding, int[] dilation, int groups, int workspace_bytes, "
        "bool[3] output_mask) -> (Tensor?, Tensor?, Tensor?)"
    )


def test_fake_kernels_infer_shapes():
    x = torch.empty(2, 3, 7, 6, 5, 4, device="meta")
    w = torch.empty(8, 3, 3, 2, 3, 1, device="meta")
    y = torch.ops.torch_convnd.conv_nd(x, w, None, [2, 1, 1, 1], [1, 0, 2, 0], [1, 2, 1, 1], 1, 1 << 20)
    assert y.shape == (2, 8, 4, 4, 7, 4)
    dx, dw, db = torch.ops.torch_convnd.conv_nd_backward(
        y, x, w, [2, 1, 1, 1], [1, 0, 2, 0], [1, 2, 1, 1], 1, 1 << 20, [True, True, False])
    assert dx.shape == x.shape and dw.shape == w.shape and db is None


@pytest.mark.parametrize(
    ("kwargs", "message"),
    [
        ({"groups": 0}, "groups must be positive"),
        ({"stride": 0}, "stride and dilation"),
        ({"padding": -1}, "padding must be nonnegative"),
        ({"workspace_bytes": 1}, "workspace_bytes is too small"),
        ({"groups": 3}, "channels must match"),
    ],
)
def test_invalid_geometry_messages(kwargs, message):
    """Same cases and messages as the reference's tests/test_convnd.py:260-275."""
    with pytest.raises(RuntimeError, match=message):
        conv_nd(torch.randn(1, 2, 3, 3, 3, 3), torch.randn(4, 2, 2, 2, 2, 2), backend="native",
                **kwargs)


def test_backward_checks_the_workspace_budget():
    """The backward operator applies the reference's patch-budget rule too
    (convnd.cpp:357-375): 4-byte elements for 16-bit inputs, and only when dx or dW is
    requested."""
    x, w = torch.randn(1, 2, 3, 3, 3, 3), torch.randn(4, 2, 2, 2, 2, 2)
    dy = torch.randn(1, 4, 2, 2, 2, 2)
    op = torch.ops.torch_convnd.conv_nd_backward
    geometry = ([1] * 4, [0] * 4, [1] * 4, 1)
    # one position's patch column: 2 channels * 16 taps * 4 bytes = 128 bytes
    with pytest.raises(RuntimeError, match="requires at least 128"):
        op(dy, x, w, *geometry, 127, [True, True, True])
    with pytest.raises(RuntimeError, match="requires at least 128"):
        op(dy.bfloat16(), x.bfloat16(), w.bfloat16(), *geometry, 127, [False, True, False])
    # enough budget: validation passes and the CPU kernel refuses to run
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        op(dy, x, w, *geometry, 128, [True, True, True])
    # a bias-only request needs no patch budget in float32
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        op(dy, x, w, *geometry, 1, [False, False, True])


def test_module_backend_torch_is_refused_like_the_function():
    """ConvNd(backend='torch') raises when called, as conv_nd(backend='torch') does."""
    layer = Conv4d(2, 4, 2, backend="torch")
    with pytest.raises(ValueError, match="not part of the B200 build"):
        layer(torch.randn(1, 2, 3, 3, 3, 3))


def test_dtype_bias_and_kernel_errors():
    """Reference tests/test_convnd.py:278-290."""
    x, w = torch.randn(1, 2, 3, 3, 3, 3), torch.randn(4, 2, 2, 2, 2, 2)
    with pytest.raises(RuntimeError, match="float16, bfloat16, float32 and float64"):
        conv_nd(x.to(torch.int64), w.to(torch.int64), backend="native")
    with pytest.raises(RuntimeError, match="same device and dtype"):
        conv_nd(x, w.double())
    with pytest.raises(RuntimeError, match="bias must match"):
        conv_nd(x, w, torch.zeros(3))
    with pytest.raises(RuntimeError, match="kernel exceeds"):
        conv_nd(x, torch.randn(4, 2, 4, 2, 2, 2))
    with pytest.raises(ValueError, match="exactly 4 integers"):
        conv_nd(x, w, stride=(1, 1))


def test_integer_overflow_is_rejected():
    """Reference tests/test_convnd.py:312-317."""
    with pytest.raises(RuntimeError, match="output spatial volume overflows"):
        conv_nd(torch.ones((1,) * 64), torch.ones((1,) * 64), padding=1)
    with pytest.raises(RuntimeError, match="padding overflows"):
        conv_nd(torch.ones(1, 1, 2), torch.ones(1, 1, 1), padding=2**63 - 1, backend="native")


def test_cpu_tensors_fail_loudly_after_validation():
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        conv_nd(torch.randn(1, 2, 3, 3, 3, 3), torch.randn(4, 2, 2, 2, 2, 2))


def test_portable_backend_is_not_offered():
    with pytest.raises(ValueError, match="not part of the B200 build"):
        conv_nd(torch.randn(1, 2, 3, 3, 3, 3), torch.randn(4, 2, 2, 2, 2, 2), backend="torch")


def test_module_api_and_state_dict():
    layer = Conv4d(4, 6, 3, padding="same", groups=2, bias=True)
    assert layer.weight.shape == (6, 2, 3, 3, 3, 3)
    assert set(layer.state_dict()) == {"weight", "bias"}
    bound = 1 / (2 * 81) ** 0.5
    assert float(layer.bias.detach().abs().max()) <= bound
    same = ConvNd(4, 6, 3, dimensions=4, padding="same", groups=2)
    same.load_state_dict(layer.state_dict())
    with pytest.raises(ValueError, match="expected 5 unbatched or 6 batched"):
        Conv4d(2, 3, 2)(torch.randn(1, 2, 3, 3))
    with pytest.raises(ValueError, match="dimensions must"):
        ConvNd(2, 3, 2, dimensions=0)
    with pytest.raises(ValueError, match="divisible"):
        ConvNd(3, 4, 2, dimensions=4, groups=2)


def test_padding_pairs():
    from torch_convnd._padding import padding_pairs

    assert padding_pairs("same", (3, 4), (1, 1), (1, 2)) == ((1, 1), (3, 3))
    assert padding_pairs("valid", (3, 3), (2, 2), (1, 1)) == ((0, 0), (0, 0))
    with pytest.raises(ValueError, match="strided"):
        padding_pairs("same", (3,), (2,), (1,))


def _declared_symbols():
    text = (ROOT / "include" / "convnd_b200.h").read_text()
    return re.findall(r"CND_API\s+[\w\s\*]+?\b(cnd_\w+)\s*\(", text)


def test_c_abi_library_exports_every_declared_symbol():
    library = ctypes.CDLL(str(_native.CORE_PATH))
    names = _declared_symbols()
    assert len(names) == len(set(names)) >= 13
    for name in names:
        assert hasattr(library, name), name


def test_c_abi_problem_init_and_budget():
    library = ctypes.CDLL(str(_native.CORE_PATH))

    class Problem(ctypes.Structure):
        _fields_ = [("rank", ctypes.c_int32), ("dtype", ctypes.c_int32),
                    ("fp32_mode", ctypes.c_int32), ("reserved", ctypes.c_int32),
                    ("batch", ctypes.c_int64), ("channels", ctypes.c_int64),
                    ("output_channels", ctypes.c_int64), ("groups", ctypes.c_int64),
                    ("input_volume", ctypes.c_int64), ("output_volume", ctypes.c_int64),
                    ("kernel_volume", ctypes.c_int64)] + [
            (name, ctypes.c_int64 * 62)
            for name in ("input", "output", "kernel", "stride", "padding", "dilation")]

    arr = lambda *v: (ctypes.c_int64 * len(v))(*v)
    problem = Problem()
    library.cnd_last_error.restype = ctypes.c_char_p
    status = library.cnd_problem_init(ctypes.byref(problem), 4, arr(16, 32, 16, 16, 16, 16),
                                      arr(64, 32, 3, 3, 3, 3), arr(1, 1, 1, 1), arr(1, 1, 1, 1),
                                      arr(1, 1, 1, 1), ctypes.c_int64(1), 1)
    assert status == 0
    assert list(problem.output[:4]) == [16, 16, 16, 16]
    assert problem.kernel_volume == 81 and problem.output_volume == 65536
    assert library.cnd_check_workspace_budget(ctypes.byref(problem), ctypes.c_int64(2),
                                              ctypes.c_int64(100)) == -1
    assert b"requires at least 10368" in library.cnd_last_error()
    library.cnd_forward_workspace_size.restype = ctypes.c_size_t
    # c2: x packed channels-last bf16 (16*65536*32*2) + packed weights (81*64*32*2), 1 KiB aligned
    assert library.cnd_forward_workspace_size(ctypes.byref(problem)) == 67108864 + 331776
    assert library.cnd_fast_path_mask(ctypes.byref(problem)) == 7
    # Plans are cached per problem, pass kind and gradient mask: sizes queried in any
    # order agree, and a changed layout field is a different problem.
    library.cnd_backward_workspace_size.restype = ctypes.c_size_t
    masks = [(1, 0, 0), (0, 1, 0), (1, 1, 1), (0, 0, 1)]
    size = lambda m: library.cnd_backward_workspace_size(ctypes.byref(problem),
                                                         (ctypes.c_int32 * 3)(*m))
    first = [size(m) for m in masks]
    assert [size(m) for m in reversed(masks)] == list(reversed(first))
    assert first[2] >= max(first[0], first[1]) and len(set(first)) > 1
    problem.reserved = 1  # channels-last input with 32 channels: read in place, no pack
    assert library.cnd_forward_workspace_size(ctypes.byref(problem)) == 331776
    problem.reserved = 0
    assert library.cnd_forward_workspace_size(ctypes.byref(problem)) == 67108864 + 331776
    status = library.cnd_problem_init(ctypes.byref(problem), 4, arr(1, 2, 3, 3, 3, 3),
                                      arr(4, 2, 4, 2, 2, 2), arr(1, 1, 1, 1), arr(0, 0, 0, 0),
                                      arr(1, 1, 1, 1), ctypes.c_int64(1), 2)
    assert status == -1 and library.cnd_last_error() == b"kernel exceeds padded input"


def test_version():
    assert torch_convnd.__version__.startswith("0.5.0")
