"""The allocation-free forward entry point (cnd_forward_noalloc), through the C ABI.

cnd_forward_noalloc serves callers that cannot allocate device memory — thin C-ABI
bindings that hold no device allocator, or processes whose GPU memory is owned by a
fixed-budget pool — by running the forward pass in a static device scratch array of the
library. These tests check that two calls in a row reproduce the regular entry point
(cnd_forward with a caller-provided workspace) within the bf16 rule the other parity
tests use, and that a problem larger than the scratch is refused with a clear error.
This file is collected last on purpose; it also runs alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tolerances import assert_matches
from torch_convnd import _native

pytestmark = pytest.mark.gpu

CND_ERR_WORKSPACE = -4


class Problem(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("fp32_mode", ctypes.c_int32), ("reserved", ctypes.c_int32)] + [
        (name, ctypes.c_int64) for name in ("batch", "channels", "output_channels", "groups",
                                            "input_volume", "output_volume", "kernel_volume")] + [
        (name, ctypes.c_int64 * 62)
        for name in ("input", "output", "kernel", "stride", "padding", "dilation")]


def _library():
    library = _native.core()
    library.cnd_forward.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_size_t, ctypes.c_void_p]
    library.cnd_forward.restype = ctypes.c_int
    library.cnd_forward_noalloc.argtypes = [ctypes.c_void_p] * 6
    library.cnd_forward_noalloc.restype = ctypes.c_int
    library.cnd_forward_workspace_size.argtypes = [ctypes.c_void_p]
    library.cnd_forward_workspace_size.restype = ctypes.c_size_t
    return library


def _problem(library, x, w, padding):
    arr = lambda values: (ctypes.c_int64 * len(values))(*values)
    problem = Problem()
    rank = x.ndim - 2
    status = library.cnd_problem_init(
        ctypes.byref(problem), rank, arr(list(x.shape)), arr(list(w.shape)), arr([1] * rank),
        arr([padding] * rank), arr([1] * rank), ctypes.c_int64(1), 1)  # 1 = bfloat16
    assert status == 0, library.cnd_last_error()
    return problem


def test_noalloc_forward_matches_regular_entry_point_twice():
    library = _library()
    generator = torch.Generator().manual_seed(2024)
    x = torch.randn(2, 32, 6, 5, 7, 8, generator=generator).bfloat16().cuda()
    w = (torch.randn(64, 32, 3, 3, 3, 3, generator=generator) / 50).bfloat16().cuda()
    b = torch.randn(64, generator=generator).bfloat16().cuda()
    problem = _problem(library, x, w, 1)
    needed = library.cnd_forward_workspace_size(ctypes.byref(problem))
    assert 0 < needed <= 16 * 1024 * 1024
    stream = torch.cuda.current_stream().cuda_stream
    shape = (2, 64, 6, 5, 7, 8)
    expected = torch.empty(shape, dtype=torch.bfloat16, device="cuda")
    workspace = torch.empty(needed, dtype=torch.uint8, device="cuda")
    status = library.cnd_forward(ctypes.byref(problem), x.data_ptr(), w.data_ptr(),
                                 b.data_ptr(), expected.data_ptr(), workspace.data_ptr(), needed,
                                 stream)
    assert status == 0, library.cnd_last_error()
    for call in range(2):
        out = torch.full(shape, float("nan"), dtype=torch.bfloat16, device="cuda")
        status = library.cnd_forward_noalloc(ctypes.byref(problem), x.data_ptr(), w.data_ptr(),
                                             b.data_ptr(), out.data_ptr(), stream)
        assert status == 0, library.cnd_last_error()
        torch.cuda.synchronize()
        assert_matches(out, expected.double(), torch.bfloat16, f"noalloc call {call}")
    assert library.cnd_device_status(ctypes.c_void_p(stream)) == 0


def test_noalloc_forward_rejects_problems_above_the_static_scratch():
    library = _library()
    # c2's full batch needs ~64 MiB of packed input: beyond the 16 MiB scratch.
    x = torch.empty(16, 32, 16, 16, 16, 16, dtype=torch.bfloat16, device="cuda")
    w = torch.empty(64, 32, 3, 3, 3, 3, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(16, 64, 16, 16, 16, 16, dtype=torch.bfloat16, device="cuda")
    problem = _problem(library, x, w, 1)
    status = library.cnd_forward_noalloc(ctypes.byref(problem), x.data_ptr(), w.data_ptr(),
                                         None, y.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream)
    assert status == CND_ERR_WORKSPACE
    message = library.cnd_last_error().decode()
    assert "static scratch" in message and "16777216" in message
