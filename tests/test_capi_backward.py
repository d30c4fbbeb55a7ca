"""cnd_backward through the C ABI, as a non-PyTorch host (ctypes, cgo, JNI) calls it.

The backward entry point replaces the reference's conv_nd_backward kernel
(src/torch_convnd/csrc/convnd.cpp:345-415, convnd_mixed.cpp:11-59). These tests drive it
with raw device pointers: every output_mask combination with NULL pointers for the
gradients that are not requested, the workspace size that cnd_backward_workspace_size
reports for that mask, and the status codes of a short workspace or a missing buffer.
Results are compared with the float64 oracle (reference convnd.cpp:345-415 restated).
"""

from __future__ import annotations

import ctypes
import itertools

import pytest
import torch

from oracle import convnd_oracle as oracle
from tolerances import assert_conv_matches, conv_magnitudes
from torch_convnd import _native

pytestmark = pytest.mark.gpu

CND_OK, CND_ERR_INVALID, CND_ERR_WORKSPACE = 0, -1, -4
CODES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2, torch.float64: 3}


class Problem(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("fp32_mode", ctypes.c_int32), ("reserved", ctypes.c_int32)] + [
        (name, ctypes.c_int64) for name in ("batch", "channels", "output_channels", "groups",
                                            "input_volume", "output_volume", "kernel_volume")] + [
        (name, ctypes.c_int64 * 62)
        for name in ("input", "output", "kernel", "stride", "padding", "dilation")]


def _library():
    library = _native.core()
    library.cnd_backward.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_void_p,
                                                             ctypes.c_size_t, ctypes.c_void_p]
    library.cnd_backward.restype = ctypes.c_int
    library.cnd_backward_workspace_size.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    library.cnd_backward_workspace_size.restype = ctypes.c_size_t
    return library


def _problem(library, x, w, stride, padding, dilation, groups):
    arr = lambda values: (ctypes.c_int64 * len(values))(*values)
    problem = Problem()
    status = library.cnd_problem_init(
        ctypes.byref(problem), x.ndim - 2, arr(list(x.shape)), arr(list(w.shape)),
        arr(stride), arr(padding), arr(dilation), ctypes.c_int64(groups), CODES[x.dtype])
    assert status == CND_OK, library.cnd_last_error()
    return problem


CASES = [
    # dtype, x shape, w shape, stride, padding, dilation, groups
    (torch.bfloat16, (2, 32, 6, 5, 7, 8), (64, 32, 3, 3, 3, 3), (1,) * 4, (1,) * 4, (1,) * 4, 1),
    (torch.float32, (1, 8, 4, 5, 4, 4, 5), (16, 8, 3, 3, 3, 3, 3), (1,) * 5, (1,) * 5, (1,) * 5,
     1),
    # strided: the input gradient runs on the generic CUDA-core kernel
    (torch.bfloat16, (2, 16, 7, 6, 8, 9), (32, 8, 3, 3, 3, 3), (2,) * 4, (1,) * 4, (1,) * 4, 2),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}".split(".")[-1] + f"_s{c[3][0]}")
def test_backward_every_output_mask_through_the_c_abi(case):
    dtype, x_shape, w_shape, stride, padding, dilation, groups = case
    library = _library()
    generator = torch.Generator().manual_seed(31)
    x = torch.randn(x_shape, generator=generator).to(dtype)
    w = (torch.randn(w_shape, generator=generator) * 0.1).to(dtype)
    out = oracle.output_shape(x_shape[2:], w_shape[2:], stride, padding, dilation)
    dy = torch.randn((x_shape[0], w_shape[0], *out), generator=generator).to(dtype)
    expected = dict(zip(("dx", "dw", "db"),
                        oracle.backward(dy, x, w, stride, padding, dilation, groups)))
    magnitudes = None
    if dtype == torch.float32:
        magnitudes = conv_magnitudes(x, w, dy, stride, padding, dilation, groups)
    xc, wc, dyc = x.cuda(), w.cuda(), dy.cuda()
    problem = _problem(library, xc, wc, stride, padding, dilation, groups)
    stream = torch.cuda.current_stream().cuda_stream
    for bits in itertools.product((0, 1), repeat=3):
        mask = (ctypes.c_int32 * 3)(*bits)
        needed = library.cnd_backward_workspace_size(ctypes.byref(problem), mask)
        workspace = torch.empty(max(needed, 1), dtype=torch.uint8, device="cuda")
        grads = {
            "dx": torch.full_like(xc, float("nan")) if bits[0] else None,
            "dw": torch.full_like(wc, float("nan")) if bits[1] else None,
            "db": torch.full((w_shape[0],), float("nan"), dtype=dtype, device="cuda")
            if bits[2] else None,
        }
        pointer = lambda t: None if t is None else t.data_ptr()
        status = library.cnd_backward(
            ctypes.byref(problem), dyc.data_ptr(), xc.data_ptr(), wc.data_ptr(),
            pointer(grads["dx"]), pointer(grads["dw"]), pointer(grads["db"]), mask,
            workspace.data_ptr() if needed else None, needed, stream)
        assert status == CND_OK, (bits, library.cnd_last_error())
        torch.cuda.synchronize()
        assert library.cnd_device_status(ctypes.c_void_p(stream)) == CND_OK
        assert_conv_matches(grads, expected, dtype, f"mask {bits}", magnitudes)

    # a workspace one byte short is refused before anything runs
    mask = (ctypes.c_int32 * 3)(1, 1, 1)
    needed = library.cnd_backward_workspace_size(ctypes.byref(problem), mask)
    if needed > 0:
        workspace = torch.empty(needed, dtype=torch.uint8, device="cuda")
        dx, dw = torch.empty_like(xc), torch.empty_like(wc)
        db = torch.empty(w_shape[0], dtype=dtype, device="cuda")
        status = library.cnd_backward(
            ctypes.byref(problem), dyc.data_ptr(), xc.data_ptr(), wc.data_ptr(), dx.data_ptr(),
            dw.data_ptr(), db.data_ptr(), mask, workspace.data_ptr(), needed - 1, stream)
        assert status == CND_ERR_WORKSPACE
        assert "workspace" in library.cnd_last_error().decode()
    # a requested gradient without a buffer is an argument error
    status = library.cnd_backward(ctypes.byref(problem), dyc.data_ptr(), xc.data_ptr(),
                                  wc.data_ptr(), None, None, None, mask, None, 0, stream)
    assert status == CND_ERR_INVALID
    assert "missing gradient buffer" in library.cnd_last_error().decode()
