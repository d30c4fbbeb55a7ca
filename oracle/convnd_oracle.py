"""CPU oracle for the N-D convolution hot path.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may
import this module, and only as the checker; the product path (torch_convnd) never
touches it.

Two independent float64 restatements of what the reference computes:

* ``forward`` / ``backward`` restate the reference's native algorithm
  (src/torch_convnd/csrc/convnd.cpp:305-415): per image, an im2col "unfold" of the input
  into columns [groups, C/g * taps, positions] using the row/position -> input-offset map
  of ``column_input_offset`` (csrc/convnd.h:57-76; -1 marks zero padding), a batched GEMM
  with the weight viewed as [groups, Cout/g, C/g * taps], the bias added afterwards
  (convnd.cpp:337-341); backward computes grad_bias = sum(dY) (convnd.cpp:388-390),
  grad_weight += dY . columns^T (convnd.cpp:402-406) and grad_input = fold(W^T . dY), the
  fold scattering each column entry back to its input offset (convnd_cuda.cu:147-169).
  Everything runs in float64 on inputs given in any dtype (upcast first), which is how
  BASELINE's oracle is defined ("an fp64 run of the reference path").

* ``tap_reference`` restates the reference tests' independent check
  (tests/test_convnd.py:38-67): one channel contraction per tap over padded, strided,
  dilated slices. No index map is shared with the first restatement. ``tap_dgrad`` and
  ``tap_wgrad`` are its adjoints, tap by tap (the input gradient scatters each tap's
  contraction back into the same padded slices; the weight gradient contracts each tap's
  slice with dY), the derivatives autograd takes of the reference tests' formula. These
  three run on whatever device their tensors are on, so full-size checks can run them
  in float64 on the GPU that is being tested (as checker only).

Both are pinned against golden vectors produced by the reference itself
(tests/golden/make_golden.py runs the reference's backend='torch' in float64).
"""

from __future__ import annotations

import itertools
import math

import torch


def output_shape(spatial, kernel, stride, padding, dilation):
    """Output extents (reference make_geometry, convnd.cpp:72-78)."""
    result = []
    for size, k, s, p, d in zip(spatial, kernel, stride, padding, dilation, strict=True):
        effective = d * (k - 1) + 1
        if size + 2 * p < effective:
            raise RuntimeError("kernel exceeds padded input")
        result.append((size + 2 * p - effective) // s + 1)
    return tuple(result)


def column_offsets(spatial, kernel, stride, padding, dilation, channels):
    """Input offsets of every (row, position) of the unfolded matrix, -1 for padding.

    Rows enumerate (channel, tap) with the tap row-major over the kernel axes; positions
    enumerate output positions row-major. Offsets index one image [C, *spatial].
    """
    out = output_shape(spatial, kernel, stride, padding, dilation)
    taps = math.prod(kernel)
    positions = math.prod(out)
    tap = torch.arange(taps).unsqueeze(1)  # [taps, 1]
    pos = torch.arange(positions).unsqueeze(0)  # [1, positions]
    offset = torch.zeros(taps, positions, dtype=torch.int64)
    inside = torch.ones(taps, positions, dtype=torch.bool)
    multiplier = 1
    t, q = tap.clone(), pos.clone()
    for axis in range(len(spatial) - 1, -1, -1):
        coord = (q % out[axis]) * stride[axis] - padding[axis] + (t % kernel[axis]) * dilation[axis]
        inside &= (coord >= 0) & (coord < spatial[axis])
        offset = offset + coord * multiplier
        multiplier *= spatial[axis]
        q = q // out[axis]
        t = t // kernel[axis]
    volume = math.prod(spatial)
    rows = []
    for c in range(channels):
        rows.append(torch.where(inside, offset + c * volume, torch.full_like(offset, -1)))
    return torch.cat(rows, 0), out  # [channels * taps, positions]


def _unfold(image, offsets):
    flat = image.reshape(-1)
    safe = offsets.clamp_min(0)
    values = flat[safe]
    return torch.where(offsets >= 0, values, torch.zeros((), dtype=values.dtype))


def forward(x, w, b, stride, padding, dilation, groups):
    """y = conv(x, w) + b in float64 via unfold + GEMM (reference convnd.cpp:305-343)."""
    x = x.detach().to(torch.float64)
    w = w.detach().to(torch.float64)
    n, c = x.shape[:2]
    spatial, kernel = tuple(x.shape[2:]), tuple(w.shape[2:])
    cout = w.shape[0]
    cg = c // groups
    offsets, out = column_offsets(spatial, kernel, stride, padding, dilation, cg)
    taps = math.prod(kernel)
    flat_w = w.reshape(groups, cout // groups, cg * taps)
    y = torch.empty(n, groups, cout // groups, math.prod(out), dtype=torch.float64)
    for image in range(n):
        for g in range(groups):
            cols = _unfold(x[image, g * cg : (g + 1) * cg], offsets)
            y[image, g] = flat_w[g] @ cols
    y = y.reshape(n, cout, *out)
    if b is not None:
        y = y + b.detach().to(torch.float64).reshape(1, -1, *([1] * len(spatial)))
    return y


def backward(dy, x, w, stride, padding, dilation, groups, mask=(True, True, True)):
    """(dx, dw, db) in float64 (reference convnd.cpp:345-415)."""
    dy = dy.detach().to(torch.float64)
    x = x.detach().to(torch.float64)
    w = w.detach().to(torch.float64)
    n, c = x.shape[:2]
    spatial, kernel = tuple(x.shape[2:]), tuple(w.shape[2:])
    cout = w.shape[0]
    cg, og = c // groups, cout // groups
    offsets, out = column_offsets(spatial, kernel, stride, padding, dilation, cg)
    taps = math.prod(kernel)
    flat_w = w.reshape(groups, og, cg * taps)
    flat_dy = dy.reshape(n, groups, og, math.prod(out))
    dx = torch.zeros_like(x) if mask[0] else None
    dw = torch.zeros(groups, og, cg * taps, dtype=torch.float64) if mask[1] else None
    db = flat_dy.sum(dim=(0, 3)).reshape(cout) if mask[2] else None
    valid = offsets >= 0
    for image in range(n):
        for g in range(groups):
            grad = flat_dy[image, g]  # [og, positions]
            if mask[1]:
                cols = _unfold(x[image, g * cg : (g + 1) * cg], offsets)
                dw[g] += grad @ cols.T
            if mask[0]:
                dcols = flat_w[g].T @ grad  # [cg*taps, positions]
                target = dx[image, g * cg : (g + 1) * cg].reshape(-1)
                target.index_add_(0, offsets[valid], dcols[valid])
    if mask[1]:
        dw = dw.reshape(w.shape)
    return dx, dw, db


def tap_reference(x, w, b, stride, padding, dilation, groups):
    """Independent tap-by-tap float64 convolution (reference tests/test_convnd.py:38-67)."""
    x = x.detach().to(torch.float64)
    w = w.detach().to(torch.float64)
    rank = x.ndim - 2
    padded = torch.nn.functional.pad(x, tuple(v for p in reversed(padding) for v in (p, p)))
    out = output_shape(x.shape[2:], w.shape[2:], stride, padding, dilation)
    total = None
    for tap in itertools.product(*(range(k) for k in w.shape[2:])):
        slices = tuple(
            slice(t * d, t * d + size * s, s)
            for t, d, size, s in zip(tap, dilation, out, stride, strict=True)
        )
        patch = padded[(slice(None), slice(None), *slices)].reshape(
            x.shape[0], groups, x.shape[1] // groups, -1
        )
        coefficient = w[(slice(None), slice(None), *tap)].reshape(
            groups, w.shape[0] // groups, x.shape[1] // groups
        )
        term = torch.einsum("goc,bgcp->bgop", coefficient, patch)
        total = term if total is None else total + term
    result = total.reshape(x.shape[0], w.shape[0], *out)
    if b is not None:
        result = result + b.detach().to(torch.float64).reshape(1, -1, *((1,) * rank))
    return result


def _tap_slices(tap, dilation, out, stride):
    return tuple(slice(t * d, t * d + size * s, s)
                 for t, d, size, s in zip(tap, dilation, out, stride, strict=True))


def tap_dgrad(dy, w, input_spatial, stride, padding, dilation, groups):
    """float64 input gradient, tap by tap: the adjoint of ``tap_reference`` (each tap's
    W^T . dY added into the padded input slice that the tap reads; padding cropped)."""
    dy = dy.detach().to(torch.float64)
    w = w.detach().to(torch.float64)
    batch, cout = dy.shape[:2]
    out = tuple(dy.shape[2:])
    cg = w.shape[1]
    padded_shape = tuple(size + 2 * p for size, p in zip(input_spatial, padding, strict=True))
    grad = torch.zeros((batch, groups * cg, *padded_shape), dtype=torch.float64,
                       device=dy.device)
    flat_dy = dy.reshape(batch, groups, cout // groups, -1)
    for tap in itertools.product(*(range(k) for k in w.shape[2:])):
        coefficient = w[(slice(None), slice(None), *tap)].reshape(groups, cout // groups, cg)
        term = torch.einsum("goc,bgop->bgcp", coefficient, flat_dy)
        region = grad[(slice(None), slice(None), *_tap_slices(tap, dilation, out, stride))]
        region += term.reshape(batch, groups * cg, *out)
    crop = tuple(slice(p, p + size) for p, size in zip(padding, input_spatial, strict=True))
    return grad[(slice(None), slice(None), *crop)].contiguous()


def tap_wgrad(dy, x, kernel, stride, padding, dilation, groups):
    """float64 weight gradient, tap by tap: each tap's padded input slice contracted
    with dY over the batch and the output positions."""
    dy = dy.detach().to(torch.float64)
    x = x.detach().to(torch.float64)
    batch, cin = x.shape[:2]
    cout = dy.shape[1]
    out = tuple(dy.shape[2:])
    padded = torch.nn.functional.pad(x, tuple(v for p in reversed(padding) for v in (p, p)))
    flat_dy = dy.reshape(batch, groups, cout // groups, -1)
    grad = torch.empty((cout, cin // groups, *kernel), dtype=torch.float64, device=dy.device)
    for tap in itertools.product(*(range(k) for k in kernel)):
        patch = padded[(slice(None), slice(None), *_tap_slices(tap, dilation, out, stride))]
        patch = patch.reshape(batch, groups, cin // groups, -1)
        term = torch.einsum("bgop,bgcp->goc", flat_dy, patch)
        grad[(slice(None), slice(None), *tap)] = term.reshape(cout, cin // groups)
    return grad


def sampled_forward(x, w, b, stride, padding, dilation, groups, points):
    """Exact float64 outputs at sampled (n, co, out-coordinate) points, for full-size
    property checks where the whole oracle would take too long (reference
    convnd.cpp:305-343 evaluated at single output positions)."""
    x = x.detach()
    w = w.detach().to(torch.float64)
    rank = x.ndim - 2
    cg = x.shape[1] // groups
    og = w.shape[0] // groups
    values = []
    for n, co, coords in points:
        g = co // og
        total = 0.0 if b is None else float(b[co])
        for tap in itertools.product(*(range(k) for k in w.shape[2:])):
            idx = []
            ok = True
            for axis in range(rank):
                c = coords[axis] * stride[axis] - padding[axis] + tap[axis] * dilation[axis]
                if c < 0 or c >= x.shape[2 + axis]:
                    ok = False
                    break
                idx.append(c)
            if not ok:
                continue
            column = x[(n, slice(g * cg, (g + 1) * cg), *idx)].to(torch.float64)
            total += float((w[(co, slice(None), *tap)] * column).sum())
        values.append(total)
    return torch.tensor(values, dtype=torch.float64)


def sampled_dgrad(dy, w, input_spatial, stride, padding, dilation, groups, points):
    """Exact float64 input gradients at sampled (n, ci, in-coordinate) points: the sum over
    the output channels of ci's group and the taps whose output position
    o = (i + p - t*d) / s is integral and in range (the fold of reference
    convnd_cuda.cu:147-169, evaluated at single input positions)."""
    dy = dy.detach()
    w = w.detach().to(torch.float64)
    rank = dy.ndim - 2
    cg = w.shape[1]
    og = w.shape[0] // groups
    out = dy.shape[2:]
    values = []
    for n, ci, coords in points:
        g, cl = divmod(ci, cg)
        total = 0.0
        for tap in itertools.product(*(range(k) for k in w.shape[2:])):
            idx = []
            for axis in range(rank):
                q = coords[axis] + padding[axis] - tap[axis] * dilation[axis]
                if q < 0 or q % stride[axis] != 0 or q // stride[axis] >= out[axis]:
                    break
                idx.append(q // stride[axis])
            else:
                grads = dy[(n, slice(g * og, (g + 1) * og), *idx)].to(torch.float64)
                total += float((w[(slice(g * og, (g + 1) * og), cl, *tap)] * grads).sum())
        values.append(total)
    del input_spatial  # the input extents bound the points, not the sum
    return torch.tensor(values, dtype=torch.float64)


def sampled_wgrad(dy, x, kernel, stride, padding, dilation, groups, entries):
    """Exact float64 weight gradients at sampled (co, ci_in_group, tap) entries: the sum
    over the batch and every output position whose input tap stays inside the input
    (reference convnd.cpp:402-406, one entry of grad_weight at a time)."""
    dy = dy.detach()
    x = x.detach()
    rank = x.ndim - 2
    cg = x.shape[1] // groups
    og = dy.shape[1] // groups
    out = dy.shape[2:]
    values = []
    for co, cl, tap in entries:
        g = co // og
        out_slices, in_slices = [], []
        empty = False
        for axis in range(rank):
            s, p, d, size = stride[axis], padding[axis], dilation[axis], x.shape[2 + axis]
            shift = tap[axis] * d - p  # input = o * s + shift
            lo = 0
            while lo < out[axis] and lo * s + shift < 0:
                lo += 1
            hi = out[axis]
            while hi > lo and (hi - 1) * s + shift >= size:
                hi -= 1
            if hi <= lo:
                empty = True
                break
            out_slices.append(slice(lo, hi))
            in_slices.append(slice(lo * s + shift, (hi - 1) * s + shift + 1, s))
        if empty:
            values.append(0.0)
            continue
        a = dy[(slice(None), co, *out_slices)].to(torch.float64)
        b = x[(slice(None), g * cg + cl, *in_slices)].to(torch.float64)
        values.append(float((a * b).sum()))
    del kernel
    return torch.tensor(values, dtype=torch.float64)
