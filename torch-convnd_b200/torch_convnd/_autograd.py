"""Fake (meta) kernels, derivative formulas and batching rule of the torch_convnd operators.

Registered from Python like the reference's ``_autograd.py`` (fake kernels :8-26,
autograd :29-46, double backward :49-90, vmap :93-149): the forward saves (input, weight) and its
backward calls ``conv_nd_backward`` with ``output_mask = [needs dx, needs dW, has bias
and needs db]``, so frozen inputs cost no work (a c5-style first layer whose input is
data runs forward + wgrad only).
"""

from __future__ import annotations

import torch

from ._layout import empty_activation, is_channels_last


def _output_extent(size, kernel, step, pad, dil):
    return (size + 2 * pad - dil * (kernel - 1) - 1) // step + 1


def _fake_forward(input, weight, bias, stride, padding, dilation, groups, workspace_bytes):
    shape = [input.shape[0], weight.shape[0]]
    for size, kernel, step, pad, dil in zip(
        input.shape[2:], weight.shape[2:], stride, padding, dilation, strict=True
    ):
        shape.append(_output_extent(size, kernel, step, pad, dil))
    # a channels-last input gives a channels-last output (the shim's layout rule)
    return empty_activation(shape, is_channels_last(input), input)


def _fake_backward(
    grad_output, input, weight, stride, padding, dilation, groups, workspace_bytes, output_mask
):
    contiguous = torch.contiguous_format
    grad_input = (empty_activation(list(input.shape), is_channels_last(input), input)
                  if output_mask[0] else None)
    grad_weight = torch.empty_like(weight, memory_format=contiguous) if output_mask[1] else None
    grad_bias = input.new_empty(weight.shape[0]) if output_mask[2] else None
    return grad_input, grad_weight, grad_bias


def _setup_context(ctx, inputs, output):
    input, weight, bias, *geometry = inputs
    ctx.save_for_backward(input, weight)
    ctx.geometry = geometry
    ctx.has_bias = bias is not None


def _backward(ctx, grad_output):
    input, weight = ctx.saved_tensors
    needs = ctx.needs_input_grad
    mask = [needs[0], needs[1], ctx.has_bias and needs[2]]
    grads = torch.ops.torch_convnd.conv_nd_backward.default(
        grad_output, input, weight, *ctx.geometry, mask
    )
    return (*grads, None, None, None, None, None)


def _setup_backward_context(ctx, inputs, output):
    grad_output, input, weight, *rest = inputs
    ctx.save_for_backward(grad_output, input, weight)
    ctx.geometry = rest[:-1]  # stride, padding, dilation, groups, workspace_bytes


def _backward_backward(ctx, gg_input, gg_weight, gg_bias):
    """Derivatives of (dx, dW, db) = conv_nd_backward(dy, x, W).

    dx is bilinear in (dy, W), dW in (dy, x) and db linear in dy, so every term is one
    more forward or backward convolution with the same geometry.
    """
    grad_output, input, weight = ctx.saved_tensors
    geometry = ctx.geometry
    needs = ctx.needs_input_grad
    d_grad_output = d_input = d_weight = None
    terms = []
    with torch.autocast(device_type=input.device.type, enabled=False):
        if gg_input is not None:
            if needs[0]:
                terms.append(
                    torch.ops.torch_convnd.conv_nd.default(gg_input, weight, None, *geometry)
                )
            if needs[2]:
                d_weight = torch.ops.torch_convnd.conv_nd_backward.default(
                    grad_output, gg_input, weight, *geometry, [False, True, False]
                )[1]
        if gg_weight is not None:
            if needs[0]:
                terms.append(
                    torch.ops.torch_convnd.conv_nd.default(input, gg_weight, None, *geometry)
                )
            if needs[1]:
                d_input = torch.ops.torch_convnd.conv_nd_backward.default(
                    grad_output, input, gg_weight, *geometry, [True, False, False]
                )[0]
        if gg_bias is not None and needs[0]:
            shape = (1, -1) + (1,) * (input.ndim - 2)
            terms.append(gg_bias.reshape(shape).expand_as(grad_output))
    for term in terms:
        d_grad_output = term if d_grad_output is None else d_grad_output + term
    return d_grad_output, d_input, d_weight, None, None, None, None, None, None


def _vmap_conv_nd(info, in_dims, input, weight, bias, stride, padding, dilation, groups,
                  workspace_bytes):
    """Batching rule of conv_nd (the reference registers one too, _autograd.py:93-134).

    The mapped dimension folds into the operator's own dimensions, so a vmapped call is
    one native launch: into the batch when only the input is mapped; into the groups when
    the weight (or the bias) is mapped: input [V, N, C, ...] -> [N, V*C, ...], weight
    [V, Cout, C/g, ...] -> [V*Cout, C/g, ...], groups g -> V*g, output [N, V*Cout, ...]
    -> [V, N, Cout, ...].
    """
    size = info.batch_size
    x_dim, w_dim, b_dim = in_dims[:3]
    if w_dim is None and b_dim is None:
        mapped = input.movedim(x_dim, 0)
        output = torch.ops.torch_convnd.conv_nd.default(
            mapped.flatten(0, 1), weight, bias, stride, padding, dilation, groups,
            workspace_bytes)
        return output.unflatten(0, (size, mapped.shape[1])), 0
    x = input.movedim(x_dim, 0) if x_dim is not None else input.expand(size, *input.shape)
    w = weight.movedim(w_dim, 0) if w_dim is not None else weight.expand(size, *weight.shape)
    batch, channels = x.shape[1], x.shape[2]
    cout = w.shape[1]
    if size == 0:
        spatial = [_output_extent(s, k, st, p, d) for s, k, st, p, d in
                   zip(x.shape[3:], w.shape[3:], stride, padding, dilation, strict=True)]
        return x.new_empty((0, batch, cout, *spatial)), 0
    folded_x = x.movedim(0, 1).reshape(batch, size * channels, *x.shape[3:])
    folded_w = w.reshape(size * cout, *w.shape[2:])
    folded_b = None
    if bias is not None:
        b = bias.movedim(b_dim, 0) if b_dim is not None else bias.expand(size, *bias.shape)
        folded_b = b.reshape(size * cout)
    output = torch.ops.torch_convnd.conv_nd.default(
        folded_x, folded_w, folded_b, stride, padding, dilation, groups * size, workspace_bytes)
    return output.unflatten(1, (size, cout)).movedim(1, 0), 0


def _fake_forward_act(input, weight, bias, stride, padding, dilation, groups, workspace_bytes,
                      activation):
    output = _fake_forward(input, weight, bias, stride, padding, dilation, groups,
                           workspace_bytes)
    return output, torch.empty_like(output)


def _fake_backward_act(grad_output, pre_activation, input, weight, stride, padding, dilation,
                       groups, workspace_bytes, activation, output_mask):
    return _fake_backward(grad_output, input, weight, stride, padding, dilation, groups,
                          workspace_bytes, output_mask)


def _setup_context_act(ctx, inputs, output):
    input, weight, bias, *geometry = inputs
    ctx.save_for_backward(input, weight, output[1])
    # An unused pre-activation output must arrive as None, not as a materialised zero
    # gradient (which would turn every backward into the eager fallback below).
    ctx.set_materialize_grads(False)
    ctx.geometry = geometry[:-1]  # stride, padding, dilation, groups, workspace_bytes
    ctx.activation = geometry[-1]
    ctx.has_bias = bias is not None


def _backward_act(ctx, grad_output, grad_pre):
    """Gradients of (activation(y), y), y = conv(x, W) + b: the activation's backward is
    fused into the native backward's dy pack. A gradient reaching the pre-activation output
    directly (rare) is added to the activation's backward in eager ops first."""
    input, weight, pre = ctx.saved_tensors
    needs = ctx.needs_input_grad
    mask = [needs[0], needs[1], ctx.has_bias and needs[2]]
    if grad_output is None and grad_pre is None:
        return (None,) * 9
    if grad_pre is None:
        grads = torch.ops.torch_convnd.conv_nd_act_backward.default(
            grad_output, pre, input, weight, *ctx.geometry, ctx.activation, mask)
    else:
        grad = grad_pre
        if grad_output is not None:
            grad = grad + torch.ops.aten.gelu_backward(grad_output, pre)
        grads = torch.ops.torch_convnd.conv_nd_backward.default(
            grad, input, weight, *ctx.geometry, mask)
    return (*grads, None, None, None, None, None, None)


def register_training() -> None:
    torch.library.register_fake("torch_convnd::conv_nd")(_fake_forward)
    torch.library.register_fake("torch_convnd::conv_nd_backward")(_fake_backward)
    torch.library.register_autograd(
        "torch_convnd::conv_nd", _backward, setup_context=_setup_context
    )
    torch.library.register_autograd(
        "torch_convnd::conv_nd_backward",
        _backward_backward,
        setup_context=_setup_backward_context,
    )
    torch.library.register_vmap("torch_convnd::conv_nd", _vmap_conv_nd)
    torch.library.register_fake("torch_convnd::conv_nd_act")(_fake_forward_act)
    torch.library.register_fake("torch_convnd::conv_nd_act_backward")(_fake_backward_act)
    torch.library.register_autograd(
        "torch_convnd::conv_nd_act", _backward_act, setup_context=_setup_context_act
    )
