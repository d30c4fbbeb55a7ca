// PyTorch dispatcher kernels for torch_convnd::conv_nd / conv_nd_backward.
//
// The reference registers its C++ implementations for the CPU, CUDA, AutocastCPU and
// AutocastCUDA keys (src/torch_convnd/csrc/convnd.cpp:435-452). This shim keeps those
// registrations and the reference's argument checks and messages, then hands dense
// device pointers to the C ABI (include/convnd_b200.h). The CPU kernels validate the
// arguments exactly like the CUDA ones (so invalid geometry reports the same error on
// any device) and then refuse: this build has no CPU implementation.
#include <ATen/ATen.h>
#include <ATen/autocast_mode.h>
#include <c10/core/DeviceGuard.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <array>
#include <string>
#include <optional>
#include <tuple>
#include <vector>

#include "convnd_b200.h"

namespace convnd_b200 {
namespace {

int32_t dtype_code(at::ScalarType type) {
  switch (type) {
    case at::kHalf:
      return CND_F16;
    case at::kBFloat16:
      return CND_BF16;
    case at::kFloat:
      return CND_F32;
    case at::kDouble:
      return CND_F64;
    default:
      return -1;
  }
}

void check_status(int status) {
  TORCH_CHECK(status == CND_OK, cnd_last_error());
}

// The reference's make_geometry checks (convnd.cpp:33-87), in its order, followed by the
// C ABI's validation of the numeric geometry.
cnd_problem make_problem(const at::Tensor& input, const at::Tensor& weight,
                         at::IntArrayRef stride, at::IntArrayRef padding,
                         at::IntArrayRef dilation, int64_t groups) {
  TORCH_CHECK(input.layout() == at::kStrided && weight.layout() == at::kStrided,
              "conv_nd requires strided tensors");
  TORCH_CHECK(input.device().is_cpu() || input.device().is_cuda(),
              "conv_nd supports CPU and CUDA tensors");
  TORCH_CHECK(dtype_code(input.scalar_type()) >= 0,
              "native conv_nd supports float16, bfloat16, float32 and float64");
  TORCH_CHECK(weight.device() == input.device() && weight.scalar_type() == input.scalar_type(),
              "input and weight must have the same device and dtype");
  TORCH_CHECK(input.dim() >= 3 && input.dim() <= CND_MAX_RANK + 2,
              "conv_nd requires 1 to 62 spatial dimensions");
  TORCH_CHECK(weight.dim() == input.dim(), "input and weight ranks must match");
  const int64_t rank = input.dim() - 2;
  TORCH_CHECK(static_cast<int64_t>(stride.size()) == rank &&
                  static_cast<int64_t>(padding.size()) == rank &&
                  static_cast<int64_t>(dilation.size()) == rank,
              "stride, padding and dilation must match the spatial rank");
  cnd_problem problem;
  const std::vector<int64_t> input_shape = input.sizes().vec();
  const std::vector<int64_t> weight_shape = weight.sizes().vec();
  check_status(cnd_problem_init(&problem, static_cast<int32_t>(rank), input_shape.data(),
                                weight_shape.data(), stride.data(), padding.data(),
                                dilation.data(), groups, dtype_code(input.scalar_type())));
  return problem;
}

std::vector<int64_t> output_shape(const at::Tensor& input, const cnd_problem& problem) {
  std::vector<int64_t> shape = {input.size(0), problem.output_channels};
  shape.insert(shape.end(), problem.output, problem.output + problem.rank);
  return shape;
}

void check_bias(const std::optional<at::Tensor>& bias, const at::Tensor& input,
                const cnd_problem& problem) {
  if (!bias.has_value()) return;
  TORCH_CHECK(bias->layout() == at::kStrided && bias->dim() == 1 &&
                  bias->size(0) == problem.output_channels && bias->device() == input.device() &&
                  bias->scalar_type() == input.scalar_type(),
              "bias must match output channels, device and dtype");
}

void check_grad_output(const at::Tensor& grad_output, const at::Tensor& input,
                       const cnd_problem& problem) {
  TORCH_CHECK(grad_output.sizes().vec() == output_shape(input, problem) &&
                  grad_output.device() == input.device() &&
                  grad_output.scalar_type() == input.scalar_type() &&
                  grad_output.layout() == at::kStrided,
              "grad_output must match the convolution output shape, device and dtype");
}

// The reference's backward validates the patch budget with 4-byte elements for 16-bit
// inputs (their gradients accumulate in fp32; on CUDA always, convnd.cpp:357-362), and
// with the element size for fp32/fp64 when dx or dW is requested on a non-empty batch
// (convnd.cpp:375, after the early return at :391-393).
void check_backward_budget(const at::Tensor& input, const cnd_problem& problem,
                           int64_t workspace_bytes, const std::array<bool, 3>& output_mask) {
  const bool low = input.scalar_type() == at::kHalf || input.scalar_type() == at::kBFloat16;
  if (!low && ((!output_mask[0] && !output_mask[1]) || input.size(0) == 0)) return;
  const int64_t element = input.element_size() > 4 ? input.element_size() : 4;
  check_status(cnd_check_workspace_budget(&problem, element, workspace_bytes));
}

// Dense channels-last activation: [N, C, d0..] stored as [N, d0.., C] (PyTorch's
// channels_last strides for any rank). A tensor that is also contiguous counts as
// channels-first. The kernels read it in place, so its data must be 16-byte aligned.
bool is_channels_last(const at::Tensor& t) {
  if (t.dim() < 3 || t.is_contiguous()) return false;
  if (reinterpret_cast<uintptr_t>(t.const_data_ptr()) % 16 != 0) return false;
  int64_t expected = 1;
  if (t.size(1) != 1 && t.stride(1) != expected) return false;
  expected *= t.size(1);
  for (int64_t a = t.dim() - 1; a >= 2; --a) {
    if (t.size(a) != 1 && t.stride(a) != expected) return false;
    expected *= t.size(a);
  }
  return t.size(0) == 1 || t.stride(0) == expected;
}

// New dense tensor of logical shape `shape` ([N, C, spatial...]), channels-last if `cl`.
at::Tensor empty_activation(std::vector<int64_t> shape, bool cl, const at::TensorOptions& options) {
  if (!cl) return at::empty(shape, options);
  std::vector<int64_t> stored = {shape[0]};
  stored.insert(stored.end(), shape.begin() + 2, shape.end());
  stored.push_back(shape[1]);
  std::vector<int64_t> order = {0, static_cast<int64_t>(shape.size()) - 1};
  for (int64_t a = 1; a + 1 < static_cast<int64_t>(shape.size()); ++a) order.push_back(a);
  return at::empty(stored, options).permute(order);
}

at::Tensor workspace_tensor(size_t bytes, const at::Tensor& like) {
  return at::empty({static_cast<int64_t>(bytes > 0 ? bytes : 1)},
                   like.options().dtype(at::kByte));
}

at::Tensor conv_nd_cuda(const at::Tensor& input, const at::Tensor& weight,
                        const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                        at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups,
                        int64_t workspace_bytes) {
  cnd_problem problem = make_problem(input, weight, stride, padding, dilation, groups);
  check_bias(bias, input, problem);
  check_status(cnd_check_workspace_budget(&problem, input.element_size(), workspace_bytes));
  const c10::cuda::CUDAGuard guard(input.device());
  // A channels-last input is read in place and gives a channels-last output (PyTorch's
  // memory-format propagation); any other layout is made contiguous, as the reference does.
  const bool cl = is_channels_last(input);
  const at::Tensor x = cl ? input : input.contiguous();
  if (cl) problem.layout = CND_LAYOUT_X_CL | CND_LAYOUT_Y_CL;
  const at::Tensor w = weight.contiguous();
  at::Tensor b;
  if (bias.has_value()) b = bias->contiguous();
  at::Tensor output = empty_activation(output_shape(input, problem), cl, input.options());
  if (input.size(0) == 0) return output;
  const size_t bytes = cnd_forward_workspace_size(&problem);
  at::Tensor workspace = workspace_tensor(bytes, input);
  const auto stream = c10::cuda::getCurrentCUDAStream(input.device().index());
  check_status(cnd_forward(&problem, x.const_data_ptr(), w.const_data_ptr(),
                           b.defined() ? b.const_data_ptr() : nullptr, output.mutable_data_ptr(),
                           workspace.mutable_data_ptr(), bytes, stream.stream()));
  return output;
}

std::tuple<std::optional<at::Tensor>, std::optional<at::Tensor>, std::optional<at::Tensor>>
conv_nd_backward_cuda(const at::Tensor& grad_output, const at::Tensor& input,
                      const at::Tensor& weight, at::IntArrayRef stride, at::IntArrayRef padding,
                      at::IntArrayRef dilation, int64_t groups, int64_t workspace_bytes,
                      std::array<bool, 3> output_mask) {
  cnd_problem problem = make_problem(input, weight, stride, padding, dilation, groups);
  check_grad_output(grad_output, input, problem);
  check_backward_budget(input, problem, workspace_bytes, output_mask);
  const c10::cuda::CUDAGuard guard(input.device());
  std::optional<at::Tensor> grad_input, grad_weight, grad_bias;
  const bool x_cl = is_channels_last(input);
  const bool dy_cl = is_channels_last(grad_output);
  problem.layout = (x_cl ? CND_LAYOUT_X_CL : 0) | (dy_cl ? CND_LAYOUT_Y_CL : 0);
  if (output_mask[0]) grad_input = empty_activation(input.sizes().vec(), x_cl, input.options());
  if (output_mask[1]) grad_weight = at::empty(weight.sizes(), weight.options());
  if (output_mask[2]) grad_bias = at::empty({problem.output_channels}, input.options());
  if (!output_mask[0] && !output_mask[1] && !output_mask[2]) {
    return {grad_input, grad_weight, grad_bias};
  }
  const at::Tensor dy = dy_cl ? grad_output : grad_output.contiguous();
  const at::Tensor x = x_cl ? input : input.contiguous();
  const at::Tensor w = weight.contiguous();
  const int32_t mask[3] = {output_mask[0], output_mask[1], output_mask[2]};
  const size_t bytes = cnd_backward_workspace_size(&problem, mask);
  at::Tensor workspace = workspace_tensor(bytes, input);
  const auto stream = c10::cuda::getCurrentCUDAStream(input.device().index());
  check_status(cnd_backward(
      &problem, dy.const_data_ptr(), x.const_data_ptr(), w.const_data_ptr(),
      grad_input ? grad_input->mutable_data_ptr() : nullptr,
      grad_weight ? grad_weight->mutable_data_ptr() : nullptr,
      grad_bias ? grad_bias->mutable_data_ptr() : nullptr, mask, workspace.mutable_data_ptr(),
      bytes, stream.stream()));
  return {grad_input, grad_weight, grad_bias};
}

int32_t activation_code(c10::string_view activation) {
  if (activation == "gelu") return CND_ACT_GELU;
  TORCH_CHECK(false, "conv_nd_act supports activation='gelu', got '", std::string(activation),
              "'");
}

// conv + bias + activation in one epilogue: (activation(y), y) with y = conv(x, w) + b, both
// in the input's layout. The pre-activation output is what the backward needs.
std::tuple<at::Tensor, at::Tensor> conv_nd_act_cuda(
    const at::Tensor& input, const at::Tensor& weight, const std::optional<at::Tensor>& bias,
    at::IntArrayRef stride, at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups,
    int64_t workspace_bytes, c10::string_view activation) {
  const int32_t act = activation_code(activation);
  cnd_problem problem = make_problem(input, weight, stride, padding, dilation, groups);
  check_bias(bias, input, problem);
  check_status(cnd_check_workspace_budget(&problem, input.element_size(), workspace_bytes));
  const c10::cuda::CUDAGuard guard(input.device());
  const bool cl = is_channels_last(input);
  const at::Tensor x = cl ? input : input.contiguous();
  problem.layout = (cl ? CND_LAYOUT_X_CL | CND_LAYOUT_Y_CL : 0) | (act << CND_LAYOUT_ACT_SHIFT);
  const at::Tensor w = weight.contiguous();
  at::Tensor b;
  if (bias.has_value()) b = bias->contiguous();
  at::Tensor output = empty_activation(output_shape(input, problem), cl, input.options());
  at::Tensor pre = empty_activation(output_shape(input, problem), cl, input.options());
  if (input.size(0) == 0) return {output, pre};
  const size_t bytes = cnd_forward_workspace_size(&problem);
  at::Tensor workspace = workspace_tensor(bytes, input);
  const auto stream = c10::cuda::getCurrentCUDAStream(input.device().index());
  check_status(cnd_forward_act(&problem, x.const_data_ptr(), w.const_data_ptr(),
                               b.defined() ? b.const_data_ptr() : nullptr,
                               output.mutable_data_ptr(), pre.mutable_data_ptr(), act,
                               workspace.mutable_data_ptr(), bytes, stream.stream()));
  return {output, pre};
}

std::tuple<std::optional<at::Tensor>, std::optional<at::Tensor>, std::optional<at::Tensor>>
conv_nd_act_backward_cuda(const at::Tensor& grad_output, const at::Tensor& pre_activation,
                          const at::Tensor& input, const at::Tensor& weight,
                          at::IntArrayRef stride, at::IntArrayRef padding,
                          at::IntArrayRef dilation, int64_t groups, int64_t workspace_bytes,
                          c10::string_view activation, std::array<bool, 3> output_mask) {
  const int32_t act = activation_code(activation);
  cnd_problem problem = make_problem(input, weight, stride, padding, dilation, groups);
  check_grad_output(grad_output, input, problem);
  check_grad_output(pre_activation, input, problem);
  check_backward_budget(input, problem, workspace_bytes, output_mask);
  const c10::cuda::CUDAGuard guard(input.device());
  std::optional<at::Tensor> grad_input, grad_weight, grad_bias;
  const bool x_cl = is_channels_last(input);
  const bool dy_cl = is_channels_last(grad_output);
  problem.layout = (x_cl ? CND_LAYOUT_X_CL : 0) | (dy_cl ? CND_LAYOUT_Y_CL : 0) |
                   (act << CND_LAYOUT_ACT_SHIFT);
  if (output_mask[0]) grad_input = empty_activation(input.sizes().vec(), x_cl, input.options());
  if (output_mask[1]) grad_weight = at::empty(weight.sizes(), weight.options());
  if (output_mask[2]) grad_bias = at::empty({problem.output_channels}, input.options());
  if (!output_mask[0] && !output_mask[1] && !output_mask[2]) {
    return {grad_input, grad_weight, grad_bias};
  }
  const at::Tensor dy = dy_cl ? grad_output : grad_output.contiguous();
  // the pre-activation is read with dy's indexing: same layout as dy
  at::Tensor pre = pre_activation;
  if (dy_cl != is_channels_last(pre) || (!dy_cl && !pre.is_contiguous())) {
    pre = empty_activation(pre_activation.sizes().vec(), dy_cl, pre_activation.options());
    pre.copy_(pre_activation);
  }
  const at::Tensor x = x_cl ? input : input.contiguous();
  const at::Tensor w = weight.contiguous();
  const int32_t mask[3] = {output_mask[0], output_mask[1], output_mask[2]};
  const size_t bytes = cnd_backward_workspace_size(&problem, mask);
  at::Tensor workspace = workspace_tensor(bytes, input);
  const auto stream = c10::cuda::getCurrentCUDAStream(input.device().index());
  check_status(cnd_backward_act(
      &problem, dy.const_data_ptr(), pre.const_data_ptr(), act, x.const_data_ptr(),
      w.const_data_ptr(), grad_input ? grad_input->mutable_data_ptr() : nullptr,
      grad_weight ? grad_weight->mutable_data_ptr() : nullptr,
      grad_bias ? grad_bias->mutable_data_ptr() : nullptr, mask, workspace.mutable_data_ptr(),
      bytes, stream.stream()));
  return {grad_input, grad_weight, grad_bias};
}

[[noreturn]] void refuse_cpu() {
  TORCH_CHECK(false,
              "torch_convnd B200 build: the native convolution runs on CUDA devices only; "
              "move the tensors to a CUDA device");
}

at::Tensor conv_nd_cpu(const at::Tensor& input, const at::Tensor& weight,
                       const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                       at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups,
                       int64_t workspace_bytes) {
  cnd_problem problem = make_problem(input, weight, stride, padding, dilation, groups);
  check_bias(bias, input, problem);
  check_status(cnd_check_workspace_budget(&problem, input.element_size(), workspace_bytes));
  refuse_cpu();
}

std::tuple<std::optional<at::Tensor>, std::optional<at::Tensor>, std::optional<at::Tensor>>
conv_nd_backward_cpu(const at::Tensor& grad_output, const at::Tensor& input,
                     const at::Tensor& weight, at::IntArrayRef stride, at::IntArrayRef padding,
                     at::IntArrayRef dilation, int64_t groups, int64_t workspace_bytes,
                     std::array<bool, 3> output_mask) {
  cnd_problem problem = make_problem(input, weight, stride, padding, dilation, groups);
  check_grad_output(grad_output, input, problem);
  // The reference's CPU path promotes 16-bit inputs to fp32 and then applies the fp32
  // rule (convnd.cpp:363-366).
  if ((output_mask[0] || output_mask[1]) && input.size(0) > 0) {
    const int64_t element = input.element_size() > 4 ? input.element_size() : 4;
    check_status(cnd_check_workspace_budget(&problem, element, workspace_bytes));
  }
  refuse_cpu();
}

std::tuple<at::Tensor, at::Tensor> conv_nd_act_cpu(
    const at::Tensor& input, const at::Tensor& weight, const std::optional<at::Tensor>& bias,
    at::IntArrayRef stride, at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups,
    int64_t workspace_bytes, c10::string_view activation) {
  activation_code(activation);
  cnd_problem problem = make_problem(input, weight, stride, padding, dilation, groups);
  check_bias(bias, input, problem);
  check_status(cnd_check_workspace_budget(&problem, input.element_size(), workspace_bytes));
  refuse_cpu();
}

std::tuple<std::optional<at::Tensor>, std::optional<at::Tensor>, std::optional<at::Tensor>>
conv_nd_act_backward_cpu(const at::Tensor& grad_output, const at::Tensor& pre_activation,
                         const at::Tensor& input, const at::Tensor& weight,
                         at::IntArrayRef stride, at::IntArrayRef padding,
                         at::IntArrayRef dilation, int64_t groups, int64_t workspace_bytes,
                         c10::string_view activation, std::array<bool, 3> output_mask) {
  activation_code(activation);
  cnd_problem problem = make_problem(input, weight, stride, padding, dilation, groups);
  check_grad_output(grad_output, input, problem);
  check_grad_output(pre_activation, input, problem);
  (void)workspace_bytes;
  (void)output_mask;
  refuse_cpu();
}

// Autocast: cast floating operands to the autocast dtype, then redispatch below the
// autocast key (the standard PyTorch pattern the reference also uses, convnd.cpp:417-431).
template <c10::DeviceType Device>
at::Tensor conv_nd_autocast(const at::Tensor& input, const at::Tensor& weight,
                            const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                            at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups,
                            int64_t workspace_bytes) {
  const c10::impl::ExcludeDispatchKeyGuard no_autocast(
      at::autocast::get_autocast_dispatch_key_from_device_type(Device));
  const at::ScalarType target = at::autocast::get_autocast_dtype(Device);
  static const auto op = c10::Dispatcher::singleton()
                             .findSchemaOrThrow("torch_convnd::conv_nd", "")
                             .typed<decltype(conv_nd_cuda)>();
  return op.call(at::autocast::cached_cast(target, input, Device),
                 at::autocast::cached_cast(target, weight, Device),
                 at::autocast::cached_cast(target, bias, Device), stride, padding, dilation,
                 groups, workspace_bytes);
}

template <c10::DeviceType Device>
std::tuple<at::Tensor, at::Tensor> conv_nd_act_autocast(
    const at::Tensor& input, const at::Tensor& weight, const std::optional<at::Tensor>& bias,
    at::IntArrayRef stride, at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups,
    int64_t workspace_bytes, c10::string_view activation) {
  const c10::impl::ExcludeDispatchKeyGuard no_autocast(
      at::autocast::get_autocast_dispatch_key_from_device_type(Device));
  const at::ScalarType target = at::autocast::get_autocast_dtype(Device);
  static const auto op = c10::Dispatcher::singleton()
                             .findSchemaOrThrow("torch_convnd::conv_nd_act", "")
                             .typed<decltype(conv_nd_act_cuda)>();
  return op.call(at::autocast::cached_cast(target, input, Device),
                 at::autocast::cached_cast(target, weight, Device),
                 at::autocast::cached_cast(target, bias, Device), stride, padding, dilation,
                 groups, workspace_bytes, activation);
}

}  // namespace
}  // namespace convnd_b200

TORCH_LIBRARY_IMPL(torch_convnd, CUDA, library) {
  library.impl("conv_nd", &convnd_b200::conv_nd_cuda);
  library.impl("conv_nd_backward", &convnd_b200::conv_nd_backward_cuda);
  library.impl("conv_nd_act", &convnd_b200::conv_nd_act_cuda);
  library.impl("conv_nd_act_backward", &convnd_b200::conv_nd_act_backward_cuda);
}

TORCH_LIBRARY_IMPL(torch_convnd, AutocastCUDA, library) {
  library.impl("conv_nd", &convnd_b200::conv_nd_autocast<c10::DeviceType::CUDA>);
  library.impl("conv_nd_act", &convnd_b200::conv_nd_act_autocast<c10::DeviceType::CUDA>);
}

TORCH_LIBRARY_IMPL(torch_convnd, CPU, library) {
  library.impl("conv_nd", &convnd_b200::conv_nd_cpu);
  library.impl("conv_nd_backward", &convnd_b200::conv_nd_backward_cpu);
  library.impl("conv_nd_act", &convnd_b200::conv_nd_act_cpu);
  library.impl("conv_nd_act_backward", &convnd_b200::conv_nd_act_backward_cpu);
}

TORCH_LIBRARY_IMPL(torch_convnd, AutocastCPU, library) {
  library.impl("conv_nd", &convnd_b200::conv_nd_autocast<c10::DeviceType::CPU>);
  library.impl("conv_nd_act", &convnd_b200::conv_nd_act_autocast<c10::DeviceType::CPU>);
}
