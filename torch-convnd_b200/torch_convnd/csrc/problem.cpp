// Geometry validation and error reporting of the C ABI (no CUDA, no torch).
//
// cnd_problem_init restates the checks of the reference's make_geometry
// (src/torch_convnd/csrc/convnd.cpp:33-87) and cnd_check_workspace_budget restates
// tile_size (convnd.cpp:89-100). The texts are kept identical because callers and
// tests match on them (tests/test_convnd.py:260-317).
#include "internal.h"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <limits>
#include <string>

namespace cnd {

namespace {
thread_local std::string g_last_error;
int g_default_fp32_mode = CND_FP32_3XTF32;
}

int default_fp32_mode() { return g_default_fp32_mode; }
void set_default_fp32_mode(int mode) { g_default_fp32_mode = mode; }

int fail(int status, const char* format, ...) {
  char buffer[1024];
  va_list args;
  va_start(args, format);
  std::vsnprintf(buffer, sizeof(buffer), format, args);
  va_end(args);
  g_last_error = buffer;
  return status;
}

void clear_error() { g_last_error.clear(); }

const char* last_error() { return g_last_error.c_str(); }

namespace {

// Overflow-checked arithmetic on nonnegative int64 (reference convnd.cpp:19-31).
bool checked_product(int64_t left, int64_t right, int64_t* result) {
  if (left < 0 || right < 0) return false;
  if (right != 0 && left > std::numeric_limits<int64_t>::max() / right) return false;
  *result = left * right;
  return true;
}

bool checked_sum(int64_t left, int64_t right, int64_t* result) {
  if (left < 0 || right < 0) return false;
  if (left > std::numeric_limits<int64_t>::max() - right) return false;
  *result = left + right;
  return true;
}

}  // namespace
}  // namespace cnd

extern "C" {

const char* cnd_last_error(void) { return cnd::last_error(); }

int cnd_set_default_fp32_mode(int32_t mode) {
  const int previous = cnd::default_fp32_mode();
  if (mode >= CND_FP32_3XTF32 && mode <= CND_FP32_SIMT) cnd::set_default_fp32_mode(mode);
  return previous;
}

const char* cnd_version(void) { return "convnd_b200 0.1.0 (sm_100a)"; }

int cnd_problem_init(cnd_problem* problem, int32_t rank, const int64_t* input_shape,
                     const int64_t* weight_shape, const int64_t* stride,
                     const int64_t* padding, const int64_t* dilation, int64_t groups,
                     int32_t dtype) {
  using cnd::fail;
  cnd::clear_error();
  if (problem == nullptr || input_shape == nullptr || weight_shape == nullptr ||
      stride == nullptr || padding == nullptr || dilation == nullptr) {
    return fail(CND_ERR_INVALID, "cnd_problem_init: null argument");
  }
  std::memset(problem, 0, sizeof(*problem));
  if (dtype < CND_F16 || dtype > CND_F64) {
    return fail(CND_ERR_UNSUPPORTED,
                "native conv_nd supports float16, bfloat16, float32 and float64");
  }
  if (rank < 1 || rank > CND_MAX_RANK) {
    return fail(CND_ERR_INVALID, "conv_nd requires 1 to 62 spatial dimensions");
  }
  problem->rank = rank;
  problem->dtype = dtype;
  problem->fp32_mode = cnd::default_fp32_mode();
  if (groups <= 0) return fail(CND_ERR_INVALID, "groups must be positive");
  problem->batch = input_shape[0];
  problem->channels = input_shape[1];
  problem->output_channels = weight_shape[0];
  problem->groups = groups;
  if (problem->batch < 0) return fail(CND_ERR_INVALID, "batch size must be nonnegative");
  if (!(problem->channels > 0 && problem->output_channels > 0 &&
        problem->channels % groups == 0 && problem->output_channels % groups == 0 &&
        weight_shape[1] == problem->channels / groups)) {
    return fail(CND_ERR_INVALID, "input/weight channels must match and be divisible by groups");
  }
  problem->input_volume = 1;
  problem->output_volume = 1;
  problem->kernel_volume = 1;
  for (int32_t axis = 0; axis < rank; ++axis) {
    const int64_t size = input_shape[axis + 2];
    const int64_t kernel = weight_shape[axis + 2];
    if (!(size > 0 && kernel > 0)) {
      return fail(CND_ERR_INVALID, "spatial and kernel dimensions must be positive");
    }
    if (!(stride[axis] > 0 && dilation[axis] > 0 && padding[axis] >= 0)) {
      return fail(CND_ERR_INVALID,
                  "stride and dilation must be positive; padding must be nonnegative");
    }
    problem->input[axis] = size;
    problem->kernel[axis] = kernel;
    problem->stride[axis] = stride[axis];
    problem->padding[axis] = padding[axis];
    problem->dilation[axis] = dilation[axis];
    int64_t span = 0, effective = 0, doubled = 0, padded = 0;
    if (!cnd::checked_product(dilation[axis], kernel - 1, &span) ||
        !cnd::checked_sum(span, 1, &effective)) {
      return fail(CND_ERR_INVALID, "dilated kernel overflows int64");
    }
    if (!cnd::checked_product(2, padding[axis], &doubled)) {
      return fail(CND_ERR_INVALID, "padding overflows int64");
    }
    if (!cnd::checked_sum(size, doubled, &padded)) {
      return fail(CND_ERR_INVALID, "padded input overflows int64");
    }
    if (padded < effective) return fail(CND_ERR_INVALID, "kernel exceeds padded input");
    problem->output[axis] = (padded - effective) / stride[axis] + 1;
    if (!cnd::checked_product(problem->input_volume, size, &problem->input_volume)) {
      return fail(CND_ERR_INVALID, "input spatial volume overflows int64");
    }
    if (!cnd::checked_product(problem->output_volume, problem->output[axis],
                              &problem->output_volume)) {
      return fail(CND_ERR_INVALID, "output spatial volume overflows int64");
    }
    if (!cnd::checked_product(problem->kernel_volume, kernel, &problem->kernel_volume)) {
      return fail(CND_ERR_INVALID, "kernel volume overflows int64");
    }
  }
  return CND_OK;
}

int cnd_check_workspace_budget(const cnd_problem* problem, int64_t element_size,
                               int64_t workspace_bytes) {
  using cnd::fail;
  cnd::clear_error();
  int64_t rows = 0, per_position = 0;
  if (!cnd::checked_product(problem->channels, problem->kernel_volume, &rows)) {
    return fail(CND_ERR_INVALID, "patch rows overflows int64");
  }
  const int64_t width = element_size > 4 ? element_size : 4;
  if (!cnd::checked_product(width, rows, &per_position)) {
    return fail(CND_ERR_INVALID, "workspace bytes per position overflows int64");
  }
  if (workspace_bytes < per_position) {
    return fail(CND_ERR_INVALID,
                "workspace_bytes is too small for one output position; requires at least %lld",
                static_cast<long long>(per_position));
  }
  return CND_OK;
}

}  // extern "C"
