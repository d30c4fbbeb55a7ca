// Host interface of the generic CUDA-core kernels in generic.cu.
#pragma once

#include <cuda_runtime.h>

#include "convnd_b200.h"

namespace cnd {

struct GenericCall {
  enum Op { kForward, kDgrad, kWgrad, kBias };
  Op op;
  const cnd_problem* problem;
  const void* a;  // forward: x; dgrad: dy; wgrad: dy; bias: dy
  const void* b;  // forward: w; dgrad: w;  wgrad: x
  const void* c;  // forward: bias (or null)
  void* out;      // y / dx / dw / db
};

int run_generic(const GenericCall& call, cudaStream_t stream);

}  // namespace cnd
