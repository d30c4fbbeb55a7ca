// Generic CUDA-core convolution kernels: any rank (1-62), stride, dilation, padding,
// groups and dtype (fp16/bf16/fp32 accumulate in fp32, fp64 in fp64), with 64-bit index
// arithmetic. They run the passes the tcgen05 kernels do not cover (fp64, strided dgrad,
// padding larger than the dilated kernel, very wide channel groups) and every pass when
// the caller asks for exact fp32 (CND_FP32_SIMT). Activations may be channels-first or
// channels-last (cnd_problem.layout).
//
// Index maps follow the reference's column_input_offset / input_column_offset
// (src/torch_convnd/csrc/convnd.h:57-104): input coordinate = out*stride - pad +
// tap*dilation, and the inverse map requires (in + pad - tap*dilation) to be a
// nonnegative multiple of the stride. All reductions run in a fixed order, so results
// are bitwise reproducible (the reference's deterministic-mode contract,
// tests/test_convnd.py:235-257).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "generic.cuh"
#include "internal.h"

namespace cnd {

namespace {

template <typename T>
struct Acc {
  using type = float;
};
template <>
struct Acc<double> {
  using type = double;
};

template <typename T>
__device__ __forceinline__ typename Acc<T>::type ld(const T* p, int64_t i) {
  return static_cast<typename Acc<T>::type>(p[i]);
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <>
__device__ __forceinline__ float ld<__half>(const __half* p, int64_t i) {
  return __half2float(p[i]);
}

template <typename T, typename A>
__device__ __forceinline__ void st(T* p, int64_t i, A v) {
  p[i] = static_cast<T>(v);
}
template <>
__device__ __forceinline__ void st<__nv_bfloat16, float>(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ void st<__half, float>(__half* p, int64_t i, float v) {
  p[i] = __float2half_rn(v);
}

// Element index of activation (n, c, position) of a tensor with `channels` channels and
// `volume` positions per image: channels-first [N][C][S], or channels-last [N][S][C] when
// `cl` (the CND_LAYOUT_* bit of that tensor).
__device__ __forceinline__ int64_t act_at(int64_t n, int64_t c, int64_t position,
                                          int64_t channels, int64_t volume, bool cl) {
  return cl ? (n * volume + position) * channels + c : (n * channels + c) * volume + position;
}

// Forward: one thread per output element (n, co, position).
template <typename T>
__global__ void generic_forward_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                       const T* __restrict__ b, T* __restrict__ y,
                                       const cnd_problem P) {
  using A = typename Acc<T>::type;
  const int rank = P.rank;
  const int64_t cin_g = P.channels / P.groups;
  const int64_t cout_g = P.output_channels / P.groups;
  const int64_t total = P.batch * P.output_channels * P.output_volume;
  const bool x_cl = (P.layout & CND_LAYOUT_X_CL) != 0, y_cl = (P.layout & CND_LAYOUT_Y_CL) != 0;
  for (int64_t index = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
       index < total; index += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t position = index % P.output_volume;
    const int64_t co = (index / P.output_volume) % P.output_channels;
    const int64_t n = index / P.output_volume / P.output_channels;
    const int64_t g = co / cout_g;
    A sum = 0;
    for (int64_t tap = 0; tap < P.kernel_volume; ++tap) {
      // Input offset of this tap (row-major, last axis fastest), or -1 in the padding.
      int64_t offset = 0, multiplier = 1, pos = position, t = tap;
      bool inside = true;
      for (int axis = rank - 1; axis >= 0; --axis) {
        const int64_t o = pos % P.output[axis];
        const int64_t k = t % P.kernel[axis];
        pos /= P.output[axis];
        t /= P.kernel[axis];
        const int64_t coord = o * P.stride[axis] - P.padding[axis] + k * P.dilation[axis];
        if (coord < 0 || coord >= P.input[axis]) {
          inside = false;
          break;
        }
        offset += coord * multiplier;
        multiplier *= P.input[axis];
      }
      if (!inside) continue;
      const int64_t w_base = (co * cin_g) * P.kernel_volume + tap;
      for (int64_t ci = 0; ci < cin_g; ++ci) {
        sum += ld(x, act_at(n, g * cin_g + ci, offset, P.channels, P.input_volume, x_cl)) *
               ld(w, w_base + ci * P.kernel_volume);
      }
    }
    if (b != nullptr) sum += ld(b, co);
    st(y, act_at(n, co, position, P.output_channels, P.output_volume, y_cl), sum);
  }
}

// dgrad: one thread per input element (n, ci, position); gathers over output channels
// and taps through the inverse index map.
template <typename T>
__global__ void generic_dgrad_kernel(const T* __restrict__ dy, const T* __restrict__ w,
                                     T* __restrict__ dx, const cnd_problem P) {
  using A = typename Acc<T>::type;
  const int rank = P.rank;
  const int64_t cin_g = P.channels / P.groups;
  const int64_t cout_g = P.output_channels / P.groups;
  const int64_t total = P.batch * P.channels * P.input_volume;
  const bool x_cl = (P.layout & CND_LAYOUT_X_CL) != 0, y_cl = (P.layout & CND_LAYOUT_Y_CL) != 0;
  for (int64_t index = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
       index < total; index += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t position = index % P.input_volume;
    const int64_t ci = (index / P.input_volume) % P.channels;
    const int64_t n = index / P.input_volume / P.channels;
    const int64_t g = ci / cin_g;
    const int64_t ci_local = ci - g * cin_g;
    A sum = 0;
    for (int64_t tap = 0; tap < P.kernel_volume; ++tap) {
      int64_t offset = 0, multiplier = 1, pos = position, t = tap;
      bool reached = true;
      for (int axis = rank - 1; axis >= 0; --axis) {
        const int64_t i = pos % P.input[axis];
        const int64_t k = t % P.kernel[axis];
        pos /= P.input[axis];
        t /= P.kernel[axis];
        const int64_t numerator = i + P.padding[axis] - k * P.dilation[axis];
        if (numerator < 0 || numerator % P.stride[axis] != 0) {
          reached = false;
          break;
        }
        const int64_t o = numerator / P.stride[axis];
        if (o >= P.output[axis]) {
          reached = false;
          break;
        }
        offset += o * multiplier;
        multiplier *= P.output[axis];
      }
      if (!reached) continue;
      for (int64_t col = 0; col < cout_g; ++col) {
        const int64_t co = g * cout_g + col;
        sum += ld(dy, act_at(n, co, offset, P.output_channels, P.output_volume, y_cl)) *
               ld(w, (co * cin_g + ci_local) * P.kernel_volume + tap);
      }
    }
    st(dx, act_at(n, ci, position, P.channels, P.input_volume, x_cl), sum);
  }
}

// wgrad: one block per weight element (co, ci_local, tap); block-wide ordered tree sum
// over (n, output position).
template <typename T>
__global__ void __launch_bounds__(256) generic_wgrad_kernel(const T* __restrict__ dy,
                                                            const T* __restrict__ x,
                                                            T* __restrict__ dw,
                                                            const cnd_problem P) {
  using A = typename Acc<T>::type;
  __shared__ A partial[256];
  const int rank = P.rank;
  const int64_t cin_g = P.channels / P.groups;
  const int64_t cout_g = P.output_channels / P.groups;
  const int64_t total = P.output_channels * cin_g * P.kernel_volume;
  const bool x_cl = (P.layout & CND_LAYOUT_X_CL) != 0, y_cl = (P.layout & CND_LAYOUT_Y_CL) != 0;
  for (int64_t element = blockIdx.x; element < total; element += gridDim.x) {
    const int64_t tap = element % P.kernel_volume;
    const int64_t ci_local = (element / P.kernel_volume) % cin_g;
    const int64_t co = element / P.kernel_volume / cin_g;
    const int64_t g = co / cout_g;
    const int64_t ci = g * cin_g + ci_local;
    A sum = 0;
    const int64_t work = P.batch * P.output_volume;
    for (int64_t item = threadIdx.x; item < work; item += blockDim.x) {
      const int64_t position = item % P.output_volume;
      const int64_t n = item / P.output_volume;
      int64_t offset = 0, multiplier = 1, pos = position, t = tap;
      bool inside = true;
      for (int axis = rank - 1; axis >= 0; --axis) {
        const int64_t o = pos % P.output[axis];
        const int64_t k = t % P.kernel[axis];
        pos /= P.output[axis];
        t /= P.kernel[axis];
        const int64_t coord = o * P.stride[axis] - P.padding[axis] + k * P.dilation[axis];
        if (coord < 0 || coord >= P.input[axis]) {
          inside = false;
          break;
        }
        offset += coord * multiplier;
        multiplier *= P.input[axis];
      }
      if (!inside) continue;
      sum += ld(dy, act_at(n, co, position, P.output_channels, P.output_volume, y_cl)) *
             ld(x, act_at(n, ci, offset, P.channels, P.input_volume, x_cl));
    }
    partial[threadIdx.x] = sum;
    __syncthreads();
    for (int width = blockDim.x / 2; width > 0; width >>= 1) {
      if (threadIdx.x < width) partial[threadIdx.x] += partial[threadIdx.x + width];
      __syncthreads();
    }
    if (threadIdx.x == 0) st(dw, element, partial[0]);
    __syncthreads();
  }
}

// Bias gradient: one block per output channel, ordered tree sum over (n, position).
template <typename T>
__global__ void __launch_bounds__(256) generic_bias_kernel(const T* __restrict__ dy,
                                                           T* __restrict__ db,
                                                           const cnd_problem P) {
  using A = typename Acc<T>::type;
  __shared__ A partial[256];
  const bool y_cl = (P.layout & CND_LAYOUT_Y_CL) != 0;
  for (int64_t co = blockIdx.x; co < P.output_channels; co += gridDim.x) {
    A sum = 0;
    const int64_t work = P.batch * P.output_volume;
    for (int64_t item = threadIdx.x; item < work; item += blockDim.x) {
      const int64_t position = item % P.output_volume;
      const int64_t n = item / P.output_volume;
      sum += ld(dy, act_at(n, co, position, P.output_channels, P.output_volume, y_cl));
    }
    partial[threadIdx.x] = sum;
    __syncthreads();
    for (int width = blockDim.x / 2; width > 0; width >>= 1) {
      if (threadIdx.x < width) partial[threadIdx.x] += partial[threadIdx.x + width];
      __syncthreads();
    }
    if (threadIdx.x == 0) st(db, co, partial[0]);
    __syncthreads();
  }
}

int blocks_for(int64_t total, int threads) {
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 64) blocks = 148 * 64;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

template <typename T>
int run_typed(const GenericCall& c, cudaStream_t stream) {
  const cnd_problem& P = *c.problem;
  switch (c.op) {
    case GenericCall::kForward: {
      const int64_t total = P.batch * P.output_channels * P.output_volume;
      if (total == 0) return CND_OK;
      generic_forward_kernel<T><<<blocks_for(total, 128), 128, 0, stream>>>(
          static_cast<const T*>(c.a), static_cast<const T*>(c.b), static_cast<const T*>(c.c),
          static_cast<T*>(c.out), P);
      break;
    }
    case GenericCall::kDgrad: {
      const int64_t total = P.batch * P.channels * P.input_volume;
      if (total == 0) return CND_OK;
      generic_dgrad_kernel<T><<<blocks_for(total, 128), 128, 0, stream>>>(
          static_cast<const T*>(c.a), static_cast<const T*>(c.b), static_cast<T*>(c.out), P);
      break;
    }
    case GenericCall::kWgrad: {
      const int64_t total = P.output_channels * (P.channels / P.groups) * P.kernel_volume;
      if (total == 0) return CND_OK;
      const int64_t blocks = total < 148 * 64 ? total : 148 * 64;
      generic_wgrad_kernel<T><<<static_cast<int>(blocks), 256, 0, stream>>>(
          static_cast<const T*>(c.a), static_cast<const T*>(c.b), static_cast<T*>(c.out), P);
      break;
    }
    case GenericCall::kBias: {
      const int64_t blocks = P.output_channels < 148 * 8 ? P.output_channels : 148 * 8;
      generic_bias_kernel<T><<<static_cast<int>(blocks), 256, 0, stream>>>(
          static_cast<const T*>(c.a), static_cast<T*>(c.out), P);
      break;
    }
  }
  count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CND_ERR_CUDA, "generic kernel launch: %s", cudaGetErrorString(e));
  return CND_OK;
}

}  // namespace

int run_generic(const GenericCall& call, cudaStream_t stream) {
  switch (call.problem->dtype) {
    case CND_F16:
      return run_typed<__half>(call, stream);
    case CND_BF16:
      return run_typed<__nv_bfloat16>(call, stream);
    case CND_F32:
      return run_typed<float>(call, stream);
    case CND_F64:
      return run_typed<double>(call, stream);
    default:
      return fail(CND_ERR_UNSUPPORTED,
                  "native conv_nd supports float16, bfloat16, float32 and float64");
  }
}

}  // namespace cnd
