// Layout kernels around the tcgen05 passes (HBM-bound transposes and small reductions).
//
// pack_act: channels-first [N][G*Cg][S] -> channels-last [N][G][S][C_pad] (zero-padded
//   channels), optionally split into TF32 big/small parts for 3xTF32, optionally
//   producing per-block channel sums (the bias gradient of the reference's
//   flat_grad.sum({0,3}), convnd.cpp:388-390, fused into the pass that reads dy anyway).
// pack_weight: [Cout][Cg][taps] -> [G][taps][n_pad][c_pad] for the forward B operand, or
//   the flipped/transposed dgrad operand [G][taps'][Cin_g pad][Cout_g pad].
// wgrad_reduce / bias_reduce: ordered (deterministic) sums of fp32 partials.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "internal.h"
#include "pack.cuh"

namespace cnd {

namespace {

template <typename T>
__device__ __forceinline__ float to_float(T v);
template <>
__device__ __forceinline__ float to_float<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_float<__half>(__half v) {
  return __half2float(v);
}

// Round-to-nearest conversion of fp32 to TF32 (result kept in fp32 storage).
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ float from_float<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_float<__half>(float v) {
  return __float2half_rn(v);
}

constexpr int kPackPositions = 64;

// Derivative of PyTorch's exact GELU: Phi(v) + v * phi(v).
__device__ __forceinline__ float gelu_grad(float v) {
  const float cdf = 0.5f * (1.0f + erff(v * 0.70710678118654752f));
  // fast exponential: the product is rounded to the operand type (or checked against the
  // float32 tolerance), far above its relative error of a few 1e-7
  const float pdf = 0.39894228040143268f * __expf(-0.5f * v * v);
  return cdf + v * pdf;
}

// Splits v into `parts` terms of type T whose sum reproduces v: TF32 big/small (kMode 1),
// a TF32 rounding (kMode 2), or bf16 hi/mid/lo (kMode 3) and hi/lo (kMode 4), the
// error-compensated operands of the split-product MMAs.
template <typename T, int kMode>
__device__ __forceinline__ void split_value(float v, T* out0, T* out1, T* out2, int64_t i) {
  if constexpr (kMode == 1) {
    const float big = tf32_round(v);
    out0[i] = from_float<T>(big);
    out1[i] = from_float<T>(tf32_round(v - big));
  } else if constexpr (kMode == 2) {
    out0[i] = from_float<T>(tf32_round(v));
  } else if constexpr (kMode == 3 || kMode == 4) {
    const T hi = from_float<T>(v);
    const float r1 = v - to_float(hi);
    const T mid = from_float<T>(r1);
    out0[i] = hi;
    out1[i] = mid;
    if constexpr (kMode == 3) out2[i] = from_float<T>(r1 - to_float(mid));
  } else {
    out0[i] = from_float<T>(v);
  }
}

// One block: 64 positions x all channels of one (n, g). Loads coalesced along positions
// (channels-first source) or along channels (channels-last source, kSrcCL), stores
// coalesced along channels; with no destination only the channel sums are produced.
template <typename Tin, typename Tout, int kMode, bool kSrcCL>
__global__ void __launch_bounds__(256) pack_act_kernel(const Tin* __restrict__ src,
                                                       Tout* __restrict__ dst0,
                                                       Tout* __restrict__ dst1,
                                                       Tout* __restrict__ dst2, int64_t S,
                                                       int Cg, int c_pad, int G,
                                                       float* __restrict__ chan_partial,
                                                       const Tin* __restrict__ pre) {
  extern __shared__ float tile[];  // [c_pad][kPackPositions + 1]
  const int64_t s0 = static_cast<int64_t>(blockIdx.x) * kPackPositions;
  const int g = blockIdx.y;
  const int64_t n = blockIdx.z;
  const int width = kPackPositions + 1;
  if constexpr (kSrcCL) {
    const int64_t row = static_cast<int64_t>(G) * Cg;
    const Tin* in = src + (n * S + s0) * row + static_cast<int64_t>(g) * Cg;
    for (int i = threadIdx.x; i < c_pad * kPackPositions; i += blockDim.x) {
      const int s = i / c_pad;
      const int c = i - s * c_pad;
      float v = 0.0f;
      if (c < Cg && s0 + s < S) {
        const int64_t at = (n * S + s0) * row + static_cast<int64_t>(g) * Cg + s * row + c;
        v = to_float(in[s * row + c]);
        if (pre != nullptr) v = to_float(from_float<Tin>(v * gelu_grad(to_float(pre[at]))));
      }
      tile[c * width + s] = v;
    }
  } else {
    const Tin* in = src + (n * G + g) * static_cast<int64_t>(Cg) * S;
    for (int i = threadIdx.x; i < c_pad * kPackPositions; i += blockDim.x) {
      const int c = i / kPackPositions;
      const int s = i - c * kPackPositions;
      float v = 0.0f;
      if (c < Cg && s0 + s < S) {
        const int64_t at = (n * G + g) * static_cast<int64_t>(Cg) * S + c * S + s0 + s;
        v = to_float(in[static_cast<int64_t>(c) * S + s0 + s]);
        if (pre != nullptr) v = to_float(from_float<Tin>(v * gelu_grad(to_float(pre[at]))));
      }
      tile[c * width + s] = v;
    }
  }
  __syncthreads();
  const int64_t base = ((n * G + g) * S + s0) * c_pad;
  const int count = static_cast<int>(S - s0 < kPackPositions ? S - s0 : kPackPositions);
  if (dst0 != nullptr) {
    for (int i = threadIdx.x; i < count * c_pad; i += blockDim.x) {
      const int s = i / c_pad;
      const int c = i - s * c_pad;
      split_value<Tout, kMode>(tile[c * width + s], dst0, dst1, dst2, base + i);
    }
  }
  if (chan_partial != nullptr) {
    // Per-channel sum of this block's positions, in position order.
    for (int c = threadIdx.x; c < Cg; c += blockDim.x) {
      float sum = 0.0f;
      for (int s = 0; s < count; ++s) sum += tile[c * width + s];
      chan_partial[((n * G + g) * gridDim.x + blockIdx.x) * Cg + c] = sum;
    }
  }
}

// Original tap index of row `row` of the packed weights. Rows are grouped by load unit:
// unit = (outer taps, t0 unless shifted, t1 unless shifted, t2 unless folded) row-major,
// and within a unit the shifted taps (t0 if shift0, t1 if shift1) row-major, or with the
// a0 fold j1-major and j0 within; with the a2 fold (fold2 = k2) j2 is innermost.
__device__ __forceinline__ int packed_row_tap(int row, int k0, int k1, int k2, int shift0,
                                              int shift1, int fold, int fold2) {
  const int n1 = shift1 ? k1 : 1;
  const int n0 = shift0 ? k0 : 1;
  const int n2 = fold2 > 1 ? k2 : 1;
  const int inner = row % (n0 * n1 * n2);
  int rest = row / (n0 * n1 * n2);
  const int ls = inner / n2;
  const int j2 = inner % n2;
  const int j1 = fold ? ls / n0 : ls % n1;
  const int j0 = fold ? ls % n0 : ls / n1;
  int t2 = j2;
  if (n2 == 1) {
    t2 = rest % k2;
    rest /= k2;
  }
  int t1 = j1, t0 = j0;
  if (!shift1) {
    t1 = rest % k1;
    rest /= k1;
  }
  if (!shift0) {
    t0 = rest % k0;
    rest /= k0;
  }
  return ((rest * k0 + t0) * k1 + t1) * k2 + t2;
}

// Fast path for 16-bit activations without splitting (bf16/fp16 problems). Every thread
// moves an 8-channel x 8-position block: eight 16-byte loads (8 positions of one channel
// each), an 8x8 transpose of the 16-bit values in registers — output word m of position p
// holds channels (2m, 2m+1) and is one byte permute of the two input words holding
// positions (p & ~1, p | 1) of those channels — and eight 16-byte stores (8 channels of
// one position each). A warp's lanes are (position group, channel group) with the
// channel group fastest, so each store instruction writes whole position rows.
// Requirements (checked by the host): c_pad in {8, 16, 32, 64}, S % 8 == 0, 16-byte
// aligned tensors.
constexpr int kFastWarps = 8;

__host__ __device__ constexpr int fast_positions_per_block(int c_pad) {
  return kFastWarps * 8 * (32 / (c_pad / 8));
}

template <typename T>
__global__ void __launch_bounds__(32 * kFastWarps)
    pack_act16_kernel(const T* __restrict__ src, T* __restrict__ dst, int64_t S, int Cg,
                      int c_pad, int G, float* __restrict__ chan_partial) {
  const int cgs = c_pad >> 3;   // channel groups of 8 (1, 2, 4 or 8)
  const int pgs = 32 / cgs;     // position groups of 8 per warp
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cg = lane % cgs;
  const int pg = lane / cgs;
  const int64_t ng = static_cast<int64_t>(blockIdx.z) * G + blockIdx.y;
  const int64_t p0 =
      static_cast<int64_t>(blockIdx.x) * fast_positions_per_block(c_pad) + (warp * pgs + pg) * 8;
  const bool active = p0 < S;
  const uint16_t* in = reinterpret_cast<const uint16_t*>(src) + ng * Cg * S;
  uint16_t* out = reinterpret_cast<uint16_t*>(dst) + ng * S * c_pad;
  uint4 a[8];
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    const int c = cg * 8 + ch;
    a[ch] = make_uint4(0, 0, 0, 0);
    if (active && c < Cg) a[ch] = __ldg(reinterpret_cast<const uint4*>(in + c * S + p0));
  }
  if (active) {
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const uint32_t sel = (p & 1) ? 0x7632u : 0x5410u;
      uint32_t w[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const uint32_t* lo = reinterpret_cast<const uint32_t*>(&a[2 * m]);
        const uint32_t* hi = reinterpret_cast<const uint32_t*>(&a[2 * m + 1]);
        w[m] = __byte_perm(lo[p >> 1], hi[p >> 1], sel);
      }
      *reinterpret_cast<uint4*>(out + (p0 + p) * c_pad + cg * 8) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  if (chan_partial != nullptr) {
    // Per-channel sums of this block's positions: 8 positions per thread in order, then a
    // fixed butterfly over the warp's position groups, then the warps in order.
    __shared__ float part[kFastWarps][64];
    float sum[8];
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      const uint16_t* v = reinterpret_cast<const uint16_t*>(&a[ch]);
      float t = 0.0f;
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        T x;
        *reinterpret_cast<uint16_t*>(&x) = v[p];
        t += to_float(x);
      }
      sum[ch] = t;
    }
    for (int off = cgs; off < 32; off <<= 1) {
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) sum[ch] += __shfl_xor_sync(0xffffffffu, sum[ch], off);
    }
    if (pg == 0) {
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) part[warp][cg * 8 + ch] = sum[ch];
    }
    __syncthreads();
    for (int c = threadIdx.x; c < Cg; c += blockDim.x) {
      float total = 0.0f;
      for (int w = 0; w < kFastWarps; ++w) total += part[w][c];
      chan_partial[(ng * gridDim.x + blockIdx.x) * Cg + c] = total;
    }
  }
}

// Per-channel sums of a 16-bit channels-last activation [N][S][C] (C a multiple of 8,
// at most 256): the bias-gradient partials when dy is read in place. Block (b, n) covers
// positions [b * kSumRows, +kSumRows) of image n; thread t reads 16-byte vectors (8
// channels) of rows t / vpr, t / vpr + per_pass, ... in order, then the threads holding
// the same channel group are added in thread order: a fixed summation order.
constexpr int kSumRows = 512;

template <typename T>
__global__ void __launch_bounds__(256) channel_sum_cl16_kernel(const T* __restrict__ src,
                                                               int64_t S, int C,
                                                               float* __restrict__ partial,
                                                               T* __restrict__ dst,
                                                               const T* __restrict__ pre) {
  __shared__ float part[256][8];
  const int vpr = C >> 3;  // 16-byte vectors per row
  const int per_pass = 256 / vpr;
  const int t = threadIdx.x;
  const int v = t % vpr;
  const int r0 = t / vpr;
  float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int64_t row_base = static_cast<int64_t>(blockIdx.x) * kSumRows;
  const int64_t image = blockIdx.z;
  if (r0 < per_pass) {
    // no early exit: the unrolled rows' loads are all in flight together
#pragma unroll 4
    for (int r = r0; r < kSumRows; r += per_pass) {
      const int64_t pos = row_base + r;
      if (pos >= S) continue;
      const int64_t at = (image * S + pos) * C;
      uint4 word = __ldg(reinterpret_cast<const uint4*>(src + at) + v);
      T* x = reinterpret_cast<T*>(&word);
      if (pre != nullptr) {
        // activation backward: dy * act'(pre), rounded once to T
        const uint4 pw = __ldg(reinterpret_cast<const uint4*>(pre + at) + v);
        const T* z = reinterpret_cast<const T*>(&pw);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = from_float<T>(to_float(x[i]) * gelu_grad(to_float(z[i])));
      }
      if (dst != nullptr) *(reinterpret_cast<uint4*>(dst + at) + v) = word;
#pragma unroll
      for (int i = 0; i < 8; ++i) sum[i] += to_float(x[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) part[t][i] = sum[i];
  __syncthreads();
  if (partial == nullptr) return;
  for (int c = t; c < C; c += blockDim.x) {
    const int group = c >> 3;
    float total = 0.0f;
    for (int r = 0; r < per_pass; ++r) total += part[r * vpr + group][c & 7];
    partial[(image * gridDim.x + blockIdx.x) * C + c] = total;
  }
}

template <typename T, typename Tout, int kMode>
__global__ void pack_weight_kernel(const T* __restrict__ w, Tout* __restrict__ dst,
                                   Tout* __restrict__ dst_small, PackWeightArgs a) {
  const int64_t total = static_cast<int64_t>(a.groups) * a.taps * a.n_pad * a.c_pad;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t r = i;
    const int c = static_cast<int>(r % a.c_pad);
    r /= a.c_pad;
    const int nn = static_cast<int>(r % a.n_pad);
    r /= a.n_pad;
    const int row = static_cast<int>(r % a.taps);
    const int g = static_cast<int>(r / a.taps);
    const int t = packed_row_tap(row, a.k_box[0], a.k_box[1], a.k_box[2], a.shift0, a.shift1,
                                 a.fold, a.fold2);
    float v = 0.0f;
    // Block-diagonal packing: weight row co holds input channels [gb * cin_b, +cin_b) of
    // its group gb = co / cout_b; the other columns stay zero.
    const int cin_b = a.cin_g / a.bd, cout_b = a.cout_g / a.bd;
    if (!a.dgrad) {
      // forward operand: B[n = output channel][k = input channel] of tap t
      if (nn < a.cout_g && c < a.cin_g && c / cin_b == nn / cout_b) {
        const int cw = c - (nn / cout_b) * cin_b;
        v = to_float(w[((static_cast<int64_t>(g) * a.cout_g + nn) * cin_b + cw) * a.taps + t]);
      }
    } else {
      // dgrad operand: B[n = input channel][k = output channel] of the flipped tap, or of
      // the phase sub-kernel's mapped tap
      if (nn < a.cin_g && c < a.cout_g && nn / cin_b == c / cout_b) {
        const int nw = nn - (c / cout_b) * cin_b;
        int tw = a.taps - 1 - t;
        int taps_w = a.taps;
        if (a.phase_rank > 0) {
          int rest = t, u[kMaxFastRank];
          for (int ax = a.phase_rank - 1; ax >= 0; --ax) {
            u[ax] = rest % a.k_sub[ax];
            rest /= a.k_sub[ax];
          }
          tw = 0;
          for (int ax = 0; ax < a.phase_rank; ++ax) {
            tw = tw * a.k_full[ax] + a.tap_first[ax] + u[ax] * a.tap_step[ax];
          }
          taps_w = a.taps_w;
        }
        v = to_float(w[((static_cast<int64_t>(g) * a.cout_g + c) * cin_b + nw) * taps_w + tw]);
      }
    }
    split_value<Tout, kMode>(v, dst, dst_small, nullptr, i);
  }
}

// Weight-gradient operand with the last axis's taps folded into the channels
// (PackActArgs::fold_taps): destination [n][g][q][c_pad], channel c = j * Cg + ci taken
// from source channel ci at q's position shifted along the last axis by j * dil - pad
// (zero outside the input). One thread per destination position gathers its channels (a
// warp's loads of one channel cover consecutive positions: coalesced for a channels-first
// source, cache-line reuse along a channels-last source's rows); the warp then writes its
// 32 positions' rows, which are contiguous in the destination, through a padded
// shared-memory stage as 512-byte runs (mode 4: bf16 hi, then lo). The pack is bound by
// instructions and store wavefronts, not bytes, so nothing here divides by a runtime value.
constexpr int kFoldMaxPad = 64;  // channels per destination row (16, 32 or 64)

// Split of one value into the destination's parts (split_value's modes): hi only (mode 0,
// or a TF32 rounding in mode 2), TF32 big + small (mode 1), bf16 hi + lo (mode 4).
template <typename Tout, int kMode>
__device__ __forceinline__ void split_two(float v, Tout& hi, Tout& lo) {
  if constexpr (kMode == 1) {
    const float big = tf32_round(v);
    hi = from_float<Tout>(big);
    lo = from_float<Tout>(tf32_round(v - big));
  } else if constexpr (kMode == 2) {
    hi = from_float<Tout>(tf32_round(v));
  } else if constexpr (kMode == 4) {
    hi = from_float<Tout>(v);
    lo = from_float<Tout>(v - to_float(hi));
  } else {
    hi = from_float<Tout>(v);
  }
}

// With chan_partial the kernel also writes the channel sums of every 64 destination
// positions (two warps): chan_partial[((n * G + g) * ceil(S_dst / 64) + block) * Cg + c],
// the layout of pack_act_kernel's partials, summed in a fixed order.
template <typename Tin, typename Tout, int kMode, bool kSrcCL, int kCg>
__global__ void __launch_bounds__(256) pack_fold_kernel(
    const Tin* __restrict__ src, Tout* __restrict__ dst0, Tout* __restrict__ dst1,
    int64_t S_src, int64_t S_dst, int64_t last_src, int64_t last_dst, int Cg_rt, int c_pad,
    int G, int taps, int dil, int pad, float* __restrict__ chan_partial) {
  static_assert(sizeof(Tout) == 2 || sizeof(Tout) == 4, "16- or 32-bit operands");
  static_assert(kCg % 8 == 0, "whole 8-channel chunks per tap");
  constexpr int kPitch = kFoldMaxPad * 2 + 16;  // bytes per staged row (bank spread)
  constexpr int kChunkVecs = 8 * static_cast<int>(sizeof(Tout)) / 16;  // uint4 per 8 channels
  constexpr bool kTwo = kMode == 1 || kMode == 4;                       // second part
  constexpr bool kRaw = kMode == 0 && sizeof(Tin) == sizeof(Tout);     // copy the bits
  (void)Cg_rt;
  __shared__ __align__(16) uint8_t stage[8][32 * kPitch];
  __shared__ float sums[8][kCg];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.y;
  const int64_t n = blockIdx.z;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + warp * 32;  // warp's first
  const int64_t q = q0 + lane;
  const bool valid = q < S_dst;
  uint8_t* row_stage = stage[warp] + lane * kPitch;
  const int64_t qc = valid ? q : 0;
  const int64_t outer = qc / last_dst;
  const int i_last = static_cast<int>(qc - outer * last_dst) - pad;
  const int64_t row0 = outer * last_src;  // source position of (outer, last-axis 0)
  const Tin* plane;   // channel 0 of this (n, g) at source position row0
  int64_t ch_step;    // elements between channels
  int64_t pos_step;   // elements between positions
  if constexpr (kSrcCL) {
    pos_step = static_cast<int64_t>(G) * kCg;
    ch_step = 1;
    plane = src + (n * S_src + row0) * pos_step + static_cast<int64_t>(g) * kCg;
  } else {
    pos_step = 1;
    ch_step = S_src;
    plane = src + (n * G + g) * kCg * S_src + row0;
  }
  uint8_t* ws = stage[warp];
  const int row_bytes = c_pad * static_cast<int>(sizeof(Tout));
  const int row_shift = __ffs(row_bytes) - 1;  // log2 of the row bytes (32, 64 or 128)
  const int64_t out_base = ((n * G + g) * S_dst + q0) * c_pad;  // elements
  const int64_t rows_here = S_dst - q0 < 32 ? S_dst - q0 : 32;
  const int run_bytes = static_cast<int>(rows_here) << row_shift;
  // One gather per destination part (the second one re-reads the source from cache): the
  // part's row goes to this lane's staged row, then the warp writes its rows.
  for (int part = 0; part < (kTwo ? 2 : 1); ++part) {
    if (part == 1) __syncwarp();  // the first part's copy-out has read the stage
    for (int j = 0; j < taps; ++j) {
      const int at = i_last + j * dil;
      const bool in = valid && at >= 0 && at < last_src;
      const Tin* p = plane + (in ? at : 0) * pos_step;
#pragma unroll
      for (int c8 = 0; c8 < kCg; c8 += 8) {
        alignas(16) Tout out[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if constexpr (kRaw) {
            out[k] = in ? p[(c8 + k) * ch_step] : Tout{};
          } else {
            const float v = in ? to_float(p[(c8 + k) * ch_step]) : 0.0f;
            Tout hi, lo;
            split_two<Tout, kMode>(v, hi, lo);
            out[k] = part == 0 ? hi : lo;
            if (chan_partial != nullptr && part == 0) {  // one tap: the bias partials
              float sum = v;
#pragma unroll
              for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
              if (lane == 0) sums[warp][c8 + k] = sum;
            }
          }
        }
        const int m = j * kCg + c8;  // first channel of the chunk
#pragma unroll
        for (int u = 0; u < kChunkVecs; ++u) {
          *reinterpret_cast<uint4*>(row_stage + m * sizeof(Tout) + u * 16) =
              reinterpret_cast<const uint4*>(out)[u];
        }
      }
    }
    for (int m = taps * kCg; m < c_pad; m += 8) {  // padding channels
#pragma unroll
      for (int u = 0; u < kChunkVecs; ++u) {
        *reinterpret_cast<uint4*>(row_stage + m * sizeof(Tout) + u * 16) = make_uint4(0, 0, 0, 0);
      }
    }
    if (chan_partial != nullptr && part == 0) {
      // channel sums of each 64-position block: warps 2b and 2b + 1, added in warp order
      __syncthreads();
      const int64_t blocks_total = (S_dst + 63) / 64;
      const int local = threadIdx.x / kCg;  // block within the CTA
      const int c = threadIdx.x % kCg;
      const int64_t block = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 64) + local;
      if (local < static_cast<int>(blockDim.x / 64) && block < blocks_total) {
        chan_partial[((n * G + g) * blocks_total + block) * kCg + c] =
            sums[2 * local][c] + sums[2 * local + 1][c];
      }
    }
    __syncwarp();
    uint8_t* dst = reinterpret_cast<uint8_t*>((part == 0 ? dst0 : dst1) + out_base);
    for (int o = lane * 16; o < run_bytes; o += 512) {
      const int row = o >> row_shift;
      const int within = o & ((1 << row_shift) - 1);
      *reinterpret_cast<uint4*>(dst + o) =
          *reinterpret_cast<const uint4*>(ws + row * kPitch + within);
    }
  }
}

// Split-K weight-gradient reduce. Element p of one split's partial block (`stride`
// floats per split) is summed over the splits and written to dw:
//  - dense groups: partial[s][g][t][ci][co] -> dw[(g*cout_g + co)*cin_g*taps + ci*taps + t]
//  - block-diagonal (bd groups run as one): p walks (t, cb, co) with co fastest and reads
//    partial[s][t][gb*cin_b + cb][co], gb = co / cout_b -> dw[co][cb][t].
// A CTA takes 32 consecutive elements (one per lane, coalesced) and its 8 warps take 8
// contiguous split ranges, each summed in split order with several loads in flight; the 8
// range sums are then added in range order. The association is fixed, so every run gives
// the same bits, and the CTAs keep enough loads in flight for HBM bandwidth even when a
// layer has few weights and many splits.
struct WgradReduceMap {
  int bd;  // 1: dense groups; > 1: block-diagonal
  int G, taps, cin, cout;  // cin / cout: per group (dense) or all channels (bd)
  int fold;  // > 1 (dense only): last-axis taps folded into the partials' channels
};

__device__ __forceinline__ void wgrad_reduce_index(const WgradReduceMap& m, int64_t p,
                                                   int64_t* src, int64_t* dst) {
  if (m.bd == 1) {
    // partial [g][t'][j * cin + ci][co] with t' over taps / fold: dw tap t' * fold + j
    const int taps_f = m.taps / m.fold;
    const int cin_f = m.cin * m.fold;
    int64_t r = p;
    const int co = static_cast<int>(r % m.cout);
    r /= m.cout;
    const int cf = static_cast<int>(r % cin_f);
    r /= cin_f;
    const int tf = static_cast<int>(r % taps_f);
    const int g = static_cast<int>(r / taps_f);
    const int j = cf / m.cin;
    const int ci = cf - j * m.cin;
    const int t = tf * m.fold + j;
    *src = p;
    *dst = ((static_cast<int64_t>(g) * m.cout + co) * m.cin + ci) * m.taps + t;
  } else {
    const int cin_b = m.cin / m.bd, cout_b = m.cout / m.bd;
    int64_t r = p;
    const int co = static_cast<int>(r % m.cout);
    r /= m.cout;
    const int cb = static_cast<int>(r % cin_b);
    const int t = static_cast<int>(r / cin_b);
    const int ci = (co / cout_b) * cin_b + cb;
    *src = (static_cast<int64_t>(t) * m.cin + ci) * m.cout + co;
    *dst = (static_cast<int64_t>(co) * cin_b + cb) * m.taps + t;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) wgrad_reduce_kernel(const float* __restrict__ partial,
                                                           int splits, int64_t stride,
                                                           int64_t total, WgradReduceMap m,
                                                           T* __restrict__ dw) {
  __shared__ float range_sum[8][32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int s_begin = (warp * splits) / 8;
  const int s_end = ((warp + 1) * splits) / 8;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * 32; base < total;
       base += static_cast<int64_t>(gridDim.x) * 32) {
    const int64_t p = base + lane;
    int64_t src = 0, dst = 0;
    if (p < total) wgrad_reduce_index(m, p, &src, &dst);
    float sum = 0.0f;
    if (p < total) {
      const float* at = partial + src;
#pragma unroll 8
      for (int s = s_begin; s < s_end; ++s) sum += at[static_cast<int64_t>(s) * stride];
    }
    range_sum[warp][lane] = sum;
    __syncthreads();
    if (warp == 0 && p < total) {
      float v = range_sum[0][lane];
#pragma unroll
      for (int j = 1; j < 8; ++j) v += range_sum[j][lane];
      dw[dst] = from_float<T>(v);
    }
    __syncthreads();
  }
}

// db[g*cg + c] = sum over (n, block) of partial[n][g][block][c], in two passes with a
// fixed association (bitwise reproducible). Pass 1: CTA (k, g) sums row chunk k of the
// batch*blocks rows; a warp's lanes take consecutive channels (coalesced reads), its 8
// warps every 8th row, and the warp sums are added in warp order into
// chunk_sums[k][g][c]. Pass 2 adds the chunks in order. One CTA per channel summing all
// rows had left c4's 16 channels to 16 CTAs (38 us).
constexpr int kBiasChunks = 64;

__global__ void __launch_bounds__(256) bias_chunk_kernel(const float* __restrict__ partial,
                                                         int64_t batch, int G, int blocks,
                                                         int cg, float* __restrict__ chunk_sums) {
  __shared__ float part[8][256];
  const int chunk = blockIdx.x;
  const int g = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = batch * blocks;
  const int64_t r0 = rows * chunk / kBiasChunks;
  const int64_t r1 = rows * (chunk + 1) / kBiasChunks;
  for (int c0 = 0; c0 < cg; c0 += 32) {
    const int c = c0 + lane;
    float sum = 0.0f;
    if (c < cg) {
      int64_t r = r0 + warp;
      int64_t n = r / blocks;
      int64_t b = r - n * blocks;
      for (; r < r1; r += 8) {
        sum += partial[((n * G + g) * blocks + b) * static_cast<int64_t>(cg) + c];
        b += 8;
        while (b >= blocks) {
          b -= blocks;
          ++n;
        }
      }
      part[warp][c] = sum;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < cg; c += blockDim.x) {
    float v = part[0][c];
#pragma unroll
    for (int w = 1; w < 8; ++w) v += part[w][c];
    chunk_sums[(static_cast<int64_t>(chunk) * G + g) * cg + c] = v;
  }
}

template <typename T>
__global__ void bias_final_kernel(const float* __restrict__ chunk_sums, int G, int cg,
                                  T* __restrict__ db) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= G * cg) return;
  float v = 0.0f;
  for (int k = 0; k < kBiasChunks; ++k) v += chunk_sums[static_cast<int64_t>(k) * G * cg + i];
  db[i] = from_float<T>(v);
}

int grid_for(int64_t total, int threads) {
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

template <typename Tin, typename Tout, int kMode, bool kSrcCL>
int launch_pack_act_impl(const PackActArgs& a, cudaStream_t stream) {
  const int64_t blocks = (a.spatial + kPackPositions - 1) / kPackPositions;
  if (blocks > 0x7FFFFFFF || a.groups > 65535 || a.batch > 65535) {
    return fail(CND_ERR_UNSUPPORTED, "pack_act: grid too large");
  }
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(a.groups),
                  static_cast<unsigned>(a.batch));
  const size_t smem = static_cast<size_t>(a.c_pad) * (kPackPositions + 1) * sizeof(float);
  if (smem > 200 * 1024) return fail(CND_ERR_UNSUPPORTED, "pack_act: too many channels");
  auto kernel = pack_act_kernel<Tin, Tout, kMode, kSrcCL>;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  kernel<<<grid, 256, smem, stream>>>(static_cast<const Tin*>(a.src), static_cast<Tout*>(a.dst),
                                      static_cast<Tout*>(a.dst_small),
                                      static_cast<Tout*>(a.dst_third), a.spatial, a.cg, a.c_pad,
                                      static_cast<int>(a.groups), a.chan_partial,
                                      a.act ? static_cast<const Tin*>(a.pre) : nullptr);
  count_launch();
  return CND_OK;
}

template <typename Tin, typename Tout, int kMode>
int launch_pack_act(const PackActArgs& a, cudaStream_t stream) {
  if (a.src_cl) return launch_pack_act_impl<Tin, Tout, kMode, true>(a, stream);
  return launch_pack_act_impl<Tin, Tout, kMode, false>(a, stream);
}

template <typename Tin, typename Tout, int kMode, bool kSrcCL>
int launch_pack_fold_impl(const PackActArgs& a, cudaStream_t stream) {
  const int64_t s_dst = a.spatial / a.fold_last_src * a.fold_last_dst;
  const int64_t blocks = (s_dst + 255) / 256;
  if (blocks > 0x7FFFFFFF || a.groups > 65535 || a.batch > 65535) {
    return fail(CND_ERR_UNSUPPORTED, "pack_fold: grid too large");
  }
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(a.groups),
                  static_cast<unsigned>(a.batch));
  auto args = [&](auto kernel) {
    kernel<<<grid, 256, 0, stream>>>(
        static_cast<const Tin*>(a.src), static_cast<Tout*>(a.dst),
        static_cast<Tout*>(a.dst_small), a.spatial, s_dst, a.fold_last_src, a.fold_last_dst,
        a.cg, a.c_pad, static_cast<int>(a.groups), a.fold_taps, a.fold_dilation,
        a.fold_padding, a.chan_partial);
  };
  if (a.cg == 8) {
    args(pack_fold_kernel<Tin, Tout, kMode, kSrcCL, 8>);
  } else if (a.cg == 16) {
    args(pack_fold_kernel<Tin, Tout, kMode, kSrcCL, 16>);
  } else if (a.cg == 32) {
    args(pack_fold_kernel<Tin, Tout, kMode, kSrcCL, 32>);
  } else {
    return fail(CND_ERR_UNSUPPORTED, "pack_fold: %d channels per group", a.cg);
  }
  count_launch();
  return CND_OK;
}

template <typename Tin, typename Tout, int kMode>
int launch_pack_fold(const PackActArgs& a, cudaStream_t stream) {
  if (a.src_cl) return launch_pack_fold_impl<Tin, Tout, kMode, true>(a, stream);
  return launch_pack_fold_impl<Tin, Tout, kMode, false>(a, stream);
}

template <typename T>
int pack_weight_typed(const PackWeightArgs& a, cudaStream_t stream) {
  const int64_t total = a.groups * a.taps * a.n_pad * a.c_pad;
  const int blocks = grid_for(total, 256);
  const T* w = static_cast<const T*>(a.w);
  T* dst = static_cast<T*>(a.dst);
  T* dst_small = static_cast<T*>(a.dst_small);
  if (a.mode == 1) {
    pack_weight_kernel<T, T, 1><<<blocks, 256, 0, stream>>>(w, dst, dst_small, a);
  } else if (a.mode == 2) {
    pack_weight_kernel<T, T, 2><<<blocks, 256, 0, stream>>>(w, dst, dst_small, a);
  } else if (a.mode == 4) {
    // float32 weights as bfloat16 hi + lo parts
    pack_weight_kernel<T, __nv_bfloat16, 4><<<blocks, 256, 0, stream>>>(
        w, static_cast<__nv_bfloat16*>(a.dst), static_cast<__nv_bfloat16*>(a.dst_small), a);
  } else {
    pack_weight_kernel<T, T, 0><<<blocks, 256, 0, stream>>>(w, dst, dst_small, a);
  }
  count_launch();
  return CND_OK;
}

}  // namespace

template <typename T>
int launch_pack_act16(const PackActArgs& a, cudaStream_t stream) {
  const int per_block = fast_positions_per_block(a.c_pad);
  const int64_t blocks = (a.spatial + per_block - 1) / per_block;
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(a.groups),
                  static_cast<unsigned>(a.batch));
  pack_act16_kernel<T><<<grid, 32 * kFastWarps, 0, stream>>>(static_cast<const T*>(a.src),
                                                 static_cast<T*>(a.dst), a.spatial, a.cg,
                                                 a.c_pad, static_cast<int>(a.groups),
                                                 a.chan_partial);
  count_launch();
  return CND_OK;
}

bool pack16_fast_ok(const PackActArgs& a) {
  return a.mode == 0 && !a.src_cl && a.dst != nullptr && a.act == 0 && (a.c_pad == 8 || a.c_pad == 16 || a.c_pad == 32 || a.c_pad == 64) &&
         a.cg <= a.c_pad && a.spatial % 8 == 0 &&
         (a.spatial + 63) / 64 <= 0x7FFFFFFF && a.groups <= 65535 &&
         a.batch <= 65535 && reinterpret_cast<uintptr_t>(a.src) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(a.dst) % 16 == 0;
}

template <typename T>
struct Wide {
  using type = float;
};
template <>
struct Wide<double> {
  using type = double;
};

template <typename T>
__device__ __forceinline__ typename Wide<T>::type widen(T v) {
  return static_cast<typename Wide<T>::type>(v);
}
template <>
__device__ __forceinline__ float widen<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float widen<__half>(__half v) {
  return __half2float(v);
}

__device__ __forceinline__ double gelu_of(double v) {
  return 0.5 * v * (1.0 + erf(v * 0.70710678118654752440));
}
__device__ __forceinline__ float gelu_of(float v) {
  return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
}
__device__ __forceinline__ double gelu_grad_of(double v) {
  return 0.5 * (1.0 + erf(v * 0.70710678118654752440)) +
         v * 0.39894228040143267794 * exp(-0.5 * v * v);
}
__device__ __forceinline__ float gelu_grad_of(float v) { return gelu_grad(v); }

template <typename T>
__global__ void activation_forward_kernel(const T* __restrict__ src, T* dst, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    dst[i] = static_cast<T>(gelu_of(widen(src[i])));
  }
}

template <typename T>
__global__ void activation_backward_kernel(const T* __restrict__ dy, const T* __restrict__ pre,
                                           T* __restrict__ dz, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    dz[i] = static_cast<T>(widen(dy[i]) * gelu_grad_of(widen(pre[i])));
  }
}

template <typename T>
int activation_typed(const void* a, const void* b, void* out, int64_t n, bool backward,
                     cudaStream_t stream) {
  if (n == 0) return CND_OK;
  const int blocks = grid_for(n, 256);
  if (backward) {
    activation_backward_kernel<T><<<blocks, 256, 0, stream>>>(
        static_cast<const T*>(a), static_cast<const T*>(b), static_cast<T*>(out), n);
  } else {
    activation_forward_kernel<T><<<blocks, 256, 0, stream>>>(static_cast<const T*>(a),
                                                             static_cast<T*>(out), n);
  }
  count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CND_ERR_CUDA, "activation launch: %s", cudaGetErrorString(e));
  return CND_OK;
}

int activation_dispatch(const void* a, const void* b, void* out, int64_t n, int dtype,
                        bool backward, cudaStream_t stream) {
  switch (dtype) {
    case CND_BF16:
      return activation_typed<__nv_bfloat16>(a, b, out, n, backward, stream);
    case CND_F16:
      return activation_typed<__half>(a, b, out, n, backward, stream);
    case CND_F32:
      return activation_typed<float>(a, b, out, n, backward, stream);
    default:
      return activation_typed<double>(a, b, out, n, backward, stream);
  }
}

bool channel_sums_fast_ok(const PackActArgs& a);
int channel_sums(const PackActArgs& a, cudaStream_t stream);

// Plain channels-first float32 packs into operand parts (TF32 big + small, a TF32
// rounding, or bf16 hi + lo), with or without the bias partials, run as a one-tap
// pack_fold_kernel: the shared-memory transpose of pack_act_kernel is bound by its
// instruction count (c4: dy 67 us, x 41 us).
bool plain_fold_ok(const PackActArgs& a) {
  const int out_es = a.mode == 4 ? 2 : 4;
  const int row = a.c_pad * out_es;
  const bool two = a.mode == 1 || a.mode == 4;
  return a.fold_taps <= 1 && !a.src_cl && a.act == 0 && a.dst != nullptr &&
         a.dtype == CND_F32 && (a.mode == 1 || a.mode == 2 || a.mode == 4) &&
         (a.cg == 8 || a.cg == 16 || a.cg == 32) && a.cg <= a.c_pad &&
         (row == 32 || row == 64 || row == 128) && a.groups <= 65535 && a.batch <= 65535 &&
         reinterpret_cast<uintptr_t>(a.dst) % 16 == 0 &&
         (!two || reinterpret_cast<uintptr_t>(a.dst_small) % 16 == 0);
}

int pack_activations(const PackActArgs& args, cudaStream_t stream) {
  int rc;
  if (plain_fold_ok(args)) {
    PackActArgs one = args;
    one.fold_taps = 1;
    one.fold_dilation = 0;
    one.fold_padding = 0;
    one.fold_last_src = one.fold_last_dst = args.spatial > 0 ? args.spatial : 1;
    if (args.spatial == 0) return CND_OK;
    if (args.mode == 4) {
      rc = launch_pack_fold<float, __nv_bfloat16, 4>(one, stream);
    } else if (args.mode == 1) {
      rc = launch_pack_fold<float, float, 1>(one, stream);
    } else {
      rc = launch_pack_fold<float, float, 2>(one, stream);
    }
  } else if (args.fold_taps > 1) {
    if (args.dst == nullptr || args.act != 0 || args.chan_partial != nullptr ||
        args.fold_last_src < 1 || args.fold_last_dst < 1 ||
        args.spatial % args.fold_last_src != 0 || args.fold_taps * args.cg > args.c_pad) {
      return fail(CND_ERR_INVALID, "pack_activations: invalid folded-tap pack");
    }
    if ((args.c_pad != 16 && args.c_pad != 32 && args.c_pad != kFoldMaxPad) ||
        reinterpret_cast<uintptr_t>(args.dst) % 16 != 0 ||
        (args.mode == 4 && reinterpret_cast<uintptr_t>(args.dst_small) % 16 != 0)) {
      return fail(CND_ERR_INVALID, "pack_activations: folded-tap pack needs 16-byte rows");
    }
    if (args.dtype == CND_BF16) {
      rc = launch_pack_fold<__nv_bfloat16, __nv_bfloat16, 0>(args, stream);
    } else if (args.dtype == CND_F16) {
      rc = launch_pack_fold<__half, __half, 0>(args, stream);
    } else if (args.dtype == CND_F32 && args.mode == 4) {
      rc = launch_pack_fold<float, __nv_bfloat16, 4>(args, stream);
    } else {
      return fail(CND_ERR_UNSUPPORTED, "pack_activations: folded taps need 16-bit operands");
    }
  } else if (channel_sums_fast_ok(args)) {
    return channel_sums(args, stream);
  } else if ((args.dtype == CND_BF16 || args.dtype == CND_F16) && pack16_fast_ok(args)) {
    rc = args.dtype == CND_BF16 ? launch_pack_act16<__nv_bfloat16>(args, stream)
                                : launch_pack_act16<__half>(args, stream);
  } else if (args.dtype == CND_BF16) {
    rc = launch_pack_act<__nv_bfloat16, __nv_bfloat16, 0>(args, stream);
  } else if (args.dtype == CND_F16) {
    rc = launch_pack_act<__half, __half, 0>(args, stream);
  } else if (args.dtype == CND_F32) {
    switch (args.mode) {
      case 1:
        rc = launch_pack_act<float, float, 1>(args, stream);
        break;
      case 2:
        rc = launch_pack_act<float, float, 2>(args, stream);
        break;
      case 3:
        rc = launch_pack_act<float, __nv_bfloat16, 3>(args, stream);
        break;
      case 4:
        rc = launch_pack_act<float, __nv_bfloat16, 4>(args, stream);
        break;
      default:
        rc = launch_pack_act<float, float, 0>(args, stream);
    }
  } else {
    return fail(CND_ERR_UNSUPPORTED, "pack_activations: unsupported dtype");
  }
  if (rc != CND_OK) return rc;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CND_ERR_CUDA, "pack_act launch: %s", cudaGetErrorString(e));
  return CND_OK;
}

int pack_weights(const PackWeightArgs& in, cudaStream_t stream) {
  PackWeightArgs args = in;
  if (args.bd < 1) args.bd = 1;
  if (args.cin_g % args.bd != 0 || args.cout_g % args.bd != 0) {
    return fail(CND_ERR_INVALID, "pack_weights: %d block-diagonal groups do not divide the "
                "channels", args.bd);
  }
  int rc;
  if (args.dtype == CND_BF16) {
    rc = pack_weight_typed<__nv_bfloat16>(args, stream);
  } else if (args.dtype == CND_F16) {
    rc = pack_weight_typed<__half>(args, stream);
  } else if (args.dtype == CND_F32) {
    rc = pack_weight_typed<float>(args, stream);
  } else {
    return fail(CND_ERR_UNSUPPORTED, "pack_weights: unsupported dtype");
  }
  if (rc != CND_OK) return rc;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(CND_ERR_CUDA, "pack_weight launch: %s", cudaGetErrorString(e));
  }
  return CND_OK;
}

int reduce_wgrad(const float* partial, int splits, int groups, int bd, int taps, int cin_g,
                 int cout_g, void* dw, int dtype, cudaStream_t stream, int fold) {
  if (fold < 1 || taps % fold != 0 || (fold > 1 && bd > 1)) {
    return fail(CND_ERR_INVALID, "wgrad_reduce: %d folded taps of %d (block-diagonal %d)",
                fold, taps, bd);
  }
  WgradReduceMap m{bd, groups, taps, cin_g, cout_g, fold};
  // elements of one split's partial block, and the dW elements the reduce writes
  const int64_t stride = static_cast<int64_t>(groups) * taps * cin_g * cout_g;
  const int64_t total = bd > 1 ? static_cast<int64_t>(taps) * (cin_g / bd) * cout_g : stride;
  const int blocks = grid_for((total + 31) / 32, 1);
  if (dtype == CND_BF16) {
    wgrad_reduce_kernel<<<blocks, 256, 0, stream>>>(partial, splits, stride, total, m,
                                                    static_cast<__nv_bfloat16*>(dw));
  } else if (dtype == CND_F16) {
    wgrad_reduce_kernel<<<blocks, 256, 0, stream>>>(partial, splits, stride, total, m,
                                                    static_cast<__half*>(dw));
  } else {
    wgrad_reduce_kernel<<<blocks, 256, 0, stream>>>(partial, splits, stride, total, m,
                                                    static_cast<float*>(dw));
  }
  count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CND_ERR_CUDA, "wgrad_reduce: %s", cudaGetErrorString(e));
  return CND_OK;
}

size_t bias_chunk_bytes(int groups, int cg) {
  return static_cast<size_t>(kBiasChunks) * groups * cg * sizeof(float);
}

int reduce_bias(const float* partial, int64_t batch, int groups, int blocks, int cg, void* db,
                int dtype, float* chunk_sums, cudaStream_t stream) {
  if (cg > 256 || groups > 65535 || blocks < 1) {
    return fail(CND_ERR_UNSUPPORTED, "bias_reduce: %d channels per group", cg);
  }
  bias_chunk_kernel<<<dim3(kBiasChunks, static_cast<unsigned>(groups)), 256, 0, stream>>>(
      partial, batch, groups, blocks, cg, chunk_sums);
  const int total = groups * cg;
  const int grid = (total + 255) / 256;
  if (dtype == CND_BF16) {
    bias_final_kernel<<<grid, 256, 0, stream>>>(chunk_sums, groups, cg,
                                                static_cast<__nv_bfloat16*>(db));
  } else if (dtype == CND_F16) {
    bias_final_kernel<<<grid, 256, 0, stream>>>(chunk_sums, groups, cg,
                                                static_cast<__half*>(db));
  } else {
    bias_final_kernel<<<grid, 256, 0, stream>>>(chunk_sums, groups, cg,
                                                static_cast<float*>(db));
  }
  count_launch();
  count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CND_ERR_CUDA, "bias_reduce: %s", cudaGetErrorString(e));
  return CND_OK;
}

bool channel_sums_fast_ok(const PackActArgs& a) {
  const int64_t channels = a.groups * a.cg;
  // channels-last 16-bit rows that already are the packed rows: channel sums only, or a
  // row copy (with the activation backward) into the packed layout
  const bool rows_match = a.groups == 1 && a.cg == a.c_pad && a.mode == 0 &&
                          (a.dst == nullptr || reinterpret_cast<uintptr_t>(a.dst) % 16 == 0);
  return a.src_cl && (a.dst == nullptr || rows_match) &&
         (a.dtype == CND_BF16 || a.dtype == CND_F16) &&
         (a.act == 0 || reinterpret_cast<uintptr_t>(a.pre) % 16 == 0) &&
         channels % 8 == 0 && channels <= 256 && 256 % (channels / 8) == 0 &&
         a.batch <= 65535 && reinterpret_cast<uintptr_t>(a.src) % 16 == 0;
}

int channel_sums(const PackActArgs& a, cudaStream_t stream) {
  const int channels = static_cast<int>(a.groups * a.cg);
  const int64_t blocks = (a.spatial + kSumRows - 1) / kSumRows;
  const dim3 grid(static_cast<unsigned>(blocks), 1, static_cast<unsigned>(a.batch));
  if (a.dtype == CND_BF16) {
    channel_sum_cl16_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(a.src), a.spatial, channels, a.chan_partial,
        static_cast<__nv_bfloat16*>(a.dst),
        a.act ? static_cast<const __nv_bfloat16*>(a.pre) : nullptr);
  } else {
    channel_sum_cl16_kernel<__half><<<grid, 256, 0, stream>>>(
        static_cast<const __half*>(a.src), a.spatial, channels, a.chan_partial,
        static_cast<__half*>(a.dst), a.act ? static_cast<const __half*>(a.pre) : nullptr);
  }
  count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CND_ERR_CUDA, "channel_sum launch: %s", cudaGetErrorString(e));
  return CND_OK;
}

int activation_forward(const void* src, void* dst, int64_t n, int dtype, int act,
                       cudaStream_t stream) {
  if (act != CND_ACT_GELU) return fail(CND_ERR_UNSUPPORTED, "unknown activation %d", act);
  return activation_dispatch(src, nullptr, dst, n, dtype, false, stream);
}

int activation_backward(const void* dy, const void* pre, void* dz, int64_t n, int dtype,
                        int act, cudaStream_t stream) {
  if (act != CND_ACT_GELU) return fail(CND_ERR_UNSUPPORTED, "unknown activation %d", act);
  return activation_dispatch(dy, pre, dz, n, dtype, true, stream);
}

int64_t pack_blocks(const PackActArgs& args) {
  if (channel_sums_fast_ok(args)) return (args.spatial + kSumRows - 1) / kSumRows;
  if ((args.dtype == CND_BF16 || args.dtype == CND_F16) && pack16_fast_ok(args)) {
    const int per_block = fast_positions_per_block(args.c_pad);
    return (args.spatial + per_block - 1) / per_block;
  }
  return (args.spatial + kPackPositions - 1) / kPackPositions;
}

}  // namespace cnd
