// Shared host/device definitions of the tcgen05 implicit-GEMM convolution kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "internal.h"

namespace cnd {

// Operand element type of a tensor-core pass.
enum OperandType { kOpF16 = 0, kOpBF16 = 1, kOpF32 = 2 };

// One implicit-GEMM convolution pass on tcgen05 whose GEMM is
//   out[pos, n] = sum_{tap, c} act[pos * s + tap * d - p, c] * wt[tap, n, c]
// i.e. the reference's forward product W . columns (convnd.cpp:333-334) without the
// columns matrix. Used for the forward pass and, with flipped weights, for dgrad.
struct ConvPass {
  int rank;
  int64_t batch, groups;
  int64_t in[kMaxFastRank], out[kMaxFastRank], k[kMaxFastRank], s[kMaxFastRank],
      d[kMaxFastRank], p[kMaxFastRank];
  int c_pad;        // activation channels per group in the packed layout
  int n_real;       // output channels per group
  int n_pad;        // MMA N (multiple of 16, <= 256)
  int op;           // OperandType
  int split3;       // 3xTF32: act/wt have big + small parts
  const void* act;  // packed [N][G][in...][c_pad]
  const void* act_small;
  const void* wt;   // packed [G][taps][n_pad][c_pad]
  const void* wt_small;
  void* dst;        // channels-first [N][G*n_real][out...] of out_dtype (channels-last
                    // [N][out...][G*n_real] when out_cl)
  const void* bias; // [G*n_real] of out_dtype, or null
  int out_dtype;    // cnd_dtype
  int out_cl;
  // Strided output (one phase of a strided input gradient): output position j of axis a
  // goes to position out_mul[a] * j + out_add[a] of a tensor whose axes have extents
  // out_full[a]; out_strided = 0 means the output is exactly out[].
  int out_strided;
  int64_t out_mul[kMaxFastRank], out_add[kMaxFastRank], out_full[kMaxFastRank];
  // Fused activation (CND_ACT_*): dst receives activation(conv + bias) and `pre` (if not
  // null) conv + bias, in the same layout.
  int activation;
  void* pre;
};

// Weight-gradient pass: dW[g][tap][ci][co] partials of
//   sum_pos act[pos * s + tap * d - p, ci] * grad[pos, co]
// (the reference's baddbmm dW += dY . columns^T, convnd.cpp:402-406 and
// convnd_mixed.cpp:39-45), split over positions into `splits` fp32 partials.
struct WgradPass {
  int rank;
  int64_t batch, groups;
  int64_t in[kMaxFastRank], out[kMaxFastRank], k[kMaxFastRank], s[kMaxFastRank],
      d[kMaxFastRank], p[kMaxFastRank];
  int c_pad;        // x channels per group (packed)
  int cin_real;
  int n_pad;        // dy channels per group (packed), MMA N
  int n_real;
  int op;           // kOpBF16 or kOpF16 (float32 problems arrive as bf16 parts)
  int parts;        // 1, or 2 / 3 bf16 terms per operand for float32 problems
  const void* act[3];   // x packed [N][G][in...][c_pad], one array per part
  const void* grad[3];  // dy packed [N][G][out...][n_pad], one array per part
  float* partial;   // [splits][G][taps][cin_real][n_real]
  int splits;       // chosen by plan_wgrad
};

// Returns true when the tcgen05 weight-gradient kernel can run the pass.
bool wgrad_pass_supported(const WgradPass& pass);

// Number of fp32 partial sets the wgrad kernel will write for this pass.
int plan_wgrad_splits(const WgradPass& pass, int sm_count);

int launch_wgrad_pass(const WgradPass& pass, cudaStream_t stream, uint64_t timeout_ns);

// One-line description of the pass's kernel plan (for the plan summary).
int describe_wgrad_pass(const WgradPass& pass, char* text, size_t size);

}  // namespace cnd
