// Host interface of the layout kernels in pack.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"

namespace cnd {

// mode: 0 = copy, 1 = TF32 big + small (3xTF32), 2 = round to TF32, 3 = fp32 -> bf16
// hi + mid + lo, 4 = fp32 -> bf16 hi + lo (modes 3/4 write bfloat16 parts).
struct PackActArgs {
  const void* src;      // channels-first [batch][groups*cg][spatial], or channels-last
                        // [batch][spatial][groups*cg] when src_cl
  void* dst;            // channels-last [batch][groups][spatial][c_pad]; null: only the
                        // channel partial sums are produced
  void* dst_small;      // second part (modes 1, 3, 4)
  void* dst_third;      // third part (mode 3)
  int64_t batch, groups, spatial;
  int cg, c_pad, dtype, mode;
  float* chan_partial;  // optional [batch][groups][pack_blocks(spatial)][cg]
  int src_cl;           // 1: the source is channels-last
  // Fused activation backward: each value is multiplied by act'(pre) (pre has the
  // source's shape and layout; CND_ACT_*) in fp32 before it is stored, rounded once.
  int act;
  const void* pre;
  // fold_taps > 1 (weight-gradient operand): the taps of the last spatial axis folded
  // into the channels. Destination channel j * cg + ci (j < fold_taps) holds source
  // channel ci at the position shifted along the last axis by j * fold_dilation -
  // fold_padding (zero outside the input); the destination's last axis has
  // fold_last_dst positions (the source's fold_last_src), so it has
  // spatial / fold_last_src * fold_last_dst positions. No activation or channel sums.
  int fold_taps;
  int fold_dilation, fold_padding;
  int64_t fold_last_src, fold_last_dst;
};

// Weights [groups*cout_g][cin_g][taps] -> [groups][taps][n_pad][c_pad] (mode as for
// activations; mode 4 writes float32 weights as bfloat16 hi + lo parts), rows in the
// convolution pass's load-unit order (k_box = kernel extents of the three box axes,
// shift0/shift1 = whether the a0 / a1 taps of a unit are served by shared-memory shifts).
struct PackWeightArgs {
  const void* w;
  void* dst;
  void* dst_small;
  int groups, cout_g, cin_g, taps, n_pad, c_pad, dtype, mode, dgrad;
  int k_box[3];
  int shift0, shift1;
  int fold;  // 1: within a unit the a0 taps are consecutive (j0 fastest), else a1 taps
  // > 1: the k2 taps of box axis a2 are inside every unit too, fastest of all (each
  // (j1, j0) block of the B operand is [j2][n]: the a2 taps folded into the MMA N)
  int fold2;
  // > 1: the weights of a problem with bd groups packed as one dense block-diagonal
  // matrix (groups == 1, cout_g / cin_g = all channels; off-diagonal blocks are zero)
  int bd;
  // > 0 (dgrad only): the packed taps are the sub-kernel of one phase of a strided input
  // gradient. Packed tap u (row-major over k_sub[0..phase_rank)) is the weight's tap
  // t_a = tap_first[a] + u_a * tap_step[a] (row-major over k_full), taken as is (the
  // phase's tap order already is the flipped one); the weight has taps_w taps per (co, ci).
  int phase_rank;
  int taps_w;
  int k_sub[kMaxFastRank], k_full[kMaxFastRank], tap_first[kMaxFastRank],
      tap_step[kMaxFastRank];
};

int pack_activations(const PackActArgs& args, cudaStream_t stream);
int pack_weights(const PackWeightArgs& args, cudaStream_t stream);
// bd > 1: the partials are of the dense block-diagonal problem (groups == 1, cin_g /
// cout_g = all channels); only the bd diagonal blocks are written to dw.
// fold > 1: the partials are of the problem whose last axis's `fold` taps were folded
// into the channels (PackActArgs::fold_taps): partial channel j * cin_g + ci of folded
// tap t' is dw's channel ci at tap t' * fold + j (taps counts dw's taps).
int reduce_wgrad(const float* partial, int splits, int groups, int bd, int taps, int cin_g,
                 int cout_g, void* dw, int dtype, cudaStream_t stream, int fold = 1);
// chunk_sums: bias_chunk_bytes(groups, cg) bytes of scratch for the first pass.
size_t bias_chunk_bytes(int groups, int cg);
int reduce_bias(const float* partial, int64_t batch, int groups, int blocks, int cg, void* db,
                int dtype, float* chunk_sums, cudaStream_t stream);
// Elementwise activation passes for problems the tcgen05 epilogue / pack do not serve:
// dst = act(src) (dst may alias src), and dz = dy * act'(pre); n elements of `dtype`.
int activation_forward(const void* src, void* dst, int64_t n, int dtype, int act,
                       cudaStream_t stream);
int activation_backward(const void* dy, const void* pre, void* dz, int64_t n, int dtype,
                        int act, cudaStream_t stream);
// Number of position blocks (and so of bias-gradient partials per (n, g)) the activation
// pack of `args` produces.
int64_t pack_blocks(const PackActArgs& args);

}  // namespace cnd
