// Host interface of the persistent tcgen05 convolution pass in fprop.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "internal.h"
#include "tc_conv.cuh"

namespace cnd {

// Kernel parameters (passed by value as a __grid_constant__).
struct FpropParams {
  // geometry: box axes a0..a2, outer axes (merged TMA dimension)
  int n_outer;
  int out_o[kMaxOuter], in_o[kMaxOuter], k_o[kMaxOuter], s_o[kMaxOuter], d_o[kMaxOuter],
      p_o[kMaxOuter];
  int64_t in_o_stride[kMaxOuter];
  int out[3], in[3], k[3], s[3], d[3], p[3];
  int64_t batch, groups, in_merged_per_gn, out_outer_vol, out_box_vol, out_volume,
      out_channels_total;
  int taps;
  // tiling
  int e0, b1, b2, mt;
  int nshift0, nshift1;  // taps of a0 / a1 served by shared-memory shifts (1 = none)
  // fold = 1: the a0 taps of a unit run as one MMA per A slice whose N spans every tap
  // block that lands on a tile of the super (N = blocks * n_pad); tile m's accumulator
  // sits at column (mt - 1 - m) * n_pad, so block j0 of slice i lands on tile i - j0.
  // Accumulators are zeroed by the epilogue and every MMA accumulates.
  int fold;
  // k2f = k2 (3): the a2 taps of a unit are folded into N as well. A tile row then is an
  // input-aligned position of a line of b2 rows and the MMA for a2 tap j2 writes the
  // column block j2 of that row; output position r of a line is the sum over j2 of block
  // j2 at row r + j2 (one warp-shuffle per tap in the epilogue, lines never cross a warp
  // boundary), so a line of b2 rows yields b2o = b2 - k2 + 1 outputs. k2f = 1 otherwise
  // (b2o = b2). n_blk = k2f * n_pad TMEM columns per M tile.
  int k2f, b2o, n_blk;
  int h0, h1;            // halo box extents (rows) along a0 / a1
  // par0 = 2 (folded a0 taps at dilation 2): a super tile covers output planes of one
  // parity, whose a0 taps read input planes of that parity only; the TMA box steps a0 by
  // 2 (element stride), so the taps are consecutive box slices as at dilation 1.
  // a0_tile_step = e0 * par0 output planes between consecutive M tiles.
  int par0, a0_tile_step;
  int nsup[3];
  int64_t supers_total;
  int units;             // load units per super tile (taps / shifted taps)
  // channels and MMA
  int cblocks, cblk_elems, ksteps, row_bytes, layout;
  int n_pad, n_real, nacc, acc_stride;
  uint32_t a_part_bytes, b_part_bytes, b_off, stage_bytes, tx_bytes, idesc, tmem_cols;
  uint32_t idesc_base;  // idesc without its N field (folded MMAs set N per slice)
  int stages;
  // epilogue groups of four warps (1 or 2); group g drains M tiles g, g + groups, ...
  int epi_groups;
  uint32_t bar_off;  // barriers after the stages (and the output staging buffers)
  // output (channels-first); tma_store = 1 stages each M tile in shared memory as
  // [channel][position] (two buffers of out_tile_bytes at out_stage_off) and writes it
  // with one TMA store, else every thread stores its position's channels directly
  int tma_store;
  // out_cl = 1: the output is channels-last [N][positions][G * n_real]. With tma_store
  // each M tile is staged as [position][channel] rows in column chunks of out_span bytes
  // (16, or 32 / 64 / 128 with the TMA swizzle of that width) and written by one TMA
  // store per chunk; otherwise each thread stores its position's channels directly.
  int out_cl;
  uint32_t out_span;
  // Strided output (ConvPass::out_strided): element offset of output position (outer o,
  // box o0..o2) is phase_base + sum o * ostride, over a tensor of out_volume_full positions
  // per image; direct stores only.
  int act;    // CND_ACT_*: the epilogue applies it after the bias
  void* pre;  // pre-activation output (same layout as dst), or null
  // pre_staged = 1: with tma_store, each tile's pre-activation is staged beside its
  // output (two buffers per tile) and written by its own TMA store through maps.pre
  int pre_staged;
  int out_strided;
  int64_t phase_base, out_volume_full;
  int64_t ostride_box[3], ostride_o[kMaxOuter];
  uint32_t out_stage_off, out_tile_bytes;
  void* dst;
  const void* bias;
  int out_dtype;
  unsigned int* err;
  uint64_t timeout_ns;
  int debug_stall;
};

struct FpropPlan {
  FpropParams params;
  int parts;         // 2 for 3xTF32 (big + small operand arrays)
  double score;      // the cost model's estimated cycles per output position (lower wins)
  size_t smem;
  // weight packing order (see PackWeightArgs::unit_order)
  int shift0, shift1, fold, fold2;
  int k_box[3];
};

// Chooses tiling, halo and pipeline depth for a pass; false if the pass does not fit.
bool plan_fprop(const ConvPass& pass, FpropPlan* plan);

// Runs a planned pass. The packed weights must follow the plan's unit order.
int launch_fprop(const ConvPass& pass, const FpropPlan& plan, cudaStream_t stream,
                 uint64_t timeout_ns, int debug_stall);

}  // namespace cnd
