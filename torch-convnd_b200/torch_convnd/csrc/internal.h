// Internal declarations shared by the C-ABI translation units (host + device).
#pragma once

#include <cstddef>
#include <cstdint>

#include "convnd_b200.h"

namespace cnd {

// ---- error reporting (problem.cpp) -----------------------------------------------------
int fail(int status, const char* format, ...);
void clear_error();
const char* last_error();
int default_fp32_mode();
void set_default_fp32_mode(int mode);

// ---- fast-path limits ------------------------------------------------------------------
constexpr int kMaxOuter = 6;       // spatial axes folded into the TMA "merged" dimension
constexpr int kMaxFastRank = kMaxOuter + 3;
constexpr int kMaxBoxes = 16;      // boxes per 128-row tile
constexpr int kTileRows = 128;     // MMA M

// Device error word (device-global, one per library instance and device).
unsigned int* device_error_word();
void count_launch(int n = 1);

// Geometry of one implicit-GEMM pass, in the "box" decomposition used by the tcgen05
// kernels: the last three spatial axes are tiled by a dense box of output positions
// (b[0] x b[1] x b[2], innermost last) that one TMA load fetches for each tap; every
// other spatial axis, the batch and the group index are folded into one "merged" TMA
// dimension whose validity per tap is decided by the producer thread.
struct BoxGeom {
  int b[3];
  int nbox[3];
  int out[3], in[3], k[3], s[3], d[3], p[3];
  int n_outer;
  int out_o[kMaxOuter], in_o[kMaxOuter], k_o[kMaxOuter], s_o[kMaxOuter], d_o[kMaxOuter],
      p_o[kMaxOuter];
  int64_t in_o_stride[kMaxOuter];  // stride of each outer axis in the merged input index
  int64_t out_o_stride[kMaxOuter]; // stride of each outer axis in the outer output index
  int64_t batch;
  int64_t groups;
  int64_t outer_count;      // batch * prod(out_o)
  int64_t boxes_per_group;  // outer_count * nbox[0]*nbox[1]*nbox[2]
  int64_t in_merged_per_ng; // prod(in_o)
  int64_t out_outer_vol;    // prod(out_o)
  int64_t out_box_vol;      // out[0]*out[1]*out[2]
  int nb;                   // boxes per tile
  int box_rows;             // b[0]*b[1]*b[2]
  int taps;                 // total kernel volume
};

}  // namespace cnd
