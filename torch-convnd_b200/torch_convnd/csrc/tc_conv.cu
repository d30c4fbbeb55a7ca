// tcgen05 implicit-GEMM convolution kernels for sm_100a.
//
// Replaces the reference's patch pipeline (unfold_cuda -> cuBLAS bmm -> fold_cuda,
// src/torch_convnd/csrc/convnd_cuda.cu:173-213 and convnd.cpp:305-415): no patch
// matrix is materialised. For every tap of the kernel, TMA loads a dense box of
// channels-last activations (out-of-bounds elements read as zero, which is the
// reference's implicit zero padding, convnd.h:57-76) straight into shared memory in the
// swizzled K-major (forward/dgrad) or MN-major (wgrad) layout that tcgen05.mma reads;
// fp32 accumulators live in tensor memory.
//
// Warp roles (192 threads): warp 0 = TMA producer (one thread) and TMEM owner,
// warp 1 = MMA issuer (one thread), warps 2-5 = epilogue (TMEM lanes 32*(warp%4)...).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "ptx.cuh"
#include "tc_conv.cuh"

namespace cnd {

namespace {

constexpr int kThreads = 192;
constexpr uint32_t kSiteWProducer = 0x201, kSiteWMma = 0x202, kSiteWEpilogue = 0x203;

// Per-box bookkeeping, decoded once per tile.
struct BoxInfo {
  int32_t valid;
  int32_t n;
  int32_t q[3];
  int32_t ib[3];                 // input coordinate of the box origin, tap 0
  int32_t ib_o[kMaxOuter];       // input coordinate along each outer axis, tap 0
  int64_t in_ng_base;            // merged input index of (n, g, outer origin 0)
  int64_t out_merged;            // merged output index (n, g, outer output position)
  int64_t outer_lin;             // linear outer output position (without n)
};

struct WgradKernelParams {
  BoxGeom g;
  // A load unit is one A slot: tpm separate tap tiles (halo == 0), or one halo box along
  // a1 holding all k1 taps of a (outer, t0, t2) combination, read as mtpu M tiles whose
  // atoms sit d1*b2 rows apart (halo == 1).
  int halo, mtpu, units_total, units_per_cta, entries_per_unit;
  uint32_t atom_bytes;  // LBO of the A operand: distance between the stacked taps
  int c_pad, cin_real, n_pad, n_real, tpm, mt_per_cta, mt_total, splits, kc_rows, ksteps;
  int a_row_bytes, a_layout, b_row_bytes, b_layout, b_blocks, b_blk_elems, a_stages;
  uint32_t a_tile_bytes, a_part_bytes, a_slot_bytes, b_part_bytes, b_slot_bytes, a_tx, b_tx,
      idesc, tmem_cols, a_base_off, bar_off;
  int64_t ptiles;
  // nfold = k0 > 0: the box-axis-0 taps are folded into N. Position tiles then run over
  // input-aligned slices q, B is the k0-slice dY box [q - k0 + 1, q] (atom j = slice
  // q - k0 + 1 + j = tap k0 - 1 - j), and each M tile's accumulator spans
  // n_cols = k0 * n_pad columns. Only slices whose input slice q - p0 exists are walked
  // (slices in the zero padding add nothing): the walk index is q - q_lo.
  int nfold, n_cols, q_lo;
  uint32_t b_lbo;  // B descriptor leading byte offset (between N atoms)
  // B buffers with a full/empty barrier pair each: 2 whole-tile slots, or, when folded, a
  // ring of b_ring one-slice slots (followed in memory by nfold - 1 mirror slots that
  // repeat slots 0.., so the nfold slices of any tile are consecutive slots).
  int b_ring;
  // Halo kernel: one A stage holds the boxes of every unit of a position tile, unit u at
  // u * a_unit_bytes (its kParts parts a_part_bytes apart).
  uint32_t a_unit_bytes;
  // Halo kernel: the last of the `chunks` tap chunks may hold fewer units than the
  // others; it runs over splits_last <= splits position ranges (proportionally fewer
  // CTAs, each as busy as a full chunk's), and its CTAs write zeros into the partial slots
  // it leaves unused.
  int chunks, splits_last;
  int outer_combos;  // product of the outer axes' kernel extents (<= 64)
  float* partial;
  unsigned int* err;
  uint64_t timeout_ns;
};

// One kernel tap of a weight-gradient CTA: offsets along the three box axes, the index
// of its outer-axis tap combination and that combination's merged-coordinate delta.
struct TapEntry {
  int32_t dx0, dx1, dx2;
  int32_t outer;
  int32_t delta;
};

// Offsets (t * dilation) of one outer-axis tap combination.
struct OuterCombo {
  int32_t off[kMaxOuter];
};

constexpr int kMaxOuterCombos = 64;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uintptr_t v = reinterpret_cast<uintptr_t>(p);
  return reinterpret_cast<uint8_t*>((v + 1023) & ~static_cast<uintptr_t>(1023));
}

// Walks box indices in order (q2 fastest, then q1, q0, outer position, batch) without
// divisions; the outer coordinates are re-derived only when the outer position changes.
struct BoxCursor {
  int64_t bt;
  int q[3];
  int64_t outer_lin, n;
  bool outer_changed;
};

__device__ __forceinline__ void cursor_init(const BoxGeom& g, int64_t bt, BoxCursor& c) {
  c.bt = bt;
  int64_t rest = bt;
  c.q[2] = static_cast<int>(rest % g.nbox[2]);
  rest /= g.nbox[2];
  c.q[1] = static_cast<int>(rest % g.nbox[1]);
  rest /= g.nbox[1];
  c.q[0] = static_cast<int>(rest % g.nbox[0]);
  rest /= g.nbox[0];
  c.outer_lin = rest % g.out_outer_vol;
  c.n = rest / g.out_outer_vol;
  c.outer_changed = true;
}

__device__ __forceinline__ void cursor_next(const BoxGeom& g, BoxCursor& c) {
  ++c.bt;
  c.outer_changed = false;
  if (++c.q[2] < g.nbox[2]) return;
  c.q[2] = 0;
  if (++c.q[1] < g.nbox[1]) return;
  c.q[1] = 0;
  if (++c.q[0] < g.nbox[0]) return;
  c.q[0] = 0;
  c.outer_changed = true;
  if (++c.outer_lin < g.out_outer_vol) return;
  c.outer_lin = 0;
  ++c.n;
}

// Same walk with q[0] fastest (then q[2], q[1], outer position, batch): folded weight
// gradients visit consecutive box-axis-0 slices of one (q1, q2) column in a row.
__device__ __forceinline__ void cursor_init_q0(const BoxGeom& g, int64_t bt, BoxCursor& c) {
  c.bt = bt;
  int64_t rest = bt;
  c.q[0] = static_cast<int>(rest % g.nbox[0]);
  rest /= g.nbox[0];
  c.q[2] = static_cast<int>(rest % g.nbox[2]);
  rest /= g.nbox[2];
  c.q[1] = static_cast<int>(rest % g.nbox[1]);
  rest /= g.nbox[1];
  c.outer_lin = rest % g.out_outer_vol;
  c.n = rest / g.out_outer_vol;
  c.outer_changed = true;
}

__device__ __forceinline__ void cursor_next_q0(const BoxGeom& g, BoxCursor& c) {
  ++c.bt;
  c.outer_changed = false;
  if (++c.q[0] < g.nbox[0]) return;
  c.q[0] = 0;
  if (++c.q[2] < g.nbox[2]) return;
  c.q[2] = 0;
  if (++c.q[1] < g.nbox[1]) return;
  c.q[1] = 0;
  c.outer_changed = true;
  if (++c.outer_lin < g.out_outer_vol) return;
  c.outer_lin = 0;
  ++c.n;
}

// Fills a BoxInfo from the cursor. The outer-axis fields (ib_o, in_ng_base without the
// tap-0 origins, out_merged) are recomputed only when `refresh_outer` is set.
__device__ __forceinline__ void cursor_box(const BoxGeom& g, const BoxCursor& c, int grp,
                                           bool refresh_outer, BoxInfo& info) {
  info.valid = c.bt < g.boxes_per_group ? 1 : 0;
  info.q[0] = c.q[0];
  info.q[1] = c.q[1];
  info.q[2] = c.q[2];
#pragma unroll
  for (int a = 0; a < 3; ++a) info.ib[a] = c.q[a] * g.b[a] * g.s[a] - g.p[a];
  if (refresh_outer) {
    info.n = static_cast<int32_t>(c.n);
    info.outer_lin = c.outer_lin;
    int64_t o = c.outer_lin;
#pragma unroll
    for (int a = kMaxOuter - 1; a >= 0; --a) {
      if (a < g.n_outer) {
        const int64_t coord = o % g.out_o[a];
        o /= g.out_o[a];
        info.ib_o[a] = static_cast<int32_t>(coord * g.s_o[a] - g.p_o[a]);
      } else {
        info.ib_o[a] = 0;
      }
    }
    int64_t base = (c.n * g.groups + grp) * g.in_merged_per_ng;
#pragma unroll
    for (int a = 0; a < kMaxOuter; ++a) {
      if (a < g.n_outer) base += static_cast<int64_t>(info.ib_o[a]) * g.in_o_stride[a];
    }
    info.in_ng_base = base;
    info.out_merged = (c.n * g.groups + grp) * g.out_outer_vol + c.outer_lin;
  }
}

// ---------------------------------------------------------------------------------------
// Weight-gradient kernel for per-tap plans (each tap tile its own TMA box; halo plans run
// wgrad_halo_kernel below). Grid (split, tap chunk, group). Each CTA accumulates
// mt_per_cta tiles of 128 (tap, channel) rows x n_pad output channels in TMEM over its
// range of position tiles, then writes one fp32 partial.
//
// kParts > 1 runs error-compensated products for float32 problems: each operand arrives
// as kParts bfloat16 terms (hi, mid[, lo]) and the MMA sums the cross products whose
// combined magnitude is above fp32 rounding, smallest first: 3 products for two terms,
// 6 for three (the latter is as accurate as fp32 accumulation).
// Number of cross products for kParts terms per operand, and the term indices of
// product q (smallest magnitude first).
template <int kParts>
__host__ __device__ constexpr int product_count() {
  return kParts == 1 ? 1 : (kParts == 2 ? 3 : 6);
}

__host__ __device__ constexpr int product_a(int parts, int q) {
  return parts == 2 ? (q == 0 ? 1 : 0)
                    : (parts == 3 ? (q == 0 ? 2 : (q == 1 || q == 3) ? 1 : 0) : 0);
}

__host__ __device__ constexpr int product_b(int parts, int q) {
  return parts == 2 ? (q == 1 ? 1 : 0)
                    : (parts == 3 ? (q == 2 ? 2 : (q == 1 || q == 4) ? 1 : 0) : 0);
}

struct WgradMaps {
  CUtensorMap act[3];
  CUtensorMap grad[3];
};

// Tables of a CTA's tap entries and of the outer-axis tap combinations, filled by the
// 128 epilogue threads (idle until the main loop ends). Non-halo: entry = one tap. Halo:
// entry = one unit, a (outer, t0, t2) combination (outer, t2 when folded) whose k1 taps
// along a1 share one box; its tap fields describe t1 = 0.
__device__ __forceinline__ void wgrad_tables(const WgradKernelParams& P, int t, int unit_first,
                                             int entry_count, OuterCombo* combos,
                                             TapEntry* taps) {
  const BoxGeom& g = P.g;
  for (int c = t; c < P.outer_combos; c += 128) {
    int rest = c;
#pragma unroll
    for (int a = kMaxOuter - 1; a >= 0; --a) {
      if (a < g.n_outer) {
        combos[c].off[a] = (rest % g.k_o[a]) * g.d_o[a];
        rest /= g.k_o[a];
      } else {
        combos[c].off[a] = 0;
      }
    }
  }
  for (int i = t; i < entry_count; i += 128) {
    int tap;
    if (P.halo) {
      const int unit = unit_first + i;
      const int t2 = unit % g.k[2];
      const int rest = unit / g.k[2];  // (outer, t0) row-major; outer alone when folded
      tap = (P.nfold ? rest * g.k[0] * g.k[1] : rest * g.k[1]) * g.k[2] + t2;
    } else {
      tap = unit_first * P.tpm + i;
    }
    TapEntry e{0, 0, 0, 0, 0};
    if (tap < g.taps) {
      int rest = tap;
      e.dx2 = (rest % g.k[2]) * g.d[2];
      rest /= g.k[2];
      e.dx1 = (rest % g.k[1]) * g.d[1];
      rest /= g.k[1];
      e.dx0 = (rest % g.k[0]) * g.d[0];
      rest /= g.k[0];
      e.outer = rest;  // row-major index over the outer tap axes
      int64_t delta = 0;
#pragma unroll
      for (int a = kMaxOuter - 1; a >= 0; --a) {
        if (a < g.n_outer) {
          delta += static_cast<int64_t>(rest % g.k_o[a]) * g.d_o[a] * g.in_o_stride[a];
          rest /= g.k_o[a];
        }
      }
      e.delta = static_cast<int32_t>(delta);
    } else {
      e.outer = -1;  // padding slot of the last M tile: loads read zeros
    }
    taps[i] = e;
  }
}

// Epilogue of a weight-gradient CTA (warps 2-5): waits for the last MMA, then writes
// its accumulators (mt_count M tiles of n_cols columns) as one fp32 partial. A chunk run
// over chunk_splits < P.splits position ranges also writes zeros into the slots
// chunk_splits..P.splits-1 of its taps (CTA `split` takes every chunk_splits-th of them),
// so that the reduction over P.splits slots finds every slot written.
__device__ __forceinline__ void wgrad_epilogue(const WgradKernelParams& P, uint32_t tmem,
                                               uint64_t* acc_bar, const volatile uint32_t* progress,
                                               int split, int grp, int unit_first, int unit_count,
                                               bool empty_range, int warp, int lane,
                                               int chunk_splits) {
  const BoxGeom& g = P.g;
  const dev::ErrorWord err{P.err};
  dev::mbar_wait_progress(acc_bar, 0, progress, err, kSiteWEpilogue, P.timeout_ns);
  dev::tc_fence_after();
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const int jt = row / P.c_pad;
  const int ci = row - jt * P.c_pad;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
  const int mt_count = unit_count * P.mtpu;
  const int64_t slot_stride = g.groups * g.taps * static_cast<int64_t>(P.cin_real) * P.n_real;
  for (int mt = 0; mt < mt_count; ++mt) {
    int tap;
    bool valid;
    if (P.halo) {
      const int unit = unit_first + mt / P.mtpu;
      const int t1 = (mt % P.mtpu) * P.tpm + jt;
      const int t2 = unit % g.k[2];
      const int rest = unit / g.k[2];  // (outer, t0), or outer alone when folded
      tap = ((P.nfold ? rest * g.k[0] : rest) * g.k[1] + t1) * g.k[2] + t2;
      valid = t1 < g.k[1] && ci < P.cin_real;
    } else {
      tap = (unit_first + mt) * P.tpm + jt;
      valid = tap < g.taps && ci < P.cin_real;
    }
    for (int c = 0; c < P.n_cols / 16; ++c) {
      // Column block j of a folded accumulator is tap k0 - 1 - j along box axis 0.
      const int block = (c * 16) / P.n_pad;
      const int co_base = c * 16 - block * P.n_pad;
      const int tap_c = P.nfold ? tap + (P.nfold - 1 - block) * g.k[1] * g.k[2] : tap;
      float* dst = P.partial +
                   ((((static_cast<int64_t>(split) * g.groups + grp) * g.taps + tap_c) *
                         P.cin_real +
                     ci) *
                    P.n_real);
      uint32_t v[16];
      __syncwarp();
      dev::tmem_load16(lane_addr + static_cast<uint32_t>(mt * P.n_cols + c * 16), v);
      dev::tmem_load_wait();
      if (valid) {
        if (empty_range) {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0u;
        }
        if ((P.n_real & 3) == 0 && co_base + 16 <= P.n_real) {
          // 16-byte stores of four consecutive output channels (row is 16-byte aligned)
          float4* d4 = reinterpret_cast<float4*>(dst + co_base);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            d4[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int co = co_base + i;
            if (co < P.n_real) dst[co] = __uint_as_float(v[i]);
          }
        }
        for (int slot = chunk_splits + split; slot < P.splits; slot += chunk_splits) {
          float* zdst = dst + static_cast<int64_t>(slot - split) * slot_stride;
          for (int i = 0; i < 16; ++i) {
            const int co = co_base + i;
            if (co < P.n_real) zdst[co] = 0.0f;
          }
        }
      }
    }
  }
}

template <int kParts, int kKSteps>
__global__ void __launch_bounds__(kThreads, 1)
    wgrad_kernel(const __grid_constant__ WgradMaps maps,
                 const __grid_constant__ WgradKernelParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* b_base = smem;                       // 2 dy slots
  uint8_t* a_base = smem + P.a_base_off;        // a_stages A slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bar_off);
  uint64_t* b_full = bars;
  uint64_t* b_empty = bars + P.b_ring;
  uint64_t* a_full = bars + 2 * P.b_ring;
  uint64_t* a_empty = a_full + P.a_stages;
  uint64_t* acc_bar = a_empty + P.a_stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
  volatile uint32_t* progress = tmem_slot + 1;
  BoxInfo* boxes = reinterpret_cast<BoxInfo*>(tmem_slot + 4);
  uint64_t* box_mask = reinterpret_cast<uint64_t*>(boxes + kMaxBoxes);
  OuterCombo* combos = reinterpret_cast<OuterCombo*>(box_mask + kMaxBoxes);
  TapEntry* taps = reinterpret_cast<TapEntry*>(combos + kMaxOuterCombos);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int chunk = blockIdx.y;
  const int grp = blockIdx.z;
  const BoxGeom& g = P.g;
  const dev::ErrorWord err{P.err};
  const int64_t p_begin = P.ptiles * split / P.splits;
  const int64_t p_end = P.ptiles * (split + 1) / P.splits;
  const int unit_first = chunk * P.units_per_cta;
  const int unit_count = min(P.units_per_cta, P.units_total - unit_first);
  const int entry_count = unit_count * P.entries_per_unit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P.b_ring; ++s) {
      dev::mbar_init(&b_full[s], 1);
      dev::mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < P.a_stages; ++s) {
      dev::mbar_init(&a_full[s], 1);
      dev::mbar_init(&a_empty[s], 1);
    }
    dev::mbar_init(acc_bar, 1);
    *progress = 0;
    dev::fence_barrier_init();
  }
  if (warp == 0) {
    __syncwarp();
    dev::tmem_alloc(tmem_slot, P.tmem_cols);
  }
  if (warp >= 2) wgrad_tables(P, threadIdx.x - 64, unit_first, entry_count, combos, taps);
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (whole warp) ----------------
    // Lane 0 keeps the position-tile bookkeeping in shared memory; the loads of a tile or
    // unit (boxes x taps x parts) are spread over the 32 lanes, which issue them in
    // parallel. One lane alone issued only one load every several hundred cycles, too
    // few for units made of many small per-tap tiles.
    if (lane == 0) {
      for (int part = 0; part < kParts; ++part) {
        dev::prefetch_tensormap(&maps.act[part]);
        dev::prefetch_tensormap(&maps.grad[part]);
      }
    }
    int a_stage = 0, b_slot = 0;
    uint32_t a_phase = 0, b_phase = 0;
    bool ok = true;
    BoxCursor cursor;
    cursor_init(g, p_begin * g.nb, cursor);
    const int b_loads = g.nb * P.b_blocks * kParts;
    const int a_loads = P.entries_per_unit * g.nb * kParts;
    for (int64_t pt = p_begin; pt < p_end && ok; ++pt) {
      // Boxes of this position tile and, per box, which outer tap combinations stay
      // inside the input (bit c of box_mask; recomputed when the outer position moves).
      if (lane == 0) {
        for (int j = 0; j < g.nb; ++j) {
          BoxInfo& B = boxes[j];
          const bool refresh = cursor.outer_changed || g.nb > 1;
          cursor_box(g, cursor, grp, refresh, B);
          if (refresh) {
            uint64_t mask = 0;
            for (int c = 0; c < P.outer_combos; ++c) {
              bool inside = true;
#pragma unroll
              for (int a = 0; a < kMaxOuter; ++a) {
                if (a < g.n_outer) {
                  const int coord = B.ib_o[a] + combos[c].off[a];
                  inside = inside && coord >= 0 && coord < g.in_o[a];
                }
              }
              if (inside) mask |= uint64_t{1} << c;
            }
            box_mask[j] = mask;
          }
          cursor_next(g, cursor);
        }
      }
      __syncwarp();
      // All TMA loads of the tile form one pool of jobs spread over the lanes: the dY
      // loads first, then every unit's activation loads. Each lane waits on the barrier of
      // its own job's slot; the first load of a slot posts the slot's expected bytes (a
      // load may complete before that: the phase cannot finish without the posting
      // arrival).
      // Rounds of jobs: each A stage appears at most once per round. Lanes of a round
      // wait concurrently, and an mbarrier parity wait is exact only for the phase right
      // after the last one known complete; a second use of a stage inside a round could
      // wait two phases ahead and pass at once.
      bool lane_ok = true;
      for (int round_first = 0; round_first < unit_count || round_first == 0;
           round_first += P.a_stages) {
        const int round_units = unit_count - round_first < P.a_stages
                                    ? unit_count - round_first
                                    : P.a_stages;
        const int round_b = round_first == 0 ? b_loads : 0;
        const int jobs = round_b + round_units * a_loads;
        for (int l = lane; l < jobs && lane_ok; l += 32) {
          if (l < round_b) {
            if (!dev::mbar_wait(&b_empty[b_slot], b_phase ^ 1u, err, kSiteWProducer,
                                P.timeout_ns)) {
              lane_ok = false;
              break;
            }
            if (l == 0) dev::mbar_arrive_expect_tx(&b_full[b_slot], P.b_tx);
            const int part = l % kParts;
            const int blk = (l / kParts) % P.b_blocks;
            const int j = l / (kParts * P.b_blocks);
            const int32_t mo = boxes[j].valid ? static_cast<int32_t>(boxes[j].out_merged) : -1;
            uint8_t* dst = b_base + b_slot * P.b_slot_bytes + blk * (P.kc_rows * 128) +
                           j * g.box_rows * P.b_row_bytes;
            dev::tma_load_5d(dst + part * P.b_part_bytes, &maps.grad[part], &b_full[b_slot],
                             blk * P.b_blk_elems, boxes[j].q[2] * g.b[2],
                             boxes[j].q[1] * g.b[1], boxes[j].q[0] * g.b[0], mo);
          } else {
            const int la = l - round_b;
            const int unit = round_first + la / a_loads;
            const int lu = la - (unit - round_first) * a_loads;
            // Padding taps past the last one (tap tiles of the last unit) are not loaded:
            // their accumulator rows are never read, so stale slot contents do no harm.
            // Their jobs return before the wait: once the unit's real loads land the MMA
            // may release the stage, and a later wait would then be one phase ahead.
            const int unit_taps = min(P.entries_per_unit, g.taps - (unit_first + unit) * P.tpm);
            const int jt = lu / (kParts * g.nb);
            if (jt >= unit_taps) continue;
            int stage = a_stage + unit;
            uint32_t par = a_phase;
            while (stage >= P.a_stages) {
              stage -= P.a_stages;
              par ^= 1u;
            }
            if (!dev::mbar_wait(&a_empty[stage], par ^ 1u, err, kSiteWProducer, P.timeout_ns)) {
              lane_ok = false;
              break;
            }
            if (lu == 0) {
              dev::mbar_arrive_expect_tx(
                  &a_full[stage], static_cast<uint32_t>(unit_taps) * (P.a_tx / P.entries_per_unit));
            }
            const int part = lu % kParts;
            const int j = (lu / kParts) % g.nb;
            const TapEntry e = taps[unit * P.entries_per_unit + jt];
            const BoxInfo& B = boxes[j];
            const bool inside = B.valid && e.outer >= 0 && ((box_mask[j] >> e.outer) & 1u);
            const int32_t mc = inside ? static_cast<int32_t>(B.in_ng_base + e.delta) : -1;
            uint8_t* dst = a_base + stage * P.a_slot_bytes + jt * P.a_tile_bytes +
                           j * g.box_rows * P.a_row_bytes;
            dev::tma_load_5d(dst + part * P.a_part_bytes, &maps.act[part], &a_full[stage], 0,
                             B.ib[2] + e.dx2, B.ib[1] + e.dx1, B.ib[0] + e.dx0, mc);
          }
        }
        if (__all_sync(0xffffffffu, lane_ok) == 0) break;
        if (round_first + P.a_stages >= unit_count) break;
      }
      ok = __all_sync(0xffffffffu, lane_ok) != 0;
      if (!ok) break;
      // advance the B slot and the A stages past this tile
      if (++b_slot == 2) {
        b_slot = 0;
        b_phase ^= 1u;
      }
      for (int u = 0; u < unit_count; ++u) {
        if (++a_stage == P.a_stages) {
          a_stage = 0;
          a_phase ^= 1u;
        }
      }
      // Every lane has read this tile's boxes before lane 0 rewrites them.
      __syncwarp();
    }
    (void)ok;
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop and executes every MMA / commit; elect.sync inside
    // each instruction picks the issuing lane, so control flow never diverges.
    const bool leader = lane == 0;
    const uint32_t tmem_u = dev::warp_uniform(tmem);
    int a_stage = 0, b_slot = 0;
    uint32_t a_phase = 0, b_phase = 0;
    // Constant descriptor parts; per MMA only the start-address field (address >> 4)
    // changes, and it never carries (shared memory is below 256 KB).
    const uint64_t a_hi = dev::make_smem_desc(0, P.atom_bytes, 8u * P.a_row_bytes, P.a_layout);
    const uint32_t group_units = (static_cast<uint32_t>(P.tpm) * P.atom_bytes) >> 4;
    const uint64_t b_hi = dev::make_smem_desc(0, P.b_lbo, 8u * P.b_row_bytes, P.b_layout);
    const uint32_t a_step = (16u * P.a_row_bytes) >> 4;  // one K step = 16 positions
    const uint32_t b_step = (16u * P.b_row_bytes) >> 4;
    const uint32_t a_part = P.a_part_bytes >> 4;
    const uint32_t b_part = P.b_part_bytes >> 4;
    bool ok = true;
    for (int64_t pt = p_begin; pt < p_end && ok; ++pt) {
      if (!dev::mbar_wait_warp(&b_full[b_slot], b_phase, err, kSiteWMma, P.timeout_ns)) break;
      const uint32_t bs =
          dev::warp_uniform(dev::smem_u32(b_base + b_slot * P.b_slot_bytes) >> 4);
      const uint32_t first_tile = pt == p_begin ? 1u : 0u;
      for (int unit = 0; unit < unit_count; ++unit) {
        if (!dev::mbar_wait_warp(&a_full[a_stage], a_phase, err, kSiteWMma, P.timeout_ns)) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const uint32_t as =
            dev::warp_uniform(dev::smem_u32(a_base + a_stage * P.a_slot_bytes) >> 4);
        for (int gi = 0; gi < P.mtpu; ++gi) {
          const uint32_t d = tmem_u + static_cast<uint32_t>((unit * P.mtpu + gi) * P.n_cols);
          const uint32_t ag = as + static_cast<uint32_t>(gi) * group_units;
          // K steps unrolled at compile time (a runtime loop between MMAs slows issue).
#pragma unroll
          for (int ks = 0; ks < kKSteps; ++ks) {
            const uint32_t aoff = ag + static_cast<uint32_t>(ks) * a_step;
            const uint32_t boff = bs + static_cast<uint32_t>(ks) * b_step;
#pragma unroll
            for (int q = 0; q < product_count<kParts>(); ++q) {
              const uint64_t ad = a_hi | (aoff + product_a(kParts, q) * a_part);
              const uint64_t bd = b_hi | (boff + product_b(kParts, q) * b_part);
              const uint32_t acc = (first_tile != 0u && ks == 0 && q == 0) ? 0u : 1u;
              dev::mma_f16_warp(d, ad, bd, P.idesc, acc);
            }
          }
        }
        dev::mma_commit_warp(&a_empty[a_stage]);
        if (++a_stage == P.a_stages) {
          a_stage = 0;
          a_phase ^= 1u;
        }
      }
      dev::mma_commit_warp(&b_empty[b_slot]);
      if (++b_slot == 2) {
        b_slot = 0;
        b_phase ^= 1u;
      }
      if (leader) *progress = static_cast<uint32_t>(pt - p_begin + 1);
      __syncwarp();
    }
    dev::mma_commit_warp(acc_bar);
  } else if (warp >= 2) {
    wgrad_epilogue(P, tmem, acc_bar, progress, split, grp, unit_first, unit_count,
                   p_begin >= p_end, warp, lane, P.splits);
  }
  dev::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, P.tmem_cols);
  }
}

// ---------------------------------------------------------------------------------------
// Weight-gradient kernel for halo plans (one box per tile, one A box per unit). Same
// decomposition, MMAs and epilogue as wgrad_kernel, with a leaner pipeline:
//  * one A stage per position tile holding every unit's box, so the MMA warp takes one
//    barrier handoff per tile instead of one per unit;
//  * the producer keeps all per-tile state in registers: lane 0 walks the boxes and
//    broadcasts each box with warp shuffles, lane u holds unit u's tap entry. Loads from
//    shared memory are slow while the tensor core streams operands from it, and a
//    producer that read its tables from there fell behind the MMAs.
template <int kParts, int kKSteps>
__global__ void __launch_bounds__(kThreads, 1)
    wgrad_halo_kernel(const __grid_constant__ WgradMaps maps,
                      const __grid_constant__ WgradKernelParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* b_base = smem;
  uint8_t* a_base = smem + P.a_base_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bar_off);
  // Every load of a position tile (its A boxes and its new dY slices) signals the tile's
  // a_full barrier: the MMA warp waits once per tile. b_empty[slot] frees a dY slot.
  uint64_t* b_empty = bars + P.b_ring;
  uint64_t* a_full = bars + 2 * P.b_ring;
  uint64_t* a_empty = a_full + P.a_stages;
  uint64_t* acc_bar = a_empty + P.a_stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
  volatile uint32_t* progress = tmem_slot + 1;
  OuterCombo* combos = reinterpret_cast<OuterCombo*>(tmem_slot + 4);
  TapEntry* taps = reinterpret_cast<TapEntry*>(combos + kMaxOuterCombos);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Grid x: `splits` CTAs for each full chunk, then splits_last for the last chunk.
  const int full_ctas = (P.chunks - 1) * P.splits;
  const int bx = static_cast<int>(blockIdx.x);
  const bool last = bx >= full_ctas;
  const int chunk = last ? P.chunks - 1 : bx / P.splits;
  const int split = last ? bx - full_ctas : bx - chunk * P.splits;
  const int chunk_splits = last ? P.splits_last : P.splits;
  const int grp = blockIdx.z;
  const BoxGeom& g = P.g;
  const dev::ErrorWord err{P.err};
  const int unit_first = chunk * P.units_per_cta;
  const int unit_count = max(0, min(P.units_per_cta, P.units_total - unit_first));
  // Position-tile range of this CTA (empty for a CTA without units).
  const int64_t p_begin = P.ptiles * split / chunk_splits;
  const int64_t p_end = unit_count > 0 ? P.ptiles * (split + 1) / chunk_splits : p_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P.b_ring; ++s) dev::mbar_init(&b_empty[s], 1);
    for (int s = 0; s < P.a_stages; ++s) {
      dev::mbar_init(&a_full[s], 1);
      dev::mbar_init(&a_empty[s], 1);
    }
    dev::mbar_init(acc_bar, 1);
    *progress = 0;
    dev::fence_barrier_init();
  }
  if (warp == 0) {
    __syncwarp();
    dev::tmem_alloc(tmem_slot, P.tmem_cols);
  }
  if (warp >= 2) wgrad_tables(P, threadIdx.x - 64, unit_first, unit_count, combos, taps);
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers (whole warps, register state) ----------------
    // Warp 0 loads the activation boxes of every tile and posts each stage's bytes;
    // warp 2 (an epilogue warp, idle until the main loop ends) loads the dY slices. Both
    // walk the same tiles and wait for a stage to be free before loading into it, and all
    // loads of a tile signal its a_full barrier.
    const bool a_role = warp == 0;
    if (lane == 0 && a_role) {
      for (int part = 0; part < kParts; ++part) {
        dev::prefetch_tensormap(&maps.act[part]);
        dev::prefetch_tensormap(&maps.grad[part]);
      }
    }
    TapEntry mine{0, 0, 0, -1, 0};
    if (lane < unit_count) mine = taps[lane];
    int a_stage = 0, b_slot = 0;
    uint32_t a_phase = 0, b_phase = 0;
    bool ok = true;
    BoxCursor cursor;
    if (P.nfold) {
      cursor_init_q0(g, p_begin, cursor);
    } else {
      cursor_init(g, p_begin, cursor);
    }
    BoxInfo box;  // lane 0's walk; broadcast per tile
    box.n = 0;
    box.outer_lin = 0;
    box.in_ng_base = 0;
    box.out_merged = 0;
    uint64_t mask = 0;
    int ring_slot = 0;
    uint32_t ring_phase = 0;
    int q0 = P.nfold ? static_cast<int>(p_begin % g.nbox[0]) : 0;
    const uint32_t stage_tx = P.a_tx * static_cast<uint32_t>(unit_count);
    const int b_loads = P.b_blocks * kParts;
    for (int64_t pt = p_begin; pt < p_end && ok; ++pt) {
      if (lane == 0) {
        const bool refresh = cursor.outer_changed;
        cursor_box(g, cursor, grp, refresh, box);
        if (refresh && a_role) {
          // outer tap combinations that stay inside the input (rare: once per outer step)
          mask = 0;
          for (int c = 0; c < P.outer_combos; ++c) {
            bool inside = true;
#pragma unroll
            for (int a = 0; a < kMaxOuter; ++a) {
              if (a < g.n_outer) {
                const int coord = box.ib_o[a] + combos[c].off[a];
                inside = inside && coord >= 0 && coord < g.in_o[a];
              }
            }
            if (inside) mask |= uint64_t{1} << c;
          }
        }
        if (P.nfold) {
          cursor_next_q0(g, cursor);
        } else {
          cursor_next(g, cursor);
        }
      }
      const unsigned full = 0xffffffffu;
      const int valid = __shfl_sync(full, box.valid, 0);
      const int ib0 = __shfl_sync(full, box.ib[0], 0);
      const int ib1 = __shfl_sync(full, box.ib[1], 0);
      const int ib2 = __shfl_sync(full, box.ib[2], 0);
      const int bq0 = __shfl_sync(full, box.q[0], 0);
      const int bq1 = __shfl_sync(full, box.q[1], 0);
      const int bq2 = __shfl_sync(full, box.q[2], 0);
      const int64_t in_base = __shfl_sync(full, box.in_ng_base, 0);
      const int32_t out_m = __shfl_sync(full, static_cast<int32_t>(box.out_merged), 0);
      const uint64_t msk = __shfl_sync(full, mask, 0);
      bool lane_ok = true;
      const bool run_start = P.nfold && (pt == p_begin || q0 == 0);
      const int new_entries = P.nfold ? (run_start ? P.nfold : 1) : 0;
      // Bytes of this tile's dY loads (folded: new ring entries, mirrored slots twice).
      uint32_t b_bytes = P.b_tx;
      if (P.nfold) {
        int copies = 0, slot = ring_slot;
        for (int e = 0; e < new_entries; ++e) {
          copies += slot < P.nfold - 1 ? 2 : 1;
          if (++slot == P.b_ring) slot = 0;
        }
        b_bytes = P.b_tx * static_cast<uint32_t>(copies);
      }
      // A: every unit's box into this tile's stage, lane u loading unit u. Lane 0 posts
      // the stage's bytes, dY included (a load may land before the posting; the phase
      // cannot complete without the posting arrival).
      if (a_role && lane < unit_count) {
        if (!dev::mbar_wait(&a_empty[a_stage], a_phase ^ 1u, err, kSiteWProducer,
                            P.timeout_ns)) {
          lane_ok = false;
        } else {
          if (lane == 0) dev::mbar_arrive_expect_tx(&a_full[a_stage], stage_tx + b_bytes);
          const bool inside = valid && mine.outer >= 0 && ((msk >> mine.outer) & 1u);
          const int32_t mc = inside ? static_cast<int32_t>(in_base + mine.delta) : -1;
          uint8_t* dst = a_base + a_stage * P.a_slot_bytes + lane * P.a_unit_bytes;
#pragma unroll
          for (int part = 0; part < kParts; ++part) {
            dev::tma_load_5d(dst + part * P.a_part_bytes, &maps.act[part], &a_full[a_stage], 0,
                             ib2 + mine.dx2, ib1 + mine.dx1, ib0 + mine.dx0, mc);
          }
        }
      }
      // B: folded — the new ring entries (a mirror copy for the first nfold - 1 slots);
      // otherwise the tile's dY box into one of two slots.
      if (a_role) {
        // the dY loads belong to warp 2
      } else if (P.nfold) {
        // job index of this lane: entries in ring order, mirrored slots twice
        int l = 0, k = 0, c = -1, slot = ring_slot;
        uint32_t par = ring_phase;
        for (int e = 0; e < new_entries; ++e) {
          const int copies = slot < P.nfold - 1 ? 2 : 1;
          if (lane >= l && lane < l + copies) {
            k = e;
            c = lane - l;
            break;
          }
          l += copies;
          if (++slot == P.b_ring) {
            slot = 0;
            par ^= 1u;
          }
        }
        if (c >= 0 && lane_ok) {
          if (!dev::mbar_wait(&a_empty[a_stage], a_phase ^ 1u, err, kSiteWProducer,
                              P.timeout_ns) ||
              !dev::mbar_wait(&b_empty[slot], par ^ 1u, err, kSiteWProducer, P.timeout_ns)) {
            lane_ok = false;
          } else {
            const int dst_slot = c == 0 ? slot : P.b_ring + slot;
#pragma unroll
            for (int part = 0; part < kParts; ++part) {
              dev::tma_load_5d(b_base + dst_slot * P.b_slot_bytes + part * P.b_part_bytes,
                               &maps.grad[part], &a_full[a_stage], 0, bq2 * g.b[2],
                               bq1 * g.b[1], P.q_lo + q0 - (new_entries - 1) + k,
                               valid ? out_m : -1);
            }
          }
        }
      } else if (lane < b_loads && lane_ok) {
        if (!dev::mbar_wait(&a_empty[a_stage], a_phase ^ 1u, err, kSiteWProducer,
                            P.timeout_ns) ||
            !dev::mbar_wait(&b_empty[b_slot], b_phase ^ 1u, err, kSiteWProducer,
                            P.timeout_ns)) {
          lane_ok = false;
        } else {
          const int part = lane % kParts;
          const int blk = lane / kParts;
          uint8_t* dst = b_base + b_slot * P.b_slot_bytes + blk * (P.kc_rows * 128);
          dev::tma_load_5d(dst + part * P.b_part_bytes, &maps.grad[part], &a_full[a_stage],
                           blk * P.b_blk_elems, bq2 * g.b[2], bq1 * g.b[1], bq0 * g.b[0],
                           valid ? out_m : -1);
        }
      }
      ok = __all_sync(0xffffffffu, lane_ok) != 0;
      if (!ok) break;
      if (P.nfold) {
        for (int e = 0; e < new_entries; ++e) {
          if (++ring_slot == P.b_ring) {
            ring_slot = 0;
            ring_phase ^= 1u;
          }
        }
        if (++q0 == g.nbox[0]) q0 = 0;
      } else if (++b_slot == 2) {
        b_slot = 0;
        b_phase ^= 1u;
      }
      if (++a_stage == P.a_stages) {
        a_stage = 0;
        a_phase ^= 1u;
      }
    }
    if (!ok) {
      // A wait expired: give loads already issued time to land (they take microseconds)
      // before the CTA's shared memory goes away.
      const uint64_t start = dev::global_timer_ns();
      while (dev::global_timer_ns() - start < 200000u) __nanosleep(1000);
    }
  }
  if (warp == 1) {
    // ---------------- MMA issuer (converged warp, elect.sync inside each MMA) ----------------
    const bool leader = lane == 0;
    const uint32_t tmem_u = dev::warp_uniform(tmem);
    int a_stage = 0, b_slot = 0;
    uint32_t a_phase = 0;
    const uint64_t a_hi = dev::make_smem_desc(0, P.atom_bytes, 8u * P.a_row_bytes, P.a_layout);
    const uint32_t group_units = (static_cast<uint32_t>(P.tpm) * P.atom_bytes) >> 4;
    const uint64_t b_hi = dev::make_smem_desc(0, P.b_lbo, 8u * P.b_row_bytes, P.b_layout);
    const uint32_t a_step = (16u * P.a_row_bytes) >> 4;
    const uint32_t b_step = (16u * P.b_row_bytes) >> 4;
    const uint32_t a_part = P.a_part_bytes >> 4;
    const uint32_t b_part = P.b_part_bytes >> 4;
    const uint32_t unit_units = P.a_unit_bytes >> 4;
    bool ok = true;
    int ring_slot = 0, first_slot = 0;
    int q0 = P.nfold ? static_cast<int>(p_begin % g.nbox[0]) : 0;
    for (int64_t pt = p_begin; pt < p_end && ok; ++pt) {
      uint32_t bs;
      bool run_end = false;
      if (P.nfold) {
        const bool run_start = pt == p_begin || q0 == 0;
        run_end = pt == p_end - 1 || q0 == g.nbox[0] - 1;
        if (++q0 == g.nbox[0]) q0 = 0;
        if (run_start) {
          first_slot = ring_slot;
        } else if (++first_slot == P.b_ring) {
          first_slot = 0;
        }
        if (run_start) {
          ring_slot += P.nfold;
          if (ring_slot >= P.b_ring) ring_slot -= P.b_ring;
        } else if (++ring_slot == P.b_ring) {
          ring_slot = 0;
        }
        bs = dev::warp_uniform(dev::smem_u32(b_base + first_slot * P.b_slot_bytes) >> 4);
      } else {
        bs = dev::warp_uniform(dev::smem_u32(b_base + b_slot * P.b_slot_bytes) >> 4);
      }
      if (!dev::mbar_wait_warp(&a_full[a_stage], a_phase, err, kSiteWMma, P.timeout_ns)) break;
      dev::tc_fence_after();
      const uint32_t first_tile = pt == p_begin ? 1u : 0u;
      const uint32_t as =
          dev::warp_uniform(dev::smem_u32(a_base + a_stage * P.a_slot_bytes) >> 4);
      for (int unit = 0; unit < unit_count; ++unit) {
        for (int gi = 0; gi < P.mtpu; ++gi) {
          const uint32_t d = tmem_u + static_cast<uint32_t>((unit * P.mtpu + gi) * P.n_cols);
          const uint32_t ag = as + static_cast<uint32_t>(unit) * unit_units +
                              static_cast<uint32_t>(gi) * group_units;
#pragma unroll
          for (int ks = 0; ks < kKSteps; ++ks) {
            const uint32_t aoff = ag + static_cast<uint32_t>(ks) * a_step;
            const uint32_t boff = bs + static_cast<uint32_t>(ks) * b_step;
#pragma unroll
            for (int q = 0; q < product_count<kParts>(); ++q) {
              const uint64_t ad = a_hi | (aoff + product_a(kParts, q) * a_part);
              const uint64_t bd = b_hi | (boff + product_b(kParts, q) * b_part);
              const uint32_t acc = (first_tile != 0u && ks == 0 && q == 0) ? 0u : 1u;
              dev::mma_f16_warp(d, ad, bd, P.idesc, acc);
            }
          }
        }
      }
      dev::mma_commit_warp(&a_empty[a_stage]);
      if (++a_stage == P.a_stages) {
        a_stage = 0;
        a_phase ^= 1u;
      }
      if (P.nfold) {
        int slot = first_slot;
        for (int k = run_end ? P.nfold : 1; k > 0; --k) {
          dev::mma_commit_warp(&b_empty[slot]);
          if (++slot == P.b_ring) slot = 0;
        }
      } else {
        dev::mma_commit_warp(&b_empty[b_slot]);
        if (++b_slot == 2) b_slot = 0;
      }
      // progress (read by the epilogue's bounded wait) every 8 tiles
      if (((pt - p_begin) & 7) == 7 && leader) *progress = static_cast<uint32_t>(pt - p_begin + 1);
      __syncwarp();
    }
    dev::mma_commit_warp(acc_bar);
  } else if (warp >= 2) {
    wgrad_epilogue(P, tmem, acc_bar, progress, split, grp, unit_first, unit_count,
                   p_begin >= p_end, warp, lane, chunk_splits);
  }
  dev::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, P.tmem_cols);
  }
}

// =======================================================================================
// Host side
// =======================================================================================

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &status) ==
            cudaSuccess &&
        status == cudaDriverEntryPointSuccess) {
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  return encode;
}

CUtensorMapDataType map_type(int op) {
  if (op == kOpBF16) return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (op == kOpF16) return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}

CUtensorMapSwizzle map_swizzle(int row_bytes) {
  if (row_bytes == 32) return CU_TENSOR_MAP_SWIZZLE_32B;
  if (row_bytes == 64) return CU_TENSOR_MAP_SWIZZLE_64B;
  return CU_TENSOR_MAP_SWIZZLE_128B;
}

// tcgen05 shared-memory descriptor layout code for a swizzle width in bytes.
uint32_t desc_layout(int row_bytes) {
  if (row_bytes == 32) return 6;
  if (row_bytes == 64) return 4;
  return 2;
}

int element_size(int op) { return op == kOpF32 ? 4 : 2; }

// Encodes a 5-D map over a packed channels-last activation tensor
// [merged][e0][e1][e2][channels] with a box of (cblk, b2*s2, b1*s1, b0*s0, 1) and
// element strides (1, s2, s1, s0, 1).
int encode_act_map(CUtensorMap* map, const void* base, int op, int64_t channels,
                   const int64_t ext[3], int64_t merged, int cblk, const int box[3],
                   const int stride[3]) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return fail(CND_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int64_t es = element_size(op);
  cuuint64_t dims[5] = {static_cast<cuuint64_t>(channels), static_cast<cuuint64_t>(ext[2]),
                        static_cast<cuuint64_t>(ext[1]), static_cast<cuuint64_t>(ext[0]),
                        static_cast<cuuint64_t>(merged)};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(channels * es),
                           static_cast<cuuint64_t>(channels * ext[2] * es),
                           static_cast<cuuint64_t>(channels * ext[2] * ext[1] * es),
                           static_cast<cuuint64_t>(channels * ext[2] * ext[1] * ext[0] * es)};
  cuuint32_t boxd[5] = {static_cast<cuuint32_t>(cblk),
                        static_cast<cuuint32_t>(box[2] * stride[2]),
                        static_cast<cuuint32_t>(box[1] * stride[1]),
                        static_cast<cuuint32_t>(box[0] * stride[0]), 1};
  cuuint32_t estr[5] = {1, static_cast<cuuint32_t>(stride[2]), static_cast<cuuint32_t>(stride[1]),
                        static_cast<cuuint32_t>(stride[0]), 1};
  const CUresult r = encode(map, map_type(op), 5, const_cast<void*>(base), dims, strides, boxd,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            map_swizzle(static_cast<int>(cblk * es)),
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(CND_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed with code %d",
                static_cast<int>(r));
  }
  return CND_OK;
}

// Chooses the box shape (outer->inner) and boxes per tile for `rows` positions per tile.
bool plan_boxes(const int out[3], const int stride[3], int rows, int* nb_out, int b_out[3]) {
  double best = 1e30;
  bool found = false;
  for (int nb = 1; nb <= kMaxBoxes; nb *= 2) {
    const int per_box = rows / nb;
    if (per_box < 8 || per_box % 8 != 0) break;
    for (int b2 = 1; b2 <= per_box; ++b2) {
      if (per_box % b2 != 0 || b2 * stride[2] > 256) continue;
      for (int b1 = 1; b1 <= per_box / b2; ++b1) {
        if ((per_box / b2) % b1 != 0 || b1 * stride[1] > 256) continue;
        const int b0 = per_box / b2 / b1;
        if (b0 * stride[0] > 256) continue;
        const int b[3] = {b0, b1, b2};
        double padded = 1.0, real = 1.0;
        for (int a = 0; a < 3; ++a) {
          padded *= static_cast<double>((out[a] + b[a] - 1) / b[a]) * b[a];
          real *= out[a];
        }
        // Waste first; then fewer boxes; then a longer innermost run.
        const double score = padded / real + 0.01 * nb - 0.0001 * b2 - 0.00001 * b1;
        if (score < best) {
          best = score;
          found = true;
          *nb_out = nb;
          b_out[0] = b0;
          b_out[1] = b1;
          b_out[2] = b2;
        }
      }
    }
  }
  return found;
}

// Splits the spatial axes of a pass into outer axes and three box axes and fills the
// BoxGeom; `rows` is the number of positions per tile.
bool build_geom(int rank, int64_t batch, int64_t groups, const int64_t* in, const int64_t* out,
                const int64_t* k, const int64_t* s, const int64_t* d, const int64_t* p, int rows,
                BoxGeom* g, const int* forced_box = nullptr) {
  std::memset(g, 0, sizeof(*g));
  if (rank < 1 || rank > kMaxFastRank) return false;
  const int n_outer = rank > 3 ? rank - 3 : 0;
  const int lead = 3 - (rank - n_outer);  // unit box axes prepended for ranks < 3
  g->n_outer = n_outer;
  const int64_t limit = (int64_t{1} << 31) - 1;
  for (int a = 0; a < 3; ++a) {
    const int src = a - lead + n_outer;
    if (a < lead) {
      g->out[a] = g->in[a] = g->k[a] = g->s[a] = g->d[a] = 1;
      g->p[a] = 0;
      continue;
    }
    if (in[src] > limit || out[src] > limit || k[src] > 4096 || s[src] > 8 || d[src] > 65536 ||
        p[src] > 65536) {
      return false;
    }
    g->out[a] = static_cast<int>(out[src]);
    g->in[a] = static_cast<int>(in[src]);
    g->k[a] = static_cast<int>(k[src]);
    g->s[a] = static_cast<int>(s[src]);
    g->d[a] = static_cast<int>(d[src]);
    g->p[a] = static_cast<int>(p[src]);
  }
  int64_t in_vol = 1, out_vol = 1, taps = 1;
  for (int a = n_outer - 1; a >= 0; --a) {
    if (in[a] > limit || out[a] > limit || k[a] > 4096 || s[a] > limit || d[a] > 65536 ||
        p[a] > 65536) {
      return false;
    }
    g->out_o[a] = static_cast<int>(out[a]);
    g->in_o[a] = static_cast<int>(in[a]);
    g->k_o[a] = static_cast<int>(k[a]);
    g->s_o[a] = static_cast<int>(s[a]);
    g->d_o[a] = static_cast<int>(d[a]);
    g->p_o[a] = static_cast<int>(p[a]);
    g->in_o_stride[a] = in_vol;
    g->out_o_stride[a] = out_vol;
    in_vol *= in[a];
    out_vol *= out[a];
  }
  for (int a = 0; a < rank; ++a) taps *= k[a];
  if (taps > limit) return false;
  g->taps = static_cast<int>(taps);
  g->batch = batch;
  g->groups = groups;
  g->in_merged_per_ng = in_vol;
  g->out_outer_vol = out_vol;
  g->outer_count = batch * out_vol;
  g->out_box_vol = static_cast<int64_t>(g->out[0]) * g->out[1] * g->out[2];
  // Merged TMA coordinates are int32.
  if (batch * groups * in_vol > limit || batch * groups * out_vol > limit) return false;
  int nb = 0, b[3] = {0, 0, 0};
  if (forced_box != nullptr) {
    nb = 1;
    for (int a = 0; a < 3; ++a) b[a] = forced_box[a];
  } else if (!plan_boxes(g->out, g->s, rows, &nb, b)) {
    return false;
  }
  g->nb = nb;
  g->box_rows = rows / nb;
  for (int a = 0; a < 3; ++a) {
    g->b[a] = b[a];
    g->nbox[a] = (g->out[a] + b[a] - 1) / b[a];
  }
  g->boxes_per_group =
      g->outer_count * static_cast<int64_t>(g->nbox[0]) * g->nbox[1] * g->nbox[2];
  return true;
}

uint32_t make_idesc(int op, int m, int n, bool a_mn, bool b_mn) {
  uint32_t desc = 0;
  desc |= 1u << 4;  // accumulator format F32
  const uint32_t fmt = op == kOpBF16 ? 1u : (op == kOpF16 ? 0u : 2u);
  desc |= fmt << 7;
  desc |= fmt << 10;
  if (a_mn) desc |= 1u << 15;
  if (b_mn) desc |= 1u << 16;
  desc |= static_cast<uint32_t>(n >> 3) << 17;
  desc |= static_cast<uint32_t>(m >> 4) << 24;
  return desc;
}

uint32_t tmem_columns(int needed) {
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(needed)) cols <<= 1;
  return cols;
}

uint32_t round_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

int sm_count() {
  static int count = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
    if (count <= 0) count = 148;
  });
  return count;
}

}  // namespace

namespace {

struct WgradPlan {
  WgradKernelParams P;
  size_t smem;
  int chunks;
  int parts;
  int halo_rows;  // box rows along a1 in halo mode
};

// Splits of the last tap chunk when the full chunks run `splits`: a CTA's time is about
// (kTileCost + units) x its position tiles, in units of one unit's MMAs per tile, where
// kTileCost is the fixed per-tile cost (dY slices, barrier handoffs, commits). The last
// chunk's CTAs get as many tiles as keep them as busy as a full chunk's. 2.2 was the
// fastest of 1.0 / 1.5 / 2.2 measured on B200 (c2 wgrad call 0.463 / 0.449 / 0.435 ms,
// c3 unchanged or slower below it).
int64_t last_chunk_splits(const WgradKernelParams& P, int64_t splits) {
  constexpr double kTileCost = 2.2;
  const int last_units = P.units_total - (P.chunks - 1) * P.units_per_cta;
  if (P.chunks <= 1 || last_units >= P.units_per_cta) return splits;
  const double ratio = (kTileCost + last_units) / (kTileCost + P.units_per_cta);
  int64_t last = static_cast<int64_t>(static_cast<double>(splits) * ratio + 0.5);
  if (last < 1) last = 1;
  if (last > splits) last = splits;
  return last;
}

bool plan_wgrad(const WgradPass& pass, int splits_hint, WgradPlan* plan) {
  WgradKernelParams& P = plan->P;
  std::memset(&P, 0, sizeof(P));
  if (pass.op == kOpF32) return false;  // wgrad runs on kind::f16 (bf16 parts for fp32)
  const int es = element_size(pass.op);
  const int parts = pass.parts < 1 ? 1 : pass.parts;
  if (parts > 3) return false;
  const int a_row = pass.c_pad * es;
  if (!(a_row == 32 || a_row == 64 || a_row == 128)) return false;
  if (pass.n_pad < 16 || pass.n_pad > 256 || pass.n_pad % 16 != 0) return false;
  const int b_row_full = pass.n_pad * es;
  int b_row = 0;
  if (b_row_full == 32 || b_row_full == 64 || b_row_full == 128) {
    b_row = b_row_full;
  } else if (b_row_full % 128 == 0) {
    b_row = 128;
  } else {
    return false;
  }
  P.c_pad = pass.c_pad;
  P.cin_real = pass.cin_real;
  P.n_pad = pass.n_pad;
  P.n_real = pass.n_real;
  P.tpm = 128 / pass.c_pad;
  P.a_row_bytes = a_row;
  P.a_layout = static_cast<int>(desc_layout(a_row));
  P.b_row_bytes = b_row;
  P.b_layout = static_cast<int>(desc_layout(b_row));
  P.b_blocks = b_row_full / b_row;
  P.b_blk_elems = b_row / es;
  // Kernel extent, stride and dilation of box axis a1 (the second-to-last spatial axis).
  const int a1 = pass.rank >= 2 ? pass.rank - 2 : -1;
  const int k1 = a1 >= 0 ? static_cast<int>(pass.k[a1]) : 1;
  const int64_t s1 = a1 >= 0 ? pass.s[a1] : 1;
  const int64_t d1 = a1 >= 0 ? pass.d[a1] : 1;
  const int64_t o1 = a1 >= 0 ? pass.out[a1] : 1;
  const int64_t o2 = pass.out[pass.rank - 1];
  const int mtpu = (k1 + P.tpm - 1) / P.tpm;
  // Box axis 0 (third-to-last spatial axis): its three taps can be folded into N.
  const int a0 = pass.rank >= 3 ? pass.rank - 3 : -1;
  const int k0 = a0 >= 0 ? static_cast<int>(pass.k[a0]) : 1;
  const bool foldable = k0 == 3 && a0 >= 0 && pass.s[a0] == 1 && pass.d[a0] == 1 &&
                        b_row_full <= 128 && 3 * pass.n_pad <= 256;
  // Halo boxes cut the TMA operations per tap by k1 at the price of padding atoms. That
  // pays down to ~1/3 atom use with one operand part, or with the a0 fold (thin channels
  // are bound by the count of small per-tap loads); float32's three unfolded parts need
  // 60 %.
  const double min_atom_use = parts == 1 || foldable ? 0.3 : 0.6;
  const bool halo_ok = k1 >= 2 && s1 == 1 && d1 <= 16 &&
                       static_cast<double>(k1) / (mtpu * P.tpm) >= min_atom_use;
  const bool fold_ok = halo_ok && foldable;
  const int fold = fold_ok ? k0 : 0;
  bool planned = false;
  if (halo_ok) {
    // Position tile [1, b1, b2] with b2 a power of two >= 8 (8-row alignment of every
    // tap window; the K chunk b1 * b2 itself need not be a power of two), least padding
    // waste first. Among K chunks within 30 % of the least waste, the longest that fits
    // comes first (every A box then feeds more MMAs per barrier handoff), skipping tiles
    // with more halo rows than rows of their own. Measured on B200: c4's 8-wide axes run
    // best on 64-row tiles [1, 8, 8], c3's 12-wide axes on 192-row tiles [1, 12, 16]
    // (128 rows pad them 1.78x, 64 rows [1, 4, 16] carry 7 halo rows per 4).
    const int halo_extra = (mtpu * P.tpm - 1) * static_cast<int>(d1);
    auto tile_waste = [&](int kc, int* b2_out) {
      double best_waste = 1e30;
      for (int b2 = 8; b2 <= kc; b2 *= 2) {
        if (kc % b2 != 0) continue;
        const int b1 = kc / b2;
        const double waste = double((o1 + b1 - 1) / b1 * b1) / o1 *
                             double((o2 + b2 - 1) / b2 * b2) / o2;
        if (waste < best_waste - 1e-9) {
          best_waste = waste;
          *b2_out = b2;
        }
      }
      return best_waste;
    };
    constexpr int kChunks[] = {256, 192, 128, 64};
    auto preferred = [&](int kc) {
      int b2 = 0;
      tile_waste(kc, &b2);
      return b2 > 0 && halo_extra <= kc / b2;
    };
    double least_waste = 1e30;
    for (int kc : kChunks) {
      int b2 = 0;
      if (!(fold && kc > 192) && preferred(kc)) {
        least_waste = std::min(least_waste, tile_waste(kc, &b2));
      }
    }
    // First the preferred chunks, then (if none fits) any chunk, longest first.
    for (int round = 0; round < 2 && !planned; ++round)
    for (int kc : kChunks) {
      if (fold && kc > 192) continue;  // ring slots of 256 rows leave too few A stages
      int b2 = 0;
      const double waste = tile_waste(kc, &b2);
      if (b2 == 0) continue;
      if (round == 0 && (!preferred(kc) || waste > 1.3 * least_waste)) continue;
      const int b1 = kc / b2;
      const int h1 = b1 + halo_extra;
      if (h1 > 256) continue;
      const uint32_t rows = static_cast<uint32_t>(h1 * b2);
      const uint32_t a_part = round_up(rows * a_row, 1024);
      const uint32_t b_part = round_up(static_cast<uint32_t>(kc * b_row_full), 1024);
      const int b_slots = fold ? fold + 4 : 2;  // folded: smallest ring plus mirrors
      if (b_slots * b_part * parts + 3 * a_part * parts > 208 * 1024) continue;
      const int box[3] = {1, b1, b2};
      if (!build_geom(pass.rank, pass.batch, pass.groups, pass.in, pass.out, pass.k, pass.s,
                      pass.d, pass.p, kc, &P.g, box)) {
        continue;
      }
      P.halo = 1;
      P.mtpu = mtpu;
      P.kc_rows = kc;
      P.a_part_bytes = a_part;
      P.a_tx = rows * a_row * parts;
      P.atom_bytes = static_cast<uint32_t>(d1 * b2 * a_row);
      P.units_total = P.g.taps / k1;
      P.entries_per_unit = 1;
      if (fold) {
        // Position tiles run over the input-aligned slices q in [q_lo, q_hi): those of
        // [0, out0 + k0 - 1) whose input slice q - p0 lies inside the input. The box
        // origin of walk index i is then input slice i - (p0 - q_lo).
        const int p0 = P.g.p[0];
        const int q_lo = std::max(0, p0);
        const int q_hi = std::min(P.g.out[0] + k0 - 1, p0 + P.g.in[0]);
        if (q_hi <= q_lo) continue;
        P.nfold = fold;
        P.q_lo = q_lo;
        P.units_total = P.g.taps / (k1 * k0);
        P.g.nbox[0] = q_hi - q_lo;
        P.g.p[0] = p0 - q_lo;
        P.g.boxes_per_group = P.g.outer_count * static_cast<int64_t>(P.g.nbox[0]) *
                              P.g.nbox[1] * P.g.nbox[2];
      }
      plan->halo_rows = h1;
      planned = true;
      break;
    }
  }
  if (!planned) {
    // Position rows per K chunk: 128, or 64 when the 128-row slots do not fit twice.
    int kc = 128;
    for (;;) {
      const uint32_t a_tile = static_cast<uint32_t>(kc * a_row);
      const uint32_t a_slot = round_up(a_tile * P.tpm, 1024) * parts;
      const uint32_t b_slot = round_up(static_cast<uint32_t>(kc * b_row_full), 1024) * parts;
      if (2 * a_slot + 2 * b_slot <= 200 * 1024 || kc == 64) break;
      kc = 64;
    }
    if (!build_geom(pass.rank, pass.batch, pass.groups, pass.in, pass.out, pass.k, pass.s,
                    pass.d, pass.p, kc, &P.g)) {
      return false;
    }
    P.halo = 0;
    P.mtpu = 1;
    P.kc_rows = kc;
    P.a_tile_bytes = static_cast<uint32_t>(kc * a_row);
    P.a_part_bytes = round_up(P.a_tile_bytes * P.tpm, 1024);
    P.a_tx = P.a_tile_bytes * P.tpm * parts;
    P.atom_bytes = P.a_tile_bytes;
    P.units_total = (P.g.taps + P.tpm - 1) / P.tpm;
    P.entries_per_unit = P.tpm;
    plan->halo_rows = 0;
  }
  const int kc = P.kc_rows;
  P.ksteps = kc / 16;
  P.a_tile_bytes = static_cast<uint32_t>(kc * a_row);
  P.a_slot_bytes = P.a_part_bytes * parts;
  const int slices = P.nfold ? P.nfold : 1;
  P.b_part_bytes = round_up(static_cast<uint32_t>(kc * b_row_full), 1024);
  P.b_slot_bytes = P.b_part_bytes * parts;
  P.b_tx = static_cast<uint32_t>(kc * b_row_full) * parts;
  P.n_cols = slices * pass.n_pad;
  // N atoms: consecutive one-slice ring slots of a folded tile, else 64-channel blocks.
  P.b_lbo = P.nfold ? P.b_slot_bytes : static_cast<uint32_t>(kc) * 128u;
  int64_t combos = 1;
  for (int a = 0; a < P.g.n_outer; ++a) combos *= P.g.k_o[a];
  if (combos > kMaxOuterCombos) return false;
  P.outer_combos = static_cast<int>(combos);
  P.mt_total = P.units_total * P.mtpu;
  const int max_units = (512 / P.n_cols) / P.mtpu;
  if (max_units < 1) return false;
  plan->chunks = (P.units_total + max_units - 1) / max_units;
  P.units_per_cta = (P.units_total + plan->chunks - 1) / plan->chunks;
  constexpr uint32_t kSmemBudget = 208 * 1024;
  if (P.halo) {
    // One A stage per position tile holding every unit's box (wgrad_halo_kernel). B: two
    // tile slots, or a ring of nfold + extra one-slice slots (the tile's slices plus
    // `extra` loaded ahead) followed by nfold - 1 mirror slots. Prefer a ring three
    // slices ahead with at least three A stages; fewer units per CTA when even two
    // stages do not fit.
    P.a_unit_bytes = P.a_part_bytes * parts;
    if (P.units_per_cta > 32) {  // one producer lane per unit
      P.units_per_cta = 32;
      plan->chunks = (P.units_total + 31) / 32;
    }
    bool fitted = false;
    for (;;) {
      P.a_slot_bytes = P.a_unit_bytes * static_cast<uint32_t>(P.units_per_cta);
      for (int extra = 3; extra >= 2 && !fitted; --extra) {
        const int ring = P.nfold ? P.nfold + extra : 2;
        const uint32_t b_region =
            static_cast<uint32_t>(P.nfold ? ring + P.nfold - 1 : 2) * P.b_slot_bytes;
        if (b_region >= kSmemBudget) continue;
        int stages = static_cast<int>((kSmemBudget - b_region) / P.a_slot_bytes);
        if (stages > 8) stages = 8;
        if (stages < (extra == 3 && P.nfold ? 3 : 2)) continue;
        P.b_ring = ring;
        P.a_stages = stages;
        P.a_base_off = b_region;
        fitted = true;
      }
      if (fitted || P.units_per_cta == 1) break;
      --P.units_per_cta;
      plan->chunks = (P.units_total + P.units_per_cta - 1) / P.units_per_cta;
    }
    if (!fitted) return false;
  } else {
    // B memory: two tile slots; the A stages (one unit of tpm tap tiles each) get the
    // rest, since A loads are the deeper stream (several units per tile).
    P.b_ring = 2;
    const uint32_t b_region = 2 * P.b_slot_bytes;
    if (b_region + 2 * P.a_slot_bytes > kSmemBudget) return false;
    int stages = static_cast<int>((kSmemBudget - b_region) / P.a_slot_bytes);
    if (stages > 12) stages = 12;
    if (stages < 2) return false;
    P.a_stages = stages;
    P.a_base_off = b_region;
  }
  P.bar_off = P.a_base_off + static_cast<uint32_t>(P.a_stages) * P.a_slot_bytes;
  P.mt_per_cta = P.units_per_cta * P.mtpu;
  P.tmem_cols = tmem_columns(P.mt_per_cta * P.n_cols);
  P.idesc = make_idesc(pass.op, 128, P.n_cols, true, true);
  plan->parts = parts;
  P.ptiles = (P.g.boxes_per_group + P.g.nb - 1) / P.g.nb;
  P.chunks = plan->chunks;
  int splits = splits_hint;
  if (splits <= 0) {
    const int64_t ctas_per_split = static_cast<int64_t>(plan->chunks) * pass.groups;
    // One CTA per SM: as many splits as fit one wave (a few CTAs of a second wave would
    // double the pass time).
    int64_t s = sm_count() / ctas_per_split;
    if (s < 1) s = 1;
    if (parts > 1) {
      // float32 problems: at most ~4096 positions per split. The tensor core's fp32
      // accumulation error grows with the number of accumulation steps; the fp32
      // partials are then summed in a fixed order by the reduction kernel.
      const int64_t tiles_per_split = 4096 / P.kc_rows > 0 ? 4096 / P.kc_rows : 1;
      const int64_t need = (P.ptiles + tiles_per_split - 1) / tiles_per_split;
      if (s < need) s = need < 1024 ? need : 1024;
    }
    if (P.halo && plan->chunks > 1 && parts == 1) {
      // The last chunk's CTAs get fewer splits, the full chunks more: the largest s with
      // (chunks - 1) * s + last(s) CTAs per group in one wave.
      for (int64_t t = 4 * s; t > s; --t) {
        if (((plan->chunks - 1) * t + last_chunk_splits(P, t)) * pass.groups <= sm_count()) {
          s = t;
          break;
        }
      }
    }
    if (s > P.ptiles) s = P.ptiles;
    if (s < 1) s = 1;
    splits = static_cast<int>(s);
  }
  P.splits = splits;
  P.chunks = plan->chunks;
  P.splits_last = splits;
  if (P.halo) P.splits_last = static_cast<int>(last_chunk_splits(P, splits));
  plan->smem = P.bar_off + (2 * P.b_ring + 2 * P.a_stages + 1) * 8 + 16 +
               (P.halo ? 0 : (sizeof(BoxInfo) + sizeof(uint64_t)) * kMaxBoxes) +
               sizeof(OuterCombo) * kMaxOuterCombos +
               sizeof(TapEntry) * static_cast<size_t>(P.units_per_cta) * P.entries_per_unit +
               1024;
  return true;
}

}  // namespace

bool wgrad_pass_supported(const WgradPass& pass) {
  WgradPlan plan;
  return pass.rank >= 1 && pass.rank <= kMaxFastRank && plan_wgrad(pass, 1, &plan);
}

int plan_wgrad_splits(const WgradPass& pass, int sm) {
  (void)sm;
  WgradPlan plan;
  if (!plan_wgrad(pass, 0, &plan)) return 0;
  return plan.P.splits;
}

int describe_wgrad_pass(const WgradPass& pass, char* text, size_t size) {
  WgradPlan plan;
  if (!plan_wgrad(pass, pass.splits, &plan)) return std::snprintf(text, size, "unplanned");
  const WgradKernelParams& P = plan.P;
  return std::snprintf(text, size,
                       "halo=%d fold=%d kc=%d boxes=%dx[%d,%d,%d] taps/M=%d units=%d/%d "
                       "chunks=%d stages=%d ring=%d N=%d",
                       P.halo, P.nfold, P.kc_rows, P.g.nb, P.g.b[0], P.g.b[1], P.g.b[2], P.tpm,
                       P.units_per_cta, P.units_total, plan.chunks, P.a_stages, P.b_ring,
                       P.n_cols);
}

int launch_wgrad_pass(const WgradPass& pass, cudaStream_t stream, uint64_t timeout_ns) {
  WgradPlan plan;
  if (!plan_wgrad(pass, pass.splits, &plan)) {
    return fail(CND_ERR_UNSUPPORTED, "weight-gradient geometry outside the tcgen05 path");
  }
  WgradKernelParams& P = plan.P;
  P.partial = pass.partial;
  P.err = device_error_word();
  P.timeout_ns = timeout_ns;
  if (plan.chunks > 65535 || pass.groups > 65535) {
    return fail(CND_ERR_UNSUPPORTED, "grid too large for the tcgen05 path");
  }
  int64_t ext_in[3], ext_out[3];
  for (int a = 0; a < 3; ++a) {
    ext_in[a] = P.g.in[a];
    ext_out[a] = P.g.out[a];
  }
  const int64_t merged_in = pass.batch * pass.groups * P.g.in_merged_per_ng;
  const int64_t merged_out = pass.batch * pass.groups * P.g.out_outer_vol;
  const int box[3] = {P.g.b[0], P.g.b[1], P.g.b[2]};
  const int strd[3] = {P.g.s[0], P.g.s[1], P.g.s[2]};
  const int ones[3] = {1, 1, 1};
  alignas(64) WgradMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  int act_box[3] = {box[0], box[1], box[2]};
  int act_strd[3] = {strd[0], strd[1], strd[2]};
  if (P.halo) {
    act_box[1] = plan.halo_rows;
    act_strd[1] = 1;
  }
  for (int part = 0; part < 3; ++part) {
    const int source = part < plan.parts ? part : 0;
    int rc = encode_act_map(&maps.act[part], pass.act[source], pass.op, pass.c_pad, ext_in,
                            merged_in, pass.c_pad, act_box, act_strd);
    if (rc != CND_OK) return rc;
    rc = encode_act_map(&maps.grad[part], pass.grad[source], pass.op, pass.n_pad, ext_out,
                        merged_out, P.b_blk_elems, box, ones);
    if (rc != CND_OK) return rc;
  }
  // Halo kernel: x enumerates the (chunk, split) CTAs of a group.
  const dim3 grid = P.halo ? dim3(static_cast<unsigned>((plan.chunks - 1) * P.splits +
                                                        P.splits_last),
                                  1u, static_cast<unsigned>(pass.groups))
                           : dim3(static_cast<unsigned>(P.splits),
                                  static_cast<unsigned>(plan.chunks),
                                  static_cast<unsigned>(pass.groups));
  using Kernel = void (*)(WgradMaps, WgradKernelParams);
  Kernel kernel = nullptr;
#define CND_WGRAD_PICK(PARTS)                                                         \
  if (P.halo) {                                                                      \
    kernel = P.ksteps == 16   ? wgrad_halo_kernel<PARTS, 16>                         \
             : P.ksteps == 12 ? wgrad_halo_kernel<PARTS, 12>                         \
             : P.ksteps == 8  ? wgrad_halo_kernel<PARTS, 8>                          \
                              : wgrad_halo_kernel<PARTS, 4>;                         \
  } else {                                                                           \
    kernel = P.ksteps == 16  ? wgrad_kernel<PARTS, 16>                               \
             : P.ksteps == 8 ? wgrad_kernel<PARTS, 8>                                \
                             : wgrad_kernel<PARTS, 4>;                               \
  }
  if (plan.parts == 3) {
    CND_WGRAD_PICK(3)
  } else if (plan.parts == 2) {
    CND_WGRAD_PICK(2)
  } else {
    CND_WGRAD_PICK(1)
  }
#undef CND_WGRAD_PICK
  if (P.ksteps != 16 && P.ksteps != 8 && P.ksteps != 4 && !(P.halo && P.ksteps == 12)) {
    return fail(CND_ERR_UNSUPPORTED, "weight-gradient K chunk outside the tcgen05 path");
  }
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(plan.smem));
  kernel<<<grid, kThreads, plan.smem, stream>>>(maps, P);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(CND_ERR_CUDA, "wgrad_kernel launch failed: %s", cudaGetErrorString(e));
  }
  count_launch();
  return CND_OK;
}

}  // namespace cnd
