// Persistent tcgen05 implicit-GEMM convolution pass (forward, and dgrad as a forward
// pass over dy with flipped/transposed weights).
//
// Work decomposition. The last three spatial axes are "box axes" a0, a1, a2; the rest,
// with batch and group, form the merged TMA dimension. An M tile is 128 output positions
// [e0, b1, b2] along (a0, a1, a2); a CTA "super tile" is MT M tiles stacked along a0, all
// sharing every weight tile it loads (weight reuse x MT). For each load unit — one value
// of every tap axis that is not "shifted", and one channel block — TMA fetches a single
// halo box of channels-last input [h0, h1, b2] that covers the super tile for every tap
// of the shifted axes (a0 always when its stride is 1; a1 too when e0 == 1): the MMA for
// tap (j0, j1) and tile m reads the box at row ((m*e0 + j0*d0)*h1 + j1*d1)*b2, a
// multiple of 8 rows, so the 32/64/128-byte swizzle pattern lines up and no data moves
// in shared memory. Out-of-range coordinates read zero (the reference's implicit zero
// padding, src/torch_convnd/csrc/convnd.h:57-76). Weights are packed so that the taps of
// one load unit are consecutive rows and arrive with one TMA box.
//
// Warp roles (192 threads): warp 0 lane 0 = TMA producer (warp 0 owns TMEM), warp 1 lane
// 0 = MMA issuer, warps 2-5 = epilogue. Accumulators are double buffered in TMEM so the
// epilogue of one super tile overlaps the main loop of the next. float32 problems
// (kind::tf32) rotate taps over several accumulators and sum them in fp32 registers,
// which keeps the tensor core's per-step accumulation error from growing with K.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "fprop.cuh"
#include "ptx.cuh"

namespace cnd {

namespace {

// Warp 0: TMA producer, warp 1: MMA issuer, then epi_groups groups of four epilogue
// warps (one per TMEM lane quarter); group g drains M tiles g, g + epi_groups, ...
constexpr int kMaxEpiGroups = 2;
constexpr int kMaxThreads = 64 + 128 * kMaxEpiGroups;
constexpr uint32_t kSiteProducer = 0x301, kSiteMma = 0x302, kSiteEpilogue = 0x303,
                   kSiteMmaAcc = 0x304, kSiteDrain = 0x305;

struct FpropMaps {
  CUtensorMap act[2];
  CUtensorMap wt[2];
  CUtensorMap out;  // channels-first output, dims (o2, o1, o0, outer, n*C): TMA stores
  CUtensorMap pre;  // the pre-activation output, same layout as `out` (pre_staged only)
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uintptr_t v = reinterpret_cast<uintptr_t>(p);
  return reinterpret_cast<uint8_t*>((v + 1023) & ~static_cast<uintptr_t>(1023));
}

// Position of a super tile: group, batch index, outer output coordinates and the tile
// indices along the box axes (q0 counts super tiles along a0).
struct Super {
  int g;
  int64_t n;
  int64_t outer_lin;  // row-major index over the outer output axes
  int o[kMaxOuter];
  int q0, q1, q2;
  int a0_first;  // output a0 coordinate of the super tile's first M tile
};

__device__ __forceinline__ void decode_super(const FpropParams& P, int64_t st, Super& s) {
  int64_t rest = st;
  s.q2 = static_cast<int>(rest % P.nsup[2]);
  rest /= P.nsup[2];
  s.q1 = static_cast<int>(rest % P.nsup[1]);
  rest /= P.nsup[1];
  s.q0 = static_cast<int>(rest % P.nsup[0]);
  rest /= P.nsup[0];
  // With a parity split (par0 = 2) super tiles alternate between even and odd a0 planes.
  const int blk = s.q0 / P.par0;
  s.a0_first = (blk * P.mt * P.e0) * P.par0 + (s.q0 - blk * P.par0);
  s.outer_lin = rest % P.out_outer_vol;
  rest /= P.out_outer_vol;
  s.n = rest % P.batch;
  s.g = static_cast<int>(rest / P.batch);
  int64_t o = s.outer_lin;
#pragma unroll
  for (int a = kMaxOuter - 1; a >= 0; --a) {
    if (a < P.n_outer) {
      s.o[a] = static_cast<int>(o % P.out_o[a]);
      o /= P.out_o[a];
    } else {
      s.o[a] = 0;
    }
  }
}

// One MMA issued by the converged MMA warp (one elected lane).
template <bool kTF32>
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                    uint32_t acc) {
  if constexpr (kTF32) {
    dev::mma_tf32_warp(d, a, b, idesc, acc);
  } else {
    dev::mma_f16_warp(d, a, b, idesc, acc);
  }
}

// Operand kinds of the kernel instantiations: the element type of activations, weights
// and output, and whether float32 runs as one or three TF32 products, or as three
// products of bfloat16 hi / lo parts (kind::f16, about 16 significant bits per operand;
// one K = 16 MMA covers what takes two K = 8 TF32 MMAs).
enum KernelOp { kKindF16 = 0, kKindBF16 = 1, kKindTF32 = 2, kKind3xTF32 = 3, kKind2xBF16 = 4 };

template <int kOp>
struct OpTraits;
template <>
struct OpTraits<kKindF16> {
  using Out = __half;
  static constexpr bool tf32 = false;
  static constexpr int parts = 1;
  static __device__ __forceinline__ Out cast(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float load(const Out* p) { return __half2float(__ldg(p)); }
};
template <>
struct OpTraits<kKindBF16> {
  using Out = __nv_bfloat16;
  static constexpr bool tf32 = false;
  static constexpr int parts = 1;
  static __device__ __forceinline__ Out cast(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float load(const Out* p) { return __bfloat162float(__ldg(p)); }
};
template <>
struct OpTraits<kKindTF32> {
  using Out = float;
  static constexpr bool tf32 = true;
  static constexpr int parts = 1;
  static __device__ __forceinline__ Out cast(float v) { return v; }
  static __device__ __forceinline__ float load(const Out* p) { return __ldg(p); }
};
template <>
struct OpTraits<kKind3xTF32> {
  using Out = float;
  static constexpr bool tf32 = true;
  static constexpr int parts = 2;
  static __device__ __forceinline__ Out cast(float v) { return v; }
  static __device__ __forceinline__ float load(const Out* p) { return __ldg(p); }
};
template <>
struct OpTraits<kKind2xBF16> {
  using Out = float;
  static constexpr bool tf32 = false;
  static constexpr int parts = 2;
  static __device__ __forceinline__ Out cast(float v) { return v; }
  static __device__ __forceinline__ float load(const Out* p) { return __ldg(p); }
};

// PyTorch's exact GELU (approximate='none'): 0.5 v (1 + erf(v / sqrt(2))).
__device__ __forceinline__ float gelu_exact(float v) {
  return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
}

// Rounding of an fp32 epilogue value to the output type.
template <typename T>
struct OpCast;
template <>
struct OpCast<float> {
  static __device__ __forceinline__ float cast(float v) { return v; }
};
template <>
struct OpCast<__nv_bfloat16> {
  static __device__ __forceinline__ __nv_bfloat16 cast(float v) { return __float2bfloat16_rn(v); }
};
template <>
struct OpCast<__half> {
  static __device__ __forceinline__ __half cast(float v) { return __float2half_rn(v); }
};

// One 16-channel chunk of an epilogue row: the sum of the `used` rotating accumulators
// of an M tile (TMEM columns tile_col + a * kMT * n_pad + c * 16) plus the bias. The
// bias chunk is fetched before the TMEM loads, so its latency is paid once per chunk.
// kZero writes zeros back over the columns read (folded passes accumulate onto them).
template <typename Traits, int kMT, bool kZero>
__device__ __forceinline__ void epilogue_chunk(uint32_t dbase, int tile_col, int c, int n_pad,
                                               int used, const typename Traits::Out* group_bias,
                                               int n_real, float (&out)[16]);

// epilogue_chunk for passes with the a2 taps folded into N (k2f > 1): the M tile's
// columns hold k2f blocks of n_pad, block j for a2 tap j at the tile row of its input
// position. Output row r of a line (b2 rows, a power of two <= 32, aligned within the
// warp) is the sum over j of block j at row r + j * d2: one shuffle per block. Rows whose
// line position is at or past b2o come out as garbage and are not stored.
template <typename Traits, int kMT>
__device__ __forceinline__ void epilogue_chunk_k2(uint32_t dbase, int tile_col, int c,
                                                  const FpropParams& P, int used,
                                                  const typename Traits::Out* group_bias,
                                                  float (&out)[16]) {
  float b[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int co = c * 16 + i;
    b[i] = (group_bias != nullptr && co < P.n_real) ? Traits::load(group_bias + co) : 0.0f;
    out[i] = 0.0f;
  }
  for (int j = 0; j < P.k2f; ++j) {
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.0f;
    const uint32_t col = dbase + static_cast<uint32_t>(tile_col + j * P.n_pad + c * 16);
    for (int a = 0; a < used; ++a) {
      uint32_t raw[16];
      const uint32_t addr = col + static_cast<uint32_t>(a * kMT * P.n_blk);
      __syncwarp();
      dev::tmem_load16(addr, raw);
      dev::tmem_load_wait();
      dev::tmem_zero16(addr);  // folded passes accumulate onto zeroed columns
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += __uint_as_float(raw[i]);
    }
    const int shift = j * P.d[2];
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] += __shfl_down_sync(0xffffffffu, v[i], shift, P.b2);
  }
  if (group_bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] += b[i];
  }
}

template <typename Traits, int kMT, bool kZero>
__device__ __forceinline__ void epilogue_chunk(uint32_t dbase, int tile_col, int c, int n_pad,
                                               int used, const typename Traits::Out* group_bias,
                                               int n_real, float (&out)[16]) {
  float b[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int co = c * 16 + i;
    b[i] = (group_bias != nullptr && co < n_real) ? Traits::load(group_bias + co) : 0.0f;
  }
  const uint32_t col = dbase + static_cast<uint32_t>(tile_col + c * 16);
  {
    uint32_t v[16];
    __syncwarp();
    dev::tmem_load16(col, v);
    dev::tmem_load_wait();
    if constexpr (kZero) dev::tmem_zero16(col);
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] = __uint_as_float(v[i]);
  }
  for (int a = 1; a < used; ++a) {
    uint32_t v[16];
    __syncwarp();
    dev::tmem_load16(col + static_cast<uint32_t>(a * kMT * n_pad), v);
    dev::tmem_load_wait();
    if constexpr (kZero) dev::tmem_zero16(col + static_cast<uint32_t>(a * kMT * n_pad));
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] += __uint_as_float(v[i]);
  }
  if (group_bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] += b[i];
  }
}

// Stores `count` (<= 16 used) consecutive channels of one channels-last output row, as
// 16-byte vectors when the run is whole and aligned.
template <typename OutT>
__device__ __forceinline__ void store_run16(OutT* dst, const float (&value)[16], int count) {
  constexpr int kPer = 16 / sizeof(OutT);  // elements per 16-byte vector
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
    for (int v = 0; v < 16 / kPer; ++v) {
      if ((v + 1) * kPer <= count) {
        alignas(16) OutT packed[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) packed[i] = OpCast<OutT>::cast(value[v * kPer + i]);
        *reinterpret_cast<uint4*>(dst + v * kPer) = *reinterpret_cast<const uint4*>(packed);
        done = (v + 1) * kPer;
      }
    }
  }
  // constant indices only: a runtime index would move `value` to local memory
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i >= done && i < count) dst[i] = OpCast<OutT>::cast(value[i]);
  }
}

template <int kOp, int kKSteps, int kMT, int kFold>
// Ten warps put three on one scheduler, whose 16 K registers then allow 168 per thread.
__global__ void __launch_bounds__(kMaxThreads, 1)
    fprop_kernel(const __grid_constant__ FpropMaps maps, const __grid_constant__ FpropParams P) {
  using Traits = OpTraits<kOp>;
  using OutT = typename Traits::Out;
  constexpr bool kTF32 = Traits::tf32;
  constexpr int kParts = Traits::parts;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P.bar_off);
  uint64_t* empty = full + P.stages;
  uint64_t* acc_full = empty + P.stages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile uint32_t* progress = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const dev::ErrorWord err{P.err};

  if (threadIdx.x == 0) {
    for (int s = 0; s < P.stages; ++s) {
      dev::mbar_init(&full[s], 1);
      dev::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      dev::mbar_init(&acc_full[b], 1);
      dev::mbar_init(&acc_empty[b], 128 * P.epi_groups);
    }
    *progress = 0;
    dev::fence_barrier_init();
  }
  if (warp == 0) {
    __syncwarp();
    dev::tmem_alloc(tmem_slot, P.tmem_cols);
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nshift = P.nshift0 * P.nshift1;
  const int work_per_super = P.units * nshift;
  const int unit_rows = nshift * P.k2f;  // packed weight rows (taps) of one load unit
  const int k2_units = P.k2f > 1 ? 1 : P.k[2];  // a2 taps walked as separate units

  if (warp == 0 && lane == 0) {
    // ------------------------------ TMA producer ------------------------------
    for (int part = 0; part < kParts; ++part) {
      dev::prefetch_tensormap(&maps.act[part]);
      dev::prefetch_tensormap(&maps.wt[part]);
    }
    int stage = 0;
    uint32_t phase = 0;
    int64_t issued = 0;
    bool ok = P.debug_stall == 0;
    for (int64_t st = blockIdx.x; st < P.supers_total && ok; st += gridDim.x) {
      Super S;
      decode_super(P, st, S);
      const int64_t m_base = (S.n * P.groups + S.g) * P.in_merged_per_gn;
      int ibo[kMaxOuter];
#pragma unroll
      for (int a = 0; a < kMaxOuter; ++a) {
        ibo[a] = a < P.n_outer ? S.o[a] * P.s_o[a] - P.p_o[a] : 0;
      }
      const int x0 = S.a0_first * P.s[0] - P.p[0];
      const int x1 = S.q1 * P.b1 * P.s[1] - P.p[1];
      const int x2 = S.q2 * P.b2o * P.s[2] - P.p[2];
      int to[kMaxOuter];
#pragma unroll
      for (int a = 0; a < kMaxOuter; ++a) to[a] = 0;
      int t0 = 0, t1 = 0, t2 = 0;
      const int32_t w_base = S.g * P.taps;
      for (int u = 0; u < P.units && ok; ++u) {
        bool valid = true;
        int64_t m = m_base;
#pragma unroll
        for (int a = 0; a < kMaxOuter; ++a) {
          if (a < P.n_outer) {
            const int c = ibo[a] + to[a] * P.d_o[a];
            valid = valid && c >= 0 && c < P.in_o[a];
            m += static_cast<int64_t>(c) * P.in_o_stride[a];
          }
        }
        const int32_t mc = valid ? static_cast<int32_t>(m) : -1;
        const int32_t c0 = x0 + (P.nshift0 > 1 ? 0 : t0 * P.d[0]);
        const int32_t c1 = x1 + (P.nshift1 > 1 ? 0 : t1 * P.d[1]);
        const int32_t c2 = x2 + t2 * P.d[2];
        const int32_t w_row = w_base + u * unit_rows;
        for (int cb = 0; cb < P.cblocks; ++cb) {
          if (!dev::mbar_wait(&empty[stage], phase ^ 1u, err, kSiteProducer, P.timeout_ns)) {
            ok = false;
            break;
          }
          uint8_t* sb = smem + stage * P.stage_bytes;
          dev::mbar_arrive_expect_tx(&full[stage], P.tx_bytes);
          const int32_t ch = cb * P.cblk_elems;
#pragma unroll
          for (int part = 0; part < kParts; ++part) {
            dev::tma_load_5d(sb + part * P.a_part_bytes, &maps.act[part], &full[stage], ch, c2,
                             c1, c0, mc);
            dev::tma_load_3d(sb + P.b_off + part * P.b_part_bytes, &maps.wt[part], &full[stage],
                             ch, 0, w_row);
          }
          ++issued;
          if (++stage == P.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        // Next unit: t2 fastest (unless folded), then the unshifted a1 / a0 taps, then the
        // outer taps.
        if (++t2 == k2_units) {
          t2 = 0;
          bool carry = true;
          if (P.nshift1 == 1) {
            if (++t1 == P.k[1]) {
              t1 = 0;
            } else {
              carry = false;
            }
          }
          if (carry && P.nshift0 == 1) {
            if (++t0 == P.k[0]) {
              t0 = 0;
            } else {
              carry = false;
            }
          }
#pragma unroll
          for (int a = kMaxOuter - 1; a >= 0; --a) {
            if (carry && a < P.n_outer) {
              if (++to[a] == P.k_o[a]) {
                to[a] = 0;
              } else {
                carry = false;
              }
            }
          }
        }
      }
    }
    if (!ok && issued > 0) {
      // Let loads already in flight land before the CTA's shared memory goes away.
      const int pending = issued < P.stages ? static_cast<int>(issued) : P.stages;
      for (int i = 1; i <= pending; ++i) {
        const int64_t kb = issued - i;
        dev::mbar_wait(&full[kb % P.stages], static_cast<uint32_t>((kb / P.stages) & 1), err,
                       kSiteDrain, P.timeout_ns / 8 + 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    // The whole warp runs the loop, waits and executes every MMA / commit instruction;
    // elect.sync inside each one picks the issuing lane, so control flow never diverges.
    const bool leader = lane == 0;
    const uint32_t tmem_u = dev::warp_uniform(tmem);
    // Descriptors differ only in their start-address field (bits 0-13, address >> 4):
    // build the constant part once and add offsets in 16-byte units. Shared memory is
    // below 256 KB, so the field never carries into the next one.
    const uint64_t desc_hi =
        dev::make_smem_desc(0, 16, 8u * static_cast<uint32_t>(P.row_bytes), P.layout);
    const uint32_t row_units = static_cast<uint32_t>(P.row_bytes) >> 4;
    const uint32_t tile_units = static_cast<uint32_t>(P.e0 * P.h1 * P.b2) * row_units;
    // a0 taps are d0 / par0 box slices apart (one slice with a parity split)
    const uint32_t j0_units =
        static_cast<uint32_t>((P.d[0] / P.par0) * P.h1 * P.b2) * row_units;
    const uint32_t j1_units = static_cast<uint32_t>(P.d[1] * P.b2) * row_units;
    // B rows and TMEM columns of one tap block: n_pad, or k2f * n_pad with the a2 fold.
    const uint32_t btap_units = static_cast<uint32_t>(P.n_blk) * row_units;
    const uint32_t a_small_units = P.a_part_bytes >> 4;
    const uint32_t b_small_units = P.b_part_bytes >> 4;
    const uint32_t tile_cols = static_cast<uint32_t>(P.n_blk);
    const uint32_t acc_cols = static_cast<uint32_t>(kMT * P.n_blk);
    // Shifted taps of a stage are walked j1 fastest with incremental addresses; the A
    // offset steps by j1_units, or back to j1 = 0 and on to the next j0 at a j1 wrap.
    const uint32_t j0_wrap = j0_units - static_cast<uint32_t>(P.nshift1 - 1) * j1_units;
    const int nshift_stage = P.nshift0 * P.nshift1;
    const int acc_mask = P.nacc - 1;  // nacc is a power of two
    int stage = 0;
    uint32_t phase = 0;
    uint32_t done = 0;
    int iter = 0;
    bool ok = true;
    for (int64_t st = blockIdx.x; st < P.supers_total && ok; st += gridDim.x, ++iter) {
      const int buf = iter & 1;
      // Folded passes wait for the epilogue's zeroing of the buffer (it arrives once at
      // start); otherwise the first use of each buffer passes at once.
      const uint32_t acc_parity = (static_cast<uint32_t>(iter >> 1) & 1u) ^ (kFold ? 0u : 1u);
      if (!dev::mbar_wait_warp(&acc_empty[buf], acc_parity, err, kSiteMmaAcc, P.timeout_ns)) {
        break;
      }
      dev::tc_fence_after();
      const uint32_t dbase = tmem_u + static_cast<uint32_t>(buf * P.acc_stride);
      for (int u = 0; u < P.units && ok; ++u) {
        const int w_unit = u * nshift_stage;  // work item (unit, shifted tap) index
        for (int cb = 0; cb < P.cblocks; ++cb) {
          if (!dev::mbar_wait_warp(&full[stage], phase, err, kSiteMma, P.timeout_ns)) {
            ok = false;
            break;
          }
          dev::tc_fence_after();
          const uint32_t sa =
              dev::warp_uniform(dev::smem_u32(smem + stage * P.stage_bytes) >> 4);
          if constexpr (kFold > 0) {
            // One MMA per A slice i (and a1 shift): tap blocks j0 in [lo, hi] with
            // 0 <= i - j0 < kMT, N = (hi - lo + 1) * n_pad, D at tile i - lo's column.
            // Float32 passes rotate the (unit, a1 shift) groups over nacc accumulator
            // sets, as the unfolded loop rotates taps.
            const uint32_t sbw = sa + (P.b_off >> 4);
            auto fold_shift = [&](int j1) {
              const uint32_t a_j1 = sa + static_cast<uint32_t>(j1) * j1_units;
              const uint32_t b_j1 = sbw + static_cast<uint32_t>(j1 * kFold) * btap_units;
              const int wi = u * P.nshift1 + j1;
              const uint32_t dset = dbase + static_cast<uint32_t>(wi & acc_mask) * acc_cols;
#pragma unroll
              for (int i = 0; i < kMT + kFold - 1; ++i) {
                constexpr int kLast = kMT - 1;
                const int lo = i > kLast ? i - kLast : 0;
                const int hi = i < kFold - 1 ? i : kFold - 1;
                const uint32_t idesc =
                    P.idesc_base | (static_cast<uint32_t>(((hi - lo + 1) * P.n_blk) >> 3) << 17);
                const uint32_t a_addr = a_j1 + static_cast<uint32_t>(i) * tile_units;
                const uint32_t b_addr = b_j1 + static_cast<uint32_t>(lo) * btap_units;
                const uint32_t d = dset + static_cast<uint32_t>(kLast - i + lo) * tile_cols;
#pragma unroll
                for (int kk = 0; kk < kKSteps; ++kk) {
                  const uint64_t ad = desc_hi | (a_addr + 2u * kk);
                  const uint64_t bd = desc_hi | (b_addr + 2u * kk);
                  if constexpr (kParts == 2) {
                    mma<kTF32>(d, desc_hi | (a_addr + a_small_units + 2u * kk), bd, idesc, 1u);
                    mma<kTF32>(d, ad, desc_hi | (b_addr + b_small_units + 2u * kk), idesc, 1u);
                    mma<kTF32>(d, ad, bd, idesc, 1u);
                  } else {
                    mma<kTF32>(d, ad, bd, idesc, 1u);
                  }
                }
              }
            };
            if (P.nshift1 == 3) {
              fold_shift(0);  // three a1 shifts: straight-line issue
              fold_shift(1);
              fold_shift(2);
            } else {
              for (int j1 = 0; j1 < P.nshift1; ++j1) fold_shift(j1);
            }
          } else {
          uint32_t a_tap = sa;
          uint32_t b_tap = sa + (P.b_off >> 4);
          int j1 = 0;
          // The M-tile and K-step loops are unrolled at compile time: a runtime loop or
          // per-tap division between MMAs slows the issue below the operand-feed rate.
          for (int t = 0; t < nshift_stage; ++t) {
            const int wi = w_unit + t;
            const uint32_t first = (wi < P.nacc && cb == 0) ? 1u : 0u;
            const uint32_t d0 = dbase + static_cast<uint32_t>(wi & acc_mask) * acc_cols;
#pragma unroll
            for (int m = 0; m < kMT; ++m) {
              const uint32_t a_addr = a_tap + static_cast<uint32_t>(m) * tile_units;
              const uint32_t d = d0 + static_cast<uint32_t>(m) * tile_cols;
#pragma unroll
              for (int kk = 0; kk < kKSteps; ++kk) {
                const uint64_t ad = desc_hi | (a_addr + 2u * kk);
                const uint64_t bd = desc_hi | (b_tap + 2u * kk);
                const uint32_t acc = (first != 0u && kk == 0) ? 0u : 1u;
                if constexpr (kParts == 2) {
                  mma<kTF32>(d, desc_hi | (a_addr + a_small_units + 2u * kk), bd, P.idesc, acc);
                  mma<kTF32>(d, ad, desc_hi | (b_tap + b_small_units + 2u * kk), P.idesc, 1u);
                  mma<kTF32>(d, ad, bd, P.idesc, 1u);
                } else {
                  mma<kTF32>(d, ad, bd, P.idesc, acc);
                }
              }
            }
            b_tap += btap_units;
            if (++j1 == P.nshift1) {
              j1 = 0;
              a_tap += j0_wrap;
            } else {
              a_tap += j1_units;
            }
          }
          }
          dev::mma_commit_warp(&empty[stage]);
          ++done;
          if (leader) *progress = done;
          __syncwarp();
          if (++stage == P.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      dev::mma_commit_warp(&acc_full[buf]);
      __syncwarp();
    }
  } else if (warp >= 2) {
    // ------------------------------ epilogue ------------------------------
    const int group = (warp - 2) >> 2;
    const int groups = P.epi_groups;
    const int quarter = warp & 3;  // TMEM lanes 32 * (warp % 4) ..
    const int row = quarter * 32 + lane;
    const int i2 = row % P.b2;
    const int i1 = (row / P.b2) % P.b1;
    const int i0 = row / (P.b2 * P.b1);
    // Output rows of a tile: the first b2o of every line (all of them unless the a2 taps
    // are folded); prow is a row's place among them, the staging order of TMA stores.
    const bool line_ok = i2 < P.b2o;
    const int prow = (i0 * P.b1 + i1) * P.b2o + i2;
    const int tile_rows = P.e0 * P.b1 * P.b2o;
    // Spatial element offset of output (outer position of S, o0, o1, o2) in the output
    // tensor, and that tensor's positions per image (a phase of a strided input gradient
    // lands on a strided sub-grid of a larger tensor).
    auto out_offset = [&](const Super& S, int o0, int o1, int o2) -> int64_t {
      if (!P.out_strided) {
        return S.outer_lin * P.out_box_vol + (static_cast<int64_t>(o0) * P.out[1] + o1) * P.out[2] + o2;
      }
      int64_t off = P.phase_base + o0 * P.ostride_box[0] + o1 * P.ostride_box[1] +
                    o2 * P.ostride_box[2];
#pragma unroll
      for (int a = 0; a < kMaxOuter; ++a) {
        if (a < P.n_outer) off += S.o[a] * P.ostride_o[a];
      }
      return off;
    };
    const int64_t out_vol = P.out_strided ? P.out_volume_full : P.out_volume;
    // Fused activation: store the pre-activation values of this thread's row (M tile m,
    // channels c * 16 ..), then apply the activation in place.
    // With pre_staged the staged branches write the pre-activation tile themselves.
    auto activate = [&](const Super& S, int m, int o1, int o2, int c, float (&value)[16]) {
      if (!P.act) return;
      const int o0 = S.a0_first + m * P.a0_tile_step + i0;
      if (P.pre != nullptr && !P.pre_staged && line_ok && o0 < P.out[0] && o1 < P.out[1] &&
          o2 < P.out[2]) {
        OutT* pre = static_cast<OutT*>(P.pre);
        const int64_t sp = out_offset(S, o0, o1, o2);
        if (P.out_cl) {
          store_run16<OutT>(pre + (S.n * out_vol + sp) * P.out_channels_total +
                                static_cast<int64_t>(S.g) * P.n_real + c * 16,
                            value, P.n_real - c * 16);
        } else {
          OutT* dst = pre + (S.n * P.out_channels_total + static_cast<int64_t>(S.g) * P.n_real) *
                                out_vol + sp;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int co = c * 16 + i;
            if (co < P.n_real) dst[static_cast<int64_t>(co) * out_vol] = Traits::cast(value[i]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) value[i] = gelu_exact(value[i]);
    };
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int used = work_per_super < P.nacc ? work_per_super : P.nacc;
    const OutT* bias = static_cast<const OutT*>(P.bias);
    OutT* out = static_cast<OutT*>(P.dst);
    const bool store_issuer = threadIdx.x == 64 + 128 * group;  // lane 0 of the group
    // Staging: one group alternates two buffers (a store may still read the older one);
    // with two groups each has one, reused once its previous store has read it.
    const int stage_slots = groups == 1 ? 2 : 1;
    const uint32_t stage_slot_bytes = (P.pre_staged ? 2 : 1) * P.out_tile_bytes;
    uint8_t* const group_stage = smem + P.out_stage_off + group * stage_slot_bytes;
    const int barrier_id = 1 + group;
    // TMEM column of M tile m's accumulator (descending when the a0 taps are folded).
    auto tile_col = [&](int m) { return (kFold > 0 ? kMT - 1 - m : m) * P.n_blk; };
    // One 16-channel chunk of this thread's output row of M tile m.
    auto chunk = [&](uint32_t dbase, int m, int c, const OutT* group_bias, float (&value)[16]) {
      if (P.k2f > 1) {
        epilogue_chunk_k2<Traits, kMT>(dbase, tile_col(m), c, P, used, group_bias, value);
      } else {
        epilogue_chunk<Traits, kMT, (kFold > 0)>(dbase, tile_col(m), c, P.n_pad, used,
                                                 group_bias, P.n_real, value);
      }
    };
    // The 16-channel chunks of tile m, each handed to body(c, value) with the bias added.
    // With one accumulator set and no a2 fold, chunk c + 1's TMEM load is issued before
    // chunk c is processed, so its latency hides behind the activation and the stores.
    auto tile_chunks = [&](uint32_t dbase, int m, const OutT* group_bias, auto&& body) {
      const int nchunks = P.n_pad / 16;
      if (P.k2f > 1 || used > 1) {
        for (int c = 0; c < nchunks; ++c) {
          float value[16];
          chunk(dbase, m, c, group_bias, value);
          body(c, value);
        }
        return;
      }
      const uint32_t col0 = dbase + static_cast<uint32_t>(tile_col(m));
      uint32_t raw[16];
      __syncwarp();
      dev::tmem_load16(col0, raw);
      for (int c = 0; c < nchunks; ++c) {
        dev::tmem_load_wait();
        float value[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) value[i] = __uint_as_float(raw[i]);
        if constexpr (kFold > 0) dev::tmem_zero16(col0 + 16u * static_cast<uint32_t>(c));
        if (c + 1 < nchunks) {
          __syncwarp();
          dev::tmem_load16(col0 + 16u * static_cast<uint32_t>(c + 1), raw);
        }
        if (group_bias != nullptr) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int co = c * 16 + i;
            if (co < P.n_real) value[i] += Traits::load(group_bias + co);
          }
        }
        body(c, value);
      }
    };
    if constexpr (kFold > 0) {
      // Folded MMAs all accumulate: start both accumulator buffers at zero.
      for (int c = 16 * group; c < 2 * P.acc_stride; c += 16 * groups) {
        __syncwarp();
        dev::tmem_zero16(lane_addr + static_cast<uint32_t>(c));
      }
      dev::tmem_store_wait();
      dev::tc_fence_before();
      dev::mbar_arrive(&acc_empty[0]);
      dev::mbar_arrive(&acc_empty[1]);
    }
    int out_tiles = 0;
    int iter = 0;
    for (int64_t st = blockIdx.x; st < P.supers_total; st += gridDim.x, ++iter) {
      const int buf = iter & 1;
      dev::mbar_wait_progress(&acc_full[buf], static_cast<uint32_t>(iter >> 1) & 1u, progress,
                              err, kSiteEpilogue, P.timeout_ns);
      dev::tc_fence_after();
      Super S;
      decode_super(P, st, S);
      const uint32_t dbase = lane_addr + static_cast<uint32_t>(buf * P.acc_stride);
      const int o1 = S.q1 * P.b1 + i1;
      const int o2 = S.q2 * P.b2o + i2;
      const int64_t channel_base =
          (S.n * P.out_channels_total + static_cast<int64_t>(S.g) * P.n_real) * out_vol;
      const OutT* group_bias = bias != nullptr ? bias + static_cast<int64_t>(S.g) * P.n_real : nullptr;
      if (P.tma_store && P.out_cl) {
        // Channels-last rows: stage the tile as [position][channel] (swizzled 16-byte
        // chunks, so a warp's row stores spread over the banks) and write each column
        // chunk with one TMA store; buffers alternate as below.
        const uint32_t span = P.out_span;
        const uint32_t mask = span == 128 ? 7u : (span == 64 ? 3u : (span == 32 ? 1u : 0u));
        const int row_bytes = P.n_real * static_cast<int>(sizeof(OutT));
        const int32_t merged = static_cast<int32_t>(S.n * P.out_outer_vol + S.outer_lin);
        // One 16-channel chunk of this thread's row into a staging buffer.
        auto stage_row = [&](uint8_t* stage, int c, const float (&value)[16]) {
          alignas(16) OutT packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) packed[i] = Traits::cast(value[i]);
#pragma unroll
          for (int v = 0; v < static_cast<int>(sizeof(OutT)); ++v) {  // 16-byte vectors
            const int off = c * 16 * static_cast<int>(sizeof(OutT)) + v * 16;
            if (off < row_bytes && line_ok) {
              const uint32_t part = static_cast<uint32_t>(off) / span;
              uint32_t addr = part * 128u * span + static_cast<uint32_t>(prow) * span +
                              static_cast<uint32_t>(off) % span;
              addr ^= ((addr >> 7) & mask) << 4;
              *reinterpret_cast<uint4*>(stage + addr) = reinterpret_cast<const uint4*>(packed)[v];
            }
          }
        };
        for (int m = group; m < kMT; m += groups, ++out_tiles) {
          // this group's buffer of the tile, and with pre_staged its pre-activation
          // buffer beside it
          uint8_t* stage = group_stage + (out_tiles & (stage_slots - 1)) * groups *
                                             stage_slot_bytes;
          uint8_t* pre_stage = stage + P.out_tile_bytes;
          if (store_issuer) {
            if (stage_slots == 2) {
              dev::bulk_wait_group_read<1>();
            } else {
              dev::bulk_wait_group_read<0>();
            }
          }
          dev::named_barrier(barrier_id, 128);
          tile_chunks(dbase, m, group_bias, [&](int c, float (&value)[16]) {
            if (P.pre_staged) stage_row(pre_stage, c, value);
            activate(S, m, o1, o2, c, value);
            stage_row(stage, c, value);
          });
          dev::fence_proxy_async();
          dev::named_barrier(barrier_id, 128);
          if (store_issuer) {
            const int32_t o0 = S.a0_first + m * P.a0_tile_step;
            for (int k = 0; k * static_cast<int>(span) < row_bytes; ++k) {
              const int32_t ch = S.g * P.n_real + k * static_cast<int>(span / sizeof(OutT));
              dev::tma_store_5d(&maps.out, stage + k * 128 * span, ch, S.q2 * P.b2o,
                                S.q1 * P.b1, o0, merged);
              if (P.pre_staged) {
                dev::tma_store_5d(&maps.pre, pre_stage + k * 128 * span, ch, S.q2 * P.b2o,
                                  S.q1 * P.b1, o0, merged);
              }
            }
            dev::bulk_commit_group();
          }
        }
        if constexpr (kFold > 0) dev::tmem_store_wait();
        dev::tc_fence_before();
        dev::mbar_arrive(&acc_empty[buf]);
        continue;
      }
      if (P.tma_store) {
        // Stage each M tile as [channel][position] and write it with one TMA store; the
        // buffer of tile t is reused by tile t + 2 once that store has read it.
        const int32_t nc0 = static_cast<int32_t>(S.n * P.out_channels_total +
                                                 static_cast<int64_t>(S.g) * P.n_real);
        auto stage_cols = [&](OutT* buf, int c, const float (&value)[16]) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int co = c * 16 + i;
            if (co < P.n_real && line_ok) buf[co * tile_rows + prow] = Traits::cast(value[i]);
          }
        };
        for (int m = group; m < kMT; m += groups, ++out_tiles) {
          OutT* stage_buf = reinterpret_cast<OutT*>(
              group_stage + (out_tiles & (stage_slots - 1)) * groups * stage_slot_bytes);
          OutT* pre_buf = reinterpret_cast<OutT*>(reinterpret_cast<uint8_t*>(stage_buf) +
                                                  P.out_tile_bytes);
          if (store_issuer) {
            if (stage_slots == 2) {
              dev::bulk_wait_group_read<1>();
            } else {
              dev::bulk_wait_group_read<0>();
            }
          }
          dev::named_barrier(barrier_id, 128);
          tile_chunks(dbase, m, group_bias, [&](int c, float (&value)[16]) {
            if (P.pre_staged) stage_cols(pre_buf, c, value);
            activate(S, m, o1, o2, c, value);
            stage_cols(stage_buf, c, value);
          });
          dev::fence_proxy_async();
          dev::named_barrier(barrier_id, 128);
          if (store_issuer) {
            const int32_t o0 = S.a0_first + m * P.a0_tile_step;
            dev::tma_store_5d(&maps.out, stage_buf, S.q2 * P.b2o, S.q1 * P.b1, o0,
                              static_cast<int32_t>(S.outer_lin), nc0);
            if (P.pre_staged) {
              dev::tma_store_5d(&maps.pre, pre_buf, S.q2 * P.b2o, S.q1 * P.b1, o0,
                                static_cast<int32_t>(S.outer_lin), nc0);
            }
            dev::bulk_commit_group();
          }
        }
        if constexpr (kFold > 0) dev::tmem_store_wait();
        dev::tc_fence_before();
        dev::mbar_arrive(&acc_empty[buf]);
        continue;
      }
      if (P.out_cl) {
        // Channels-last rows: this thread's position holds n_real consecutive channels.
        for (int m = group; m < kMT; m += groups) {
          const int o0 = S.a0_first + m * P.a0_tile_step + i0;
          const bool valid = line_ok && o0 < P.out[0] && o1 < P.out[1] && o2 < P.out[2];
          const int64_t sp = out_offset(S, o0, o1, o2);
          OutT* dst = out + (S.n * out_vol + sp) * P.out_channels_total +
                      static_cast<int64_t>(S.g) * P.n_real;
          tile_chunks(dbase, m, group_bias, [&](int c, float (&value)[16]) {
            activate(S, m, o1, o2, c, value);
            if (valid) store_run16<OutT>(dst + c * 16, value, P.n_real - c * 16);
          });
        }
        if constexpr (kFold > 0) dev::tmem_store_wait();
        dev::tc_fence_before();
        dev::mbar_arrive(&acc_empty[buf]);
        continue;
      }
      for (int m = group; m < kMT; m += groups) {
        const int o0 = S.a0_first + m * P.a0_tile_step + i0;
        const bool valid = line_ok && o0 < P.out[0] && o1 < P.out[1] && o2 < P.out[2];
        const int64_t sp = out_offset(S, o0, o1, o2);
        OutT* dst = out + channel_base + sp;
        tile_chunks(dbase, m, group_bias, [&](int c, float (&value)[16]) {
          activate(S, m, o1, o2, c, value);
          if (valid) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int co = c * 16 + i;
              if (co < P.n_real) dst[static_cast<int64_t>(co) * out_vol] = Traits::cast(value[i]);
            }
          }
        });
      }
      if constexpr (kFold > 0) dev::tmem_store_wait();
      dev::tc_fence_before();
      dev::mbar_arrive(&acc_empty[buf]);
    }
    // The staged stores must be complete before the CTA's shared memory goes away.
    if (P.tma_store && store_issuer) dev::bulk_wait_group<0>();
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

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
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

int elem_size(int op) { return op == kOpF32 ? 4 : 2; }

CUtensorMapDataType map_dtype(int op) {
  if (op == kOpBF16) return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (op == kOpF16) return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}

CUtensorMapSwizzle swizzle_for(int row_bytes) {
  if (row_bytes == 32) return CU_TENSOR_MAP_SWIZZLE_32B;
  if (row_bytes == 64) return CU_TENSOR_MAP_SWIZZLE_64B;
  return CU_TENSOR_MAP_SWIZZLE_128B;
}

uint32_t layout_for(int row_bytes) {
  if (row_bytes == 32) return 6;
  if (row_bytes == 64) return 4;
  return 2;
}

int row_bytes_for(int op, int c_pad) {
  const int row = c_pad * elem_size(op);
  if (row == 32 || row == 64 || row == 128) return row;
  if (row > 128 && row % 128 == 0) return 128;
  return 0;
}

uint32_t round_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

uint32_t pow2_columns(int needed) {
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(needed)) cols <<= 1;
  return cols;
}

int device_sms() {
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

uint32_t make_idesc(int op, int m, int n) {
  uint32_t desc = 1u << 4;  // fp32 accumulator
  const uint32_t fmt = op == kOpBF16 ? 1u : (op == kOpF16 ? 0u : 2u);
  desc |= fmt << 7;
  desc |= fmt << 10;
  desc |= static_cast<uint32_t>(n >> 3) << 17;
  desc |= static_cast<uint32_t>(m >> 4) << 24;
  return desc;
}

constexpr int64_t kInt32Max = (int64_t{1} << 31) - 1;

// Fills the geometry part of the parameters (axes split, extents). False when a value
// does not fit the kernel's 32-bit coordinates.
bool fill_geometry(const ConvPass& pass, FpropParams* P) {
  const int rank = pass.rank;
  if (rank < 1 || rank > kMaxFastRank) return false;
  const int n_outer = rank > 3 ? rank - 3 : 0;
  const int lead = 3 - (rank - n_outer);
  P->n_outer = n_outer;
  for (int a = 0; a < 3; ++a) {
    const int src = a - lead + n_outer;
    if (a < lead) {
      P->out[a] = P->in[a] = P->k[a] = P->s[a] = P->d[a] = 1;
      P->p[a] = 0;
      continue;
    }
    if (pass.in[src] > kInt32Max / 4 || pass.out[src] > 65536 || pass.k[src] > 4096 ||
        pass.s[src] > 8 || pass.d[src] > 65536 || pass.p[src] > 65536) {
      return false;
    }
    P->out[a] = static_cast<int>(pass.out[src]);
    P->in[a] = static_cast<int>(pass.in[src]);
    P->k[a] = static_cast<int>(pass.k[src]);
    P->s[a] = static_cast<int>(pass.s[src]);
    P->d[a] = static_cast<int>(pass.d[src]);
    P->p[a] = static_cast<int>(pass.p[src]);
  }
  int64_t in_vol = 1, out_vol = 1, taps = 1;
  for (int a = kMaxOuter - 1; a >= 0; --a) {
    if (a >= n_outer) {
      P->out_o[a] = P->in_o[a] = P->k_o[a] = P->s_o[a] = P->d_o[a] = 1;
      P->p_o[a] = 0;
      P->in_o_stride[a] = 0;
      continue;
    }
    if (pass.in[a] > kInt32Max || pass.out[a] > kInt32Max || pass.k[a] > 4096 ||
        pass.s[a] > 65536 || pass.d[a] > 65536 || pass.p[a] > 65536) {
      return false;
    }
    P->out_o[a] = static_cast<int>(pass.out[a]);
    P->in_o[a] = static_cast<int>(pass.in[a]);
    P->k_o[a] = static_cast<int>(pass.k[a]);
    P->s_o[a] = static_cast<int>(pass.s[a]);
    P->d_o[a] = static_cast<int>(pass.d[a]);
    P->p_o[a] = static_cast<int>(pass.p[a]);
    P->in_o_stride[a] = in_vol;
    in_vol *= pass.in[a];
    out_vol *= pass.out[a];
  }
  for (int a = 0; a < rank; ++a) taps *= pass.k[a];
  if (taps > 1 << 20) return false;
  P->taps = static_cast<int>(taps);
  P->batch = pass.batch;
  P->groups = pass.groups;
  P->in_merged_per_gn = in_vol;
  P->out_outer_vol = out_vol;
  P->out_box_vol = static_cast<int64_t>(P->out[0]) * P->out[1] * P->out[2];
  P->out_volume = out_vol * P->out_box_vol;
  if (pass.batch * pass.groups * in_vol > kInt32Max) return false;
  return true;
}

struct Candidate {
  int e0, b1, b2, mt, shift0, shift1, row_bytes, fold, k2f;
};

// Cycles of one M=128, K=16 (or tf32 K=8) MMA with N columns on this part: the larger of
// the tensor-pipe time and the shared-memory operand feed (A 4 KB + B 32 B per column at
// 128 B per clock), both measured on B200.
double mma_cycles(int n) {
  const double compute = n / 2.0;
  const double feed = (4096.0 + 32.0 * n) / 128.0;
  return compute > feed ? compute : feed;
}

// Shared-memory stage layout of a candidate; false when it does not fit.
bool layout_candidate(const ConvPass& pass, FpropParams* P, const Candidate& c, int parts) {
  const int row_bytes = c.row_bytes;
  const int es = pass.op == kOpF32 ? 4 : 2;
  P->cblk_elems = row_bytes / es;
  P->cblocks = pass.c_pad / P->cblk_elems;
  P->ksteps = row_bytes / 32;
  P->layout = static_cast<int>(layout_for(row_bytes));
  P->fold = c.fold;
  const int k0 = P->k[0], k1 = P->k[1];
  P->e0 = c.e0;
  P->b1 = c.b1;
  P->b2 = c.b2;
  P->mt = c.mt;
  P->k2f = c.k2f;
  P->b2o = c.b2;
  if (c.k2f > 1) {
    // a line of b2 input-aligned rows completes b2 - (k2 - 1) * d2 outputs; one line
    // covers a short axis whole
    P->b2o = c.b2 - (c.k2f - 1) * P->d[2];
    if (P->b2o > P->out[2]) P->b2o = P->out[2];
  }
  P->n_blk = c.k2f * pass.n_pad;
  P->nshift0 = c.shift0 ? k0 : 1;
  P->nshift1 = c.shift1 ? k1 : 1;
  P->par0 = (c.fold && P->d[0] == 2) ? 2 : 1;
  P->a0_tile_step = c.e0 * P->par0;
  P->h0 = c.mt * c.e0 + (c.shift0 ? (k0 - 1) * (P->d[0] / P->par0) : 0);
  P->h1 = c.b1 + (c.shift1 ? (k1 - 1) * P->d[1] : 0);
  // TMA box extents (elements of the packed tensor, before element striding).
  const int box0 = c.shift0 ? P->h0 * P->par0 : c.mt * c.e0 * P->s[0];
  const int box1 = c.shift1 ? P->h1 : c.b1 * P->s[1];
  const int box2 = c.b2 * P->s[2];
  if (box0 > 256 || box1 > 256 || box2 > 256) return false;
  const uint32_t rows = static_cast<uint32_t>(P->h0 * P->h1 * c.b2);
  P->row_bytes = row_bytes;
  P->a_part_bytes = round_up(rows * row_bytes, 1024);
  const int nshift = P->nshift0 * P->nshift1 * c.k2f;  // weight rows (taps) per unit
  P->b_part_bytes = round_up(static_cast<uint32_t>(nshift * pass.n_pad * row_bytes), 1024);
  P->b_off = P->a_part_bytes * parts;
  P->stage_bytes = P->b_off + P->b_part_bytes * parts;
  P->tx_bytes = (rows * row_bytes + static_cast<uint32_t>(nshift * pass.n_pad * row_bytes)) * parts;
  return P->stage_bytes <= 100 * 1024;
}

}  // namespace

bool plan_fprop(const ConvPass& pass, FpropPlan* plan) {
  std::memset(plan, 0, sizeof(*plan));
  FpropParams& P = plan->params;
  if (pass.n_pad < 16 || pass.n_pad > 256 || pass.n_pad % 16 != 0) return false;
  const int row_max = row_bytes_for(pass.op, pass.c_pad);
  if (row_max == 0) return false;
  if (!fill_geometry(pass, &P)) return false;
  const bool tf32 = pass.op == kOpF32;
  // split3: float32 operands as two parts (TF32 big + small, or bf16 hi + lo)
  const int parts = pass.split3 ? 2 : 1;
  const int es = elem_size(pass.op);
  const int out_es = pass.out_dtype == CND_F32 ? 4 : 2;  // the output's element size
  P.n_pad = pass.n_pad;
  P.n_real = pass.n_real;
  const int products = parts == 2 ? 3 : 1;
  const int64_t outer_count = pass.batch * P.out_outer_vol * pass.groups;

  double best = 1e300;
  FpropParams chosen{};
  bool found = false;
  for (int row_bytes = row_max; row_bytes >= 32; row_bytes /= 2) {
   // Narrower channel blocks (more K passes, down to a quarter row) only when the full
   // row already fills 128 B: they make room for more M tiles per super tile (c2 dgrad:
   // 8 tiles of 32-byte blocks, fewer narrow edge MMAs of the a0 fold).
   if (row_bytes != row_max &&
       (row_max < 64 || row_bytes < row_max / 4 || (pass.c_pad * es) % row_bytes != 0)) {
     break;
   }
   for (int fold = 0; fold <= 2; ++fold) {
    // Folding the a0 taps into N needs unit-stride a0 tiles of one slice, three a0 taps
    // and 3 * n_pad <= 256. fold = 2 folds the a2 taps as well (k2f = k2): unit-stride a2,
    // 3 * k2 * n_pad <= 256, lines of 16 or 32 rows.
    // Dilation 2 folds too, over output planes of one parity (FpropParams::par0).
    if (fold && (P.k[0] != 3 || (P.d[0] != 1 && P.d[0] != 2) || P.s[0] != 1 ||
                 3 * pass.n_pad > 256)) {
      continue;
    }
    const int k2f = fold == 2 ? P.k[2] : 1;
    if (fold == 2 && (P.k[2] < 2 || P.s[2] != 1 || 3 * k2f * pass.n_pad > 256)) continue;
    for (int e0 = 1; e0 <= 128; e0 *= 2) {
    if (fold && e0 != 1) continue;
    for (int b2 = 8; b2 <= 128; b2 *= 2) {
      if (128 % (e0 * b2) != 0) continue;
      if (fold == 2 && (b2 < 16 || b2 > 32 || b2 - (k2f - 1) * P.d[2] < 1)) continue;
      const int b1 = 128 / (e0 * b2);
      for (int mt : {1, 2, 4, 6, 8, 12}) {
        if (fold && mt < 2) continue;
        // 6 and 12 tiles per super tile (12-wide a0 axes without padding slices) are
        // instantiated for the folded 16-bit kernels only.
        if ((mt == 6 || mt == 12) && (!fold || parts > 1)) continue;
        for (int shift0 = 0; shift0 <= 1; ++shift0) {
          if (shift0 && (P.s[0] != 1 || P.k[0] == 1)) continue;
          if (fold && !shift0) continue;
          for (int shift1 = 0; shift1 <= 1; ++shift1) {
            if (shift1 && (P.s[1] != 1 || P.k[1] == 1 || e0 != 1)) continue;
            FpropParams trial = P;
            const Candidate cand{e0, b1, b2, mt, shift0, shift1, row_bytes, fold ? 1 : 0, k2f};
            if (!layout_candidate(pass, &trial, cand, parts)) continue;
            const int n_blk = k2f * pass.n_pad;
            int nacc = 1;
            if (parts > 1 || tf32) {
              nacc = 8;
              while (nacc > 1 && 2 * nacc * mt * n_blk > 512) nacc /= 2;
              // split-product (float32) passes keep at least two rotating accumulators
              // (one accumulator over a whole unit walk grows the accumulation error);
              // with the a2 fold the k2f column blocks already split every chain
              if (nacc < 2 && k2f < 2) continue;
            }
            if (2 * nacc * mt * n_blk > 512) continue;
            // Estimated cycles per useful output position.
            const int b2o = trial.b2o;
            // super tiles along a0 (per parity with a parity split) times their tiles
            const int par0 = trial.par0;
            const int per_parity = (P.out[0] + par0 - 1) / par0;
            const double tiles0 = par0 * ((per_parity + mt * e0 - 1) / (mt * e0));
            const double waste = (tiles0 * mt * e0 / P.out[0]) *
                                 (double((P.out[1] + b1 - 1) / b1) * b1 / P.out[1]) *
                                 (double((P.out[2] + b2o - 1) / b2o) * b2 / P.out[2]);
            const int nshift = trial.nshift0 * trial.nshift1 * k2f;
            const double units = double(P.taps) / nshift * trial.cblocks;
            double mma_total;
            if (fold) {
              // one MMA per (slice, a1 shift), N = taps of the slice that hit a tile
              double per_pass = 0.0;
              for (int i = 0; i < mt + 2; ++i) {
                const int lo = i > mt - 1 ? i - (mt - 1) : 0;
                const int hi = i < 2 ? i : 2;
                per_pass += mma_cycles((hi - lo + 1) * n_blk);
              }
              mma_total = units * trial.nshift1 * trial.ksteps * products * per_pass;
            } else {
              mma_total = double(mt) * P.taps * trial.cblocks * trial.ksteps * products *
                          mma_cycles(pass.n_pad);
            }
            const double l2_cycles = units * trial.tx_bytes / 70.0;
            const double issue_cycles = units * 250.0;
            double cycles = mma_total;
            if (l2_cycles > cycles) cycles = l2_cycles;
            if (issue_cycles > cycles) cycles = issue_cycles;
            // Bound plus a small preference for less L2 traffic and fewer load units
            // (both shorten the latency chain the bound ignores).
            const double per_position =
                (cycles + 0.15 * l2_cycles + 0.05 * issue_cycles) * waste / (mt * 128.0);
            // Enough super tiles to fill the machine.
            const double supers = double(outer_count) * tiles0 *
                                  ((P.out[1] + b1 - 1) / b1) * ((P.out[2] + b2o - 1) / b2o);
            const double fill = supers >= device_sms() ? 1.0 : device_sms() / supers;
            const double score = per_position * fill;
            if (score < best) {
              best = score;
              chosen = trial;
              chosen.nacc = nacc;
              found = true;
            }
          }
        }
      }
    }
    }
   }
  }
  if (!found) return false;
  plan->score = best;
  P = chosen;
  P.units = P.taps / (P.nshift0 * P.nshift1 * P.k2f);
  P.nsup[0] = P.par0 * (((P.out[0] + P.par0 - 1) / P.par0 + P.mt * P.e0 - 1) / (P.mt * P.e0));
  P.nsup[1] = (P.out[1] + P.b1 - 1) / P.b1;
  P.nsup[2] = (P.out[2] + P.b2o - 1) / P.b2o;
  P.supers_total = outer_count * P.nsup[0] * P.nsup[1] * P.nsup[2];
  P.acc_stride = P.nacc * P.mt * P.n_blk;
  P.tmem_cols = pow2_columns(2 * P.acc_stride);
  P.stages = static_cast<int>((200 * 1024) / P.stage_bytes);
  if (P.stages > 8) P.stages = 8;
  if (P.stages < 2) return false;
  // Output through staged TMA stores when the channels-first rows allow 16-byte aligned
  // boxes (innermost output extent and tile width multiples of 16 bytes) and the two
  // staging buffers fit beside at least two stages, without giving up two CTAs per SM.
  const size_t extra = 1024 + (2 * 8 + 4) * 8 + 64;
  P.tma_store = 0;
  P.pre_staged = 0;
  P.out_tile_bytes = round_up(static_cast<uint32_t>(pass.n_real * 128 * out_es), 1024);
  P.out_cl = pass.out_cl;
  P.act = pass.activation;
  P.out_strided = pass.out_strided;
  if (pass.out_strided) {
    // element strides of the full tensor's axes (row-major), times the phase multipliers
    int64_t stride_full[kMaxFastRank];
    int64_t vol = 1;
    for (int a = pass.rank - 1; a >= 0; --a) {
      stride_full[a] = vol;
      vol *= pass.out_full[a];
    }
    P.out_volume_full = vol;
    P.phase_base = 0;
    for (int a = 0; a < pass.rank; ++a) P.phase_base += pass.out_add[a] * stride_full[a];
    const int n_outer = P.n_outer;
    const int lead = 3 - (pass.rank - n_outer);
    for (int a = 0; a < kMaxOuter; ++a) {
      P.ostride_o[a] = a < n_outer ? pass.out_mul[a] * stride_full[a] : 0;
    }
    for (int a = 0; a < 3; ++a) {
      const int src = a - lead + n_outer;
      P.ostride_box[a] = a < lead ? 0 : pass.out_mul[src] * stride_full[src];
    }
  }
  // Channels-last rows go through TMA stores when one position's channels form 16 bytes
  // or a swizzle width (32 / 64 / 128 bytes), or whole 128-byte chunks.
  const int cl_row = pass.n_real * out_es;
  P.out_span = 0;
  if (pass.out_cl) {
    if (cl_row == 16 || cl_row == 32 || cl_row == 64 || cl_row == 128) {
      P.out_span = static_cast<uint32_t>(cl_row);
    } else if (cl_row % 128 == 0) {
      P.out_span = 128;
    }
  }
  const bool store_shape = pass.out_strided ? false :
      pass.out_cl
          ? (P.out_span > 0 && pass.n_real <= 256 &&
             pass.batch * P.out_outer_vol <= kInt32Max &&
             (pass.groups * pass.n_real * out_es) % 16 == 0)
          : ((static_cast<int64_t>(P.out[2]) * out_es) % 16 == 0 && (P.b2o * out_es) % 16 == 0 &&
             pass.n_real <= 256 && pass.batch * pass.groups * pass.n_real <= kInt32Max &&
             P.out_outer_vol <= kInt32Max);
  // Two epilogue groups whenever a super tile has two M tiles to share: the epilogue's
  // TMEM loads, activation math and stores are latency-bound with one warp per
  // scheduler. A CTA of ten warps holds its SM alone, so it gets the full shared memory.
  P.epi_groups = P.mt >= 2 ? 2 : 1;
  if (store_shape) {
    const bool two = P.epi_groups == 1 &&
                     static_cast<size_t>(P.stages) * P.stage_bytes + extra <= 110 * 1024 &&
                     pow2_columns(2 * P.nacc * P.mt * P.n_blk) <= 256;
    const size_t cap = two ? 110 * 1024 - extra : 216 * 1024;
    // a fused activation also stages its pre-activation tile: two buffers per tile
    const int buffers = pass.activation != 0 ? 4 : 2;
    const size_t staging = buffers * static_cast<size_t>(P.out_tile_bytes);
    if (cap > staging) {
      int st = static_cast<int>((cap - staging) / P.stage_bytes);
      if (st > 8) st = 8;
      if (st >= 2) {
        P.stages = st;
        P.tma_store = 1;
        P.pre_staged = pass.activation != 0 ? 1 : 0;
      }
    }
  }
  P.out_stage_off = static_cast<uint32_t>(P.stages) * P.stage_bytes;
  P.bar_off = P.out_stage_off + (P.tma_store ? (P.pre_staged ? 4 : 2) * P.out_tile_bytes : 0);
  P.idesc = make_idesc(pass.op, 128, pass.n_pad);
  P.idesc_base = P.idesc & ~(0x3Fu << 17);
  P.out_dtype = pass.out_dtype;
  P.out_channels_total = pass.groups * pass.n_real;
  plan->parts = parts;
  plan->smem = static_cast<size_t>(P.bar_off) + 1024 + (2 * P.stages + 4) * 8 + 64;
  // Weight packing order: one load unit's shifted taps are consecutive rows.
  plan->shift0 = P.nshift0 > 1;
  plan->shift1 = P.nshift1 > 1;
  plan->fold = P.fold;
  plan->fold2 = P.k2f;
  plan->k_box[0] = P.k[0];
  plan->k_box[1] = P.k[1];
  plan->k_box[2] = P.k[2];
  return true;
}

int launch_fprop(const ConvPass& pass, const FpropPlan& plan_in, cudaStream_t stream,
                 uint64_t timeout_ns, int debug_stall) {
  FpropPlan plan = plan_in;
  FpropParams& P = plan.params;
  P.dst = pass.dst;
  P.bias = pass.bias;
  P.act = pass.activation;  // set per call: plans are made before the activation is known
  P.pre = pass.pre;
  // staged pre-activation tiles need a fused activation and a pre-activation tensor
  P.pre_staged = P.pre_staged && P.act != 0 && pass.pre != nullptr ? 1 : 0;
  P.err = device_error_word();
  P.timeout_ns = timeout_ns;
  P.debug_stall = debug_stall;
  if (P.supers_total == 0) return CND_OK;
  auto encode = encoder();
  if (encode == nullptr) return fail(CND_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int es = elem_size(pass.op);
  alignas(64) FpropMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  const void* act[2] = {pass.act, pass.act_small};
  const void* wt[2] = {pass.wt, pass.wt_small};
  for (int part = 0; part < plan.parts; ++part) {
    cuuint64_t dims[5] = {static_cast<cuuint64_t>(pass.c_pad), static_cast<cuuint64_t>(P.in[2]),
                          static_cast<cuuint64_t>(P.in[1]), static_cast<cuuint64_t>(P.in[0]),
                          static_cast<cuuint64_t>(pass.batch * pass.groups * P.in_merged_per_gn)};
    const cuuint64_t c = static_cast<cuuint64_t>(pass.c_pad) * es;
    cuuint64_t strides[4] = {c, c * P.in[2], c * P.in[2] * P.in[1], c * P.in[2] * P.in[1] * P.in[0]};
    const int box0 = P.nshift0 > 1 ? P.h0 * P.par0 : P.mt * P.e0 * P.s[0];
    const int box1 = P.nshift1 > 1 ? P.h1 : P.b1 * P.s[1];
    cuuint32_t boxd[5] = {static_cast<cuuint32_t>(P.cblk_elems),
                          static_cast<cuuint32_t>(P.b2 * P.s[2]), static_cast<cuuint32_t>(box1),
                          static_cast<cuuint32_t>(box0), 1};
    cuuint32_t estr[5] = {1, static_cast<cuuint32_t>(P.s[2]),
                          static_cast<cuuint32_t>(P.nshift1 > 1 ? 1 : P.s[1]),
                          static_cast<cuuint32_t>(P.nshift0 > 1 ? P.par0 : P.s[0]), 1};
    CUresult r = encode(&maps.act[part], map_dtype(pass.op), 5, const_cast<void*>(act[part]),
                        dims, strides, boxd, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_for(P.row_bytes), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      return fail(CND_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed with code %d",
                  static_cast<int>(r));
    }
    const int nshift = P.nshift0 * P.nshift1 * P.k2f;
    cuuint64_t wdims[3] = {static_cast<cuuint64_t>(pass.c_pad), static_cast<cuuint64_t>(pass.n_pad),
                           static_cast<cuuint64_t>(pass.groups * P.taps)};
    cuuint64_t wstrides[2] = {c, c * pass.n_pad};
    cuuint32_t wbox[3] = {static_cast<cuuint32_t>(P.cblk_elems),
                          static_cast<cuuint32_t>(pass.n_pad), static_cast<cuuint32_t>(nshift)};
    cuuint32_t westr[3] = {1, 1, 1};
    r = encode(&maps.wt[part], map_dtype(pass.op), 3, const_cast<void*>(wt[part]), wdims,
               wstrides, wbox, westr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(P.row_bytes),
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      return fail(CND_ERR_CUDA, "cuTensorMapEncodeTiled (weights) failed with code %d",
                  static_cast<int>(r));
    }
  }
  if (P.tma_store && P.out_cl) {
    // channels-last output: dims (channels, o2, o1, o0, batch x outer positions)
    const cuuint64_t e = pass.out_dtype == CND_F32 ? 4u : 2u;
    const CUtensorMapDataType out_type = pass.out_dtype == CND_F32
                                             ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                             : (pass.out_dtype == CND_BF16
                                                    ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    const cuuint64_t row = static_cast<cuuint64_t>(pass.groups * pass.n_real) * e;
    cuuint64_t odims[5] = {static_cast<cuuint64_t>(pass.groups * pass.n_real),
                           static_cast<cuuint64_t>(P.out[2]), static_cast<cuuint64_t>(P.out[1]),
                           static_cast<cuuint64_t>(P.out[0]),
                           static_cast<cuuint64_t>(pass.batch * P.out_outer_vol)};
    // byte strides of dims 1..4 (o2, o1, o0, merged); dim 0 (channels) is contiguous
    cuuint64_t ostrides[4] = {row, row * P.out[2], row * P.out[2] * P.out[1],
                              row * static_cast<cuuint64_t>(P.out_box_vol)};
    // The map must stay inside the output tensor: its furthest element is the last one.
    cuuint64_t last = (odims[0] - 1) * e;
    for (int d = 1; d < 5; ++d) last += (odims[d] - 1) * ostrides[d - 1];
    const cuuint64_t bytes = static_cast<cuuint64_t>(pass.batch) * P.out_volume * row;
    if (last + e != bytes) {
      return fail(CND_ERR_INVALID, "channels-last output map spans %llu bytes, tensor has %llu",
                  static_cast<unsigned long long>(last + e),
                  static_cast<unsigned long long>(bytes));
    }
    cuuint32_t obox[5] = {static_cast<cuuint32_t>(P.out_span / e), static_cast<cuuint32_t>(P.b2o),
                          static_cast<cuuint32_t>(P.b1), static_cast<cuuint32_t>(P.e0), 1};
    cuuint32_t oestr[5] = {1, 1, 1, 1, 1};
    const CUtensorMapSwizzle swizzle =
        P.out_span == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
        : P.out_span == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
        : P.out_span == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                           : CU_TENSOR_MAP_SWIZZLE_NONE;
    for (int which = 0; which < (P.pre_staged ? 2 : 1); ++which) {
      const CUresult r = encode(which == 0 ? &maps.out : &maps.pre, out_type, 5,
                                which == 0 ? pass.dst : pass.pre, odims, ostrides, obox, oestr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) {
        return fail(CND_ERR_CUDA,
                    "cuTensorMapEncodeTiled (channels-last output) failed with code %d",
                    static_cast<int>(r));
      }
    }
  } else if (P.tma_store) {
    // the output's own element type (float32 problems may run bf16-part operands)
    const cuuint64_t e = pass.out_dtype == CND_F32 ? 4u : 2u;
    const CUtensorMapDataType out_type = pass.out_dtype == CND_F32
                                             ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                             : (pass.out_dtype == CND_BF16
                                                    ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    cuuint64_t odims[5] = {static_cast<cuuint64_t>(P.out[2]), static_cast<cuuint64_t>(P.out[1]),
                           static_cast<cuuint64_t>(P.out[0]),
                           static_cast<cuuint64_t>(P.out_outer_vol),
                           static_cast<cuuint64_t>(pass.batch * pass.groups * pass.n_real)};
    cuuint64_t ostrides[4] = {static_cast<cuuint64_t>(P.out[2]) * e,
                              static_cast<cuuint64_t>(P.out[1]) * P.out[2] * e,
                              static_cast<cuuint64_t>(P.out_box_vol) * e,
                              static_cast<cuuint64_t>(P.out_volume) * e};
    cuuint64_t last = (odims[0] - 1) * e;
    for (int d = 1; d < 5; ++d) last += (odims[d] - 1) * ostrides[d - 1];
    if (last + e != static_cast<cuuint64_t>(pass.batch * pass.groups * pass.n_real) *
                        static_cast<cuuint64_t>(P.out_volume) * e) {
      return fail(CND_ERR_INVALID, "output map does not cover the output tensor exactly");
    }
    cuuint32_t obox[5] = {static_cast<cuuint32_t>(P.b2o), static_cast<cuuint32_t>(P.b1),
                          static_cast<cuuint32_t>(P.e0), 1, static_cast<cuuint32_t>(pass.n_real)};
    cuuint32_t oestr[5] = {1, 1, 1, 1, 1};
    for (int which = 0; which < (P.pre_staged ? 2 : 1); ++which) {
      const CUresult r = encode(which == 0 ? &maps.out : &maps.pre, out_type, 5,
                                which == 0 ? pass.dst : pass.pre, odims, ostrides, obox, oestr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) {
        return fail(CND_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed with code %d",
                    static_cast<int>(r));
      }
    }
  }
  // Persistent grid: two CTAs per SM when both fit (shared memory and TMEM), else one,
  // enforced through the shared-memory request.
  const bool two_per_sm = P.epi_groups == 1 && plan.smem <= 110 * 1024 && P.tmem_cols <= 256;
  size_t smem = plan.smem;
  if (!two_per_sm && smem < 120 * 1024) smem = 120 * 1024;
  int64_t grid = P.supers_total;
  const int64_t resident = static_cast<int64_t>(device_sms()) * (two_per_sm ? 2 : 1);
  if (grid > resident) grid = resident;
  using Kernel = void (*)(FpropMaps, FpropParams);
  Kernel kernel = nullptr;
  const int kind = pass.op == kOpF16 ? kKindF16
                   : pass.op == kOpBF16 ? (plan.parts == 2 ? kKind2xBF16 : kKindBF16)
                   : (plan.parts == 2 ? kKind3xTF32 : kKindTF32);
#define CND_FPROP_CASE(KIND, KSTEPS, MT)                                                 \
  if (kind == KIND && P.ksteps == KSTEPS && P.mt == MT && !P.fold)                        \
    kernel = fprop_kernel<KIND, KSTEPS, MT, 0>;
#define CND_FPROP_FOLD(KIND, KSTEPS, MT)                                                 \
  if (kind == KIND && P.ksteps == KSTEPS && P.mt == MT && P.fold)                         \
    kernel = fprop_kernel<KIND, KSTEPS, MT, 3>;
#define CND_FPROP_MT(KIND, KSTEPS)                                                  \
  CND_FPROP_CASE(KIND, KSTEPS, 1) CND_FPROP_CASE(KIND, KSTEPS, 2) CND_FPROP_CASE(KIND, KSTEPS, 4) \
  CND_FPROP_CASE(KIND, KSTEPS, 8)
#define CND_FPROP_FOLDS(KIND, KSTEPS) \
  CND_FPROP_FOLD(KIND, KSTEPS, 2) CND_FPROP_FOLD(KIND, KSTEPS, 4) CND_FPROP_FOLD(KIND, KSTEPS, 8)
#define CND_FPROP_FOLDS16(KIND, KSTEPS) \
  CND_FPROP_FOLDS(KIND, KSTEPS) CND_FPROP_FOLD(KIND, KSTEPS, 6) CND_FPROP_FOLD(KIND, KSTEPS, 12)
#define CND_FPROP_KS(KIND) CND_FPROP_MT(KIND, 1) CND_FPROP_MT(KIND, 2) CND_FPROP_MT(KIND, 4)
#define CND_FPROP_KSF(KIND) CND_FPROP_FOLDS(KIND, 1) CND_FPROP_FOLDS(KIND, 2) CND_FPROP_FOLDS(KIND, 4)
#define CND_FPROP_KSF16(KIND) \
  CND_FPROP_FOLDS16(KIND, 1) CND_FPROP_FOLDS16(KIND, 2) CND_FPROP_FOLDS16(KIND, 4)
  CND_FPROP_KS(kKindF16) CND_FPROP_KS(kKindBF16) CND_FPROP_KS(kKindTF32) CND_FPROP_KS(kKind3xTF32)
  CND_FPROP_KS(kKind2xBF16)
  CND_FPROP_KSF16(kKindF16) CND_FPROP_KSF16(kKindBF16) CND_FPROP_KSF(kKindTF32)
  CND_FPROP_KSF(kKind3xTF32) CND_FPROP_KSF(kKind2xBF16)
#undef CND_FPROP_KSF16
#undef CND_FPROP_KSF
#undef CND_FPROP_FOLDS16
#undef CND_FPROP_FOLDS
#undef CND_FPROP_FOLD
#undef CND_FPROP_KS
#undef CND_FPROP_MT
#undef CND_FPROP_CASE
  if (kernel == nullptr) return fail(CND_ERR_UNSUPPORTED, "no fprop kernel for this operand");
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  kernel<<<static_cast<unsigned>(grid), 64 + 128 * P.epi_groups, smem, stream>>>(maps, P);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(CND_ERR_CUDA, "fprop_kernel launch failed: %s", cudaGetErrorString(e));
  }
  count_launch();
  return CND_OK;
}

}  // namespace cnd
