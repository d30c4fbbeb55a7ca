// Thin inline-PTX wrappers for the sm_100a features the convolution kernels use:
// mbarriers with bounded waits, TMA tiled loads, tcgen05 TMEM allocation, MMA, commit
// and TMEM loads. Every wait is bounded by a %globaltimer deadline; on expiry it records
// a site code in the library's device error word and returns false instead of spinning
// forever, so a stalled pipeline ends the kernel with an error status the host can read.
#pragma once

#include <cuda.h>
#include <cstdint>

namespace cnd {
namespace dev {

// Device error word: 0 = ok, otherwise the site code of the first expired wait.
struct ErrorWord {
  unsigned int* word;
};

__device__ __forceinline__ uint32_t smem_u32(const void* pointer) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(pointer));
}

// One lane of a converged warp (elect.sync); returns true on that lane only.
__device__ __forceinline__ bool elect_one() {
  uint32_t elected;
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(elected));
  return elected != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete. Returns false (after recording
// `site` in the error word) once `timeout_ns` has passed without completion.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, ErrorWord err,
                                          unsigned int site, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63u) == 63u && global_timer_ns() - start > timeout_ns) {
      atomicCAS(err.word, 0u, site);
      return false;
    }
  }
}

// mbar_wait for a whole converged warp with one warp-uniform answer: lanes that poll
// independently could disagree at the deadline, and a warp that must stay converged
// (elect.sync issue) takes the failure path together.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, ErrorWord err,
                                               unsigned int site, uint64_t timeout_ns) {
  const bool ok = mbar_wait(bar, parity, err, site, timeout_ns);
  return __all_sync(0xffffffffu, ok) != 0;
}

// Like mbar_wait, for long waits (an epilogue waiting for a whole main loop): the
// deadline restarts whenever the shared counter `progress` changes, so the limit
// bounds a stall rather than the total work. Polls with a short sleep between tries.
__device__ __forceinline__ bool mbar_wait_progress(uint64_t* bar, uint32_t parity,
                                                   const volatile uint32_t* progress,
                                                   ErrorWord err, unsigned int site,
                                                   uint64_t timeout_ns) {
  uint64_t start = global_timer_ns();
  uint32_t seen = *progress;
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(200);
    const uint32_t now_progress = *progress;
    const uint64_t now = global_timer_ns();
    if (now_progress != seen) {
      seen = now_progress;
      start = now;
    } else if (now - start > timeout_ns) {
      atomicCAS(err.word, 0u, site);
      return false;
    }
  }
}

// TMA tiled loads (global -> shared), completion signalled on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3,
                                            int32_t c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "r"(c4)
      : "memory");
}

// TMA tiled store (shared -> global) of a whole box, tracked by the issuing thread's
// bulk async-group. Coordinates are never negative (out-of-range parts of the box are
// clipped by the hardware), and the innermost one is a multiple of 16 bytes.
__device__ __forceinline__ void tma_store_5d(const CUtensorMap* map, const void* src, int32_t c0,
                                             int32_t c1, int32_t c2, int32_t c3, int32_t c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5, %6}], [%1];" ::
          "l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until at most N of this thread's bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until at most N of this thread's bulk groups are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Barrier over a subset of the CTA's warps (ids 1..15; id 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 -------------------------------------------------------------------------

// Allocates `columns` TMEM columns (power of two >= 32); the base address is written to
// shared memory at `result`. Executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* result, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(result)),
               "r"(columns)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base),
               "r"(columns)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T for kind::f16 (fp16/bf16 operands, fp32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same for kind::tf32 (fp32 storage, tf32 multiply, fp32 accumulate).
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once all previously issued tcgen05 MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Warp-wide forms of the MMA and commit: every lane of a converged warp executes them
// and elect.sync picks the single issuing lane inside the instruction sequence, so the
// warp never branches around the MMA. Issue loops built from these run at the operand
// feed rate; the same MMAs inside a divergent `if (lane is leader) { loop }` issue at
// roughly half that rate.
__device__ __forceinline__ void mma_f16_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|q, 0xffffffff;\n\t"
      "@q tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_tf32_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|q, 0xffffffff;\n\t"
      "@q tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "elect.sync _|q, 0xffffffff;\n\t"
      "@q tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Makes a value provably warp-uniform (lane 0's copy) for the compiler.
__device__ __forceinline__ uint32_t warp_uniform(uint32_t v) {
  return __shfl_sync(0xffffffffu, v, 0);
}

// Loads 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_load16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_load_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Stores zero into 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_zero16(uint32_t taddr) {
  const uint32_t z = 0;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32"
      " [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
      "r"(z)
      : "memory");
}

__device__ __forceinline__ void tmem_store_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 "version 1" format).
//   start: byte address in shared memory (16-byte aligned)
//   lbo/sbo: leading / stride byte offsets (multiples of 16)
//   layout: 0 = interleave (no swizzle), 2 = 128B, 4 = 64B, 6 = 32B swizzle
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo,
                                                   uint32_t layout) {
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((start >> 4) & 0x3FFFu);
  desc |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  desc |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  desc |= static_cast<uint64_t>(1u) << 46;  // descriptor version for tcgen05
  desc |= static_cast<uint64_t>(layout & 7u) << 61;
  return desc;
}

}  // namespace dev
}  // namespace cnd
