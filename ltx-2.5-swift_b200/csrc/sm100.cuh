// sm100.cuh -- thin inline-PTX layer for sm_100a: mbarriers with bounded waits,
// TMA tensor loads, tcgen05 (TMEM alloc, UMMA issue/commit, TMEM load/store)
// and the UMMA shared-memory / instruction descriptors.
//
// Descriptor bit layouts follow the PTX ISA "tcgen05 matrix descriptor" and
// "instruction descriptor" tables (cross-checked against CUTLASS 4.5
// cute/arch/mma_sm100_desc.hpp: SmemDescriptor, InstrDescriptor).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ltxattn_internal.h"

namespace ltx {

// ---------------------------------------------------------------------------
// error reporting from device code.  Every wait is bounded; a wait that runs
// out records (site, block) in the module's error word and the kernel unwinds.
// The host reads the word with ltxattn_device_status().

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wall-clock bound on any single wait.  Generous: a healthy wait is
// microseconds; this only ends waits that can never complete.
#ifndef LTX_WAIT_LIMIT_NS
#define LTX_WAIT_LIMIT_NS 2000000000ull
#endif

// Bounded wait on an mbarrier phase.  `abort_flag` (shared) lets one thread's
// timeout release every other waiter of the CTA quickly.  Returns false when
// the wait gave up; the caller must then stop issuing work.
// `limit_ns` is LTX_WAIT_LIMIT_NS everywhere but in the failure-detection
// self-test, which gives a short one.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag, int* err_word, int site,
                                          uint64_t limit_ns = LTX_WAIT_LIMIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        *abort_flag = 1;
        if (err_word) atomicCAS(err_word, 0, (site << 8) | kErrTimeout);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// fences

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Tiled bulk store shared -> global (same box and swizzle as the map's
// loads).  Rows past the tensor's extent are not written.  The source may be
// reused once bulk_wait_read() returns.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Barrier over `count` threads (a multiple of 32) with id `id` (1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Programmatic dependent launch.  A grid launched with the programmatic
// stream-serialization attribute may start while the grid before it in the
// stream is finishing; grid_dep_wait() then holds the calling thread until that
// grid has completed and its memory is visible (a no-op without the
// attribute).  grid_dep_launch_dependents() lets the next grid start launching
// once every CTA of this grid has issued it or exited.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The same barrier, returning whether `pred` held in every participating thread.
__device__ __forceinline__ bool named_barrier_and(uint32_t id, uint32_t count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------
// TMEM allocation (one full warp executes these)

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors

// Shared-memory matrix descriptor, SWIZZLE_128B (layout type 2), version 1.
//   [0,14)  start address >> 4
//   [16,30) leading-dimension byte offset >> 4
//   [32,46) stride-dimension byte offset >> 4
//   [46,48) version = 1 (sm100)
//   [49,52) base offset = 0 (atoms are 1024-byte aligned)
//   [61,64) layout type
// K-major SW128: rows of 128 B, 8-row atoms; SBO = atom stride, LBO unused (1).
// MN-major SW128: 64-element MN chunks at LBO, 8-row K groups at SBO.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 accumulate.
//   [4,6) D fmt = 1 (F32); [7,10) A fmt = 1 (BF16); [10,13) B fmt = 1 (BF16)
//   [15] A major (0 K, 1 MN); [16] B major; [17,23) N>>3; [24,29) M>>4
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn_major,
                                                      int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// D(tmem) (+)= A(smem desc) * B(smem desc).  Issued by one thread.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc).  A is M lanes x K/2 packed columns.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Split descriptor form for hot issue loops.  Every shared address in this
// library is below 256 KB, so the 14-bit start-address field never carries:
// desc(addr + off) == desc(addr) + (off >> 4) in the low word.  Issue loops
// keep {lo, hi} of a base descriptor and add compile-time offsets to lo.
struct SDesc {
  uint32_t lo, hi;
};

__device__ __forceinline__ SDesc sdesc_split(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  const uint64_t d = sdesc_sw128(saddr, lbo_bytes, sbo_bytes);
  return SDesc{static_cast<uint32_t>(d), static_cast<uint32_t>(d >> 32)};
}

// D(tmem) (+)= A(smem) * B(smem) with descriptors given as {lo, hi} words.
__device__ __forceinline__ void umma_ss2(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                         uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "mov.b64 da, {%1, %2};\n\tmov.b64 db, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, {%7, %8, %9, %10}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem) with B's descriptor given as {lo, hi}.
__device__ __forceinline__ void umma_ts2(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, {%6, %7, %8, %9}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Warp-level issue: every lane of the warp executes these with the same
// (warp-uniform) operands and one elected lane issues the instruction.  Keeping
// the descriptors warp-uniform lets them live in the uniform datapath, so an
// MMA issues without per-instruction register moves; measured, this keeps the
// tensor pipe near peak while a dense FP32 warp shares the issuing SMSP (the
// single-lane form drops to ~29% of peak there).
__device__ __forceinline__ void umma_ss_warp(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                             uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 da, db;\n\t"
      "mov.b64 da, {%1, %2};\n\tmov.b64 db, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, {%7, %8, %9, %10}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 db;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "setp.ne.b32 p, %5, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, {%6, %7, %8, %9}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
      : "memory");
}

// Make `bar` track completion of every tcgen05 op this thread issued so far.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// TMEM <-> registers, 32x32b shape: warp w (w % 4 = quadrant) touches lanes
// [32*quadrant, 32*quadrant+32); thread t gets lane 32*quadrant+t and N
// consecutive 32-bit columns.

#define LTX_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), \
                  "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define LTX_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), \
                  "r"(r[i + 4]), "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : LTX_R8(0), LTX_R8(8), LTX_R8(16), LTX_R8(24)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : LTX_R8(0), LTX_R8(8)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      LTX_W8(0), LTX_W8(8), LTX_W8(16), LTX_W8(24)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      LTX_W8(0), LTX_W8(8)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

#undef LTX_R8
#undef LTX_W8

// ---------------------------------------------------------------------------
// CTA-level helpers shared by the attention kernels

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Whole-warp wait: every lane polls the barrier and the lanes then agree, so
// a timeout seen by one lane is seen by all.  (A lane-0 poll with the other 31
// lanes parked at a shuffle was measured to resume the warp several hundred
// cycles after the phase completed.)  The lanes read the same barrier state
// and the same timer in each converged poll, so they leave the loop together.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int site, uint64_t limit_ns = LTX_WAIT_LIMIT_NS) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err, site, limit_ns);
  return __all_sync(0xffffffffu, ok);
}

// Drain wait used only on the way out: bounded, ignores the abort flag.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > LTX_WAIT_LIMIT_NS) break;
  }
}

// 1D bulk copy global -> shared, completion counted on `bar` (16-byte aligned,
// size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Warpgroup register re-split (all four warps of a warpgroup execute it).
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}

// ---------------------------------------------------------------------------
// paired fp32 arithmetic (sm_100 f32x2) and the 3-input max

__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x on the FMA pipe, for two values at once; x <= 8 in this library.
// Round-to-nearest split x = n + f with f in [-1/2, 1/2] (adding 1.5*2^23
// leaves n in the low mantissa bits), a degree-3 polynomial for 2^f, and n
// added to the exponent field.  The coefficients are this library's own
// relative-error least-squares fit of 2^f on [-1/2, 1/2] (iteratively
// reweighted towards minimax): max relative error 7.5e-5, far below the
// bf16 rounding P receives.  Arguments are clamped at -126: below that the
// result is at most 2^-126 (callers zero masked columns themselves).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float2 xc = make_float2(fmaxf(x.x, -126.f), fmaxf(x.y, -126.f));
  const float2 t = add2(xc, make_float2(kMagic, kMagic));
  const float2 n = add2(t, make_float2(-kMagic, -kMagic));
  const float2 f = fma2(n, make_float2(-1.f, -1.f), xc);  // exact: x - n
  float2 q = fma2(f, make_float2(0.0551716573536396f, 0.0551716573536396f),
                  make_float2(0.2426111400127411f, 0.2426111400127411f));
  q = fma2(q, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  q = fma2(q, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
  // bits(t) = bits(kMagic) + n, so bits(q) + (n << 23) = bits(q) + (bits(t) << 23) - (bits(kMagic) << 23)
  constexpr uint32_t kBias = 0x4B400000u << 23;
  float2 r;
  r.x = __uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23) - kBias);
  r.y = __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23) - kBias);
  return r;
}

// ---------------------------------------------------------------------------
// Split RoPE on 8 rotary pairs held as bf16x8 vectors (x1 = first half, x2 =
// second half of the rows, c / s the table entries):
//     o1 = x1*c - x2*s ,  o2 = x2*c + x1*s
// with every product and every sum rounded to bf16 (round to nearest even),
// the arithmetic of a bf16 tensor times a bf16 table (DiTAttention.swift:226-234).
// The native bf16x2 instructions round the exact result once.  That equals
// "evaluate in fp32, round to bf16": a product of two bf16 values is exact in
// fp32, and the fp32 sum of two bf16 values is either exact or (operands 2^16
// apart or more) too far from any bf16 rounding midpoint for the second
// rounding to differ.  tests/test_rope_gpu.py checks it bit for bit against
// the oracle.
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ void rope_bf16x8(const uint4& x1, const uint4& x2, const uint4& c, const uint4& s,
                                           uint4& o1, uint4& o2) {
  o1.x = bsub2(bmul2(x1.x, c.x), bmul2(x2.x, s.x));
  o1.y = bsub2(bmul2(x1.y, c.y), bmul2(x2.y, s.y));
  o1.z = bsub2(bmul2(x1.z, c.z), bmul2(x2.z, s.z));
  o1.w = bsub2(bmul2(x1.w, c.w), bmul2(x2.w, s.w));
  o2.x = badd2(bmul2(x2.x, c.x), bmul2(x1.x, s.x));
  o2.y = badd2(bmul2(x2.y, c.y), bmul2(x1.y, s.y));
  o2.z = badd2(bmul2(x2.z, c.z), bmul2(x1.z, s.z));
  o2.w = badd2(bmul2(x2.w, c.w), bmul2(x1.w, s.w));
}

// ---------------------------------------------------------------------------
// small numeric helpers

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The per-head output gate of DiTAttention.swift:395-399: 2 * sigmoid(logit),
// the sigmoid evaluated in fp32 as 1 / (1 + e^-x) (CUDA's expf, IEEE division)
// and, for bf16 activations, cast back to bf16 before the exact doubling
// (DiTAttention.swift:240-242).
__device__ __forceinline__ float gate_f32(float logit) { return 2.0f * (1.0f / (1.0f + expf(-logit))); }
__device__ __forceinline__ float gate_bf16(float logit) {
  return 2.0f * __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-logit))));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace ltx
