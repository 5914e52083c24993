// Thin inline-PTX wrappers for the sm_100a features the kernels use:
// mbarriers, cp.async (16 B, zero-fill), TMA tiled loads, and the tcgen05
// family (TMEM alloc/dealloc, UMMA issue, commit, TMEM loads).
//
// Every wait here is bounded.  A wait that runs out of iterations records an
// error code in `g_lotus_device_error` and returns false; callers propagate
// that through a shared abort flag so the CTA drains its own copies, frees its
// TMEM and exits instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace lotus_dev {

// Error word written by a kernel whose bounded wait expired (0 = none).
// Read and cleared on the host through lotus_device_error().  Each
// translation unit that includes this header has its own copy (the library
// is built without relocatable device code); the host reads all of them.
static __device__ int g_lotus_device_error = 0;

enum : int {
  kErrNone = 0,
  kErrWaitFull = 1,    // consumer gave up waiting for a filled stage
  kErrWaitEmpty = 2,   // producer gave up waiting for a free stage
  kErrWaitAccum = 3,   // epilogue gave up waiting for the accumulator
};

// Every try_wait carries a suspend-time hint: the waiting thread is suspended
// until the phase completes or the hint runs out, instead of polling.  Without
// the hint a try_wait returns after a short hardware-defined interval, and
// the polling threads (MMA issuers, producers, epilogue warps waiting on an
// accumulator) take issue slots from the warps that share their scheduler.
// kMaxWaitIters rounds bound a lost arrival to a few seconds at most.  The
// kernels take their limit as a launch parameter (this value by default), so
// that a test can shorten it and make a withheld arrival expire quickly.
constexpr uint32_t kWaitSuspendNs = 1000;
constexpr uint32_t kMaxWaitIters = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(kWaitSuspendNs)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int err_code,
                                          uint32_t limit = kMaxWaitIters) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  atomicExch(&g_lotus_device_error, err_code);
  return false;
}

// Relaxed-semantics variant for the thread that issues tcgen05.mma.  An
// acquiring try_wait (or any shared-memory load) issued behind queued MMAs
// waits for them to drain, which serialises the tensor pipe stage by stage;
// the relaxed form does not.  Callers follow it with
// tcgen05.fence::after_thread_sync, which orders the MMAs they issue next
// after the observed phase (the TMA bytes counted by that phase are in
// shared memory once it completes).
__device__ __forceinline__ bool mbar_try_wait_relaxed(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.relaxed.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(kWaitSuspendNs)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_relaxed(uint64_t* bar, uint32_t parity, int err_code,
                                                  uint32_t limit = kMaxWaitIters) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait_relaxed(bar, parity)) return true;
  }
  atomicExch(&g_lotus_device_error, err_code);
  return false;
}

// One lane of a converged warp (the lowest) returns true.  Issuing tcgen05
// work from warp-uniform code through elect.sync keeps the descriptors and
// loop state uniform across the warp.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Named-barrier AND-reduction over `count` threads (whole warps, converged):
// every participant blocks until all have arrived and gets the AND of their
// `v`.  A named barrier is not a shared-memory operation, so a thread with
// tcgen05.mma instructions in flight passes it without waiting for them
// (an mbarrier wait from that thread is held behind them).
__device__ __forceinline__ bool bar_red_and(uint32_t id, uint32_t count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------- cp.async
// 16-byte global->shared copy; `src_bytes` = 0 writes 16 zero bytes.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor cores / TMA) before it signals a barrier.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled load (no multicast): box lands at `dst`, completion is counted in
// bytes on `bar`.  x is the innermost coordinate and must be a multiple of
// 16 bytes / element size; callers only pass multiples of 64 fp16 elements.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 4-D tiled load (no multicast), coordinates innermost first.  The innermost
// coordinate obeys the same 16-byte rule as tma_load_2d; the others may be
// negative or past the end (those box elements read as zero).
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// 4-D im2col load (no multicast) of `pixels x channels` rows of an NHWC
// tensor: coordinates (c, w, h, n) of the first output pixel's window corner
// inside the map's bounding box, plus the filter tap offsets (s, r).
__device__ __forceinline__ void tma_load_im2col_4d(void* dst, const void* tmap, uint64_t* bar, int c, int w, int h,
                                                   int n, uint16_t off_w, uint16_t off_h) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c), "r"(w), "r"(h), "r"(n), "h"(off_w),
      "h"(off_h)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 op this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Instruction descriptor, kind::f16: A=B=F16, D=F32, both operands K-major,
// M=128, N=n.  Bit positions follow the PTX ISA tcgen05 instruction
// descriptor table (c_format bits 4-5, a/b format 7-9/10-12, major bits
// 15/16, N>>3 at 17-22, M>>4 at 24-28).
__host__ __device__ constexpr uint32_t make_idesc_f16_m128(uint32_t n) {
  return (1u << 4)            // D format F32
         | (0u << 7)          // A format F16
         | (0u << 10)         // B format F16
         | (0u << 15)         // A K-major
         | (0u << 16)         // B K-major
         | ((n >> 3) << 17)   // N
         | ((128u >> 4) << 24);  // M
}

// Shared-memory matrix descriptor for a K-major tile stored as 128-byte rows
// with the 128B swizzle (8-row / 1024-byte atoms, tile base 1024-aligned).
// SBO = 1024 bytes between 8-row groups; LBO is unused for this layout.
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;            // LBO (ignored)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // SBO
  d |= static_cast<uint64_t>(1u) << 46;            // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

// 32 lanes x 32 columns of fp32 from TMEM into 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 columns of fp32 from TMEM into 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 lanes x 16 columns of fp32 zeros into TMEM (one lane per thread).
__device__ __forceinline__ void tmem_st_zero_32x32b_x16(uint32_t taddr) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(0u)
      : "memory");
}
// 32 lanes x 32 columns of fp32 zeros into TMEM (one lane per thread).
__device__ __forceinline__ void tmem_st_zero_32x32b_x32(uint32_t taddr) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
          taddr),
      "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Epilogue activation, same enum values as the reference's ActivationFunction.
__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == 1) return fmaxf(v, 0.0f);
  if (act == 2) return 1.0f / (1.0f + expf(-v));
  return v;
}

}  // namespace lotus_dev
