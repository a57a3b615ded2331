// sm100.cuh — hand-written PTX building blocks for the sm_100a GEMM kernels.
//
// Covers the four hardware units the kernels drive directly:
//   * mbarrier     (arrive / expect_tx / bounded try_wait)
//   * TMA          (cp.async.bulk.tensor 2-D tile loads and stores)
//   * tcgen05      (TMEM alloc/dealloc, UMMA issue, commit, TMEM loads, fences)
//   * UMMA shared-memory and instruction descriptors.
//
// The reference reaches the same instructions through CuTe atoms
// (arc/include/ptx/tcgen05.cuh:144-207, arc/include/utils.cuh:8-24,
// arc/include/mm.cuh:108-157). Here every instruction is written out so that the
// kernel files show exactly what is issued, and no TMA load anywhere uses cluster
// multicast (each CTA fetches its own tiles).
//
// Every wait is bounded: a wait that has not completed after kWaitTimeoutNs of
// %globaltimer sets a shared abort flag plus a bit in the device status word and
// returns false, so a protocol bug surfaces as an error code on the host instead
// of a hung GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace arcb {

// ---------------------------------------------------------------------------------
// Device status word (read back by arc_device_status()).
// ---------------------------------------------------------------------------------
enum : uint32_t {
  kStatusTimeoutProducer = 1u << 0,
  kStatusTimeoutMma = 1u << 1,
  kStatusTimeoutUnpack = 1u << 2,
  kStatusTimeoutEpilogue = 1u << 3,
  kStatusTimeoutDrain = 1u << 4,
  kStatusTimeoutScales = 1u << 5,
  kStatusTimeoutPeer = 1u << 6,
};

// One word per loaded module; every kernel in this translation unit ORs into it.
__device__ uint32_t g_arc_status;

// 2 s: far above any legitimate pipeline stall of these kernels (micro- to
// milliseconds), far below anything that would look like a hung GPU.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

// ---------------------------------------------------------------------------------
// Probe build (-DARC_PROBE): per-CTA %clock64 stamps (SM cycles; compare only
// within one CTA) at pipeline milestones,
// written to a device buffer attached with arc_probe_attach(). The reference's
// equivalent prints %clock64 stamps from the kernel (arc/include/common.cuh:30-39,
// arc/include/mm.cuh:201-211, selected by the ARC_PROBE environment variable).
// ---------------------------------------------------------------------------------
constexpr uint32_t kProbeSlots = 64;  // stamps per CTA
__device__ unsigned long long* g_arc_probe;

// A stamp is a clock read, one load of the buffer pointer (an L1 hit after the
// first) and a store, so it barely perturbs the pipeline it measures.
__device__ __forceinline__ void probe_mark(uint32_t slot) {
#if defined(ARC_PROBE)
  unsigned long long t;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
  unsigned long long* buf = g_arc_probe;
  if (buf != nullptr && slot < kProbeSlots) buf[blockIdx.x * kProbeSlots + slot] = t;
#else
  (void)slot;
#endif
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Bytes to skip from the dynamic shared-memory base to the next 1024-byte boundary
// (the 128-byte swizzle atoms need it). Used as `smem_raw + pad` so the compiler
// still sees a shared-memory pointer and emits shared (not generic) loads/stores.
__device__ __forceinline__ uint32_t smem_align_pad(const void* base) {
  return (1024u - (smem_u32(base) & 1023u)) & 1023u;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t warp_idx_sync() {
  return __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, %1;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// ---------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
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

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Same test, but the thread may sleep up to `hint_ns` waiting for the phase (it is
// woken when the phase completes), so waiting warps leave the issue slots to the
// warps doing work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with parity `parity` to complete.
// Returns false when the wait was abandoned: either this thread timed out (it then
// raises *abort and ORs `err_bit` into the device status word) or another role of
// the CTA already raised *abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile uint32_t* abort, uint32_t err_bit) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t start = globaltimer_ns();
#pragma unroll 1
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(addr, parity, 20000u)) return true;
    if ((it & 15u) == 0u) {
      if (*abort) return false;
      if (globaltimer_ns() - start > kWaitTimeoutNs) {
        *abort = 1u;
        atomicOr(&g_arc_status, err_bit);
        return false;
      }
    }
  }
}

// The same bounded wait, polling with the non-blocking test instead of letting the
// thread be suspended: a suspended thread resumes some hundreds of nanoseconds after the
// phase completes, a polling one within one test (~200 cycles). For the few waits on a
// short critical path; polling takes issue slots from the other warps of the SM.
__device__ __forceinline__ bool mbar_wait_poll(uint64_t* bar, uint32_t parity,
                                               volatile uint32_t* abort, uint32_t err_bit) {
  const uint32_t addr = smem_u32(bar);
  uint64_t start = 0;
#pragma unroll 1
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 63u) == 0u) {
      if (it == 0) {
        start = globaltimer_ns();
      } else {
        if (*abort) return false;
        if (globaltimer_ns() - start > kWaitTimeoutNs) {
          *abort = 1u;
          atomicOr(&g_arc_status, err_bit);
          return false;
        }
      }
    }
  }
}

// Non-blocking test of a phase (acquire when it reports completion). On B200 even a
// test of an already-completed phase takes ~180 cycles to answer, so code that
// checks several barriers issues all the tests first and lets their latencies
// overlap, then blocks (mbar_wait) only on the ones that were not complete.
__device__ __forceinline__ uint32_t mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok;
}

// Warp-wide bounded wait on up to two barriers. Every lane tests and waits for
// itself (each lane's wait is its own acquire), skipping a barrier whose completion
// it already saw in an earlier mbar_test (`pre1`, `pre2`; pass 1 for "no wait"),
// and the warp leaves together through a vote. On B200 this is measurably faster
// than one lane waiting and broadcasting the outcome. Every lane of the warp must
// call it, never from inside a branch that splits the warp.
__device__ __forceinline__ bool mbar_wait_all2(uint64_t* bar1, uint32_t parity1, uint32_t pre1,
                                               uint64_t* bar2, uint32_t parity2, uint32_t pre2,
                                               volatile uint32_t* abort, uint32_t err_bit) {
  const bool ok = (pre1 != 0u || mbar_wait(bar1, parity1, abort, err_bit)) &&
                  (pre2 != 0u || mbar_wait(bar2, parity2, abort, err_bit));
  return __all_sync(0xffffffffu, ok);
}

// Per-warpgroup register budget moves (all four warps of a warpgroup execute the
// same one). An increase waits until other warpgroups have released enough of the
// registers the CTA was launched with, so the shares must add up to at most
// threads x launch registers.
template <uint32_t N>
__device__ __forceinline__ void regs_release() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_claim() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Bounded wait that ignores the abort flag: used on the teardown path to let
// copies already in flight land before the CTA exits.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t start = globaltimer_ns();
#pragma unroll 1
  while (!mbar_try_wait(addr, parity)) {
    if (globaltimer_ns() - start > kWaitTimeoutNs) {
      atomicOr(&g_arc_status, kStatusTimeoutDrain);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------------
// Fences and named barriers
// ---------------------------------------------------------------------------------
// Make generic-proxy shared-memory writes visible to the async proxy (TMA store,
// tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------------
// TMA (tensor maps are passed as __grid_constant__ kernel parameters)
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// L2 cache-policy hints (createpolicy encodings used by cp.async.bulk .L2::cache_hint).
constexpr uint64_t kCacheEvictNormal = 0x1000000000000000ull;
constexpr uint64_t kCacheEvictFirst = 0x12F0000000000000ull;
constexpr uint64_t kCacheEvictLast = 0x14F0000000000000ull;

// 2-D tiled load into this CTA's shared memory; completion is signalled on `bar`
// as transaction bytes. x is the innermost (contiguous) coordinate in elements.
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int32_t x, int32_t y, uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y),
      "l"(cache_hint)
      : "memory");
}

// 3-D tiled load (coordinates innermost first), same completion mechanism.
__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int32_t x, int32_t y, int32_t z, uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z),
      "l"(cache_hint)
      : "memory");
}

// 2-D tiled store from shared memory; elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x,
                                             int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed store groups still read shared memory.
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N committed store groups are still writing global memory.
template <int N>
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------------
// tcgen05: TMEM management
// ---------------------------------------------------------------------------------
// Whole warp; writes the TMEM base address into *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
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

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------------
// tcgen05: UMMA issue (one thread) and completion tracking
// ---------------------------------------------------------------------------------
// D[tmem] (+)= A[smem desc] x B[smem desc]^T, bf16 inputs, fp32 accumulation.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc]^T, s8 inputs, s32 accumulation.
__device__ __forceinline__ void umma_s8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] x B[smem desc]^T, s8 inputs, s32 accumulation. A (M=128) sits in
// TMEM with row m in lane m and K along the columns, four int8 per 32-bit column in
// ascending K (byte 0 = lowest k): a K=32 step reads 8 consecutive columns from a_tmem.
__device__ __forceinline__ void umma_s8_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` (once) when every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------------------------
// tcgen05: TMEM -> registers. Warp w of a warpgroup may only touch lanes
// 32*(w%4) .. 32*(w%4)+31; thread t receives lane 32*(w%4)+t.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Registers -> TMEM: the same 32-bit value into 8 consecutive columns of this
// thread's lane (same lane-quarter rule as the loads).
__device__ __forceinline__ void tmem_st_32x32b_x8_fill(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};"
      :
      : "r"(taddr), "r"(v)
      : "memory");
}

// Registers -> TMEM: v[j] into column taddr + j of this thread's lane.
__device__ __forceinline__ void tmem_st_32x32b_x4(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3])
               : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------------
// Shared-memory matrix descriptor for a K-major operand stored in the 128-byte
// swizzle layout that a TMA SWIZZLE_128B load produces: rows of 128 bytes, 8-row
// (1024-byte) swizzle atoms stacked along M/N, atom base 1024-byte aligned.
//   bits  0-13 start address >> 4
//   bits 16-29 leading-dimension byte offset >> 4 (unused for swizzled K-major; 1)
//   bits 32-45 stride-dimension byte offset >> 4  (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 61-63 layout: 2 = SWIZZLE_128B
// A K step inside the 128-byte row is taken by adding the byte offset to the start
// address (the hardware applies the swizzle to the final address bits).
__device__ __forceinline__ uint64_t make_sw128_kmajor_desc(const void* smem_tile) {
  const uint32_t addr = smem_u32(smem_tile);
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  desc |= static_cast<uint64_t>(1u) << 16;
  desc |= static_cast<uint64_t>(1024u >> 4) << 32;
  desc |= static_cast<uint64_t>(1u) << 46;
  desc |= static_cast<uint64_t>(2u) << 61;
  return desc;
}

// Advance a descriptor's start address by `bytes` (multiple of 16).
__device__ __forceinline__ uint64_t desc_advance(uint64_t desc, uint32_t bytes) {
  return desc + static_cast<uint64_t>(bytes >> 4);
}

// Instruction descriptor for dense tcgen05.mma (kind::f16 / kind::i8), both operands
// K-major:
//   bits 4-5   D format  (1 = f32, 2 = s32)
//   bits 7-9   A format  (kind::f16: 1 = bf16; kind::i8: 1 = signed)
//   bits 10-12 B format  (same encoding)
//   bit  15/16 A/B major (0 = K-major)
//   bits 17-22 N >> 3
//   bits 24-28 M >> 4
__host__ __device__ constexpr uint32_t make_idesc(uint32_t d_fmt, uint32_t a_fmt, uint32_t b_fmt,
                                                  uint32_t m, uint32_t n) {
  return (d_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16_f32(uint32_t m, uint32_t n) {
  return make_idesc(1, 1, 1, m, n);
}
__host__ __device__ constexpr uint32_t idesc_s8_s32(uint32_t m, uint32_t n) {
  return make_idesc(2, 1, 1, m, n);
}

// ---------------------------------------------------------------------------------
// Thread-block clusters
// ---------------------------------------------------------------------------------
// All threads of all CTAs of the cluster; release/acquire orders shared-memory
// writes before the barrier with distributed-shared-memory reads after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// The two halves of cluster_sync_all, for a thread that can announce early that it is
// done and wait later (every thread of the cluster arrives once, then waits once).
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrival that orders no memory: for a barrier that only marks an event whose data is
// synchronised otherwise (e.g. by mbarrier transaction counts). A release arrival at
// cluster scope costs the arriving warp on the order of a thousand cycles.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

// Address of the same shared-memory object in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Bulk copy of `bytes` (a multiple of 16) from this CTA's shared memory into the
// shared memory of a CTA of the cluster. `dst` and `remote_bar` are shared::cluster
// addresses (map_to_rank); the bytes complete as transaction count on remote_bar.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, const void* src, uint32_t bytes,
                                                  uint32_t remote_bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst),
      "r"(smem_u32(src)), "r"(bytes), "r"(remote_bar)
      : "memory");
}

// ---------------------------------------------------------------------------------
// CTA pairs (cta_group::2): two CTAs of a 2-CTA cluster share one UMMA. The MMA of
// M=256 takes A rows 0-127 from rank 0's shared memory and 128-255 from rank 1's (same
// offset), B's N/2 halves likewise, and writes D rows 0-127 / 128-255 into the TMEM of
// rank 0 / rank 1. Rank 0 issues it; its completion can be signalled to both CTAs.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Arrive (release at cluster scope) on an mbarrier given by its shared::cluster address
// (map_to_rank), possibly in the peer CTA.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is signalled on an
// mbarrier of either CTA of the pair (`bar` is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar, void* dst,
                                                 int32_t x, int32_t y, uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(cache_hint)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(const CUtensorMap* map, uint32_t bar, void* dst, int32_t x,
                                                 int32_t y, int32_t z, uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "l"(cache_hint)
      : "memory");
}

// TMEM allocation shared by the pair: one warp of each CTA (same warp index) executes
// it with the same destination offset; both CTAs receive the same column base.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Pair UMMA, bf16 inputs, fp32 accumulation (idesc with M = 256).
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at `bar`'s offset in every CTA of `cta_mask` when all
// pair tcgen05 operations issued so far by this thread have completed. (This is the
// completion signal of tcgen05, not a memory load.)
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Programmatic dependent launch: let the next grid in the stream start its
// prologue, and wait for the previous grid's completion (and memory) before
// touching global memory.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------------------------
// Numeric helpers
// ---------------------------------------------------------------------------------
// Two fp32 -> packed bf16x2 (round to nearest even); lo goes to the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Packed fp32 pair arithmetic (sm_100): one instruction for two lanes of work.
__device__ __forceinline__ uint64_t f32x2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f32x2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

// acc = x * s + acc, elementwise on pairs, round to nearest even.
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t x, uint64_t s, uint64_t acc) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(s), "l"(acc));
  return r;
}

__device__ __forceinline__ uint64_t f32x2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

}  // namespace arcb
