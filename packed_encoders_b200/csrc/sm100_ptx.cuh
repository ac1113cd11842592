// Thin inline-PTX wrappers for the Blackwell (sm_100a) features the attention kernels use:
// mbarriers, TMA tiled loads, tcgen05 MMA / TMEM load-store / alloc, and their fences.
//
// Descriptor bit layouts follow the PTX ISA for tcgen05 (shared-memory matrix descriptor and
// the kind::f16 instruction descriptor); the same fields are spelled out in CUTLASS's
// cute/arch/mma_sm100_desc.hpp (SmemDescriptor, InstrDescriptor).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace pe_b200 {

// ---------------------------------------------------------------------------------------------
// Error bits written to the workspace error word (never a trap, never an early exit).
enum : int {
  kErrWaitTimeout = 1,      // an mbarrier wait ran past its bound
  kErrScheduleOverflow = 2, // more work items than the workspace holds
  kErrBadSegments = 4,      // cu_seqlens not monotonic / out of range
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0); }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\telect.sync _|P, %1;\n\tselp.b32 %0, 1, 0, P;\n\t}\n"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// ---------------------------------------------------------------------------------------------
// mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\tmbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Non-blocking probe (about 21 clk on a completed phase against about 52 for a try_wait with a
// suspend hint, measured on B200).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\tmbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: spins on try_wait (each try suspends up to ~1 ms in hardware) and gives up
// after `kWaitBudgetCycles` SM clocks, recording kErrWaitTimeout. Callers continue as if the
// phase completed, so a lost arrival yields wrong numbers plus an error flag, never a hang.
constexpr long long kWaitBudgetCycles = 4000000000LL;  // ~2 s at 1.9 GHz

// After a wait of this launch gave up (the error word is set), the roles went on without their
// barriers, so copies and MMAs of this CTA may still be in flight: give them ~200 us to land before
// the CTA frees its TMEM and exits. Called by every thread before the final barrier; free when no
// wait gave up.
__device__ __forceinline__ void drain_after_timeout(const int* err) {
  if (err && *reinterpret_cast<const volatile int*>(err) != 0)
    for (int k = 0; k < 200; ++k) __nanosleep(1000);
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_test_wait(bar, parity)) return true;
  if (mbar_try_wait(bar, parity)) return true;
  // Once any wait of this launch has given up, later waits fail fast instead of each
  // spending the full budget (a broken launch ends in milliseconds, not minutes).
  if (err && *reinterpret_cast<volatile int*>(err) != 0) return false;
  long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitBudgetCycles) {
      if (err) atomicOr(err, kErrWaitTimeout);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------------------------
// TMA (tiled, 3-D) global -> shared, completion on an mbarrier via complete_tx.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Warp-uniform forms: the whole warp executes the call and one elected lane issues the
// instruction (elect.sync inside the asm). Keeping the surrounding loop warp-uniform lets the
// compiler hold descriptors and addresses in uniform registers; a single-lane branch around
// tcgen05.mma measured about 2.4x slower issue on sm_100a.
__device__ __forceinline__ void tma_load_3d_w(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                              int c2) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];\n\t}\n" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 4-D tiled load (one elected lane): all 64-column panels of a wide row block in one copy.
__device__ __forceinline__ void tma_load_4d_w(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                              int c2, int c3) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];\n\t}\n" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_hint_w(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                                   int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%3, %4, %5, %6}], [%2], %7;\n\t}\n" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}

// As tma_load_3d_w with an L2 cache policy (createpolicy) for the copied lines.
__device__ __forceinline__ void tma_load_3d_hint_w(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                                   int c1, int c2, uint64_t policy) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%3, %4, %5}], [%2], %6;\n\t}\n" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

// L2 eviction policies for cache-hinted copies.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Raise the barrier's expected transaction bytes without arriving (one elected lane).
__device__ __forceinline__ void mbar_expect_tx_w(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;\n\t}\n" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_w(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b64 st;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}\n" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

// TMA tiled store shared -> global (bulk-group completion), and its group bookkeeping.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d_hint(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2,
                                                  uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4}], [%1], %5;" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until this thread's committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until this thread's committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Make this thread's generic-proxy shared-memory writes visible to the async proxy (TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Orders this thread's async-proxy global accesses (completed bulk stores) with later generic ones.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation (whole warp), fences, MMA, commit, TMEM load/store.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, cta_group::1, kind::f16 (bf16 in, fp32 accumulate).
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Warp-uniform forms of the MMA issue and commit (see tma_load_3d_w).
__device__ __forceinline__ void mma_ss_w(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Four MMAs (the k-steps of one 64-deep slice) from one lane elected once for the group; the
// first takes `accumulate`, the other three accumulate.
__device__ __forceinline__ void mma_ss4_w(uint32_t d_tmem, const uint64_t (&a)[4], const uint64_t (&b)[4],
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e, t;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %9, 0;\n\t"
      "setp.eq.b32 t, %9, %9;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %5, %10, p;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %6, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %10, t;\n\t}\n" ::"r"(d_tmem),
      "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(accumulate),
      "r"(idesc));
}
__device__ __forceinline__ void mma_ts4_w(uint32_t d_tmem, const uint32_t (&a_tmem)[4], const uint64_t (&b)[4],
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e, t;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %9, 0;\n\t"
      "setp.eq.b32 t, %9, %9;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %5, %10, p;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %6, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %7, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %8, %10, t;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem[0]), "r"(a_tmem[1]), "r"(a_tmem[2]), "r"(a_tmem[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]),
      "r"(accumulate), "r"(idesc));
}
// Four SS MMAs (as mma_ss4_w) followed by commits to `bar0`, `bar1` and, when `third` is
// nonzero, `bar2`, all from one elected lane of one asm block.
__device__ __forceinline__ void mma_ss4_commit_w(uint32_t d_tmem, const uint64_t (&a)[4], const uint64_t (&b)[4],
                                                 uint32_t idesc, uint32_t accumulate, uint64_t* bar0,
                                                 uint64_t* bar1, uint64_t* bar2, uint32_t third) {
  asm volatile(
      "{\n\t.reg .pred p, e, t, x;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %9, 0;\n\t"
      "setp.eq.b32 t, %9, %9;\n\tsetp.ne.and.b32 x, %14, 0, e;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %5, %10, p;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %6, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %10, t;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%11];\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%12];\n\t"
      "@x tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%13];\n\t}\n" ::"r"(d_tmem),
      "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(accumulate),
      "r"(idesc), "r"(smem_u32(bar0)), "r"(smem_u32(bar1)), "r"(smem_u32(bar2)), "r"(third)
      : "memory");
}
// Four TS MMAs (as mma_ts4_w), then a commit to `first_bar` when `first` is nonzero and one to `bar`,
// from one elected lane of one asm block.
__device__ __forceinline__ void mma_ts4_commit_w(uint32_t d_tmem, const uint32_t (&a_tmem)[4],
                                                 const uint64_t (&b)[4], uint32_t idesc, uint32_t accumulate,
                                                 uint64_t* first_bar, uint32_t first, uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred p, e, t, x;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %9, 0;\n\t"
      "setp.eq.b32 t, %9, %9;\n\tsetp.ne.and.b32 x, %12, 0, e;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %5, %10, p;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %6, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %7, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %8, %10, t;\n\t"
      "@x tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%11];\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%13];\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem[0]), "r"(a_tmem[1]), "r"(a_tmem[2]), "r"(a_tmem[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]),
      "r"(accumulate), "r"(idesc), "r"(smem_u32(first_bar)), "r"(first), "r"(smem_u32(bar))
      : "memory");
}
// Four shared-memory -> TMEM copies of 128 rows x 256 bits (16 bf16 of each row) from one elected
// lane: copy j reads the matrix that descriptor d[j] describes and lands in TMEM columns
// taddr + 8j .. +7, row r in lane r (the layout of an A operand read from TMEM).
__device__ __forceinline__ void tc_cp4_w(uint32_t taddr, const uint64_t (&d)[4]) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 t1, t2, t3;\n\telect.sync _|e, 0xffffffff;\n\t"
      "add.u32 t1, %0, 8;\n\tadd.u32 t2, %0, 16;\n\tadd.u32 t3, %0, 24;\n\t"
      "@e tcgen05.cp.cta_group::1.128x256b [%0], %1;\n\t"
      "@e tcgen05.cp.cta_group::1.128x256b [t1], %2;\n\t"
      "@e tcgen05.cp.cta_group::1.128x256b [t2], %3;\n\t"
      "@e tcgen05.cp.cta_group::1.128x256b [t3], %4;\n\t}\n" ::"r"(taddr),
      "l"(d[0]), "l"(d[1]), "l"(d[2]), "l"(d[3])
      : "memory");
}
// Four SS MMAs (as mma_ss4_w), then commits to those of `bar0`, `bar1`, `bar2` whose bit is set in
// `mask` (bit 0 = bar0), from one elected lane of one asm block.
__device__ __forceinline__ void mma_ss4_commits_w(uint32_t d_tmem, const uint64_t (&a)[4], const uint64_t (&b)[4],
                                                  uint32_t idesc, uint32_t accumulate, uint64_t* bar0,
                                                  uint64_t* bar1, uint64_t* bar2, uint32_t mask) {
  asm volatile(
      "{\n\t.reg .pred p, e, t, x0, x1, x2;\n\t.reg .b32 m;\n\telect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %9, 0;\n\tsetp.eq.b32 t, %9, %9;\n\t"
      "and.b32 m, %14, 1;\n\tsetp.ne.and.b32 x0, m, 0, e;\n\t"
      "and.b32 m, %14, 2;\n\tsetp.ne.and.b32 x1, m, 0, e;\n\t"
      "and.b32 m, %14, 4;\n\tsetp.ne.and.b32 x2, m, 0, e;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %5, %10, p;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %6, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %10, t;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %10, t;\n\t"
      "@x0 tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%11];\n\t"
      "@x1 tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%12];\n\t"
      "@x2 tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%13];\n\t}\n" ::"r"(d_tmem),
      "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(accumulate),
      "r"(idesc), "r"(smem_u32(bar0)), "r"(smem_u32(bar1)), "r"(smem_u32(bar2)), "r"(mask)
      : "memory");
}
__device__ __forceinline__ void mma_commit_w(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]; A is K-major in TMEM (lane = row, 2 bf16 per column).
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrive once on `bar` when every tcgen05 operation issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (quarter*32 + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}

// ---------------------------------------------------------------------------------------------
// Shared-memory matrix descriptors (tcgen05 format, version 1), 128-byte swizzle.
//   bits  0-13  start address >> 4
//   bits 16-29  leading-dimension byte offset >> 4
//   bits 32-45  stride-dimension byte offset >> 4
//   bits 46-47  version (1 on sm_100)
//   bits 49-51  base offset (0: atoms are 1024-byte aligned)
//   bits 61-63  layout (2 = 128-byte swizzle)
// K-major (rows of 64 bf16 = 128 B, 8-row atoms of 1024 B): SBO = 1024 B between 8-row groups,
// LBO unused; a K step of 16 elements moves the start address by 32 B inside the atom.
// MN-major (the V operand, rows = keys): SBO = 1024 B between 8-key groups, LBO = distance
// between 64-element column panels; a K step of 16 keys moves the start by 16 * 128 B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulator, bf16 A and B, M x N.
//   bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16), 10-12 B format (1 = bf16),
//   bit 15 A MN-major, bit 16 B MN-major, bits 17-22 N >> 3, bits 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------------------------
// Math helpers.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 3-input max (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Packed fp32 pair arithmetic (sm_100 f32x2): one instruction for two lanes of work.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// 2^x for a pair of x <= 0 on the FMA pipe (no MUFU): round x to the nearest integer j with the
// 1.5 * 2^23 magic-number add, evaluate 2^(x - j) on [-0.5, 0.5] with a cubic, add j to the
// exponent. The cubic is a relative least-squares fit made for this kernel (max relative error
// 7.5e-5 in fp32, far below the 2^-9 of the bf16 P it feeds). x is clamped at -125 so the
// biased exponent of the result stays >= 1 (2^(x-j) >= 2^-0.5 has biased exponent >= 126);
// 2^-125 stands in for exp2(-inf) (it is 0 in every sum it enters to fp32 precision).
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 magic = make_float2(12582912.f, 12582912.f);
  const float2 t = fadd2(x, magic);
  const float2 j = fadd2(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = ffma2(j, make_float2(-1.f, -1.f), x);
  float2 p = ffma2(make_float2(0.05517115443944931f, 0.05517115443944931f), f,
                   make_float2(0.2426101416349411f, 0.2426101416349411f));
  p = ffma2(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = ffma2(p, f, make_float2(0.9999281167984009f, 0.9999281167984009f));
  const uint32_t bx = __float_as_uint(p.x) + (__float_as_uint(t.x) << 23);
  const uint32_t by = __float_as_uint(p.y) + (__float_as_uint(t.y) << 23);
  return make_float2(__uint_as_float(bx), __uint_as_float(by));
}

// Four fp32 additions into global memory with one vector reduction (sm_90+).
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

}  // namespace pe_b200
