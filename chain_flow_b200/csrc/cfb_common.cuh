// cfb_common.cuh -- device helpers shared by the sm_100a kernels of libcfb.so.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#define CFB_DEV __device__ __forceinline__

#include "../../include/cfb.h"
// Host: record the CUDA error of the last launch (if any) for cfb_last_cuda_error(); returns the
// status the C ABI reports. Defined in cfb_engine.cu.
cfb_status cfb_launch_status(const char* what);

namespace cfb {

// Device error word values (written into the workspace, read by cfb_plan_error).
enum DevErr : int { DEV_OK = 0, DEV_TIMEOUT_GRID = 1, DEV_TIMEOUT_FULL = 2, DEV_TIMEOUT_EMPTY = 3,
                    DEV_TIMEOUT_SLOT = 4, DEV_BAD_PHASE = 5, DEV_TIMEOUT_FIXUP = 6,
                    DEV_BAD_INDEX = 7 };   // a token / row id outside its table: never dereferenced

// Every device-side wait is bounded by this many nanoseconds of %globaltimer. On expiry the
// waiter records an error and returns, so a broken schedule ends the launch instead of hanging
// the GPU.
constexpr unsigned long long kWaitBudgetNs = 1000000000ull;   // 1 s

CFB_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

CFB_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------------------------
CFB_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
CFB_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
CFB_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
               :: "r"(smem_u32(bar)) : "memory");
}
CFB_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
               :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
CFB_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.b32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// non-suspending form: reports at once whether the phase has completed
CFB_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.b32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
CFB_DEV int ld_volatile_int(const int* p);

// Polls between two looks at the clock and the error word in a bounded wait. Each look costs a
// global-memory round trip, during which the waiter cannot notice that its wait is over.
constexpr unsigned kPollsPerCheck = 64;

// A wait budget below the default is a caller forcing waits to expire, to test the failure path:
// such a wait looks at the clock at every poll (polls_per_check), and a budget of n ns expires
// once n - 1 ns have passed (wait_expired), so a budget of 1 ns gives up at the first poll that
// finds the wait unfinished, whatever the resolution of %globaltimer.
CFB_DEV unsigned polls_per_check(unsigned long long budget) {
  return budget < kWaitBudgetNs ? 1u : kPollsPerCheck;
}
CFB_DEV bool wait_expired(unsigned long long t0, unsigned long long budget) {
  return globaltimer() - t0 + 1ull >= budget;
}

// Bounded wait; returns false on timeout, or soon after `err` (if given) is set, so that after
// the first failure the rest of a launch runs through without waiting. A forced short budget
// polls with the non-suspending test_wait (try_wait may suspend the thread until the phase
// completes, which would hide the expiry).
CFB_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, const int* err = nullptr,
                       unsigned long long budget = kWaitBudgetNs) {
  if (budget < kWaitBudgetNs) {
    const unsigned long long t0 = globaltimer();
    for (;;) {
      if (mbar_test_wait(bar, parity)) return true;
      if (wait_expired(t0, budget)) return false;
      if (err && ld_volatile_int(err) != 0) return false;
    }
  }
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (unsigned it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (it % kPollsPerCheck == 0) {
      if (wait_expired(t0, budget)) return false;
      if (err && ld_volatile_int(err) != 0) return false;
    }
  }
}

// The same bounded wait (default budget) on a barrier given by its shared-memory address, for
// loops that keep their barrier addresses in registers.
CFB_DEV bool mbar_try_wait_a(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.b32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
CFB_DEV bool mbar_test_wait_a(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.b32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// (a first non-suspending look: a phase already complete, the common case of a streaming ring,
// costs less this way)
CFB_DEV bool mbar_wait_a(uint32_t bar, uint32_t parity, const int* err) {
  if (mbar_test_wait_a(bar, parity)) return true;
  if (mbar_try_wait_a(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (unsigned it = 1;; ++it) {
    if (mbar_try_wait_a(bar, parity)) return true;
    if (it % kPollsPerCheck == 0) {
      if (wait_expired(t0, kWaitBudgetNs)) return false;
      if (err && ld_volatile_int(err) != 0) return false;
    }
  }
}

// ---- bulk copy global -> shared (the TMA unit, 1-D form; no multicast) -------------------
CFB_DEV void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      :: "r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Order earlier generic-proxy global accesses (made visible to this thread by an acquire) before
// subsequent async-proxy (bulk copy) reads of global memory.
CFB_DEV void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- named barrier among the consumer warps ------------------------------------------------
CFB_DEV void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" :: "r"(nthreads) : "memory");
}

CFB_DEV uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
CFB_DEV float2 unpack_half2(uint32_t u) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  return __half22float2(h);
}

// ---- gpu-scope atomics / loads with explicit ordering ------------------------------------
CFB_DEV unsigned atom_add_acqrel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
CFB_DEV unsigned atom_add_release(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.release.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
CFB_DEV unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
CFB_DEV int ld_volatile_int(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---- 5th-generation tensor cores (tcgen05) and tensor memory ---------------------------------
CFB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CFB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// whole warp; writes the allocated TMEM address to *slot
CFB_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
CFB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[smem] · B[smem]ᵀ, kind::f16 (fp16 × fp16 -> fp32)
CFB_DEV void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// arrive on `bar` once every tcgen05 op this thread issued before has completed
CFB_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(bar)) : "memory");
}
// Warp forms: the whole warp executes these converged, with warp-uniform operands, and one
// elected lane issues. Kept converged, the operands stay in the uniform datapath: measured on
// B200, a warp issues an M = 64 MMA in about 44 cycles this way against about 80 for one lane
// running the same loop alone.
CFB_DEV void tc_mma_f16_warp(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "setp.ne.b32 q, %4, 0;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, q;\n\t}"
      :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
CFB_DEV void tc_commit_warp_a(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
      :: "r"(bar) : "memory");
}
CFB_DEV void tc_commit_warp(uint64_t* bar) { tc_commit_warp_a(smem_u32(bar)); }
// A whole 128-k unit in one statement: one elected lane issues the 8 MMAs of k blocks 0-3 (the
// 64-k half at descriptors a0 / b0) and 4-7 (a1 / b1), each k block 32 bytes (+2 in the
// descriptors' 16-byte address field) after the last, then the commit on `bar`. One election and
// one statement per unit measured ~15 % less issue time per unit than eight single-MMA statements.
CFB_DEV void tc_unit8_warp(uint32_t td, uint64_t a0, uint64_t b0, uint64_t a1, uint64_t b1, uint32_t idesc,
                           uint32_t accumulate, uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "setp.ne.b32 q, %6, 0;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %5, q;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %8, %9, %5, 1;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %10, %11, %5, 1;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %12, %13, %5, 1;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %4, %5, 1;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %14, %15, %5, 1;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %16, %17, %5, 1;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %18, %19, %5, 1;\n\t"
      "@p tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n\t}"
      :: "r"(td), "l"(a0), "l"(b0), "l"(a1), "l"(b1), "r"(idesc), "r"(accumulate), "r"(bar),
         "l"(a0 + 2), "l"(b0 + 2), "l"(a0 + 4), "l"(b0 + 4), "l"(a0 + 6), "l"(b0 + 6),
         "l"(a1 + 2), "l"(b1 + 2), "l"(a1 + 4), "l"(b1 + 4), "l"(a1 + 6), "l"(b1 + 6)
      : "memory");
}
// 32 lanes × 16 consecutive fp32 columns of TMEM (lane = row of the accumulator)
CFB_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the 128-byte swizzle:
// 128-byte rows, 8-row groups 1024 bytes apart (SBO), leading offset unused (1), version 1,
// layout SWIZZLE_128B (2). The tile base must be 1024-byte aligned; stepping K by 16 elements
// inside the 64-element swizzle row adds 32 bytes to the start address.
CFB_DEV uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor of kind::f16 with an fp32 accumulator, fp16 A and B, both K-major
// (bit 4: D format f32; bits 17-22: N / 8; bits 24-28: M / 16).
CFB_DEV constexpr uint32_t tc_idesc(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

CFB_DEV float gelu_erf(float x) {   // nn.GELU() default (exact erf form)
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

}  // namespace cfb
