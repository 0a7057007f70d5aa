// Shared device helpers for the sm_100a kernels: error plumbing, mbarriers
// with bounded waits, TMA, and tcgen05 (UMMA / TMEM) wrappers in inline PTX.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <string>

#include "../../include/svdq_b200.h"

namespace svdq {

// ---------------------------------------------------------------------------
// host-side error reporting
// ---------------------------------------------------------------------------
int set_error(int status, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);
int check_launch(const char* what);

#define SVDQ_REQUIRE(cond, msg)                                                \
  do {                                                                         \
    if (!(cond)) return ::svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, (msg));   \
  } while (0)

// Encodes a 2-D tiled tensor map through the driver entry point.
int make_tma_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);

// Number of SMs on the current device (cached per device).
int num_sms();

// The calling thread's current CUDA context (the runtime's primary context of the current
// device unless the caller made another context current).
int current_context(CUcontext* out);

// Device address of a file-scope __device__ variable in the current context, looked up with
// cudaGetSymbolAddress once per (context, symbol) and cached.
int symbol_address(const void* symbol, void** out, const char* what);

// Device address of this library's error word on the current device: bounded
// in-kernel waits record there where they gave up (kernels take it as a
// parameter).  Returns nullptr if the symbol address cannot be obtained.
int* device_error_word();

// Wait limit for any in-kernel spin (ns of %globaltimer).  Normal waits are
// microseconds; this only ends waits that can no longer complete.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Up to 64 polls of the phase in one tight PTX loop; each poll may suspend the
// thread for up to `hint_ns` while the phase is incomplete.  Returns true once
// the phase with the given parity has completed.
template <bool CLUSTER>
__device__ __forceinline__ bool mbar_poll64(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  constexpr uint32_t hint_ns = 20000;
  if (CLUSTER) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .u32 i;\n\t"
        "mov.u32 i, 0;\n"
        "MBAR_POLL:\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "@p bra.uni MBAR_DONE;\n\t"
        "add.u32 i, i, 1;\n\t"
        "setp.lt.u32 p, i, 64;\n\t"
        "@p bra.uni MBAR_POLL;\n\t"
        "mov.u32 %0, 0;\n\t"
        "bra.uni MBAR_END;\n"
        "MBAR_DONE:\n\t"
        "mov.u32 %0, 1;\n"
        "MBAR_END:\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .u32 i;\n\t"
        "mov.u32 i, 0;\n"
        "MBAR_POLL:\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "@p bra.uni MBAR_DONE;\n\t"
        "add.u32 i, i, 1;\n\t"
        "setp.lt.u32 p, i, 64;\n\t"
        "@p bra.uni MBAR_POLL;\n\t"
        "mov.u32 %0, 0;\n\t"
        "bra.uni MBAR_END;\n"
        "MBAR_DONE:\n\t"
        "mov.u32 %0, 1;\n"
        "MBAR_END:\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
  }
  return ok != 0;
}

// Bounded wait on the phase with the given parity.  Returns false (and raises
// the CTA-wide abort flag plus the device error word) if the wait ran out, or
// if another role of the CTA already aborted.  CLUSTER selects cluster-scope
// acquire, for barriers that also receive arrivals from the other CTA of a pair.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          volatile int* abort_flag, int* err, int where,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_poll64<CLUSTER>(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit_ns) {
      *abort_flag = 1;
      atomicCAS(err, 0, where);
      return false;
    }
    if (mbar_poll64<CLUSTER>(bar, parity)) return true;
  }
}

// Non-blocking check: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test_parity(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait by spinning on test_wait: a phase that has already completed costs one test, and
// a completion is seen within a poll.  (try_wait with a suspend-time hint, as in mbar_wait, was
// measured at 0.13-0.36 us per wait even on completed phases: too slow for pipelines whose stages
// are a fraction of a microsecond.)  Gives up like mbar_wait.
__device__ __forceinline__ bool mbar_spin_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err,
                                               int where, unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_test_parity(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test_parity(bar, parity)) return true;
    if ((i & 127u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > limit_ns) {
        *abort_flag = 1;
        atomicCAS(err, 0, where);
        return false;
      }
    }
  }
}

// Bounded wait for the multi-warp roles: test_wait polls with a short nanosleep between them, so
// that waiting warps leave the issue slots of their SM sub-partition to the single-thread MMA and
// TMA roles (a spinning warp takes a share of them; a suspending try_wait is slow to wake).
__device__ __forceinline__ bool wait_spin(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int where) {
  if (mbar_test_parity(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(32);
    if (mbar_test_parity(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        atomicCAS(err, 0, where);
        return false;
      }
    }
  }
}

// Bounded wait that ignores the abort flag: used while draining in-flight
// copies or MMAs after an abort.  Returns false if the limit ran out.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity,
                                                unsigned long long limit_ns) {
  if (mbar_poll64<false>(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_poll64<false>(bar, parity)) {
    if (globaltimer() - t0 > limit_ns) return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// clusters (CTA pairs for cta_group::2 MMAs)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory location in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// arrive on an mbarrier given by a shared::cluster address (own CTA or the peer)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// ---------------------------------------------------------------------------
// TMA (no cluster multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// Pair load for cta_group::2 MMAs: the data lands in this CTA's shared memory and
// the transaction bytes are counted on the mbarrier at `bar_cluster`, which may be
// the even (leader) CTA's barrier.  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// Tile store shared -> global through the bulk-async group of the issuing thread.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until all but the newest N bulk-store groups of the issuing thread have finished reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until the issuing thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory accesses before later async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tma_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- CTA-pair (cta_group::2) forms ----
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
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
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at the same offset in both CTAs of the pair once all
// previously issued tcgen05 ops of this thread complete (commit, not a load).
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair_local(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// ---- single-CTA (cta_group::1) forms ----
__device__ __forceinline__ void tmem_alloc_1(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_1() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_1(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_f16_1(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// As umma_f16_1 with the A operand in tensor memory (a_tmem: lane = row of A, each 32-bit column
// two consecutive K elements, the lower K in the low half) and B in shared memory.
__device__ __forceinline__ void umma_f16_1_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns from registers: thread i of the warp writes lane (base + i).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns from registers: thread i of the warp writes lane (base + i).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrive on this CTA's mbarrier once all previously issued tcgen05 ops of this thread complete.
__device__ __forceinline__ void umma_commit_1(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp gets lane (base + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait_regs16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Waits for outstanding tcgen05.ld and ties the 32 destination registers to the
// wait, so the compiler cannot read them before the load has completed.
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
        "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
        "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// Packed two-lane fp32 arithmetic (sm_100): each operand holds {lo, hi} floats.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | (uint64_t)__float_as_uint(lo);
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms
// stacked at a 1024-byte stride.  Fields: start>>4 [0,14), LBO>>4 [16,30)
// (unused for swizzled K-major, set to 1), SBO>>4 [32,46), version 1 [46,48),
// layout type 2 = SWIZZLE_128B [61,64).
__device__ __forceinline__ uint64_t desc_k_sw128(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) |
         ((uint64_t)(1024u >> 4) << 32) | ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor for kind::f16 with fp32 accumulation,
// K-major A and B: c_format [4,6) = 1 (f32), a_format [7,10), b_format [10,13),
// N>>3 at [17,23), M>>4 at [24,29).
__host__ __device__ constexpr uint32_t make_idesc(uint32_t a_fmt, uint32_t b_fmt, int m, int n) {
  return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}
constexpr uint32_t kFmtBF16 = 1;  // kind::f16 format code

// Programmatic dependent launch.  pdl_wait: block until the grids this launch depends on
// have completed and their writes are visible (a no-op without a programmatic dependency).
// pdl_trigger: allow the next programmatically dependent launch to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace svdq
