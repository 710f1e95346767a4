// Shared helpers for the PagedKV-Fusion sm_100a kernels: status codes, the
// device error word, bounded mbarrier waits and TMA bulk-tensor loads.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace pkv {

// Host-visible status codes (mirrored in include/pagedkv_fusion.h).
enum Status : int {
  kOk = 0,
  kInvalidArgument = 1,
  kUnsupported = 2,
  kWorkspace = 3,
  kCudaError = 4,
  kDeviceInput = 5,
};

// Codes a kernel records in the per-device error word.  The first error
// wins; kernels never trap.
enum DeviceError : int {
  kDevNone = 0,
  kDevBadBlockId = 1,     // block table entry outside [0, num_blocks)
  kDevWaitTimeout = 2,    // a bounded barrier wait gave up
  kDevBadSlot = 3,        // slot_mapping entry outside the cache
  kDevSeqTooLong = 4,     // seq_len needs more pages than the block table has
};

// Pages a decode split may read for a sequence: ceil(L / bs), clamped to the
// block-table width (a longer seq_len is recorded as kDevSeqTooLong and only
// the covered tokens are attended).  Negative lengths count as 0.
__device__ __forceinline__ int covered_pages(int L, int bs, int max_blocks_per_seq) {
  const int want = L > 0 ? (L + bs - 1) / bs : 0;
  return want < max_blocks_per_seq ? want : max_blocks_per_seq;
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// Arrival on a GPU-wide counter that publishes this CTA's earlier global
// writes and acquires the other arrivals' writes: release / acquire at GPU
// scope on the one atomic (cumulative, so writes of other threads of the CTA
// ordered before it by a CTA barrier are covered), instead of a
// sequentially consistent fence in every writing thread.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}

// 64-bit add with release / acquire at GPU scope.
__device__ __forceinline__ unsigned long long atomic_add_acq_rel_gpu_u64(unsigned long long* p,
                                                                       unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;"
               : "=l"(old)
               : "l"(p), "l"(v)
               : "memory");
  return old;
}

// 64-bit relaxed load at GPU scope (a hint: no ordering with other accesses).
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}

// 64-bit compare-and-swap with release / acquire at GPU scope.
__device__ __forceinline__ unsigned long long atomic_cas_acq_rel_gpu(unsigned long long* p,
                                                                   unsigned long long cmp,
                                                                   unsigned long long val) {
  unsigned long long old;
  asm volatile("atom.acq_rel.gpu.global.cas.b64 %0, [%1], %2, %3;"
               : "=l"(old)
               : "l"(p), "l"(cmp), "l"(val)
               : "memory");
  return old;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// Raises the barrier's expected transaction bytes without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Bulk copy from global memory into this CTA's shared memory; the bytes
// complete on bar.  Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait that suspends the thread in hardware (up to hint_ns) until the
// phase completes, so waiting warps do not take issue slots from working ones.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity,
                                                      uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Suspend-time hint of a waiting poll, in ns (0: polls without a hint).
#ifndef PKV_MBAR_SUSPEND_NS
#define PKV_MBAR_SUSPEND_NS 100000u
#endif

__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity) {
#if PKV_MBAR_SUSPEND_NS > 0
  return mbar_try_wait_suspend(bar, parity, PKV_MBAR_SUSPEND_NS);
#else
  return mbar_try_wait(bar, parity);
#endif
}

// Waits for the phase with the given parity to complete.  Gives up after
// `limit_ns` nanoseconds of wall time, or as soon as any CTA has recorded a
// wait timeout in the error word (both checked after every poll), and
// returns false; the caller records kDevWaitTimeout and unwinds.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  const int* err,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_poll(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
    if (err != nullptr && *reinterpret_cast<const volatile int*>(err) == kDevWaitTimeout)
      return false;
  }
}

// Waits (at most limit_ns, ignoring the error word) for the phase of a
// barrier that this thread's own copies complete: a producer calls it for
// every load it issued before it exits, so that no copy can land in shared
// memory after the CTA is gone -- also on an error path, where the
// consumers stopped waiting.  Copies complete on their own, so this ends
// promptly.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity,
                                           uint64_t limit_ns = 200000000ull) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_poll(bar, parity))
    if (global_timer_ns() - t0 > limit_ns) return;
}

// Drains the last min(issued, stages) loads of a ring of `stages` full
// barriers, load n having used stage n % stages in phase n / stages.
__device__ __forceinline__ void drain_ring(uint64_t* full, int stages, int issued) {
  for (int n = issued > stages ? issued - stages : 0; n < issued; ++n)
    mbar_drain(&full[n % stages], (uint32_t)(n / stages) & 1u);
}

// ---------------------------------------------------------------------------
// TMA: 3-D tiled bulk-tensor load into this CTA's shared memory.  No
// multicast: every copy reads this GPU's own global memory only.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int32_t c0, int32_t c1,
                                            int32_t c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "l"(policy)
      : "memory");
}

// 4-D tiled load (same rules as tma_load_3d).
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int32_t c0, int32_t c1, int32_t c2,
                                            int32_t c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// Selection key: unsigned order == (score ascending, -0 == +0, NaN last).
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t orderable_key(float s) {
  uint32_t u = __float_as_uint(s);
  if (s != s) return 0xFFFFFFFFu;
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}


// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in tensor memory)
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor for a 128-byte-swizzled tile whose base is
// 1024-byte aligned: rows of 128 B, 8-row atoms.  K-major operands: atoms
// follow each other along M/N at `sbo` bytes, lbo unused (16).  MN-major
// operands: atoms along K at `sbo` bytes, lbo the stride between 128-byte
// atoms along M/N.  Version 1 (sm_100), swizzle mode 2 (128 B).
__device__ __forceinline__ uint64_t umma_sw128_desc(uint32_t smem_addr, uint32_t lbo,
                                                    uint32_t sbo) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of tcgen05.mma .kind::i8 with an s32 accumulator:
// A / B signed (1) or unsigned (0) 8-bit, K-major (0) or MN-major (1).
__host__ __device__ constexpr uint32_t umma_i8_idesc(int a_signed, int b_signed, int a_mn,
                                                     int b_mn, int m, int n) {
  return (2u << 4) | ((uint32_t)a_signed << 7) | ((uint32_t)b_signed << 10) |
         ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A * B^T for one K step of 32 int8 values; issued by one thread.
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Arrives once on bar when every tcgen05 operation this thread issued so
// far has completed (their shared-memory operands may then be reused).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole-warp tensor-memory allocation of `cols` columns (power of two >= 32);
// the base address is written to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(cols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols));
}

// Loads 32-bit columns [col, col + N) of this warp's 32 tensor-memory lanes
// (lane base 32 * (warp % 4) is part of taddr): thread i gets lane i.
template <int N>
__device__ __forceinline__ void tmem_load(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_load<8>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_load<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_load<32>(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_load() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Generic-proxy writes to shared memory made visible to the async proxy
// (tensor-core operands written by threads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Byte offset of (row, byte) in a 128-byte-swizzled tile (1024-byte aligned).
__device__ __forceinline__ uint32_t sw128_offset(int row, int byte) {
  return (uint32_t)(row * 128 + ((((byte >> 4) ^ row) & 7) << 4) + (byte & 15));
}

}  // namespace pkv
