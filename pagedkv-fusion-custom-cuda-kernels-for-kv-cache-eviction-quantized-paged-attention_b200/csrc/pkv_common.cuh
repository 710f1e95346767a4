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

// Waits for the phase with the given parity to complete.  Gives up after
// `limit_ns` nanoseconds of wall time, or as soon as any CTA has recorded a
// wait timeout in the error word (both checked after every suspended poll of
// at most 100 us), and returns false; the caller records kDevWaitTimeout and
// unwinds.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  const int* err,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_suspend(bar, parity, 100000u)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
    if (err != nullptr && *reinterpret_cast<const volatile int*>(err) == kDevWaitTimeout)
      return false;
  }
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

}  // namespace pkv
