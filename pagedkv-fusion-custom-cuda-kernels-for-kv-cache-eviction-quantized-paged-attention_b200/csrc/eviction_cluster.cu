// Single-launch eviction score + bottom-k for up to 16,384 blocks.
//
// The latency path of the eviction decision (16K blocks, k = 2,458): one
// thread-block cluster (16 CTAs of 1024 threads, or 8 CTAs where 16 cannot
// be co-scheduled) does all of it in shared memory:
//
//   1. each CTA scores its slice of the blocks (bit-exact,
//      eviction_score.cuh) into 32-bit orderable keys in its shared memory;
//   2. each CTA pushes its slice to every other CTA with one DSMEM bulk copy
//      (cp.async.bulk shared::cta -> shared::cluster, completion counted on
//      the receiver's mbarrier), so every CTA then holds all keys locally --
//      no remote loads;
//   3. every CTA (identically) histograms all keys into 2,048 bins spanning
//      [min key, max key], finds the bin holding rank k-1, and cuts the bins
//      up to it into one contiguous key range per CTA with ~C / cluster-size
//      candidates each;
//   4. each CTA ranks the candidates of its own range by counting (64-bit
//      keys orderable(score) << 32 | block id are unique) and writes rank =
//      range offset + local rank for ranks below k.
//
// Order = ascending (score, id) with -0.0 == +0.0 and NaN last, i.e. the
// reference's lexsort (pagedkv_fusion/reference.py:74-81).  A range with
// more than 1,024 candidates (skewed data, e.g. many equal scores) is
// sorted with a shared-memory bitonic network instead of counted.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "eviction_score.cuh"
#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace cg = cooperative_groups;

namespace pkv {
namespace {

constexpr int kCT = 1024;       // threads per CTA
constexpr int kMaxN = 16384;    // blocks per launch
constexpr int kKPT = kMaxN / kCT;  // keys per thread in the histogram pass
constexpr int kBins = 2 * kCT;  // key histogram bins
constexpr uint64_t kPad = ~0ull;

template <int CL>
struct CCfg {
  static constexpr int kCap = kMaxN / CL;         // blocks scored per CTA
  static constexpr int kEPT = kCap / kCT;         // blocks per thread
  static constexpr int kSlice = kCap + 4;         // u32: keys, then (min, max, -, -)
  static constexpr int kOffKeys = 0;              // u32 [CL][kSlice]
  static constexpr int kOffHist = kOffKeys + CL * kSlice * 4;
  static constexpr int kOffCum = kOffHist + kBins * 4;
  static constexpr int kOffBinJ = kOffCum + kBins * 4;  // bucket of each bin (u8)
  static constexpr int kOffCand = kOffBinJ + kBins;     // u64 [kMaxN] candidates
  static constexpr int kOffMisc = kOffCand + kMaxN * 8;
  static constexpr int kOffBar = kOffMisc + 512;
  static constexpr int kSmem = kOffBar + 16;
};

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, int cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(cta));
  return r;
}

// Bulk copy of `bytes` from this CTA's shared memory into CTA `dst`'s shared
// memory; the bytes are counted on the mbarrier at `bar` (also in `dst`).
__device__ __forceinline__ void push_to_cta(uint32_t dst_cluster, uint32_t src_local,
                                            uint32_t bytes, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst_cluster),
      "r"(src_local), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

template <int CL>
__global__ void __launch_bounds__(kCT, 1)
    evict_cluster_kernel(const float* __restrict__ rec, const float* __restrict__ freq,
                         const float* __restrict__ attn, const uint8_t* __restrict__ valid,
                         const float* __restrict__ scores_in, float* __restrict__ scores_out,
                         int n, int bs, bool fast16, float wr, float wf, float wa, int k,
                         int64_t* __restrict__ out_ids, int* err) {
  using C = CCfg<CL>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint32_t* s_keys = reinterpret_cast<uint32_t*>(smem + C::kOffKeys);
  uint32_t* s_hist = reinterpret_cast<uint32_t*>(smem + C::kOffHist);
  uint32_t* s_cum = reinterpret_cast<uint32_t*>(smem + C::kOffCum);
  uint8_t* s_binj = smem + C::kOffBinJ;
  uint64_t* s_cand = reinterpret_cast<uint64_t*>(smem + C::kOffCand);
  uint32_t* s_misc = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  // s_misc: [0..63] per-warp scratch, [70] candidate fill, [71] threshold
  // bin, [72] min key, [73] max key, [80..80+CL] range offsets
  uint32_t* s_warp = s_misc;
  uint32_t* s_off = s_misc + 80;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::kOffBar);

  cg::cluster_group cluster = cg::this_cluster();
  const int me = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t slice_bytes = C::kSlice * 4;

  // ---- 1. scores -> keys of this CTA's slice ---------------------------------
  // Inputs are loaded before the launch-time cluster barrier (which only
  // orders the mbarrier set-up against the remote pushes), so the loads are
  // in flight while the barrier completes.
  float sv[C::kEPT];
#pragma unroll
  for (int e = 0; e < C::kEPT; ++e) {
    const int i = me * C::kCap + e * kCT + tid;
    sv[e] = 0.0f;
    if (i < n) {
      sv[e] = scores_in != nullptr
                  ? scores_in[i]
                  : (fast16 ? score16(attn, valid, i, rec[i], freq[i], wr, wf, wa)
                            : score_generic(attn, valid, i, bs, rec[i], freq[i], wr, wf, wa));
    }
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
    // every other CTA pushes one slice here
    mbar_arrive_expect_tx(bar, (uint32_t)(CL - 1) * slice_bytes);
  }
  for (int b = tid; b < kBins; b += kCT) s_hist[b] = 0u;
  cluster.sync();  // (A) barriers armed everywhere

  uint32_t* my_slice = s_keys + me * C::kSlice;
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
#pragma unroll
  for (int e = 0; e < C::kEPT; ++e) {
    const int i = me * C::kCap + e * kCT + tid;
    uint32_t key = 0xFFFFFFFFu;
    if (i < n) {
      if (scores_in == nullptr && scores_out != nullptr) scores_out[i] = sv[e];
      key = orderable_key(sv[e]);
      kmin = min(kmin, key);
      kmax = max(kmax, key);
    }
    my_slice[e * kCT + tid] = key;
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  if (lane == 0) {
    s_warp[warp] = kmin;
    s_warp[32 + warp] = kmax;
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t a = __reduce_min_sync(0xffffffffu, s_warp[lane]);
    const uint32_t b = __reduce_max_sync(0xffffffffu, s_warp[32 + lane]);
    if (lane == 0) {
      my_slice[C::kCap] = a;
      my_slice[C::kCap + 1] = b;
    }
  }
  __syncthreads();
  // generic-proxy writes -> visible to the bulk-copy (async) proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

  // ---- 2. push this slice to every other CTA ---------------------------------
  if (tid < CL && tid != me) {
    const uint32_t src = smem_u32(my_slice);
    push_to_cta(cluster_addr(src, tid), src, slice_bytes, cluster_addr(smem_u32(bar), tid));
  }
  if (!mbar_wait_bounded(bar, 0, err)) {
    record_error(err, kDevWaitTimeout);
    mbar_drain(bar, 0);  // no push may land after this CTA has exited
  }
  // Every push into this CTA has landed.  Arrive on the cluster barrier now
  // and wait on it only before exiting: once all CTAs have arrived, every
  // push has landed everywhere, so no CTA -- a push source -- exits while a
  // copy still reads its shared memory.  (A full cluster barrier at the end
  // cost ~1.3 us on the critical path.)  Nothing below touches another
  // CTA's shared memory, and this CTA's pushed slice is not written again.
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");

  // ---- 3. histogram of all keys over [min, max] ------------------------------
  if (warp == 0) {
    uint32_t a = 0xFFFFFFFFu, b = 0u;
    if (lane < CL) {
      a = s_keys[lane * C::kSlice + C::kCap];
      b = s_keys[lane * C::kSlice + C::kCap + 1];
    }
    a = __reduce_min_sync(0xffffffffu, a);
    b = __reduce_max_sync(0xffffffffu, b);
    if (lane == 0) {
      s_misc[72] = a;
      s_misc[73] = b;
    }
  }
  uint32_t keys[kKPT];  // block i = j * kCT + tid
#pragma unroll
  for (int j = 0; j < kKPT; ++j) {
    const int i = j * kCT + tid;
    keys[j] = s_keys[(i / C::kCap) * C::kSlice + (i % C::kCap)];
  }
  __syncthreads();
  const uint32_t gmin = s_misc[72], gmax = s_misc[73];
  const int span = (gmin == gmax) ? 0 : 32 - __clz(gmin ^ gmax);  // bits that differ
  const int shift = span > 11 ? span - 11 : 0;
  const uint32_t base = gmin >> shift;
#pragma unroll
  for (int j = 0; j < kKPT; ++j)
    if (j * kCT + tid < n) atomicAdd(&s_hist[(keys[j] >> shift) - base], 1u);
  __syncthreads();

  // inclusive cumulative counts; thread t owns bins 2t, 2t+1
  const uint32_t c0 = s_hist[2 * tid], c1 = s_hist[2 * tid + 1];
  const uint32_t incl = warp_incl_scan(c0 + c1, lane);
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = s_warp[lane];
    s_warp[lane] = warp_incl_scan(w, lane) - w;  // exclusive prefix of warp totals
  }
  __syncthreads();
  const uint32_t ex = s_warp[warp] + incl - (c0 + c1);
  s_cum[2 * tid] = ex + c0;
  s_cum[2 * tid + 1] = ex + c0 + c1;
  __syncthreads();
#pragma unroll
  for (int h = 0; h < 2; ++h) {  // threshold bin: first bin reaching k
    const int b = 2 * tid + h;
    const uint32_t before = b ? s_cum[b - 1] : 0u;
    if (s_cum[b] >= (uint32_t)k && before < (uint32_t)k) s_misc[71] = (uint32_t)b;
  }
  __syncthreads();
  const int bstar = (int)s_misc[71];
  const uint32_t cand = s_cum[bstar];
  // range of bin b (b <= bstar): floor(cum_before(b) * CL / cand), monotone
  // in b; 0xFF past the threshold bin.  s_off[j] = first rank of range j.
  for (int j = tid; j <= CL; j += kCT) s_off[j] = cand;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int b = 2 * tid + h;
    const uint32_t before = b ? s_cum[b - 1] : 0u;
    s_binj[b] = b <= bstar ? (uint8_t)(before * (uint32_t)CL / cand) : (uint8_t)0xFF;
  }
  if (tid == 0) s_misc[70] = 0u;
  __syncthreads();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int b = 2 * tid + h;
    if (b <= bstar) {
      const int jb = s_binj[b];
      const int jp = b ? (int)s_binj[b - 1] : -1;
      const uint32_t before = b ? s_cum[b - 1] : 0u;
      for (int j = jp + 1; j <= jb; ++j) s_off[j] = before;
    }
  }

  // ---- 4. candidates of this CTA's range ---------------------------------------
#pragma unroll
  for (int j = 0; j < kKPT; ++j) {
    const int i = j * kCT + tid;
    if (i < n && s_binj[(keys[j] >> shift) - base] == me)
      s_cand[atomicAdd(&s_misc[70], 1u)] = ((uint64_t)keys[j] << 32) | (uint32_t)i;
  }
  __syncthreads();
  const int m = (int)s_misc[70];
  const uint32_t off = s_off[me];
  if (m <= kCT / 4) {
    // rank by counting (keys are unique), 4 lanes per candidate
    const int c = tid >> 2, part = tid & 3;
    const uint64_t mine = c < m ? s_cand[c] : 0ull;
    uint32_t r = 0;
    if (c < m)
      for (int j = part; j < m; j += 4) r += (uint32_t)(s_cand[j] < mine);
    r += __shfl_xor_sync(0xffffffffu, r, 1);
    r += __shfl_xor_sync(0xffffffffu, r, 2);
    if (c < m && part == 0 && off + r < (uint32_t)k)
      out_ids[off + r] = (int64_t)(mine & 0xffffffffull);
  } else if (m <= kCT) {
    if (tid < m) {
      const uint64_t mine = s_cand[tid];
      uint32_t r = 0;
      for (int j = 0; j < m; ++j) r += (uint32_t)(s_cand[j] < mine);
      if (off + r < (uint32_t)k) out_ids[off + r] = (int64_t)(mine & 0xffffffffull);
    }
  } else {
    int P = 2;
    while (P < m) P <<= 1;
    for (int i = m + tid; i < P; i += kCT) s_cand[i] = kPad;
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int p = tid; p < P / 2; p += kCT) {
          const int lo = 2 * stride * (p / stride) + (p % stride);
          const bool asc = (lo & size) == 0;
          const uint64_t a = s_cand[lo], b = s_cand[lo + stride];
          if ((a > b) == asc) {
            s_cand[lo] = b;
            s_cand[lo + stride] = a;
          }
        }
        __syncthreads();
      }
    }
    for (int p = tid; p < m; p += kCT)
      if (off + p < (uint32_t)k) out_ids[off + p] = (int64_t)(s_cand[p] & 0xffffffffull);
  }
  // the arrivals above: every CTA has received every push
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

template <int CL>
cudaError_t launch_cluster_t(const float* rec, const float* freq, const float* attn,
                             const uint8_t* valid, const float* scores_in, float* scores_out,
                             int n, int bs, bool fast16, float wr, float wf, float wa, int k,
                             int64_t* out, cudaStream_t stream) {
  auto kern = evict_cluster_kernel<CL>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, 1, 1);
  cfg.blockDim = dim3(kCT, 1, 1);
  cfg.dynamicSmemBytes = CCfg<CL>::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, rec, freq, attn, valid, scores_in, scores_out, n, bs,
                            fast16, wr, wf, wa, k, out, device_error_word());
}

template <int CL>
bool prepare_cluster_t() {
  auto kern = evict_cluster_kernel<CL>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           CCfg<CL>::kSmem) != cudaSuccess)
    return false;
  if (CL > 8 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, 1, 1);
  cfg.blockDim = dim3(kCT, 1, 1);
  cfg.dynamicSmemBytes = CCfg<CL>::kSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) return false;
  return clusters > 0;
}

// Cluster size usable on the current device: 16, else 8, else 0 (none).
int cluster_size_for_device() {
  static int chosen[64];
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    // PKV_EVICTION_CLUSTER=8 pins the 8-CTA variant (tuning and tests)
    const char* pin = std::getenv("PKV_EVICTION_CLUSTER");
    const bool want8 = pin != nullptr && std::atoi(pin) == 8;
    chosen[dev] = (!want8 && prepare_cluster_t<16>()) ? 16 : (prepare_cluster_t<8>() ? 8 : 0);
    cudaGetLastError();  // a refused probe leaves no sticky error
    done[dev] = true;
  }
  return chosen[dev];
}

}  // namespace

int cluster_select_max_blocks() { return kMaxN; }

bool cluster_select_available() { return cluster_size_for_device() != 0; }

// Returns kUnsupported (without launching) when the cluster path cannot
// run here, so the caller can use the multi-kernel path instead.
int launch_cluster_select(const float* rec, const float* freq, const float* attn,
                          const uint8_t* valid, const float* scores_in, float* scores_out,
                          int64_t n, int bs, float wr, float wf, float wa, int64_t k,
                          int64_t* out_ids, cudaStream_t stream) {
  if (k > n) k = n;
  if (n <= 0 || k <= 0 || n > kMaxN) return kUnsupported;
  const int CL = cluster_size_for_device();
  if (CL == 0) return kUnsupported;
  // score16 reads each row with 16-byte loads: only for aligned rows
  const bool fast16 = scores_in == nullptr && bs == 16 &&
                      reinterpret_cast<uintptr_t>(attn) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(valid) % 16 == 0;
  const cudaError_t e =
      CL == 16 ? launch_cluster_t<16>(rec, freq, attn, valid, scores_in, scores_out, (int)n, bs,
                                      fast16, wr, wf, wa, (int)k, out_ids, stream)
               : launch_cluster_t<8>(rec, freq, attn, valid, scores_in, scores_out, (int)n, bs,
                                     fast16, wr, wf, wa, (int)k, out_ids, stream);
  if (e != cudaSuccess) {
    set_error(std::string("cluster eviction launch failed: ") + cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

}  // namespace pkv
