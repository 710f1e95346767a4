// Single-launch eviction score + bottom-k for up to 16,384 blocks.
//
// The latency path of the eviction decision (16K blocks, k = 2,458): one
// thread-block cluster (16 CTAs of 1024 threads, or 8 CTAs where 16 cannot
// be co-scheduled) does all of it, with distributed shared memory instead
// of global round trips:
//
//   1. every thread scores one or two blocks (bit-exact, eviction_score.cuh)
//      and forms the unique 64-bit key orderable(score) << 32 | block id;
//   2. the cluster agrees on the min / max 32-bit key, and histograms the
//      keys into 2,048 bins spanning [min, max] (each CTA its own, summed
//      through DSMEM); the bin holding rank k-1 is the threshold bin, and
//      the bins up to it hold C >= k candidates;
//   3. the candidate bins are cut into one contiguous key range per CTA
//      with ~C / cluster-size keys each; every CTA gathers its range's keys
//      from all CTAs' shared memory and sorts them (bitonic, shared memory);
//   4. a key's global rank is its range's start offset + its local rank;
//      ranks below k are written out.
//
// Order = ascending (score, id) with -0.0 == +0.0 and NaN last, i.e. the
// reference's lexsort (pagedkv_fusion/reference.py:74-81).  Keys are unique,
// so the result does not depend on how the gather interleaves.  Skewed data
// (one bin holding most keys) only makes one CTA sort a longer range.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

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
constexpr int kBins = 2 * kCT;  // key histogram bins
constexpr uint64_t kPad = ~0ull;

template <int CL>
struct CCfg {
  static constexpr int kEPT = kMaxN / (CL * kCT);  // keys per thread
  static constexpr int kCap = kEPT * kCT;          // keys per CTA
  static constexpr int kOffKeys = 0;
  static constexpr int kOffHist = kOffKeys + kCap * 8;
  static constexpr int kOffCum = kOffHist + kBins * 4;
  static constexpr int kOffBucket = kOffCum + kBins * 4;
  static constexpr int kOffMisc = kOffBucket + kMaxN * 8;
  static constexpr int kSmem = kOffMisc + 512;
};

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

template <int CL>
__global__ void __launch_bounds__(kCT, 1)
    evict_cluster_kernel(const float* __restrict__ rec, const float* __restrict__ freq,
                         const float* __restrict__ attn, const uint8_t* __restrict__ valid,
                         const float* __restrict__ scores_in, float* __restrict__ scores_out,
                         int n, int bs, bool fast16, float wr, float wf, float wa, int k,
                         int64_t* __restrict__ out_ids) {
  using C = CCfg<CL>;
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* s_keys = reinterpret_cast<uint64_t*>(smem + C::kOffKeys);
  uint32_t* s_hist = reinterpret_cast<uint32_t*>(smem + C::kOffHist);
  uint32_t* s_cum = reinterpret_cast<uint32_t*>(smem + C::kOffCum);
  uint64_t* s_bucket = reinterpret_cast<uint64_t*>(smem + C::kOffBucket);
  uint32_t* s_misc = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  // s_misc: [0] CTA min key, [1] CTA max key, [2..65] per-warp scratch,
  //         [70] bucket fill, [71] threshold bin, [80..80+CL] bucket offsets
  uint32_t* s_warp = s_misc + 2;
  uint32_t* s_off = s_misc + 80;

  cg::cluster_group cluster = cg::this_cluster();
  const int me = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // ---- 1. scores and keys --------------------------------------------------
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
#pragma unroll
  for (int e = 0; e < C::kEPT; ++e) {
    const int idx = e * kCT + tid;
    const int i = me * C::kCap + idx;
    uint64_t key = kPad;
    if (i < n) {
      float s;
      if (scores_in != nullptr) {
        s = scores_in[i];
      } else {
        s = fast16 ? score16(attn, valid, i, rec[i], freq[i], wr, wf, wa)
                   : score_generic(attn, valid, i, bs, rec[i], freq[i], wr, wf, wa);
        if (scores_out != nullptr) scores_out[i] = s;
      }
      const uint32_t k32 = orderable_key(s);
      key = ((uint64_t)k32 << 32) | (uint32_t)i;
      kmin = min(kmin, k32);
      kmax = max(kmax, k32);
    }
    s_keys[idx] = key;
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
      s_misc[0] = a;
      s_misc[1] = b;
    }
  }
  for (int b = tid; b < kBins; b += kCT) s_hist[b] = 0u;
  if (tid < CL + 1) s_off[tid] = 0u;
  cluster.sync();  // (A) every CTA's min / max published, histograms zeroed

  // ---- 2. cluster histogram over [gmin, gmax] --------------------------------
  uint32_t gmin = 0xFFFFFFFFu, gmax = 0u;
#pragma unroll
  for (int c = 0; c < CL; ++c) {
    const uint32_t* rm = cluster.map_shared_rank(s_misc, c);
    gmin = min(gmin, rm[0]);
    gmax = max(gmax, rm[1]);
  }
  const int span = (gmin == gmax) ? 0 : 32 - __clz(gmin ^ gmax);  // bits that differ
  const int shift = span > 11 ? span - 11 : 0;
  const uint32_t base = gmin >> shift;
#pragma unroll
  for (int e = 0; e < C::kEPT; ++e) {
    const uint64_t key = s_keys[e * kCT + tid];
    if (key != kPad) atomicAdd(&s_hist[((uint32_t)(key >> 32) >> shift) - base], 1u);
  }
  cluster.sync();  // (B) local histograms complete

  // thread t owns bins 2t and 2t+1
  uint32_t c0 = 0, c1 = 0;
#pragma unroll
  for (int c = 0; c < CL; ++c) {
    const uint2 h = reinterpret_cast<const uint2*>(cluster.map_shared_rank(s_hist, c))[tid];
    c0 += h.x;
    c1 += h.y;
  }
  uint32_t incl = warp_incl_scan(c0 + c1, lane);
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = s_warp[lane];
    const uint32_t wi = warp_incl_scan(w, lane);
    s_warp[lane] = wi - w;  // exclusive prefix of warp totals
  }
  __syncthreads();
  const uint32_t ex = s_warp[warp] + incl - (c0 + c1);
  s_cum[2 * tid] = ex + c0;  // inclusive cumulative counts
  s_cum[2 * tid + 1] = ex + c0 + c1;
  __syncthreads();
  // threshold bin: first bin whose cumulative count reaches k
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int b = 2 * tid + h;
    const uint32_t before = b ? s_cum[b - 1] : 0u;
    if (s_cum[b] >= (uint32_t)k && before < (uint32_t)k) s_misc[71] = (uint32_t)b;
  }
  __syncthreads();
  const int bstar = (int)s_misc[71];
  const uint32_t cand = s_cum[bstar];
  // bucket of bin b (b <= bstar): floor(cum_before(b) * CL / cand); buckets
  // are monotone in b, so each is a contiguous key range.  s_off[j] = first
  // candidate rank of bucket j.
  for (int j = tid; j <= CL; j += kCT) s_off[j] = cand;
  __syncthreads();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int b = 2 * tid + h;
    if (b <= bstar) {
      const uint32_t before = b ? s_cum[b - 1] : 0u;
      const int jb = (int)((uint64_t)before * CL / cand);
      const int jp = b ? (int)((uint64_t)(b > 1 ? s_cum[b - 2] : 0u) * CL / cand) : -1;
      for (int j = jp + 1; j <= jb; ++j) s_off[j] = before;
    }
  }
  if (tid == 0) s_misc[70] = 0u;
  __syncthreads();

  // ---- 3. gather this CTA's key range from every CTA, sort it ---------------
  for (int c = 0; c < CL; ++c) {
    const uint64_t* rk = cluster.map_shared_rank(s_keys, c);
#pragma unroll
    for (int e = 0; e < C::kEPT; ++e) {
      const uint64_t key = rk[e * kCT + tid];
      if (key == kPad) continue;
      const int b = (int)(((uint32_t)(key >> 32) >> shift) - base);
      if (b > bstar) continue;
      const uint32_t before = b ? s_cum[b - 1] : 0u;
      if ((int)((uint64_t)before * CL / cand) == me) s_bucket[atomicAdd(&s_misc[70], 1u)] = key;
    }
  }
  cluster.sync();  // (C) no CTA reads another's shared memory after this
  const int m = (int)s_misc[70];
  int P = 2;
  while (P < m) P <<= 1;
  for (int i = m + tid; i < P; i += kCT) s_bucket[i] = kPad;
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int p = tid; p < P / 2; p += kCT) {
        const int lo = 2 * stride * (p / stride) + (p % stride);
        const bool asc = (lo & size) == 0;
        const uint64_t a = s_bucket[lo], b = s_bucket[lo + stride];
        if ((a > b) == asc) {
          s_bucket[lo] = b;
          s_bucket[lo + stride] = a;
        }
      }
      __syncthreads();
    }
  }

  // ---- 4. write ranks below k ---------------------------------------------------
  const uint32_t off = s_off[me];
  for (int p = tid; p < m; p += kCT) {
    const uint32_t r = off + (uint32_t)p;
    if (r < (uint32_t)k) out_ids[r] = (int64_t)(s_bucket[p] & 0xffffffffull);
  }
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
                            fast16, wr, wf, wa, k, out);
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
    chosen[dev] = prepare_cluster_t<16>() ? 16 : (prepare_cluster_t<8>() ? 8 : 0);
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
