// KV-block eviction: fused per-block score and deterministic bottom-k.
//
// Score (pagedkv_fusion/reference.py:38-71), bit for bit with NumPy:
//   a[t]  = valid[b, t] ? attn[b, t] : +0.0f
//   S     = 0.0f + NumPy float32 pairwise sum of a[0:bs] (8 interleaved
//           partial sums, fixed tree, sequential tail, halving above 128
//           terms; the reduction output starts at +0.0)
//   mean  = S / n_valid (IEEE; equal to NumPy's float64 quotient rounded
//           to float32 because n_valid is exact and 53 >= 2*24 + 2), 0 if
//           the block has no valid token
//   score = (w_r*rec + w_f*freq) + w_a*mean, each op rounded, no FMA.
//
// Selection (reference.py:74-81): ascending (score, block id), -0.0 ==
// +0.0, NaN after every number.  Each block becomes the unique 64-bit key
// orderable(score) << 32 | id, so "the k smallest keys, ascending" is the
// reference's lexsort prefix exactly.  Keys are ordered by a bitonic
// network: small sets entirely in shared memory, larger ones with global
// merge steps between shared-memory passes.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "eviction_score.cuh"
#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {
namespace {

template <bool BS16>
__global__ void __launch_bounds__(256)
    eviction_score_kernel(const float* __restrict__ rec, const float* __restrict__ freq,
                          const float* __restrict__ attn, const uint8_t* __restrict__ valid,
                          float* __restrict__ scores, uint64_t* __restrict__ keys, int64_t n,
                          int64_t n_pad, int bs, float wr, float wf, float wa) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b < n) {
    const float s = BS16 ? score16(attn, valid, b, rec[b], freq[b], wr, wf, wa)
                         : score_generic(attn, valid, b, bs, rec[b], freq[b], wr, wf, wa);
    if (scores) scores[b] = s;
    if (keys) keys[b] = ((uint64_t)orderable_key(s) << 32) | (uint64_t)b;
  } else if (keys && b < n_pad) {
    keys[b] = ~0ull;
  }
}

// ---------------------------------------------------------------------------
// Keys
// ---------------------------------------------------------------------------

__global__ void make_keys_kernel(const float* __restrict__ scores,
                                 const uint64_t* __restrict__ keys_in, int64_t n, int64_t n_pad,
                                 uint64_t* __restrict__ keys) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_pad) return;
  if (i >= n)
    keys[i] = ~0ull;
  else if (keys_in)
    keys[i] = keys_in[i];
  else
    keys[i] = ((uint64_t)orderable_key(scores[i]) << 32) | (uint64_t)i;
}

// ---------------------------------------------------------------------------
// Bitonic network.  Sub-sequence direction for merge size `size` is
// ascending iff (global index & size) == 0, so the final pass (size =
// n_pad) is ascending everywhere.
// ---------------------------------------------------------------------------

constexpr int kTile = 2048;  // keys per shared-memory tile (16 KB)
constexpr int kTileThreads = 512;

__device__ __forceinline__ void cas(uint64_t& a, uint64_t& b, bool asc) {
  if ((a > b) == asc) {
    const uint64_t t = a;
    a = b;
    b = t;
  }
}

// Sorts each tile completely (sizes 2 .. tile) in shared memory.
__global__ void __launch_bounds__(kTileThreads)
    bitonic_tile_sort(uint64_t* __restrict__ keys, int tile) {
  extern __shared__ uint64_t s[];
  const int64_t base = (int64_t)blockIdx.x * tile;
  for (int i = threadIdx.x; i < tile; i += blockDim.x) s[i] = keys[base + i];
  __syncthreads();
  for (int size = 2; size <= tile; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int p = threadIdx.x; p < tile / 2; p += blockDim.x) {
        const int lo = 2 * stride * (p / stride) + (p % stride);
        const bool asc = ((base + lo) & size) == 0;
        cas(s[lo], s[lo + stride], asc);
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < tile; i += blockDim.x) keys[base + i] = s[i];
}

// Three global steps in one pass (strides s, s/2, s/4, all >= tile): each
// thread owns the eight keys lo + a * s/4 (a = 0 .. 7), closed under the
// three steps and in one 2s-aligned run (one direction).
__global__ void bitonic_global_step3(uint64_t* __restrict__ keys, int64_t n_pad, int64_t size,
                                     int64_t s) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n_pad / 8) return;
  const int64_t q = s / 4;
  const int64_t lo = 8 * q * (t / q) + (t % q);
  const bool asc = (lo & size) == 0;
  uint64_t v[8];
#pragma unroll
  for (int a = 0; a < 8; ++a) v[a] = keys[lo + a * q];
#pragma unroll
  for (int a = 0; a < 4; ++a) cas(v[a], v[a + 4], asc);  // stride s
  cas(v[0], v[2], asc);  // stride s/2
  cas(v[1], v[3], asc);
  cas(v[4], v[6], asc);
  cas(v[5], v[7], asc);
#pragma unroll
  for (int a = 0; a < 8; a += 2) cas(v[a], v[a + 1], asc);  // stride s/4
#pragma unroll
  for (int a = 0; a < 8; ++a) keys[lo + a * q] = v[a];
}

// Register form of the tile kernels: a warp holds 128 consecutive keys of
// the tile, key j of a thread at tile index warp * 128 + 32 * j + lane.
// Strides 64 and 32 pair a thread's own keys, strides 16 .. 1 pair lanes
// (shuffles); only strides >= 128 go through shared memory, so a 4,096-key
// tile sort takes 25 block barriers instead of 78.
constexpr int kWarpKeys = 128;

__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int m) {
  const unsigned int lo = __shfl_xor_sync(0xffffffffu, (unsigned int)v, m);
  const unsigned int hi = __shfl_xor_sync(0xffffffffu, (unsigned int)(v >> 32), m);
  return ((uint64_t)hi << 32) | lo;
}

// Steps of strides top .. 1 (top <= 64) of merge size `size`; g0 is the
// global index of the thread's key 0.
__device__ __forceinline__ void bitonic_reg_steps(uint64_t (&v)[4], int64_t g0, int64_t size,
                                                  int top, int lane) {
  if (top >= 64) {
    cas(v[0], v[2], (g0 & size) == 0);
    cas(v[1], v[3], ((g0 + 32) & size) == 0);
  }
  if (top >= 32) {
    cas(v[0], v[1], (g0 & size) == 0);
    cas(v[2], v[3], ((g0 + 64) & size) == 0);
  }
  for (int st = top < 16 ? top : 16; st >= 1; st >>= 1) {
    const bool lower = (lane & st) == 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint64_t y = shfl_xor_u64(v[j], st);
      const bool asc = ((g0 + 32 * j) & size) == 0;
      const bool take_min = lower == asc;
      v[j] = take_min ? (y < v[j] ? y : v[j]) : (y > v[j] ? y : v[j]);
    }
  }
}

// bitonic_tile_sort for tiles of at least 128 keys, tile / 4 threads.
__global__ void __launch_bounds__(kTileThreads)
    bitonic_tile_sort_reg(uint64_t* __restrict__ keys, int tile) {
  extern __shared__ uint64_t s[];
  const int64_t base = (int64_t)blockIdx.x * tile;
  const int lane = threadIdx.x & 31;
  const int t0 = (threadIdx.x >> 5) * kWarpKeys + lane;
  const int64_t g0 = base + t0;
  uint64_t v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = keys[g0 + 32 * j];
  for (int size = 2; size <= kWarpKeys && size <= tile; size <<= 1)
    bitonic_reg_steps(v, g0, size, size / 2, lane);
  if (tile > kWarpKeys) {
#pragma unroll
    for (int j = 0; j < 4; ++j) s[t0 + 32 * j] = v[j];
    __syncthreads();
    for (int size = 2 * kWarpKeys; size <= tile; size <<= 1) {
      for (int stride = size >> 1; stride >= kWarpKeys; stride >>= 1) {
        for (int p = threadIdx.x; p < tile / 2; p += blockDim.x) {
          const int lo = 2 * stride * (p / stride) + (p % stride);
          cas(s[lo], s[lo + stride], ((base + lo) & size) == 0);
        }
        __syncthreads();
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = s[t0 + 32 * j];
      bitonic_reg_steps(v, g0, size, kWarpKeys / 2, lane);
      if (size < tile) {
#pragma unroll
        for (int j = 0; j < 4; ++j) s[t0 + 32 * j] = v[j];
        __syncthreads();
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) keys[g0 + 32 * j] = v[j];
}

// Finishes merge size `size` (> tile) for strides tile/2 .. 1: the
// shared-memory strides, then the register ones (tile of at least 256 keys,
// tile / 4 threads).
__global__ void __launch_bounds__(kTileThreads)
    bitonic_tile_merge_reg(uint64_t* __restrict__ keys, int tile, int64_t size) {
  extern __shared__ uint64_t s[];
  const int64_t base = (int64_t)blockIdx.x * tile;
  for (int i = threadIdx.x; i < tile; i += blockDim.x) s[i] = keys[base + i];
  __syncthreads();
  const bool asc = (base & size) == 0;
  for (int stride = tile >> 1; stride >= kWarpKeys; stride >>= 1) {
    for (int p = threadIdx.x; p < tile / 2; p += blockDim.x) {
      const int lo = 2 * stride * (p / stride) + (p % stride);
      cas(s[lo], s[lo + stride], asc);
    }
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int t0 = (threadIdx.x >> 5) * kWarpKeys + lane;
  const int64_t g0 = base + t0;
  uint64_t v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = s[t0 + 32 * j];
  bitonic_reg_steps(v, g0, size, kWarpKeys / 2, lane);
#pragma unroll
  for (int j = 0; j < 4; ++j) keys[g0 + 32 * j] = v[j];
}

// One global compare-exchange step (stride >= tile).
__global__ void bitonic_global_step(uint64_t* __restrict__ keys, int64_t n_pad, int64_t size,
                                    int64_t stride) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n_pad / 2) return;
  const int64_t lo = 2 * stride * (p / stride) + (p % stride);
  const bool asc = (lo & size) == 0;
  uint64_t a = keys[lo], b = keys[lo + stride];
  if ((a > b) == asc) {
    keys[lo] = b;
    keys[lo + stride] = a;
  }
}

// Two global compare-exchange steps in one pass (strides s and s/2, both
// >= tile): each thread owns the quad lo, lo + s/2, lo + s, lo + 3s/2,
// which both steps touch only among themselves.  All four lie in one
// 2s-aligned run, so they share the direction.
__global__ void bitonic_global_step2(uint64_t* __restrict__ keys, int64_t n_pad, int64_t size,
                                     int64_t s) {
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= n_pad / 4) return;
  const int64_t h = s / 2;
  const int64_t lo = 2 * s * (q / h) + (q % h);
  const bool asc = (lo & size) == 0;
  uint64_t a = keys[lo], b = keys[lo + h], c = keys[lo + s], d = keys[lo + s + h];
  cas(a, c, asc);  // stride s
  cas(b, d, asc);
  cas(a, b, asc);  // stride s/2
  cas(c, d, asc);
  keys[lo] = a;
  keys[lo + h] = b;
  keys[lo + s] = c;
  keys[lo + s + h] = d;
}

__global__ void emit_kernel(const uint64_t* __restrict__ keys, int64_t k, int64_t id_offset,
                            int64_t* __restrict__ out_ids, uint64_t* __restrict__ out_keys) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= k) return;
  const uint64_t key = keys[i];
  if (out_ids) out_ids[i] = (int64_t)(key & 0xffffffffull);
  if (out_keys) out_keys[i] = key + (uint64_t)id_offset;
}

// ---------------------------------------------------------------------------
// Radix prefilter for large selections.  Up to four passes over 16-bit
// digits of the 64-bit keys (most significant first) find the prefix P of
// the k-th smallest key: each pass histograms the digit of the keys whose
// higher digits equal P, and the pass's last CTA appends the digit holding
// rank k-1 to P.  The search stops as soon as the keys at or below P number
// at most `cap` (for unique keys four digits always get there; the fourth
// pass stops it regardless).  Those keys
// -- the k smallest and possibly a few more -- are compacted and sorted, and
// the first k emitted: the same output as sorting everything.  Keys strictly
// below P fill the front of the candidate buffer (fewer than k of them) and
// keys equal to P the rest, stopping at `cap`: a caller's merge keys with
// more duplicates of the k-th key than fit still select exactly.
// ---------------------------------------------------------------------------

constexpr int kRadixBins = 1 << 16;
constexpr int kRadixScanThreads = 1024;

struct RadixState {
  unsigned long long prefix;  // digits found so far
  unsigned int below;         // keys below the prefix (their higher digits smaller)
  unsigned int depth;         // digits in the prefix
  unsigned int done;          // at most cap keys at or below the prefix
  unsigned int n_below;       // keys below the prefix compacted so far
  unsigned int n_equal;       // keys equal to the prefix compacted so far
  unsigned int arrived;       // CTAs of the current histogram pass that finished
};
static_assert(sizeof(RadixState) <= 256, "radix state outgrew its workspace slot");

__device__ void radix_scan_block(unsigned int* __restrict__ hist, RadixState* __restrict__ st,
                                 int64_t k, int64_t cap, int pass);

// End of a histogram pass (blocks of kRadixScanThreads threads): the last CTA
// to finish runs the scan.  Every CTA fences its counts before it arrives,
// so the last one reads the complete histogram from L2.  No CTA waits.
__device__ __forceinline__ void radix_scan_if_last(unsigned int* __restrict__ hist,
                                                   RadixState* __restrict__ st, int64_t k,
                                                   int64_t cap, int pass) {
  __shared__ unsigned int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&st->arrived, 1u) == gridDim.x - 1 ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;  // uniform
  __threadfence();
  radix_scan_block(hist, st, k, cap, pass);
  if (threadIdx.x == 0) st->arrived = 0u;  // for the next pass's kernel
}

// Digits 2-4 (pass >= 1): only keys whose higher digits equal the prefix
// count; returns at once when an earlier pass already stopped the search.
__global__ void __launch_bounds__(kRadixScanThreads)
    radix_hist_kernel(const uint64_t* __restrict__ keys, int64_t n, RadixState* __restrict__ st,
                      unsigned int* __restrict__ hist, int64_t k, int64_t cap, int pass) {
  if (st->done) return;  // uniform
  const int shift = 48 - 16 * pass;
  const unsigned long long prefix = st->prefix;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t key = keys[i];
    if ((key >> (shift + 16)) == prefix) atomicAdd(&hist[(key >> shift) & 0xFFFFu], 1u);
  }
  radix_scan_if_last(hist, st, k, cap, pass);
}

// First digit: every key counts, and uniform scores crowd a few hundred of
// the 65,536 bins, where global atomics would serialise.  Each CTA counts
// into shared memory instead -- two 16-bit counters per word, so the whole
// histogram is 128 KB -- and flushes only its nonzero bins.  A CTA sees at
// most kRadixHist0MaxKeys keys, so no 16-bit counter overflows.
constexpr int kRadixHist0Threads = 1024;
constexpr int kRadixHist0Keys = 63;  // keys per thread at most
constexpr int64_t kRadixHist0MaxKeys = (int64_t)kRadixHist0Keys * kRadixHist0Threads;
constexpr size_t kRadixHist0Smem = (kRadixBins / 2) * sizeof(unsigned int);
static_assert(kRadixHist0MaxKeys < 65536, "16-bit shared counters could overflow");

__global__ void __launch_bounds__(kRadixHist0Threads)
    radix_hist0_kernel(const uint64_t* __restrict__ keys, int64_t n, RadixState* __restrict__ st,
                       unsigned int* __restrict__ hist, int64_t k, int64_t cap) {
  extern __shared__ uint4 s_hist4[];
  unsigned int* s_hist = reinterpret_cast<unsigned int*>(s_hist4);
  for (int w = threadIdx.x; w < kRadixBins / 8; w += kRadixHist0Threads)
    s_hist4[w] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * kRadixHist0Threads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kRadixHist0Threads) {
    const unsigned int bin = (unsigned int)(keys[i] >> 48);
    atomicAdd(&s_hist[bin >> 1], (bin & 1u) ? 0x10000u : 1u);
  }
  __syncthreads();
  for (int w = threadIdx.x; w < kRadixBins / 2; w += kRadixHist0Threads) {
    const unsigned int v = s_hist[w];
    if (v & 0xFFFFu) atomicAdd(&hist[2 * w], v & 0xFFFFu);
    if (v >> 16) atomicAdd(&hist[2 * w + 1], v >> 16);
  }
  radix_scan_if_last(hist, st, k, cap, 0);
}

// Grid of radix_hist0_kernel: enough CTAs that none sees more than
// kRadixHist0MaxKeys keys, at least one per SM.
unsigned radix_hist0_grid(int64_t n) {
  const int64_t per_pass = kRadixHist0MaxKeys;
  const int64_t need = (n + per_pass - 1) / per_pass;
  return (unsigned)std::max<int64_t>(need, 148);
}

bool radix_hist0_prepare() {
  static bool ok[64];
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    ok[dev] = cudaFuncSetAttribute(radix_hist0_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kRadixHist0Smem) == cudaSuccess;
    cudaGetLastError();
    done[dev] = true;
  }
  return ok[dev];
}

// One CTA (the last of a histogram pass): the bin holding rank k-1 among the
// keys counted, appended to the prefix; the histogram is zeroed for the next
// pass.  The bins are read in
// kRadixScanRounds coalesced rounds of four per thread (one uint4), each
// round a block-wide scan on top of the previous rounds' total.
constexpr int kRadixScanRounds = kRadixBins / (4 * kRadixScanThreads);

__device__ __noinline__ void radix_scan_block(unsigned int* __restrict__ hist,
                                              RadixState* __restrict__ st, int64_t k, int64_t cap,
                                              int pass) {
  static_assert(kRadixHist0Threads == kRadixScanThreads, "the scan runs in a histogram CTA");
  __shared__ unsigned int s_warp[32];
  __shared__ unsigned int s_total;
  if (st->done) return;  // uniform
  // read before the one writing thread below can change them
  const unsigned int below = st->below;
  const unsigned long long prefix = st->prefix;
  const unsigned int target = (unsigned int)(k - 1) - below;  // rank among the counted keys
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint4* h4 = reinterpret_cast<uint4*>(hist);
  constexpr int kAhead = 8;  // rounds loaded ahead of the scan
  uint4 c[kAhead];
#pragma unroll
  for (int r = 0; r < kAhead; ++r) c[r] = __ldcg(&h4[r * kRadixScanThreads + tid]);
  unsigned int carry = 0;  // keys in the rounds before this one
#pragma unroll
  for (int r = 0; r < kRadixScanRounds; ++r) {
    const uint4 cur = c[r % kAhead];
    if (r + kAhead < kRadixScanRounds)
      c[r % kAhead] = __ldcg(&h4[(r + kAhead) * kRadixScanThreads + tid]);
    h4[r * kRadixScanThreads + tid] = make_uint4(0u, 0u, 0u, 0u);
    const unsigned int cnt[4] = {cur.x, cur.y, cur.z, cur.w};
    const unsigned int sum = cnt[0] + cnt[1] + cnt[2] + cnt[3];
    unsigned int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const unsigned int w = s_warp[lane];
      unsigned int x = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
      }
      s_warp[lane] = x - w;  // exclusive prefix of warp totals
      if (lane == 31) s_total = x;
    }
    __syncthreads();
    unsigned int run = carry + s_warp[warp] + incl - sum;  // keys in bins before mine
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (run <= target && target < run + cnt[j]) {  // exactly one bin holds the rank
        const unsigned int bin = (unsigned int)(r * 4 * kRadixScanThreads + 4 * tid + j);
        st->prefix = (prefix << 16) | (unsigned long long)bin;
        st->below = below + run;
        st->depth = (unsigned int)pass + 1;
        st->done = ((unsigned long long)below + run + cnt[j] <= (unsigned long long)cap ||
                    pass == 3) ? 1u : 0u;
      }
      run += cnt[j];
    }
    carry += s_total;
    __syncthreads();  // s_warp and s_total are rewritten next round
  }
}

// Compaction in chunks of kCompactThreads x kCompactPer keys: each CTA
// reserves its chunk's slots with one atomic per class (below / equal), so
// the two counters see a few thousand atomics instead of one per key.
constexpr int kCompactThreads = 256;
constexpr int kCompactPer = 4;

__device__ __forceinline__ unsigned int warp_incl_scan(unsigned int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

__global__ void __launch_bounds__(kCompactThreads)
    radix_compact_kernel(const uint64_t* __restrict__ keys, int64_t n, RadixState* __restrict__ st,
                         uint64_t* __restrict__ cand, int64_t cap) {
  constexpr int kWarps = kCompactThreads / 32;
  constexpr int64_t kChunk = (int64_t)kCompactThreads * kCompactPer;
  __shared__ unsigned int s_below[kWarps], s_equal[kWarps];
  __shared__ unsigned int s_base[2];
  const int shift = 64 - 16 * (int)st->depth;
  const unsigned long long prefix = st->prefix;
  const unsigned int below = st->below;  // < k <= cap
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t c0 = (int64_t)blockIdx.x * kChunk; c0 < n; c0 += (int64_t)gridDim.x * kChunk) {
    uint64_t key[kCompactPer];
    unsigned int cls = 0;  // 2 bits per key: 1 below, 2 equal
    unsigned int nb = 0, ne = 0;
#pragma unroll
    for (int j = 0; j < kCompactPer; ++j) {
      const int64_t i = c0 + (int64_t)j * kCompactThreads + tid;
      key[j] = i < n ? keys[i] : 0ull;
      const unsigned long long p = key[j] >> shift;
      const unsigned int c = i >= n ? 0u : (p < prefix ? 1u : (p == prefix ? 2u : 0u));
      cls |= c << (2 * j);
      nb += c == 1u;
      ne += c == 2u;
    }
    const unsigned int ib = warp_incl_scan(nb, lane), ie = warp_incl_scan(ne, lane);
    if (lane == 31) {
      s_below[warp] = ib;
      s_equal[warp] = ie;
    }
    __syncthreads();
    if (tid == 0) {
      unsigned int tb = 0, te = 0;
      for (int w = 0; w < kWarps; ++w) {
        const unsigned int b = s_below[w], e = s_equal[w];
        s_below[w] = tb;
        s_equal[w] = te;
        tb += b;
        te += e;
      }
      s_base[0] = tb ? atomicAdd(&st->n_below, tb) : 0u;
      s_base[1] = te ? atomicAdd(&st->n_equal, te) : 0u;
    }
    __syncthreads();
    unsigned int ob = s_base[0] + s_below[warp] + ib - nb;
    unsigned int oe = below + s_base[1] + s_equal[warp] + ie - ne;
#pragma unroll
    for (int j = 0; j < kCompactPer; ++j) {
      const unsigned int c = (cls >> (2 * j)) & 3u;
      if (c == 1u) {
        cand[ob++] = key[j];
      } else if (c == 2u) {
        if (oe < (unsigned long long)cap) cand[oe] = key[j];
        ++oe;
      }
    }
    __syncthreads();  // the shared counters are rewritten next chunk
  }
}

// PKV_EVICTION_MULTI_KERNEL=1 selects the multi-kernel sort for every size
// (used to cross-check the two paths).
bool force_multi_kernel() {
  const char* v = std::getenv("PKV_EVICTION_MULTI_KERNEL");
  return v != nullptr && v[0] == '1';
}

int64_t next_pow2(int64_t n) {
  int64_t p = 2;
  while (p < n) p <<= 1;
  return p;
}

unsigned blocks_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + " launch failed: " + cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

// Sorts keys[0 .. n_pad) ascending (n_pad a power of two).
int sort_keys(uint64_t* keys, int64_t n_pad, cudaStream_t stream) {
  const int tile = (int)(n_pad < kTile ? n_pad : kTile);
  const int threads = tile / 2 < kTileThreads ? tile / 2 : kTileThreads;
  const size_t smem = (size_t)tile * sizeof(uint64_t);
  static_assert(kTile / 4 == kTileThreads, "register tile kernels: four keys per thread");
  if (tile >= kWarpKeys)
    bitonic_tile_sort_reg<<<(unsigned)(n_pad / tile), tile / 4, smem, stream>>>(keys, tile);
  else
    bitonic_tile_sort<<<(unsigned)(n_pad / tile), threads, smem, stream>>>(keys, tile);
  for (int64_t size = (int64_t)tile * 2; size <= n_pad; size <<= 1) {
    for (int64_t stride = size / 2; stride >= tile;) {
      if (stride / 4 >= tile) {
        bitonic_global_step3<<<blocks_for(n_pad / 8, 256), 256, 0, stream>>>(keys, n_pad, size,
                                                                              stride);
        stride >>= 3;
      } else if (stride / 2 >= tile) {
        bitonic_global_step2<<<blocks_for(n_pad / 4, 256), 256, 0, stream>>>(keys, n_pad, size,
                                                                              stride);
        stride >>= 2;
      } else {
        bitonic_global_step<<<blocks_for(n_pad / 2, 256), 256, 0, stream>>>(keys, n_pad, size,
                                                                             stride);
        stride >>= 1;
      }
    }
    bitonic_tile_merge_reg<<<(unsigned)(n_pad / tile), tile / 4, smem, stream>>>(keys, tile, size);
  }
  return check_launch("bitonic sort");
}

// PKV_EVICTION_RADIX=0 turns the radix prefilter off (every selection then
// sorts all keys); read once per process so the workspace sizes stay fixed.
bool radix_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("PKV_EVICTION_RADIX");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

// The radix prefilter pays off above kRadixMinKeys keys when the sorted
// candidates (a power of two >= k + 1,024) are a small enough part of the
// padded keys: an eighth up to 2^16 padded keys, a quarter below 2^20, half
// from 2^20 on (where each merge level the full sort adds costs more than
// the prefilter's passes).
constexpr int64_t kRadixMinKeys = 16384;
int64_t radix_cap(int64_t n, int64_t k) {
  if (n <= kRadixMinKeys || k <= 0 || !radix_enabled()) return 0;
  const int64_t cap = next_pow2(k + 1024);
  const int64_t n_pad = next_pow2(n);
  const int64_t ratio = n_pad >= (int64_t(1) << 20) ? 2 : (n_pad > 65536 ? 4 : 8);
  return cap * ratio <= n_pad ? cap : 0;
}

// Workspace of the radix path after the n_pad keys: 16 bytes of alignment
// slack, cap candidates, the histogram, the state.
size_t radix_extra_bytes(int64_t cap) {
  return 16 + (size_t)cap * sizeof(uint64_t) + kRadixBins * sizeof(unsigned int) + 256;
}

// keys[0 .. n) hold the keys (n_pad >= n of them); emits the k smallest,
// ascending.  `extra` is the radix workspace when radix_cap(n, k) > 0.
int select_sorted(uint64_t* keys, int64_t n, int64_t n_pad, int64_t k, int64_t id_offset,
                  int64_t* out_ids, uint64_t* out_keys, uint8_t* extra, cudaStream_t stream) {
  const int64_t cap = radix_cap(n, k);
  uint64_t* sorted = keys;
  if (cap > 0) {
    extra = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(extra) + 15) & ~uintptr_t(15));
    uint64_t* cand = reinterpret_cast<uint64_t*>(extra);  // cap * 8 bytes: hist stays 16-aligned
    unsigned int* hist = reinterpret_cast<unsigned int*>(extra + cap * sizeof(uint64_t));
    RadixState* st = reinterpret_cast<RadixState*>(extra + cap * sizeof(uint64_t) +
                                                   kRadixBins * sizeof(unsigned int));
    cudaError_t e = cudaMemsetAsync(hist, 0, kRadixBins * sizeof(unsigned int) + sizeof(RadixState),
                                    stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(cand, 0xFF, cap * sizeof(uint64_t), stream);
    if (e != cudaSuccess) {
      set_error(std::string("eviction select reset failed: ") + cudaGetErrorString(e));
      return kCudaError;
    }
    const unsigned grid = (unsigned)std::min<int64_t>(blocks_for(n, kRadixScanThreads), 2 * 148);
    if (!radix_hist0_prepare()) {
      set_error("eviction select: radix histogram shared memory refused");
      return kCudaError;
    }
    // each pass ends with the scan in its last CTA
    radix_hist0_kernel<<<radix_hist0_grid(n), kRadixHist0Threads, kRadixHist0Smem, stream>>>(
        keys, n, st, hist, k, cap);
    for (int pass = 1; pass < 4; ++pass)
      radix_hist_kernel<<<grid, kRadixScanThreads, 0, stream>>>(keys, n, st, hist, k, cap, pass);
    radix_compact_kernel<<<(unsigned)std::min<int64_t>(
                               blocks_for(n, kCompactThreads * kCompactPer), 4 * 148),
                           kCompactThreads, 0, stream>>>(keys, n, st, cand, cap);
    const int rc = check_launch("eviction radix prefilter");
    if (rc != kOk) return rc;
    sorted = cand;
    n_pad = cap;
  }
  int rc = sort_keys(sorted, n_pad, stream);
  if (rc != kOk) return rc;
  emit_kernel<<<blocks_for(k, 256), 256, 0, stream>>>(sorted, k, id_offset, out_ids, out_keys);
  return check_launch("eviction emit");
}

}  // namespace

int launch_eviction_scores(const float* recency, const float* frequency, const float* attn,
                           const uint8_t* valid, float* scores, int64_t num_blocks,
                           int block_size, float w_r, float w_f, float w_a,
                           cudaStream_t stream) {
  if (num_blocks == 0) return kOk;
  const bool fast16 = block_size == 16 && reinterpret_cast<uintptr_t>(attn) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(valid) % 16 == 0;
  const unsigned grid = blocks_for(num_blocks, 256);
  if (fast16)
    eviction_score_kernel<true><<<grid, 256, 0, stream>>>(recency, frequency, attn, valid, scores,
                                                          nullptr, num_blocks, num_blocks, 16, w_r,
                                                          w_f, w_a);
  else
    eviction_score_kernel<false><<<grid, 256, 0, stream>>>(recency, frequency, attn, valid,
                                                           scores, nullptr, num_blocks,
                                                           num_blocks, block_size, w_r, w_f, w_a);
  return check_launch("eviction score");
}

size_t select_workspace_size(int64_t n, int64_t k) {
  const size_t keys = (size_t)next_pow2(n < 2 ? 2 : n) * sizeof(uint64_t);
  const int64_t cap = radix_cap(n, k < n ? k : n);
  return cap > 0 ? keys + radix_extra_bytes(cap) : keys;
}

// Selections of at most 16,384 scores run in one cluster launch with no
// workspace when this device can schedule the cluster.
static size_t select_workspace_size_for_call(int64_t n, int64_t k) {
  if (k > 0 && n <= cluster_select_max_blocks() && !force_multi_kernel() &&
      cluster_select_available())
    return 0;
  return select_workspace_size(n, k);
}

int launch_select(const float* scores, const uint64_t* keys_in, int64_t n, int64_t k,
                  int64_t id_offset, int64_t* out_ids, uint64_t* out_keys, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream) {
  if (k > n) k = n;
  if (k <= 0) return kOk;
  if (scores != nullptr && keys_in == nullptr && out_keys == nullptr && id_offset == 0 &&
      n <= cluster_select_max_blocks() && !force_multi_kernel()) {
    const int rc = launch_cluster_select(nullptr, nullptr, nullptr, nullptr, scores, nullptr, n,
                                         0, 0.f, 0.f, 0.f, k, out_ids, stream);
    if (rc != kUnsupported) return rc;
  }
  const int64_t n_pad = next_pow2(n);
  if (workspace == nullptr || workspace_bytes < select_workspace_size(n, k)) {
    set_error("workspace too small for eviction select");
    return kWorkspace;
  }
  uint64_t* keys = static_cast<uint64_t*>(workspace);
  make_keys_kernel<<<blocks_for(n_pad, 256), 256, 0, stream>>>(scores, keys_in, n, n_pad, keys);
  return select_sorted(keys, n, n_pad, k, id_offset, out_ids, out_keys,
                       static_cast<uint8_t*>(workspace) + n_pad * sizeof(uint64_t), stream);
}

size_t fused_select_workspace_size(int64_t n, int64_t k) {
  return select_workspace_size_for_call(n, k);
}

size_t scores_select_workspace_size(int64_t n, int64_t k) {
  return select_workspace_size_for_call(n, k);
}

int launch_scores_select(const float* recency, const float* frequency, const float* attn,
                         const uint8_t* valid, float* scores, int64_t num_blocks,
                         int block_size, float w_r, float w_f, float w_a, int64_t k,
                         int64_t* out_ids, void* workspace, size_t workspace_bytes,
                         cudaStream_t stream) {
  if (k > num_blocks) k = num_blocks;
  if (num_blocks == 0) return kOk;
  if (k > 0 && num_blocks <= cluster_select_max_blocks() && !force_multi_kernel()) {
    const int rc = launch_cluster_select(recency, frequency, attn, valid, nullptr, scores,
                                         num_blocks, block_size, w_r, w_f, w_a, k, out_ids,
                                         stream);
    if (rc != kUnsupported) return rc;
  }
  const int64_t n_pad = next_pow2(num_blocks < 2 ? 2 : num_blocks);
  if (k > 0 && (workspace == nullptr || workspace_bytes < select_workspace_size(num_blocks, k))) {
    set_error("workspace too small for fused eviction");
    return kWorkspace;
  }
  uint64_t* keys = k > 0 ? static_cast<uint64_t*>(workspace) : nullptr;
  const bool fast16 = block_size == 16 && reinterpret_cast<uintptr_t>(attn) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(valid) % 16 == 0;
  const unsigned grid = blocks_for(keys ? n_pad : num_blocks, 256);
  if (fast16)
    eviction_score_kernel<true><<<grid, 256, 0, stream>>>(recency, frequency, attn, valid, scores,
                                                          keys, num_blocks, n_pad, 16, w_r, w_f,
                                                          w_a);
  else
    eviction_score_kernel<false><<<grid, 256, 0, stream>>>(recency, frequency, attn, valid,
                                                           scores, keys, num_blocks, n_pad,
                                                           block_size, w_r, w_f, w_a);
  int rc = check_launch("eviction score");
  if (rc != kOk || k <= 0) return rc;
  return select_sorted(keys, num_blocks, n_pad, k, 0, out_ids, nullptr,
                       static_cast<uint8_t*>(workspace) + n_pad * sizeof(uint64_t), stream);
}

}  // namespace pkv
