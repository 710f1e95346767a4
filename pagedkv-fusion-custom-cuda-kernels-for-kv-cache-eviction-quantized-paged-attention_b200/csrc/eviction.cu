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

#include <cstdlib>
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

constexpr int kTile = 4096;  // keys per shared-memory tile (32 KB)
constexpr int kTileThreads = 1024;

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

// Finishes merge size `size` for strides tile/2 .. 1 in shared memory.
__global__ void __launch_bounds__(kTileThreads)
    bitonic_tile_merge(uint64_t* __restrict__ keys, int tile, int64_t size) {
  extern __shared__ uint64_t s[];
  const int64_t base = (int64_t)blockIdx.x * tile;
  for (int i = threadIdx.x; i < tile; i += blockDim.x) s[i] = keys[base + i];
  __syncthreads();
  const bool asc = (base & size) == 0;
  for (int stride = tile >> 1; stride > 0; stride >>= 1) {
    for (int p = threadIdx.x; p < tile / 2; p += blockDim.x) {
      const int lo = 2 * stride * (p / stride) + (p % stride);
      cas(s[lo], s[lo + stride], asc);
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < tile; i += blockDim.x) keys[base + i] = s[i];
}

__global__ void emit_kernel(const uint64_t* __restrict__ keys, int64_t k, int64_t id_offset,
                            int64_t* __restrict__ out_ids, uint64_t* __restrict__ out_keys) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= k) return;
  const uint64_t key = keys[i];
  if (out_ids) out_ids[i] = (int64_t)(key & 0xffffffffull);
  if (out_keys) out_keys[i] = key + (uint64_t)id_offset;
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
  bitonic_tile_sort<<<(unsigned)(n_pad / tile), threads, smem, stream>>>(keys, tile);
  for (int64_t size = (int64_t)tile * 2; size <= n_pad; size <<= 1) {
    for (int64_t stride = size / 2; stride >= tile; stride >>= 1)
      bitonic_global_step<<<blocks_for(n_pad / 2, 256), 256, 0, stream>>>(keys, n_pad, size,
                                                                           stride);
    bitonic_tile_merge<<<(unsigned)(n_pad / tile), threads, smem, stream>>>(keys, tile, size);
  }
  return check_launch("bitonic sort");
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
  (void)k;
  return (size_t)next_pow2(n < 2 ? 2 : n) * sizeof(uint64_t);
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
  if (workspace == nullptr || workspace_bytes < (size_t)n_pad * sizeof(uint64_t)) {
    set_error("workspace too small for eviction select");
    return kWorkspace;
  }
  uint64_t* keys = static_cast<uint64_t*>(workspace);
  make_keys_kernel<<<blocks_for(n_pad, 256), 256, 0, stream>>>(scores, keys_in, n, n_pad, keys);
  int rc = sort_keys(keys, n_pad, stream);
  if (rc != kOk) return rc;
  emit_kernel<<<blocks_for(k, 256), 256, 0, stream>>>(keys, k, id_offset, out_ids, out_keys);
  return check_launch("eviction emit");
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
  if (k > 0 && (workspace == nullptr || workspace_bytes < (size_t)n_pad * sizeof(uint64_t))) {
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
  rc = sort_keys(keys, n_pad, stream);
  if (rc != kOk) return rc;
  emit_kernel<<<blocks_for(k, 256), 256, 0, stream>>>(keys, k, 0, out_ids, nullptr);
  return check_launch("eviction emit");
}

}  // namespace pkv
