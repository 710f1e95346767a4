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

#include <string>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {
namespace {

// ---------------------------------------------------------------------------
// Score
// ---------------------------------------------------------------------------

__device__ __forceinline__ float masked(const float* a, const uint8_t* m, int64_t i) {
  return m[i] ? a[i] : 0.0f;
}

// NumPy's pairwise float32 sum (see file header), on masked values.
__device__ float pairwise_masked_sum(const float* a, const uint8_t* m, int64_t n) {
  if (n < 8) {
    float r = 0.0f;
    for (int64_t i = 0; i < n; ++i) r = __fadd_rn(r, masked(a, m, i));
    return r;
  }
  if (n <= 128) {
    float r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = masked(a, m, j);
    int64_t i = 8;
    const int64_t stop = n - (n % 8);
    for (; i < stop; i += 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], masked(a, m, i + j));
    }
    float res = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                          __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
    for (; i < n; ++i) res = __fadd_rn(res, masked(a, m, i));
    return res;
  }
  // n > 128: split as NumPy does (first half rounded down to a multiple of
  // 8) and recurse, iteratively over the right spine to bound the stack.
  int64_t half = n / 2;
  half -= half % 8;
  return __fadd_rn(pairwise_masked_sum(a, m, half),
                   pairwise_masked_sum(a + half, m + half, n - half));
}

__device__ __forceinline__ float blend(float rec, float freq, float mean, float wr, float wf,
                                       float wa) {
  return __fadd_rn(__fadd_rn(__fmul_rn(wr, rec), __fmul_rn(wf, freq)), __fmul_rn(wa, mean));
}

// block_size 16: one thread per block, 4 x 16-byte attention loads and one
// 16-byte mask load.
__device__ __forceinline__ float score16(const float* attn, const uint8_t* valid, int64_t b,
                                         float rec, float freq, float wr, float wf, float wa) {
  const float4* ap = reinterpret_cast<const float4*>(attn + b * 16);
  const float4 x0 = ap[0], x1 = ap[1], x2 = ap[2], x3 = ap[3];
  const uint4 mw = *reinterpret_cast<const uint4*>(valid + b * 16);
  const float a[16] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w,
                       x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
  const uint32_t mws[4] = {mw.x, mw.y, mw.z, mw.w};
  float v[16];
  int nv = 0;
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const bool ok = ((mws[t >> 2] >> ((t & 3) * 8)) & 0xffu) != 0u;
    v[t] = ok ? a[t] : 0.0f;
    nv += ok;
  }
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(v[j], v[j + 8]);
  // NumPy reduces into an output initialised to 0.0, so the pairwise
  // result is added to +0.0 (only visible for an all -0.0 row).
  const float S = __fadd_rn(
      0.0f, __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                      __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7]))));
  const float mean = nv > 0 ? __fdiv_rn(S, (float)nv) : 0.0f;
  return blend(rec, freq, mean, wr, wf, wa);
}

__device__ __forceinline__ float score_generic(const float* attn, const uint8_t* valid,
                                               int64_t b, int bs, float rec, float freq,
                                               float wr, float wf, float wa) {
  const float* a = attn + b * bs;
  const uint8_t* m = valid + b * bs;
  int nv = 0;
  for (int t = 0; t < bs; ++t) nv += m[t] != 0;
  const float S = __fadd_rn(0.0f, pairwise_masked_sum(a, m, bs));
  const float mean = nv > 0 ? __fdiv_rn(S, (float)nv) : 0.0f;
  return blend(rec, freq, mean, wr, wf, wa);
}

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

int launch_select(const float* scores, const uint64_t* keys_in, int64_t n, int64_t k,
                  int64_t id_offset, int64_t* out_ids, uint64_t* out_keys, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream) {
  if (k > n) k = n;
  if (k <= 0) return kOk;
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

size_t fused_select_workspace_size(int64_t n, int64_t k) { return select_workspace_size(n, k); }

int launch_scores_select(const float* recency, const float* frequency, const float* attn,
                         const uint8_t* valid, float* scores, int64_t num_blocks,
                         int block_size, float w_r, float w_f, float w_a, int64_t k,
                         int64_t* out_ids, void* workspace, size_t workspace_bytes,
                         cudaStream_t stream) {
  if (k > num_blocks) k = num_blocks;
  const int64_t n_pad = next_pow2(num_blocks < 2 ? 2 : num_blocks);
  if (k > 0 && (workspace == nullptr || workspace_bytes < (size_t)n_pad * sizeof(uint64_t))) {
    set_error("workspace too small for fused eviction");
    return kWorkspace;
  }
  if (num_blocks == 0) return kOk;
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
