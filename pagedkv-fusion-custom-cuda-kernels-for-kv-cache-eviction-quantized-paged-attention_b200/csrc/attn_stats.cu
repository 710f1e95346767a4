// Attention statistics derived from the keys: the per-token weights the
// eviction score reads (attn_weights[NB, bs]), produced from a K pool and one
// query vector per KV head instead of being supplied by the caller.  The
// reference has no such producer (its eviction inputs are given arrays,
// pagedkv_fusion/reference.py:38-71); the definition here is
//
//   s_h[b, t]  = sm_scale * (q_h . K[b, t, h, :])
//   attn[b, t] = mean_h exp(s_h[b, t] - max_{b', t'} s_h[b', t'])
//
// each token's weight relative to the pool's most-attended token, per KV
// head, averaged over heads: in (0, 1], like the reference's statistics.
//
// Two launches: logits (the HBM-bound pass over K: one warp per (block,
// head), lanes over channels, a 16-shuffle reduce-scatter for bs 16, and a
// running per-head maximum folded into one atomic per warp), then the
// normalization (one thread per token).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {
namespace {

constexpr float kLog2eStats = 1.4426950408889634f;

template <typename T>
__device__ __forceinline__ void load4f(const T* p, float (&f)[4]);
template <>
__device__ __forceinline__ void load4f<float>(const float* p, float (&f)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}
template <>
__device__ __forceinline__ void load4f<__half>(const __half* p, float (&f)[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
template <>
__device__ __forceinline__ void load4f<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

__device__ __forceinline__ uint32_t max_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float from_max_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Warp w handles head w % hkv and blocks w / hkv, w / hkv + W / hkv, ...
// (W, the warp count, is a multiple of hkv).  Lane l holds channels
// 4l..4l+3; each token's 32 lane partials are reduced so that lanes 2t and
// 2t + 1 end with token t (BS = 16) or lane t with token t (BS = 32).
template <typename T, int BS>
__global__ void __launch_bounds__(256)
    attn_logits_kernel(const T* __restrict__ k, const float* __restrict__ q,
                       float* __restrict__ logits, uint32_t* __restrict__ head_max, int64_t nb,
                       int hkv, float scale_log2) {
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t W = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int h = (int)(w % hkv);
  const int64_t per_head = W / hkv;
  float qv[4];
  load4f<float>(q + (int64_t)h * 128 + lane * 4, qv);
#pragma unroll
  for (int i = 0; i < 4; ++i) qv[i] *= scale_log2;
  float run = -INFINITY;
  for (int64_t b = w / hkv; b < nb; b += per_head) {
    float v[BS];
    const T* base = k + ((b * BS) * hkv + h) * 128 + lane * 4;
#pragma unroll
    for (int t = 0; t < BS; ++t) {
      float f[4];
      load4f<T>(base + (int64_t)t * hkv * 128, f);
      v[t] = qv[0] * f[0] + qv[1] * f[1] + qv[2] * f[2] + qv[3] * f[3];
    }
    // reduce-scatter: each step halves the values a lane keeps
#pragma unroll
    for (int half = BS / 2, bit = 16; half >= 1; half >>= 1, bit >>= 1) {
      const bool upper = (lane & bit) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = upper ? v[i] : v[i + half];
        const float keep = upper ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
      }
    }
    int t;
    if constexpr (BS == 32) {
      t = ((lane >> 4) & 1) << 4 | ((lane >> 3) & 1) << 3 | ((lane >> 2) & 1) << 2 |
          ((lane >> 1) & 1) << 1 | (lane & 1);
    } else {  // BS == 16: one more exchange completes the sum over 32 lanes
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
      t = ((lane >> 4) & 1) << 3 | ((lane >> 3) & 1) << 2 | ((lane >> 2) & 1) << 1 |
          ((lane >> 1) & 1);
    }
    if (BS == 32 || (lane & 1) == 0) logits[(b * BS + t) * hkv + h] = v[0];
    run = fmaxf(run, v[0]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) run = fmaxf(run, __shfl_xor_sync(0xffffffffu, run, o));
  if (lane == 0 && run != -INFINITY) atomicMax(&head_max[h], max_key(run));
}

__global__ void __launch_bounds__(256)
    attn_normalize_kernel(const float* __restrict__ logits, const uint32_t* __restrict__ head_max,
                          float* __restrict__ attn, int64_t tokens, int hkv) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= tokens) return;
  float s = 0.0f;
  for (int h = 0; h < hkv; ++h)
    s += exp2f(logits[i * hkv + h] - from_max_key(head_max[h]));
  attn[i] = s / (float)hkv;
}

int sm_count_stats() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

template <typename T>
int launch_stats_t(const T* k, const float* q, float* attn, int64_t nb, int bs, int hkv,
                   float sm_scale, float* logits, uint32_t* head_max, cudaStream_t stream) {
  // all resident CTAs, the grid a multiple of hkv / gcd(hkv, 8)
  // so that the warp count (grid x 8) is a multiple of hkv
  constexpr int cta = 256;
  int g = hkv, a = 8;
  while (a != 0) {
    const int r = g % a;
    g = a;
    a = r;
  }
  const int64_t unit = hkv / g;
  // every resident CTA slot: each warp keeps one (block, head) of loads in
  // flight, so occupancy is the queue depth
  int per_sm = 0;
  if (bs == 16)
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_logits_kernel<T, 16>, cta, 0);
  else
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_logits_kernel<T, 32>, cta, 0);
  const int64_t want = (int64_t)std::max(per_sm, 1) * sm_count_stats();
  const unsigned grid = (unsigned)std::max<int64_t>(unit, want / unit * unit);
  const float scale_log2 = sm_scale * kLog2eStats;
  if (bs == 16)
    attn_logits_kernel<T, 16><<<grid, cta, 0, stream>>>(k, q, logits, head_max, nb, hkv, scale_log2);
  else
    attn_logits_kernel<T, 32><<<grid, cta, 0, stream>>>(k, q, logits, head_max, nb, hkv, scale_log2);
  const int64_t tokens = nb * bs;
  attn_normalize_kernel<<<(unsigned)((tokens + 255) / 256), 256, 0, stream>>>(logits, head_max,
                                                                             attn, tokens, hkv);
  return kOk;
}

}  // namespace

size_t attention_stats_workspace_size(int64_t num_blocks, int block_size, int num_kv_heads) {
  return (size_t)num_blocks * block_size * num_kv_heads * sizeof(float) + 256 +
         (size_t)num_kv_heads * sizeof(uint32_t) + 256;
}

int launch_attention_stats(const void* k, int dtype, const float* q, float* attn,
                           int64_t num_blocks, int block_size, int num_kv_heads, float sm_scale,
                           void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (num_blocks == 0) return kOk;
  const size_t need = attention_stats_workspace_size(num_blocks, block_size, num_kv_heads);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("workspace too small for attention statistics: need " + std::to_string(need) +
              " bytes");
    return kWorkspace;
  }
  uintptr_t base = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~(uintptr_t)255;
  float* logits = reinterpret_cast<float*>(base);
  uintptr_t mx = (base + (size_t)num_blocks * block_size * num_kv_heads * sizeof(float) + 255) &
                 ~(uintptr_t)255;
  uint32_t* head_max = reinterpret_cast<uint32_t*>(mx);
  cudaError_t e = cudaMemsetAsync(head_max, 0, (size_t)num_kv_heads * sizeof(uint32_t), stream);
  if (e != cudaSuccess) {
    set_error(std::string("attention-stats reset failed: ") + cudaGetErrorString(e));
    return kCudaError;
  }
  int rc;
  switch (dtype) {
    case 0: rc = launch_stats_t(static_cast<const float*>(k), q, attn, num_blocks, block_size,
                                num_kv_heads, sm_scale, logits, head_max, stream); break;
    case 1: rc = launch_stats_t(static_cast<const __half*>(k), q, attn, num_blocks, block_size,
                                num_kv_heads, sm_scale, logits, head_max, stream); break;
    case 2: rc = launch_stats_t(static_cast<const __nv_bfloat16*>(k), q, attn, num_blocks,
                                block_size, num_kv_heads, sm_scale, logits, head_max, stream);
            break;
    default: set_error("unknown key dtype code"); return kInvalidArgument;
  }
  if (rc != kOk) return rc;
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("attention-stats launch failed: ") + cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

}  // namespace pkv
