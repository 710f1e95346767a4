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
// Two passes: logits (the HBM-bound pass over K), then the normalization
// (one thread per token; the logits are 1/16 of the keys' bytes at fp16).
//
// Bulk path (blocks of at most 32 KB whose KV-head count divides 8 and
// whose bs * hkv / 8 rows per warp is a power of two from 2 to 32: the
// eviction pool's fp16 / bf16 blocks of 8 heads x 16 tokens): persistent
// CTAs, two per SM, each with a producer warp that streams whole blocks --
// contiguous in the [nb, bs, hkv, 128] layout -- into a 3-stage
// shared-memory ring with one bulk copy per block, and 8 consumer warps,
// each owning one head's share of the block's token rows: dots with the
// query by a register reduce-scatter, and a running maximum per head.  Each CTA writes its per-head maxima to its own workspace row, so
// no reset precedes the launch; the normalization reduces the rows.
//
// Other shapes: one warp per (block, head) reading global memory directly,
// a 16-shuffle reduce-scatter for bs 16, and a running per-head maximum
// folded into one atomic per warp (after a reset of the maxima).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
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

// ---- bulk path ----------------------------------------------------------------
constexpr int kStatStages = 3;
constexpr int kStatConsumerWarps = 8;
constexpr int kStatThreads = (kStatConsumerWarps + 1) * 32;  // + the producer warp
constexpr uint32_t kStatMaxBlock = 32 * 1024;
constexpr int kStatMaxHeads = 8;  // a CTA's maxima row

// Consumer warp w owns head h = w % hkv and NV = bs * hkv / 8 consecutive
// token rows of every block.  Its NV row loads are issued together, each
// lane forms the 4-channel partial dot of every row, and a reduce-scatter
// over the lanes (each step halves the values a lane keeps, then butterfly
// steps finish the sum) leaves lane l with the full dot of one row: NV - 1
// + log2(32 / NV) shuffles for NV rows.
template <typename T, int NV>
__global__ void __launch_bounds__(kStatThreads, 2)
    attn_logits_bulk_kernel(const T* __restrict__ k, const float* __restrict__ q,
                            float* __restrict__ logits, float* __restrict__ cta_max, int64_t nb,
                            int bs, int hkv, float scale_log2, int* err) {
  static_assert(NV >= 2 && NV <= 32 && (NV & (NV - 1)) == 0, "rows per warp");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int64_t elems = (int64_t)bs * hkv * 128;
  const uint32_t block_bytes = (uint32_t)(elems * sizeof(T));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + kStatStages * block_bytes);
  uint64_t* empty = full + kStatStages;
  float* s_max = reinterpret_cast<float*>(empty + kStatStages);  // [kStatConsumerWarps]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kStatStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kStatConsumerWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kStatConsumerWarps) {  // producer
    if (lane == 0) {
      int n = 0;
      for (int64_t b = blockIdx.x; b < nb; b += gridDim.x, ++n) {
        const int st = n % kStatStages;
        if (!mbar_wait_bounded(&empty[st], ((uint32_t)(n / kStatStages) & 1u) ^ 1u, err)) {
          record_error(err, kDevWaitTimeout);
          break;
        }
        mbar_arrive_expect_tx(&full[st], block_bytes);
        bulk_load_g2s(smem_raw + st * block_bytes, k + b * elems, block_bytes, &full[st]);
      }
      drain_ring(full, kStatStages, n);  // no copy outlives the CTA
    }
    return;
  }

  const int h = warp % hkv;
  const int t0 = (warp / hkv) * NV;
  const int64_t row_stride = (int64_t)hkv * 128;
  // the row whose full dot this lane ends with, and whether it writes it
  int t_lane = 0;
#pragma unroll
  for (int half = NV / 2, bit = 16; half >= 1; half >>= 1, bit >>= 1)
    if (lane & bit) t_lane += half;
  const bool writer = (lane & (32 / NV - 1)) == 0;
  float qv[4];
  load4f<float>(q + (int64_t)h * 128 + lane * 4, qv);
#pragma unroll
  for (int i = 0; i < 4; ++i) qv[i] *= scale_log2;
  float run = -INFINITY;
  bool live = true;
  int n = 0;
  for (int64_t b = blockIdx.x; b < nb; b += gridDim.x, ++n) {
    const int st = n % kStatStages;
    if (live && !mbar_wait_bounded(&full[st], (uint32_t)(n / kStatStages) & 1u, err)) {
      record_error(err, kDevWaitTimeout);
      live = false;
    }
    if (live) {
      const T* rows = reinterpret_cast<const T*>(smem_raw + st * block_bytes) +
                      (int64_t)t0 * row_stride + h * 128 + lane * 4;
      float v[NV];
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        float f[4];
        load4f<T>(rows + j * row_stride, f);
        v[j] = qv[0] * f[0] + qv[1] * f[1] + qv[2] * f[2] + qv[3] * f[3];
      }
#pragma unroll
      for (int half = NV / 2, bit = 16; half >= 1; half >>= 1, bit >>= 1) {
        const bool upper = (lane & bit) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float send = upper ? v[i] : v[i + half];
          const float keep = upper ? v[i + half] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
        }
      }
#pragma unroll
      for (int bit = 16 / NV; bit >= 1; bit >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], bit);
      if (writer) logits[(b * bs + t0 + t_lane) * hkv + h] = v[0];
      run = fmaxf(run, v[0]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  // this CTA's maxima row: lanes, then the warps of one head
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) run = fmaxf(run, __shfl_xor_sync(0xffffffffu, run, o));
  if (lane == 0) s_max[warp] = run;
  named_barrier(1, kStatConsumerWarps * 32);
  if (tid < kStatMaxHeads) {
    float m = -INFINITY;
    if (tid < hkv)
      for (int w = tid; w < kStatConsumerWarps; w += hkv) m = fmaxf(m, s_max[w]);
    cta_max[(int64_t)blockIdx.x * kStatMaxHeads + tid] = m;
  }
}

// Normalization against the maxima rows of n_rows CTAs: each CTA folds the
// rows into its shared memory first.
__global__ void __launch_bounds__(256)
    attn_normalize_rows_kernel(const float* __restrict__ logits,
                               const float* __restrict__ cta_max, int n_rows,
                               float* __restrict__ attn, int64_t tokens, int hkv) {
  __shared__ float s_red[8][kStatMaxHeads];
  __shared__ float s_m[kStatMaxHeads];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float m[kStatMaxHeads];
#pragma unroll
  for (int h = 0; h < kStatMaxHeads; ++h) m[h] = -INFINITY;
  for (int r = tid; r < n_rows; r += blockDim.x) {
    const float4 a = *reinterpret_cast<const float4*>(cta_max + (int64_t)r * kStatMaxHeads);
    const float4 c = *reinterpret_cast<const float4*>(cta_max + (int64_t)r * kStatMaxHeads + 4);
    m[0] = fmaxf(m[0], a.x); m[1] = fmaxf(m[1], a.y); m[2] = fmaxf(m[2], a.z);
    m[3] = fmaxf(m[3], a.w); m[4] = fmaxf(m[4], c.x); m[5] = fmaxf(m[5], c.y);
    m[6] = fmaxf(m[6], c.z); m[7] = fmaxf(m[7], c.w);
  }
#pragma unroll
  for (int h = 0; h < kStatMaxHeads; ++h) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m[h] = fmaxf(m[h], __shfl_xor_sync(0xffffffffu, m[h], o));
    if (lane == 0) s_red[warp][h] = m[h];
  }
  __syncthreads();
  if (tid < kStatMaxHeads) {
    float x = s_red[0][tid];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) x = fmaxf(x, s_red[w][tid]);
    s_m[tid] = x;
  }
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + tid; i < tokens;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int h = 0; h < hkv; ++h) s += exp2f(logits[i * hkv + h] - s_m[h]);
    attn[i] = s / (float)hkv;
  }
}

int sm_count_stats() {
  static int cached[64] = {0};
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] > 0) return cached[dev];
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  cached[dev] = n;
  return n;
}

// Launches the bulk logits kernel for NV rows per warp; the shared-memory
// limit of each instantiation is raised once per device.
template <typename T, int NV>
cudaError_t launch_bulk_nv(const T* k, const float* q, float* logits, float* cta_max, int64_t nb,
                           int bs, int hkv, float scale_log2, int ctas, size_t smem,
                           cudaStream_t stream) {
  static bool ready[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  auto kern = attn_logits_bulk_kernel<T, NV>;
  if (!ready[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)((size_t)kStatStages * kStatMaxBlock + 256));
    if (e != cudaSuccess) return e;
    ready[dev] = true;
  }
  kern<<<ctas, kStatThreads, smem, stream>>>(k, q, logits, cta_max, nb, bs, hkv, scale_log2,
                                             device_error_word());
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_bulk(const T* k, const float* q, float* logits, float* cta_max, int64_t nb,
                        int bs, int hkv, float scale_log2, int ctas, size_t smem,
                        cudaStream_t stream) {
  switch (bs * hkv / kStatConsumerWarps) {
    case 2: return launch_bulk_nv<T, 2>(k, q, logits, cta_max, nb, bs, hkv, scale_log2, ctas, smem, stream);
    case 4: return launch_bulk_nv<T, 4>(k, q, logits, cta_max, nb, bs, hkv, scale_log2, ctas, smem, stream);
    case 8: return launch_bulk_nv<T, 8>(k, q, logits, cta_max, nb, bs, hkv, scale_log2, ctas, smem, stream);
    case 16: return launch_bulk_nv<T, 16>(k, q, logits, cta_max, nb, bs, hkv, scale_log2, ctas, smem, stream);
    default: return launch_bulk_nv<T, 32>(k, q, logits, cta_max, nb, bs, hkv, scale_log2, ctas, smem, stream);
  }
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
  // logits, then the atomic maxima (other shapes) or one maxima row per CTA
  // of the bulk grid (at most 2 CTAs on each of 1,024 SMs)
  const size_t maxima = std::max<size_t>((size_t)num_kv_heads * sizeof(uint32_t),
                                         (size_t)2 * 1024 * kStatMaxHeads * sizeof(float));
  return (size_t)num_blocks * block_size * num_kv_heads * sizeof(float) + 256 + maxima + 256;
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
  const size_t esz = dtype == 0 ? 4 : 2;
  const uint64_t block_bytes = (uint64_t)block_size * num_kv_heads * 128 * esz;
  const int nv = block_size * num_kv_heads / kStatConsumerWarps;
  if (dtype >= 0 && dtype <= 2 && block_bytes <= kStatMaxBlock &&
      kStatMaxHeads % num_kv_heads == 0 && block_size * num_kv_heads % kStatConsumerWarps == 0 &&
      nv >= 2 && nv <= 32 && (nv & (nv - 1)) == 0 && reinterpret_cast<uintptr_t>(k) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(q) % 16 == 0 && std::getenv("PKV_ATTN_STATS_WARP") == nullptr) {
    const int ctas = (int)std::min<int64_t>(num_blocks, 2LL * std::min(sm_count_stats(), 1024));
    float* cta_max = reinterpret_cast<float*>(mx);
    const size_t smem = kStatStages * block_bytes + 2 * kStatStages * sizeof(uint64_t) +
                        kStatConsumerWarps * sizeof(float);
    const float scale_log2 = sm_scale * kLog2eStats;
    cudaError_t le;
    switch (dtype) {
      case 0: le = launch_bulk(static_cast<const float*>(k), q, logits, cta_max, num_blocks,
                               block_size, num_kv_heads, scale_log2, ctas, smem, stream); break;
      case 1: le = launch_bulk(static_cast<const __half*>(k), q, logits, cta_max, num_blocks,
                               block_size, num_kv_heads, scale_log2, ctas, smem, stream); break;
      default: le = launch_bulk(static_cast<const __nv_bfloat16*>(k), q, logits, cta_max,
                                num_blocks, block_size, num_kv_heads, scale_log2, ctas, smem,
                                stream); break;
    }
    if (le == cudaSuccess) {
      const int64_t tokens = num_blocks * block_size;
      const int64_t grid = std::min<int64_t>((tokens + 255) / 256, 4LL * sm_count_stats());
      attn_normalize_rows_kernel<<<(unsigned)grid, 256, 0, stream>>>(logits, cta_max, ctas, attn,
                                                                      tokens, num_kv_heads);
      le = cudaGetLastError();
    }
    if (le != cudaSuccess) {
      set_error(std::string("attention-stats launch failed: ") + cudaGetErrorString(le));
      return kCudaError;
    }
    return kOk;
  }
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
