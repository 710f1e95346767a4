// Per-(block, head) symmetric INT8 quantization of a paged KV tensor, and
// the scatter-quantize used by the vLLM-shaped cache writer.
//
// Numerics follow pagedkv_fusion/reference.py:88-105 bit for bit:
//   absmax = max |x| over (token, channel) of one (block, head)
//   scale  = absmax / 127.0f  (IEEE division), or 1.0f when absmax == 0
//   code   = clamp(rint_half_even(x / scale), -127, 127)   (IEEE division)
// A NaN anywhere in a (block, head) makes absmax NaN and the scale 1.0, as
// NumPy's NaN-propagating max does.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {
namespace {

constexpr int kQThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

__device__ __forceinline__ int quantize_one(float x, float scale) {
  float r = rintf(__fdiv_rn(x, scale));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return __float2int_rn(r);
}

// Loads 16 bytes as VEC values of T and widens them to float.
template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const T* p, float (&f)[VEC]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < VEC; ++i) f[i] = to_f32<T>(e[i]);
}

// One CTA per physical block.  Rows (token, head) of head_dim values are
// handed to warps; pass 1 reduces |x| per head into shared memory, pass 2
// re-reads the block (now L2-resident) and writes the codes.
template <typename T, bool VECTOR>
__global__ void __launch_bounds__(kQThreads)
    quantize_kernel(const T* __restrict__ kv, int8_t* __restrict__ q, float* __restrict__ scale,
                    int bs, int hkv, int hd) {
  constexpr int VEC = 16 / sizeof(T);
  extern __shared__ uint32_t s_amax[];  // [hkv] float bits, then reused as scales
  const int64_t b = blockIdx.x;
  const int64_t elems = (int64_t)bs * hkv * hd;
  const T* src = kv + b * elems;
  int8_t* dst = q + b * elems;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = kQThreads / 32;
  const int rows = bs * hkv;
  for (int h = threadIdx.x; h < hkv; h += kQThreads) s_amax[h] = 0u;
  __syncthreads();

  for (int r = warp; r < rows; r += nwarps) {
    const T* row = src + (int64_t)r * hd;
    uint32_t m = 0u;
    if constexpr (VECTOR) {
      for (int j = lane; j < hd / VEC; j += 32) {
        float f[VEC];
        load_vec<T, VEC>(row + j * VEC, f);
#pragma unroll
        for (int i = 0; i < VEC; ++i) m = max(m, __float_as_uint(f[i]) & 0x7fffffffu);
      }
    } else {
      for (int j = lane; j < hd; j += 32)
        m = max(m, __float_as_uint(to_f32<T>(row[j])) & 0x7fffffffu);
    }
    m = __reduce_max_sync(0xffffffffu, m);  // NaN bits exceed +inf: NaN wins
    if (lane == 0) atomicMax(&s_amax[r % hkv], m);
  }
  __syncthreads();
  float* s_scale = reinterpret_cast<float*>(s_amax);
  for (int h = threadIdx.x; h < hkv; h += kQThreads) {
    const float amax = __uint_as_float(s_amax[h]);
    const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    s_scale[h] = s;
    scale[b * hkv + h] = s;
  }
  __syncthreads();

  for (int r = warp; r < rows; r += nwarps) {
    const T* row = src + (int64_t)r * hd;
    int8_t* orow = dst + (int64_t)r * hd;
    const float s = s_scale[r % hkv];
    if constexpr (VECTOR) {
      for (int j = lane; j < hd / VEC; j += 32) {
        float f[VEC];
        load_vec<T, VEC>(row + j * VEC, f);
        uint32_t w[VEC / 4];
#pragma unroll
        for (int i = 0; i < VEC / 4; ++i)
          w[i] = (uint32_t)(quantize_one(f[4 * i], s) & 255) |
                 ((uint32_t)(quantize_one(f[4 * i + 1], s) & 255) << 8) |
                 ((uint32_t)(quantize_one(f[4 * i + 2], s) & 255) << 16) |
                 ((uint32_t)(quantize_one(f[4 * i + 3], s) & 255) << 24);
        if constexpr (VEC == 4) {
          *reinterpret_cast<uint32_t*>(orow + j * VEC) = w[0];
        } else {
          *reinterpret_cast<uint2*>(orow + j * VEC) = make_uint2(w[0], w[1]);
        }
      }
    } else {
      for (int j = lane; j < hd; j += 32) orow[j] = (int8_t)quantize_one(to_f32<T>(row[j]), s);
    }
  }
}

// head_dim 128: one warp per (block, kv head).  Lane l holds channels
// 4l .. 4l+3 of all BS tokens in registers (BS independent loads in flight),
// so the block is read once: warp max -> scale -> codes, no shared memory.
template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&f)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&f)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}
template <>
__device__ __forceinline__ void load4<__half>(const __half* p, float (&f)[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

template <typename T, int BS>
__global__ void __launch_bounds__(kQThreads)
    quantize_d128_kernel(const T* __restrict__ kv, int8_t* __restrict__ q,
                         float* __restrict__ scale, int64_t units, int hkv) {
  const int lane = threadIdx.x & 31;
  const int64_t unit = (int64_t)blockIdx.x * (kQThreads / 32) + (threadIdx.x >> 5);
  if (unit >= units) return;  // whole warp
  const int64_t b = unit / hkv;
  const int h = (int)(unit - b * hkv);
  const int64_t tok_stride = (int64_t)hkv * 128;
  const int64_t base = (b * BS * hkv + h) * 128 + lane * 4;
  float v[BS][4];
  uint32_t m = 0u;
#pragma unroll
  for (int t = 0; t < BS; ++t) {
    load4<T>(kv + base + t * tok_stride, v[t]);
#pragma unroll
    for (int i = 0; i < 4; ++i) m = max(m, __float_as_uint(v[t][i]) & 0x7fffffffu);
  }
  m = __reduce_max_sync(0xffffffffu, m);  // NaN bits exceed +inf: NaN wins
  const float amax = __uint_as_float(m);
  const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  if (lane == 0) scale[unit] = s;
#pragma unroll
  for (int t = 0; t < BS; ++t) {
    const uint32_t w = (uint32_t)(quantize_one(v[t][0], s) & 255) |
                       ((uint32_t)(quantize_one(v[t][1], s) & 255) << 8) |
                       ((uint32_t)(quantize_one(v[t][2], s) & 255) << 16) |
                       ((uint32_t)(quantize_one(v[t][3], s) & 255) << 24);
    *reinterpret_cast<uint32_t*>(q + base + t * tok_stride) = w;
  }
}

template <typename T>
int launch_quantize_t(const T* kv, int8_t* q, float* scale, int64_t nb, int bs, int hkv, int hd,
                      cudaStream_t stream) {
  constexpr int VEC = 16 / sizeof(T);
  if (hd == 128 && (bs == 16 || bs == 32) &&
      reinterpret_cast<uintptr_t>(kv) % (4 * sizeof(T)) == 0 &&
      reinterpret_cast<uintptr_t>(q) % 4 == 0) {
    const int64_t units = nb * hkv;
    const unsigned grid = (unsigned)((units + kQThreads / 32 - 1) / (kQThreads / 32));
    if (bs == 16)
      quantize_d128_kernel<T, 16><<<grid, kQThreads, 0, stream>>>(kv, q, scale, units, hkv);
    else
      quantize_d128_kernel<T, 32><<<grid, kQThreads, 0, stream>>>(kv, q, scale, units, hkv);
    return kOk;
  }
  const bool vec = hd % VEC == 0 && reinterpret_cast<uintptr_t>(kv) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(q) % VEC == 0;
  const size_t smem = (size_t)hkv * sizeof(uint32_t);
  if (vec)
    quantize_kernel<T, true><<<(unsigned)nb, kQThreads, smem, stream>>>(kv, q, scale, bs, hkv, hd);
  else
    quantize_kernel<T, false><<<(unsigned)nb, kQThreads, smem, stream>>>(kv, q, scale, bs, hkv, hd);
  return kOk;
}

// ---------------------------------------------------------------------------
// write_to_cache: the tokens of one call that land in the same physical
// block form one synthetic block (integration/vllm/pagedkv_fusion_backend.py
// :81-95): their per-head absmax sets a fresh scale that overwrites
// scale_cache[:, block], and only their slots receive codes.
// ---------------------------------------------------------------------------

// Pass 1: per-token, per-head absmax of K and V (float bits).
template <typename T>
__global__ void __launch_bounds__(128)
    token_absmax_kernel(const T* __restrict__ key, const T* __restrict__ value,
                        uint32_t* __restrict__ tok_amax, int hkv, int hd) {
  const int64_t t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = warp; r < 2 * hkv; r += 4) {
    const T* src = (r < hkv ? key : value) + (t * hkv + (r % hkv)) * (int64_t)hd;
    uint32_t m = 0u;
    for (int j = lane; j < hd; j += 32) m = max(m, __float_as_uint(to_f32<T>(src[j])) & 0x7fffffffu);
    m = __reduce_max_sync(0xffffffffu, m);
    if (lane == 0) tok_amax[t * 2 * hkv + r] = m;
  }
}

// Pass 2: one CTA per token.  The group absmax is the max over every token
// of this call mapped to the same block (a scan of slot_mapping, which is
// short: one decode step writes one token per sequence).
template <typename T>
__global__ void __launch_bounds__(128)
    scatter_quantize_kernel(const T* __restrict__ key, const T* __restrict__ value,
                            const int64_t* __restrict__ slots, const uint32_t* __restrict__ tok_amax,
                            int8_t* __restrict__ kv_cache, float* __restrict__ scale_cache,
                            int64_t num_tokens, int64_t num_blocks, int bs, int hkv, int hd,
                            int* err) {
  extern __shared__ float s_sc[];  // [2 * hkv]
  const int64_t t = blockIdx.x;
  const int64_t slot = slots[t];
  const int64_t total_slots = num_blocks * bs;
  if (slot < 0 || slot >= total_slots) {
    if (threadIdx.x == 0) record_error(err, kDevBadSlot);
    return;
  }
  const int64_t blk = slot / bs;
  const int off = (int)(slot % bs);
  for (int r = threadIdx.x; r < 2 * hkv; r += blockDim.x) {
    uint32_t m = 0u;
    bool first = true;
    for (int64_t u = 0; u < num_tokens; ++u) {
      const int64_t su = slots[u];
      if (su >= 0 && su < total_slots && su / bs == blk) {
        m = max(m, tok_amax[u * 2 * hkv + r]);
        if (u < t) first = false;
      }
    }
    const float amax = __uint_as_float(m);
    const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    s_sc[r] = s;
    // the first token of the group (lowest index) publishes the scale
    if (first) scale_cache[(r < hkv ? 0 : num_blocks * hkv) + blk * hkv + (r % hkv)] = s;
  }
  __syncthreads();
  const int64_t plane = num_blocks * bs * (int64_t)hkv * hd;
  for (int e = threadIdx.x; e < 2 * hkv * hd; e += blockDim.x) {
    const int r = e / hd, d = e % hd;
    const int kvh = r % hkv;
    const T* src = (r < hkv ? key : value) + (t * hkv + kvh) * (int64_t)hd + d;
    const int code = quantize_one(to_f32<T>(*src), s_sc[r]);
    kv_cache[(r < hkv ? 0 : plane) + ((blk * bs + off) * hkv + kvh) * (int64_t)hd + d] =
        (int8_t)code;
  }
}

template <typename T>
int launch_wtc_t(const T* key, const T* value, int8_t* kv_cache, float* scale_cache,
                 const int64_t* slots, int64_t nt, int64_t nb, int bs, int hkv, int hd,
                 uint32_t* tok_amax, cudaStream_t stream) {
  token_absmax_kernel<T><<<(unsigned)nt, 128, 0, stream>>>(key, value, tok_amax, hkv, hd);
  scatter_quantize_kernel<T><<<(unsigned)nt, 128, 2 * hkv * sizeof(float), stream>>>(
      key, value, slots, tok_amax, kv_cache, scale_cache, nt, nb, bs, hkv, hd,
      device_error_word());
  return kOk;
}

}  // namespace

int launch_quantize(const void* kv, int dtype, int8_t* q, float* scale, int64_t num_blocks,
                    int block_size, int num_kv_heads, int head_dim, cudaStream_t stream) {
  if (num_blocks == 0) return kOk;
  int rc;
  switch (dtype) {
    case 0: rc = launch_quantize_t(static_cast<const float*>(kv), q, scale, num_blocks, block_size,
                                   num_kv_heads, head_dim, stream); break;
    case 1: rc = launch_quantize_t(static_cast<const __half*>(kv), q, scale, num_blocks,
                                   block_size, num_kv_heads, head_dim, stream); break;
    case 2: rc = launch_quantize_t(static_cast<const __nv_bfloat16*>(kv), q, scale, num_blocks,
                                   block_size, num_kv_heads, head_dim, stream); break;
    default: set_error("unknown kv dtype code"); return kInvalidArgument;
  }
  if (rc != kOk) return rc;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("quantize launch failed: ") + cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

size_t write_to_cache_workspace_size(int64_t num_tokens, int num_kv_heads) {
  return (size_t)num_tokens * 2 * num_kv_heads * sizeof(uint32_t);
}

int launch_write_to_cache(const void* key, const void* value, int dtype, int8_t* kv_cache,
                          float* scale_cache, const int64_t* slot_mapping, int64_t num_tokens,
                          int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                          void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (num_tokens == 0) return kOk;
  if (workspace == nullptr ||
      workspace_bytes < write_to_cache_workspace_size(num_tokens, num_kv_heads)) {
    set_error("workspace too small for write_to_cache");
    return kWorkspace;
  }
  uint32_t* tok_amax = static_cast<uint32_t*>(workspace);
  int rc;
  switch (dtype) {
    case 0: rc = launch_wtc_t(static_cast<const float*>(key), static_cast<const float*>(value),
                              kv_cache, scale_cache, slot_mapping, num_tokens, num_blocks,
                              block_size, num_kv_heads, head_dim, tok_amax, stream); break;
    case 1: rc = launch_wtc_t(static_cast<const __half*>(key), static_cast<const __half*>(value),
                              kv_cache, scale_cache, slot_mapping, num_tokens, num_blocks,
                              block_size, num_kv_heads, head_dim, tok_amax, stream); break;
    case 2: rc = launch_wtc_t(static_cast<const __nv_bfloat16*>(key),
                              static_cast<const __nv_bfloat16*>(value), kv_cache, scale_cache,
                              slot_mapping, num_tokens, num_blocks, block_size, num_kv_heads,
                              head_dim, tok_amax, stream); break;
    default: set_error("unknown kv dtype code"); return kInvalidArgument;
  }
  if (rc != kOk) return rc;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("write_to_cache launch failed: ") + cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

}  // namespace pkv
