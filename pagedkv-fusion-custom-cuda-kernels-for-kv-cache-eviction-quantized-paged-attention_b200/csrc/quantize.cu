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

#include <algorithm>
#include <cstdlib>
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

// Four int8 codes packed little-endian, by exact division (the rare path of
// quantize_word, kept out of line so the hot loops stay small).
__device__ __noinline__ uint32_t quantize_word_exact(float x0, float x1, float x2, float x3,
                                                     float scale) {
  return (uint32_t)(quantize_one(x0, scale) & 255) |
         ((uint32_t)(quantize_one(x1, scale) & 255) << 8) |
         ((uint32_t)(quantize_one(x2, scale) & 255) << 16) |
         ((uint32_t)(quantize_one(x3, scale) & 255) << 24);
}

// Two fp32 lanes in one 64-bit register, for Blackwell's packed f32x2
// arithmetic (each lane rounded exactly like the scalar instruction).
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Four codes packed little-endian.  Fast path, for a head whose absmax is
// finite and whose scale has a finite reciprocal rcp = 1/scale (rounded to
// nearest): y = x * rcp differs from fl(x/scale) by at most
// 1.5 * 2^-23 * |x/scale| <= 2^-15.5, because |x| <= absmax keeps
// |x/scale| <= 127 * (1 + 2^-24).  With d = 2^-15 and K = 1.5 * 2^23:
// y - d and y + d are exact (|y| < 128, whose ulp is at most 2^-17), and
// adding K rounds each to an integer half-to-even, left two's complement in
// the low mantissa bits.  If both round to the same integer, no half-integer
// lies in [y - d, y + d], so every value within 2^-15.5 of y -- fl(x/scale)
// among them -- rounds to that integer too, and it is the code.  Otherwise
// (about 2.4e-4 of words) the exact division decides.  |y| < 127.5, so the
// clamp to [-127, 127] never binds.  Heads with a non-finite absmax, or a
// scale below 2^-128 (reciprocal overflows), take the exact division.  The
// arithmetic runs two values per instruction (f32x2), which matters: the
// bulk quantizer is bound by instruction issue, not by HBM.
__device__ __forceinline__ uint32_t quantize_word(const float (&f)[4], float scale, float rcp,
                                                  bool fast) {
  if (fast) {
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
    constexpr float kWin = 0x1p-15f;
    const uint64_t r2 = f32x2(rcp, rcp), k2 = f32x2(kRound, kRound), w2 = f32x2(kWin, kWin);
    const uint64_t y01 = mul_f32x2(f32x2(f[0], f[1]), r2);
    const uint64_t y23 = mul_f32x2(f32x2(f[2], f[3]), r2);
    const uint64_t hi01 = add_f32x2(add_f32x2(y01, w2), k2);
    const uint64_t lo01 = add_f32x2(sub_f32x2(y01, w2), k2);
    const uint64_t hi23 = add_f32x2(add_f32x2(y23, w2), k2);
    const uint64_t lo23 = add_f32x2(sub_f32x2(y23, w2), k2);
    if (((hi01 ^ lo01) | (hi23 ^ lo23)) == 0ull) {
      const uint32_t b0 = (uint32_t)hi01, b1 = (uint32_t)(hi01 >> 32);
      const uint32_t b2 = (uint32_t)hi23, b3 = (uint32_t)(hi23 >> 32);
      return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
    }
  }
  return quantize_word_exact(f[0], f[1], f[2], f[3], scale);
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
                    int bs, int hkv, int hd, const uint8_t* __restrict__ skip) {
  constexpr int VEC = 16 / sizeof(T);
  extern __shared__ uint32_t s_amax[];  // [hkv] float bits, then reused as scales
  const int64_t b = blockIdx.x;
  if (skip != nullptr && skip[b]) return;  // whole CTA: block left untouched
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
                         float* __restrict__ scale, int64_t units, int hkv,
                         const uint8_t* __restrict__ skip) {
  const int lane = threadIdx.x & 31;
  const int64_t unit = (int64_t)blockIdx.x * (kQThreads / 32) + (threadIdx.x >> 5);
  if (unit >= units) return;  // whole warp
  const int64_t b = unit / hkv;
  if (skip != nullptr && skip[b]) return;  // whole warp: block left untouched
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
  const float rcp = __frcp_rn(s);
  const bool fast = isfinite(amax) && !isinf(rcp);
#pragma unroll
  for (int t = 0; t < BS; ++t) {
    const uint32_t w = quantize_word(v[t], s, rcp, fast);
    *reinterpret_cast<uint32_t*>(q + base + t * tok_stride) = w;
  }
}

// head_dim 128, 16-token blocks of at most kBulkMaxBlock bytes (fp16/bf16
// with <= 9 KV heads, fp32 with <= 4): a persistent kernel streams whole
// blocks (contiguous in the [NB, bs, Hkv, D] layout) into a ring of shared
// memory stages with one cp.async.bulk each.  The 16 consumer warps take the
// blocks two at a time: every warp waits for both blocks of a pair -- so
// every warp passes every stage phase in order (a warp that skipped blocks
// could wait on a stage's next phase while the current one is incomplete
// and, the parities of phases k-1 and k+1 being equal, pass it early) --
// then warps 0-7 quantize the first block and warps 8-15 the second, one
// head per warp.  A stage is refilled only after all 16 warps released it
// (those not quantizing it after their own block, with a wait of their own
// on it), so no warp can still be waiting on a phase of a stage that has
// moved on.  Deep queues with few registers: the register kernel above
// keeps one block-head in flight per warp and its CTAs turn over every few
// microseconds.
constexpr int kBulkHalfWarps = 8;
constexpr int kBulkConsumerWarps = 2 * kBulkHalfWarps;
constexpr int kBulkThreads = kBulkConsumerWarps * 32 + 32;
constexpr uint32_t kBulkMaxBlock = 36 * 1024;
constexpr int kBulkMaxHeads = 9;
constexpr int kBulkStages = 3;

template <typename T>
__device__ __forceinline__ void load4_shared(const T* p, float (&f)[4]) {
  load4<T>(p, f);
}

// Bits of max |x| over a lane's four values of one row.  32-bit inputs: the
// float bits with the sign cleared (unsigned order = magnitude order, NaN
// above +inf).  16-bit inputs: |x| and a NaN-propagating max on the packed
// pair; the surviving pair is widened once per head (absmax_float_bits).
template <typename T>
__device__ __forceinline__ uint32_t absmax_bits4(const T* p);
template <>
__device__ __forceinline__ uint32_t absmax_bits4<float>(const float* p) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  return max(max(__float_as_uint(v.x) & 0x7fffffffu, __float_as_uint(v.y) & 0x7fffffffu),
             max(__float_as_uint(v.z) & 0x7fffffffu, __float_as_uint(v.w) & 0x7fffffffu));
}
template <>
__device__ __forceinline__ uint32_t absmax_bits4<__half>(const __half* p) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const __half2 m = __hmax2_nan(__habs2(*reinterpret_cast<const __half2*>(&v.x)),
                                __habs2(*reinterpret_cast<const __half2*>(&v.y)));
  return *reinterpret_cast<const uint32_t*>(&m);
}
template <>
__device__ __forceinline__ uint32_t absmax_bits4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 m =
      __hmax2_nan(__habs2(*reinterpret_cast<const __nv_bfloat162*>(&v.x)),
                  __habs2(*reinterpret_cast<const __nv_bfloat162*>(&v.y)));
  return *reinterpret_cast<const uint32_t*>(&m);
}
template <typename T>
__device__ __forceinline__ uint32_t absmax_fold(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t absmax_fold<float>(uint32_t a, uint32_t b) { return max(a, b); }
template <>
__device__ __forceinline__ uint32_t absmax_fold<__half>(uint32_t a, uint32_t b) {
  const __half2 m = __hmax2_nan(*reinterpret_cast<const __half2*>(&a),
                                *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&m);
}
template <>
__device__ __forceinline__ uint32_t absmax_fold<__nv_bfloat16>(uint32_t a, uint32_t b) {
  const __nv_bfloat162 m = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                       *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<const uint32_t*>(&m);
}
template <typename T>
__device__ __forceinline__ uint32_t absmax_float_bits(uint32_t m);
template <>
__device__ __forceinline__ uint32_t absmax_float_bits<float>(uint32_t m) { return m; }
template <>
__device__ __forceinline__ uint32_t absmax_float_bits<__half>(uint32_t m) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&m));
  return max(__float_as_uint(f.x) & 0x7fffffffu, __float_as_uint(f.y) & 0x7fffffffu);
}
template <>
__device__ __forceinline__ uint32_t absmax_float_bits<__nv_bfloat16>(uint32_t m) {
  const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&m));
  return max(__float_as_uint(f.x) & 0x7fffffffu, __float_as_uint(f.y) & 0x7fffffffu);
}

template <typename T>
__global__ void __launch_bounds__(kBulkThreads, 2)
    quantize_bulk_kernel(const T* __restrict__ kv, int8_t* __restrict__ q,
                         float* __restrict__ scale, int64_t nb, int hkv,
                         const uint8_t* __restrict__ skip, int* err) {
  constexpr int BS = 16;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int64_t elems = (int64_t)BS * hkv * 128;
  const uint32_t block_bytes = (uint32_t)(elems * sizeof(T));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + kBulkStages * block_bytes);
  uint64_t* empty = full + kBulkStages;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kBulkStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kBulkConsumerWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kBulkConsumerWarps) {  // producer
    if (lane == 0) {
      int n = 0;
      for (int64_t b = blockIdx.x; b < nb; b += gridDim.x) {
        if (skip != nullptr && skip[b]) continue;
        const int st = n % kBulkStages;
        const uint32_t ph = (uint32_t)(n / kBulkStages) & 1u;
        if (!mbar_wait_bounded(&empty[st], ph ^ 1u, err)) {
          record_error(err, kDevWaitTimeout);
          break;
        }
        mbar_arrive_expect_tx(&full[st], block_bytes);
        bulk_load_g2s(smem_raw + st * block_bytes, kv + b * elems, block_bytes, &full[st]);
        ++n;
      }
      drain_ring(full, kBulkStages, n);  // no copy outlives this warp
    }
    return;
  }

  const int half = warp / kBulkHalfWarps;  // which block of the pair
  const int h0 = warp % kBulkHalfWarps;    // heads h0, h0 + 8
  const int64_t tok = (int64_t)hkv * 128;
  bool live = true;
  int n = 0;  // blocks of this CTA consumed so far (skipped ones excluded)
  int64_t b = blockIdx.x;
  for (;;) {
    int64_t first = 0, second = 0;
    int cnt = 0;
    for (; cnt < 2 && b < nb; b += gridDim.x)
      if (skip == nullptr || !skip[b]) {
        if (cnt == 0) first = b; else second = b;
        ++cnt;
      }
    if (cnt == 0) break;
    // Every warp waits for both blocks of the pair and releases each after
    // its wait, so a stage is refilled only after all 16 warps have passed
    // its phase.  The warps quantizing the second block release the first
    // before quantizing (it landed first), so its stage refills as soon as
    // its own warps are done; the warps quantizing the first block do that
    // first and only then wait for the second, so no block waits for its
    // neighbour's arrival to start.
    auto release_other = [&]() {  // the pair's other block (the only one when cnt == 1)
      const int i = cnt == 2 ? (half ^ 1) : 0;
      const int st = (n + i) % kBulkStages;
      if (live && !mbar_wait_bounded(&full[st], (uint32_t)((n + i) / kBulkStages) & 1u, err)) {
        record_error(err, kDevWaitTimeout);
        live = false;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    };
    if (half == 1) release_other();
    if (half < cnt) {
      const int st = (n + half) % kBulkStages;
      if (live && !mbar_wait_bounded(&full[st], (uint32_t)((n + half) / kBulkStages) & 1u, err)) {
        record_error(err, kDevWaitTimeout);
        live = false;
      }
      const int64_t blk_id = half ? second : first;
      const T* blk = reinterpret_cast<const T*>(smem_raw + st * block_bytes);
      if (live) {
        for (int h = h0; h < hkv; h += kBulkHalfWarps) {
          const T* row0 = blk + (int64_t)h * 128 + lane * 4;
          uint32_t m = absmax_bits4<T>(row0);
#pragma unroll 5
          for (int t = 1; t < BS; ++t) m = absmax_fold<T>(m, absmax_bits4<T>(row0 + t * tok));
          m = __reduce_max_sync(0xffffffffu, absmax_float_bits<T>(m));  // NaN wins
          const float amax = __uint_as_float(m);
          const float sc = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
          if (lane == 0) scale[blk_id * hkv + h] = sc;
          const float rcp = __frcp_rn(sc);
          const bool fast = isfinite(amax) && !isinf(rcp);
          int8_t* out = q + blk_id * elems + (int64_t)h * 128 + lane * 4;
#pragma unroll 2
          for (int t = 0; t < BS; ++t) {
            float f[4];
            load4_shared<T>(row0 + t * tok, f);
            *reinterpret_cast<uint32_t*>(out + t * tok) = quantize_word(f, sc, rcp, fast);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (half == 0 && cnt == 2) release_other();
    n += cnt;
  }
}

int sm_count_quant() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

template <typename T>
int launch_quantize_t(const T* kv, int8_t* q, float* scale, int64_t nb, int bs, int hkv, int hd,
                      const uint8_t* skip, cudaStream_t stream) {
  constexpr int VEC = 16 / sizeof(T);
  const uint64_t block_bytes = (uint64_t)bs * hkv * hd * sizeof(T);
  if (hd == 128 && bs == 16 && block_bytes <= kBulkMaxBlock && hkv <= kBulkMaxHeads &&
      reinterpret_cast<uintptr_t>(kv) % 16 == 0 && reinterpret_cast<uintptr_t>(q) % 4 == 0 &&
      std::getenv("PKV_QUANTIZE_REGISTER") == nullptr) {
    const size_t smem = kBulkStages * block_bytes + 2 * kBulkStages * sizeof(uint64_t);
    auto kern = quantize_bulk_kernel<T>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int64_t ctas = std::min<int64_t>(nb, 2LL * sm_count_quant());
    kern<<<(unsigned)ctas, kBulkThreads, smem, stream>>>(kv, q, scale, nb, hkv, skip,
                                                          device_error_word());
    return kOk;
  }
  if (hd == 128 && (bs == 16 || bs == 32) &&
      reinterpret_cast<uintptr_t>(kv) % (4 * sizeof(T)) == 0 &&
      reinterpret_cast<uintptr_t>(q) % 4 == 0) {
    const int64_t units = nb * hkv;
    const unsigned grid = (unsigned)((units + kQThreads / 32 - 1) / (kQThreads / 32));
    if (bs == 16)
      quantize_d128_kernel<T, 16><<<grid, kQThreads, 0, stream>>>(kv, q, scale, units, hkv, skip);
    else
      quantize_d128_kernel<T, 32><<<grid, kQThreads, 0, stream>>>(kv, q, scale, units, hkv, skip);
    return kOk;
  }
  const bool vec = hd % VEC == 0 && reinterpret_cast<uintptr_t>(kv) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(q) % VEC == 0;
  const size_t smem = (size_t)hkv * sizeof(uint32_t);
  if (vec)
    quantize_kernel<T, true><<<(unsigned)nb, kQThreads, smem, stream>>>(kv, q, scale, bs, hkv, hd,
                                                                         skip);
  else
    quantize_kernel<T, false><<<(unsigned)nb, kQThreads, smem, stream>>>(kv, q, scale, bs, hkv, hd,
                                                                          skip);
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
                    int block_size, int num_kv_heads, int head_dim, const uint8_t* skip,
                    cudaStream_t stream) {
  if (num_blocks == 0) return kOk;
  int rc;
  switch (dtype) {
    case 0: rc = launch_quantize_t(static_cast<const float*>(kv), q, scale, num_blocks, block_size,
                                   num_kv_heads, head_dim, skip, stream); break;
    case 1: rc = launch_quantize_t(static_cast<const __half*>(kv), q, scale, num_blocks,
                                   block_size, num_kv_heads, head_dim, skip, stream); break;
    case 2: rc = launch_quantize_t(static_cast<const __nv_bfloat16*>(kv), q, scale, num_blocks,
                                   block_size, num_kv_heads, head_dim, skip, stream); break;
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
