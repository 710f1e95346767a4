// Per-block eviction score, bit-identical to NumPy's evaluation of
// pagedkv_fusion/reference.py:38-71 (see eviction.cu for the contract).
// Shared by the multi-kernel path (eviction.cu) and the single-launch
// cluster path (eviction_cluster.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace pkv {

// ---------------------------------------------------------------------------
// Score
// ---------------------------------------------------------------------------

__device__ __forceinline__ float masked(const float* a, const uint8_t* m, int64_t i) {
  return m[i] ? a[i] : 0.0f;
}

// NumPy's pairwise float32 sum (see file header), on masked values.
__device__ inline float pairwise_masked_sum(const float* a, const uint8_t* m, int64_t n) {
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
  // 8) and recurse.
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

}  // namespace pkv
