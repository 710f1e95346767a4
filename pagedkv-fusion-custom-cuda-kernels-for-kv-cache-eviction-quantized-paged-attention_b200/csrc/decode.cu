// INT8 paged decode attention for sm_100a: split-K over pages plus a
// cross-split combine.
//
// Semantics follow pagedkv_fusion/reference.py:117-173 (decode step, one
// query token per sequence, per-(block, head) INT8 scales, GQA by
// kv_head = h / (H / Hkv)).  The launcher contract mirrors
// csrc/quant_paged_attention.cu:172-225 of the reference (same argument
// meaning and shape checks); a sequence of length 0 produces zeros.
//
// Two kernels do the streaming work:
//
//  * decode_fast_kernel  (head_dim 128, block_size 16/32, H/Hkv a power of
//    two <= 8).  One CTA = one (sequence, split of pages, group of HG KV
//    heads).  A producer warp streams each page's [block_size x HG x 128]
//    int8 tile with one TMA (cp.async.bulk.tensor, 128-byte swizzle) into a
//    4-stage ring guarded by mbarriers; 8 consumer warps compute.  K pages
//    of the split are streamed first, then V pages, so the softmax of a
//    split needs one barrier and no rescaling.  q.k uses IDP4A: the fp32
//    query is written as a 24-bit fixed-point integer split into three
//    signed 8-bit digits, so each 4-byte K word costs three integer dot
//    products and no int8->float conversion.  p.V converts V bytes with a
//    byte-permute into the mantissa of 2^23 and one float subtract.
//
//  * decode_generic_kernel  (any head_dim % 32 == 0 <= 256, block_size <=
//    64, any group size): plain loads, one CTA per (sequence, split, query
//    head).
//
// Logits are kept pre-multiplied by log2(e) so the softmax uses exp2; each
// split writes (m, l, acc[D]) and decode_combine_kernel merges splits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <random>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kQFix = 127 * 65536;  // largest |integer| of the 3-digit query

// ===========================================================================
// Tensor maps for the paged caches
// ===========================================================================

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// View the cache [NB, BS, Hkv, 128] int8 as a 3-D tensor (d, kv_head,
// token row) and load boxes of (128, hg, BS).
bool make_cache_map(CUtensorMap* map, const int8_t* cache, int64_t num_blocks, int bs,
                    int hkv, int hg) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {128, (cuuint64_t)hkv, (cuuint64_t)(num_blocks * bs)};
  cuuint64_t strides[2] = {128, (cuuint64_t)hkv * 128};
  cuuint32_t box[3] = {128, (cuuint32_t)hg, (cuuint32_t)bs};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(cache), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 4-D view (d, token, head, block) of the cache [NB, 16, hkv, 128] int8: a
// page box (128, 16, hkv, 1) lands as [head][token][128 B].
bool make_page_map(CUtensorMap* map, const int8_t* cache, int64_t num_blocks, int hkv) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[4] = {128, 16, (cuuint64_t)hkv, (cuuint64_t)num_blocks};
  cuuint64_t strides[3] = {(cuuint64_t)hkv * 128, 128, (cuuint64_t)16 * hkv * 128};
  cuuint32_t box[4] = {128, 16, (cuuint32_t)hkv, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(cache), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Small cache of encoded maps: a serving loop calls decode with the same
// cache tensors every step.
struct MapKey {
  const void* ptr;
  int64_t nb;
  int bs, hkv, hg;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && nb == o.nb && bs == o.bs && hkv == o.hkv && hg == o.hg;
  }
};

bool cached_cache_map(CUtensorMap* out, const int8_t* cache, int64_t nb, int bs, int hkv,
                      int hg) {
  static std::mutex mu;
  static MapKey keys[16];
  static CUtensorMap maps[16];
  static int used = 0, next = 0;
  MapKey key{cache, nb, bs, hkv, hg};
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (keys[i] == key) {
      *out = maps[i];
      return true;
    }
  if (!(hg < 0 ? make_page_map(out, cache, nb, hkv) : make_cache_map(out, cache, nb, bs, hkv, hg)))
    return false;
  keys[next] = key;
  maps[next] = *out;
  next = (next + 1) % 16;
  used = std::min(used + 1, 16);
  return true;
}

// ===========================================================================
// Small device helpers
// ===========================================================================

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Balanced base-256 digits of an integer |n| <= 127*65536: n = d2*65536 +
// d1*256 + d0 with every digit in [-128, 127].
__device__ __forceinline__ void to_digits(int n, int& d0, int& d1, int& d2) {
  d0 = ((n + 128) & 255) - 128;
  const int n1 = (n - d0) >> 8;
  d1 = ((n1 + 128) & 255) - 128;
  d2 = (n1 - d1) >> 8;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) |
         ((uint32_t)(d & 255) << 24);
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// ===========================================================================
// Fast kernel
// ===========================================================================

constexpr int kFastStages = 4;
constexpr int kStageBytes = 128 * 128;  // 128 cache lines of 128 B
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kFastThreads = kConsumers + 32;

template <int BS, int HG, int G>
struct FastCfg {
  static constexpr int kLinesPerPage = BS * HG;
  static_assert(128 % kLinesPerPage == 0 && kLinesPerPage >= 8, "page tile shape");
  static constexpr int kPPS = 128 / kLinesPerPage;  // pages per stage
  static constexpr int kPageBytes = kLinesPerPage * 128;
  static constexpr int kTokPerStage = kPPS * BS;
  static constexpr int kNHG = HG * G;  // query heads handled by one CTA
  static_assert(kNHG <= 16, "query heads per CTA");
  static constexpr int kMaxTok = kNHG <= 8 ? 512 : 256;  // tokens per split
  static constexpr int kMaxPages = kMaxTok / BS;
  // p.V work units: (kv head, pair of its query heads); token slices split
  // the 8 consumer warps between units.
  static constexpr int kGPW = G < 2 ? G : 2;
  static constexpr int kUnits = HG * (G / kGPW);
  static_assert(kUnits <= kConsumerWarps && kConsumerWarps % kUnits == 0, "p.V warp map");
  static constexpr int kVR = kConsumerWarps / kUnits;
  static constexpr int kQdStride = 3 * 128 + 16;  // padded: spreads banks
  static constexpr int kOffLogit = kFastStages * kStageBytes;
  static constexpr int kOffPd = kOffLogit + kNHG * kMaxTok * 4;  // [kNHG][3][kMaxTok] bytes
  static constexpr int kOffQd = kOffPd + kNHG * 3 * kMaxTok;
  static constexpr int kOffQs = kOffQd + (G > 1 ? kNHG * kQdStride : 0);
  static constexpr int kOffVsc = kOffQs + 64;
  static constexpr int kOffMl = kOffVsc + 64;
  static constexpr int kOffPhys = kOffMl + 16 * 8;
  static constexpr int kOffKs = kOffPhys + kMaxPages * 4;
  static constexpr int kOffVs = kOffKs + kMaxPages * HG * 4;
  static constexpr int kOffBar = ((kOffVs + kMaxPages * HG * 4) + 15) & ~15;
  static constexpr int kOffFlag = kOffBar + 2 * kFastStages * 8;
  static constexpr int kSmemBytes = kOffFlag + 16 + 1024;  // + alignment slack
};

// Signed int8 bytes of a times unsigned bytes of b, summed into c.
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <int BS, int HG, int G>
__global__ void __launch_bounds__(kFastThreads, 2)
    decode_fast_kernel(const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const float* __restrict__ q,
                       const float* __restrict__ k_scale, const float* __restrict__ v_scale,
                       const int32_t* __restrict__ block_tables,
                       const int32_t* __restrict__ seq_lens, float* __restrict__ out,
                       float* __restrict__ ws_acc, float2* __restrict__ ws_ml, int num_heads,
                       int num_kv_heads, int64_t num_blocks, int max_blocks_per_seq,
                       float qk_scale, int pages_per_split, int max_splits, int* err) {
  using C = FastCfg<BS, HG, G>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* s_logit = reinterpret_cast<float*>(smem + C::kOffLogit);
  float* s_qs = reinterpret_cast<float*>(smem + C::kOffQs);
  float2* s_ml = reinterpret_cast<float2*>(smem + C::kOffMl);
  int* s_phys = reinterpret_cast<int*>(smem + C::kOffPhys);
  float* s_ks = reinterpret_cast<float*>(smem + C::kOffKs);
  float* s_vs = reinterpret_cast<float*>(smem + C::kOffVs);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + kFastStages;
  const uint32_t stage_base = smem_u32(smem);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int seq = blockIdx.x;
  const int split = blockIdx.y;
  const int j0 = blockIdx.z * HG;  // first KV head of this CTA

  const int L_req = seq_lens[seq];
  const int n_pages = covered_pages(L_req, BS, max_blocks_per_seq);
  const int L = min(max(L_req, 0), n_pages * BS);
  if (L != max(L_req, 0) && split == 0 && blockIdx.z == 0 && threadIdx.x == 0)
    record_error(err, kDevSeqTooLong);
  const int p0 = split * pages_per_split;
  if (p0 >= n_pages) return;  // uniform across the CTA
  const int np = min(n_pages - p0, pages_per_split);
  const int t_begin = p0 * BS;
  const int T = min(L, (p0 + np) * BS) - t_begin;
  const int n_stages = (np + C::kPPS - 1) / C::kPPS;
  const int n_splits = (n_pages + pages_per_split - 1) / pages_per_split;

  // ---- prologue: block table, scales, query digits -----------------------
  const int32_t* bt_row = block_tables + (int64_t)seq * max_blocks_per_seq + p0;
  for (int i = tid; i < np * HG; i += kFastThreads) {
    const int pg = i / HG, jj = i - pg * HG;
    const int phys = bt_row[pg];
    const bool ok = phys >= 0 && (int64_t)phys < num_blocks;
    if (jj == 0) {
      s_phys[pg] = ok ? phys : -1;
      if (!ok) record_error(err, kDevBadBlockId);
    }
    const int64_t si = (int64_t)(ok ? phys : 0) * num_kv_heads + j0 + jj;
    s_ks[i] = ok ? k_scale[si] : 0.0f;
    s_vs[i] = ok ? v_scale[si] : 0.0f;
  }

  // query digits: for G == 1 every consumer keeps its own slice in
  // registers; for G > 1 they live in shared memory.
  uint4 qd[4][3];
  float my_qs = 0.0f;
  const int k_line = tid >> 1;  // K phase: two threads per cache line
  const int k_half = tid & 1;
  const int k_jj = k_line % HG;
  if constexpr (G == 1) {
    if (warp < kConsumerWarps) {
      const float4* qrow = reinterpret_cast<const float4*>(
          q + ((int64_t)seq * num_heads + (j0 + k_jj)) * 128 + k_half * 64);
      float4 v[16];
      float m = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[i] = qrow[i];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)),
                           fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
      }
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      const float inv = m > 0.0f ? (float)kQFix / m : 0.0f;
      my_qs = m > 0.0f ? m / (float)kQFix : 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t w[3][4];
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const float4 x = v[c * 4 + wi];
          int d[4][3];
          const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            int n = __float2int_rn(xs[e] * inv);
            n = max(-kQFix, min(kQFix, n));
            to_digits(n, d[e][0], d[e][1], d[e][2]);
          }
#pragma unroll
          for (int j = 0; j < 3; ++j) w[j][wi] = pack4(d[0][j], d[1][j], d[2][j], d[3][j]);
        }
#pragma unroll
        for (int j = 0; j < 3; ++j) qd[c][j] = make_uint4(w[j][0], w[j][1], w[j][2], w[j][3]);
      }
    }
  } else {
    uint8_t* s_qd = smem + C::kOffQd;
    for (int hg = warp; hg < C::kNHG; hg += kConsumerWarps + 1) {
      const int hq = (j0 + hg / G) * G + hg % G;
      const float4 x = reinterpret_cast<const float4*>(
          q + ((int64_t)seq * num_heads + hq) * 128)[lane];
      float m = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
      m = warp_max(m);
      const float inv = m > 0.0f ? (float)kQFix / m : 0.0f;
      const float xs[4] = {x.x, x.y, x.z, x.w};
      int d[4][3];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int n = __float2int_rn(xs[e] * inv);
        n = max(-kQFix, min(kQFix, n));
        to_digits(n, d[e][0], d[e][1], d[e][2]);
      }
#pragma unroll
      for (int j = 0; j < 3; ++j)
        reinterpret_cast<uint32_t*>(s_qd + hg * C::kQdStride + j * 128)[lane] =
            pack4(d[0][j], d[1][j], d[2][j], d[3][j]);
      if (lane == 0) s_qs[hg] = m > 0.0f ? m / (float)kQFix : 0.0f;
    }
  }

  if (tid == 0) {
    for (int s = 0; s < kFastStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  // ---- producer warp -----------------------------------------------------
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
      const uint64_t policy = l2_policy_evict_first();
      const int total = 2 * n_stages;
      int i = 0;
      for (; i < total; ++i) {
        const int slot = i % kFastStages;
        const uint32_t ph = (uint32_t)(i / kFastStages) & 1u;
        if (!mbar_wait_bounded(&empty[slot], ph ^ 1u, err)) {
          record_error(err, kDevWaitTimeout);
          break;
        }
        const bool is_v = i >= n_stages;
        const int st = is_v ? i - n_stages : i;
        const int pb = st * C::kPPS;
        const int pe = min(np, pb + C::kPPS);
        mbar_arrive_expect_tx(&full[slot], (uint32_t)((pe - pb) * C::kPageBytes));
        for (int pg = pb; pg < pe; ++pg) {
          const int phys = max(s_phys[pg], 0);
          tma_load_3d(smem + slot * kStageBytes + (pg - pb) * C::kPageBytes,
                      is_v ? &map_v : &map_k, &full[slot], 0, j0, phys * BS, policy);
        }
      }
      drain_ring(full, kFastStages, i);  // no copy outlives the CTA
    }
    return;
  }

  // ---- consumers: K phase -------------------------------------------------
  bool live = true;
  for (int st = 0; st < n_stages; ++st) {
    const int slot = st % kFastStages;
    const uint32_t ph = (uint32_t)(st / kFastStages) & 1u;
    if (live && !mbar_wait_bounded(&full[slot], ph, err)) {
      record_error(err, kDevWaitTimeout);
      live = false;
    }
    if (live) {
      const int tok = st * C::kTokPerStage + k_line / HG;
      const uint32_t line_addr = stage_base + slot * kStageBytes + k_line * 128;
      int acc[G][3];
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = acc[g][2] = 0;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int c = k_half * 4 + cc;
        const uint4 kw = lds128(line_addr + ((c ^ (k_line & 7)) << 4));
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            uint4 qw;
            if constexpr (G == 1) {
              qw = qd[cc][j];
            } else {
              qw = lds128(smem_u32(smem + C::kOffQd + (k_jj * G + g) * C::kQdStride + j * 128 +
                                   c * 16));
            }
            int a = acc[g][j];
            a = __dp4a((int)kw.x, (int)qw.x, a);
            a = __dp4a((int)kw.y, (int)qw.y, a);
            a = __dp4a((int)kw.z, (int)qw.z, a);
            a = __dp4a((int)kw.w, (int)qw.w, a);
            acc[g][j] = a;
          }
        }
      }
      const int pg = tok / BS;
      const bool valid = tok < T && s_phys[pg] >= 0;
      const float ks = s_ks[pg * HG + k_jj];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float part = (float)acc[g][2] * 65536.0f + ((float)acc[g][1] * 256.0f + (float)acc[g][0]);
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        const float qs = (G == 1) ? my_qs : s_qs[k_jj * G + g];
        if (k_half == 0 && tok < T)
          s_logit[(k_jj * G + g) * C::kMaxTok + tok] = valid ? part * (qs * ks * qk_scale) : -INFINITY;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  named_barrier(1, kConsumers);

  // ---- softmax over the split (per query head) ---------------------------
  // p_t = 2^(logit_t - m).  For p.V each p_t * vs(page) is written as a
  // 24-bit fixed-point fraction of the split's largest V scale, in three
  // unsigned byte planes (tokens up to the next multiple of 4 included, as
  // zeros past T).
  uint8_t* s_pd = smem + C::kOffPd;
  float* s_vsc = reinterpret_cast<float*>(smem + C::kOffVsc);
  const int T4 = (T + 3) & ~3;
  for (int hg = warp; hg < C::kNHG; hg += kConsumerWarps) {
    const float* row = s_logit + hg * C::kMaxTok;
    float m = -INFINITY;
    for (int t = lane; t < T; t += 32) m = fmaxf(m, row[t]);
    m = warp_max(m);
    const int jj = hg / G;
    float vmax = 0.0f;
    for (int pg = lane; pg < np; pg += 32) vmax = fmaxf(vmax, s_vs[pg * HG + jj]);
    vmax = warp_max(vmax);
    const float to_fix = vmax > 0.0f ? 16777215.0f / vmax : 0.0f;
    uint8_t* pd = s_pd + hg * 3 * C::kMaxTok;
    float l = 0.0f;
    for (int t = lane; t < T4; t += 32) {
      uint32_t n = 0;
      if (t < T && m != -INFINITY) {
        const float p = exp2f(row[t] - m);
        l += p;
        n = __float2uint_rn(fminf(p * s_vs[(t / BS) * HG + jj] * to_fix, 16777215.0f));
      }
      pd[t] = (uint8_t)(n & 255u);
      pd[C::kMaxTok + t] = (uint8_t)((n >> 8) & 255u);
      pd[2 * C::kMaxTok + t] = (uint8_t)(n >> 16);
    }
    l = warp_sum(l);
    if (lane == 0) {
      s_ml[hg] = make_float2(m, l);
      s_vsc[hg] = vmax * (1.0f / 16777215.0f);
    }
  }
  named_barrier(1, kConsumers);

  // ---- V phase: integer p.V ----------------------------------------------
  // A warp owns (kv head v_jj, query heads g0 .. g0+kGPW-1, token slice v_r);
  // lane w owns channels 4w .. 4w+3.  Per 4 tokens: 4 V words, a 4x4 byte
  // transpose (8 prmt) to put one channel of 4 tokens in a word, then one
  // dp4a per (channel, digit plane, query head).
  const int unit = warp % C::kUnits;
  const int v_r = warp / C::kUnits;
  const int v_jj = unit / (G / C::kGPW);
  const int g0 = (unit % (G / C::kGPW)) * C::kGPW;
  int iacc[C::kGPW][3][4];
#pragma unroll
  for (int g = 0; g < C::kGPW; ++g)
#pragma unroll
    for (int j = 0; j < 3; ++j) iacc[g][j][0] = iacc[g][j][1] = iacc[g][j][2] = iacc[g][j][3] = 0;
  const uint32_t word_off = (uint32_t)((lane & 3) << 2);
  const int chunk = lane >> 2;
  for (int st = 0; st < n_stages; ++st) {
    const int i = n_stages + st;
    const int slot = i % kFastStages;
    const uint32_t ph = (uint32_t)(i / kFastStages) & 1u;
    if (live && !mbar_wait_bounded(&full[slot], ph, err)) {
      record_error(err, kDevWaitTimeout);
      live = false;
    }
    if (live) {
      const uint32_t base = stage_base + slot * kStageBytes;
      const int tok0 = st * C::kTokPerStage;
      const int ngroups = (min(C::kTokPerStage, T - tok0) + 3) >> 2;
#pragma unroll 2
      for (int gi = v_r; gi < ngroups; gi += C::kVR) {
        const int ts = gi * 4;
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int line = (ts + u) * HG + v_jj;
          w[u] = lds32(base + line * 128 + ((chunk ^ (line & 7)) << 4) + word_off);
        }
        const uint32_t t0 = __byte_perm(w[0], w[1], 0x5140), t1 = __byte_perm(w[0], w[1], 0x7362);
        const uint32_t t2 = __byte_perm(w[2], w[3], 0x5140), t3 = __byte_perm(w[2], w[3], 0x7362);
        const uint32_t c[4] = {__byte_perm(t0, t2, 0x5410), __byte_perm(t0, t2, 0x7632),
                               __byte_perm(t1, t3, 0x5410), __byte_perm(t1, t3, 0x7632)};
#pragma unroll
        for (int g = 0; g < C::kGPW; ++g) {
          const uint8_t* pd = s_pd + (v_jj * G + g0 + g) * 3 * C::kMaxTok + tok0 + ts;
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const uint32_t pw = lds32(smem_u32(pd + j * C::kMaxTok));
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) iacc[g][j][ch] = dp4a_su(c[ch], pw, iacc[g][j][ch]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  // integer planes -> fp32 (each plane sum < 2^24: exact)
  float acc[C::kGPW][4];
#pragma unroll
  for (int g = 0; g < C::kGPW; ++g) {
    const float sc = s_vsc[v_jj * G + g0 + g];
#pragma unroll
    for (int ch = 0; ch < 4; ++ch)
      acc[g][ch] = sc * ((float)iacc[g][2][ch] * 65536.0f +
                         ((float)iacc[g][1][ch] * 256.0f + (float)iacc[g][0][ch]));
  }

  // ---- reduce token slices, then write -------------------------------------
  if constexpr (C::kVR > 1) {
    named_barrier(1, kConsumers);  // every stage consumed: the ring is free
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int g = 0; g < C::kGPW; ++g)
      reinterpret_cast<float4*>(red + ((v_r * C::kUnits + unit) * C::kGPW + g) * 128)[lane] =
          make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    named_barrier(1, kConsumers);
    if (v_r == 0) {
#pragma unroll
      for (int g = 0; g < C::kGPW; ++g) {
        for (int r = 1; r < C::kVR; ++r) {
          const float4 o = reinterpret_cast<const float4*>(
              red + ((r * C::kUnits + unit) * C::kGPW + g) * 128)[lane];
          acc[g][0] += o.x;
          acc[g][1] += o.y;
          acc[g][2] += o.z;
          acc[g][3] += o.w;
        }
      }
    }
  }
  if (v_r == 0) {
#pragma unroll
    for (int g = 0; g < C::kGPW; ++g) {
      const int hg = v_jj * G + g0 + g;
      const int hq = (j0 + v_jj) * G + g0 + g;
      const float2 ml = s_ml[hg];
      if (n_splits == 1) {
        const float inv = ml.y > 0.0f ? 1.0f / ml.y : 0.0f;
        reinterpret_cast<float4*>(out + ((int64_t)seq * num_heads + hq) * 128)[lane] =
            make_float4(acc[g][0] * inv, acc[g][1] * inv, acc[g][2] * inv, acc[g][3] * inv);
      } else {
        const int64_t slot = ((int64_t)seq * max_splits + split) * num_heads + hq;
        reinterpret_cast<float4*>(ws_acc + slot * 128)[lane] =
            make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
        if (lane == 0) ws_ml[slot] = ml;
      }
    }
  }
}

// ===========================================================================
// Stream kernel: persistent CTAs over a balanced share of all pages
// ===========================================================================
//
// The split kernel above gives every (sequence, split) its own CTA, so a
// batch whose splits do not fill whole waves of the GPU (64 sequences of
// 2,048 tokens: 1,024 CTAs for 296 slots) idles SMs in the last wave, and
// every short CTA pays the block-table / scale / query prologue.  Here the
// grid is ~2 CTAs per SM.  All pages of all (sequence, KV-head group) units
// form one flattened range; CTA c takes pages [P*c/C, P*(c+1)/C), walks
// them in chunks of <= kMaxTok tokens (K pages, softmax, V pages, as
// above) and merges consecutive chunks of one unit with the online-softmax
// rescale.
//
// A table warp fills a double-buffered chunk table (block-table entries,
// scales, token count and, for a new unit, the query rows by bulk copy) and
// publishes each half in two steps: the block ids (phys_full), then the rest
// (meta_full).  It fetches the first two chunks together before any page
// load is issued, so these small loads do not queue behind the GPU-wide
// burst of page loads, and later chunks one chunk ahead.  The TMA warp only
// waits for a chunk's block ids before issuing its K and V pages back to
// back, so the scale loads overlap the first page loads.  The per-head maximum of a
// chunk's logits is gathered while the K pages are read, so the softmax is
// a single vectorised pass.
//
// A unit owned by one CTA is written directly.  A unit that straddles CTAs
// leaves one partial (acc, m, l) per CTA at slot unit + c; the CTA whose
// arrival on the unit's counter completes the set merges them in segment
// order (so the result does not depend on which CTA arrives last) and
// writes the output.  The counters carry a per-launch tag (arrive_on_unit),
// so no memset precedes the launch.  A small batch (fewer than min_pages
// pages per CTA of the grid) is spread over fewer CTAs.

constexpr int kStreamMaxSeqs = 1024;
constexpr int kStreamThreads = kConsumers + 64;  // + TMA warp + table warp
constexpr int kTmaWarp = kConsumerWarps;
constexpr int kTableWarp = kConsumerWarps + 1;

template <int BS, int HG, int G>
struct StreamCfg {
  using F = FastCfg<BS, HG, G>;
  // one half of the double-buffered chunk table
  static constexpr int kMetaPhys = 0;                                  // int [kMaxPages]
  static constexpr int kMetaKs = kMetaPhys + F::kMaxPages * 4;         // float [kMaxPages][HG]
  static constexpr int kMetaVs = kMetaKs + F::kMaxPages * HG * 4;      // float [kMaxPages][HG]
  static constexpr int kMetaVmax = kMetaVs + F::kMaxPages * HG * 4;    // float [HG]
  static constexpr int kMetaT = kMetaVmax + 32;                        // int: tokens in chunk
  static constexpr int kMetaQ = (kMetaT + 4 + 15) & ~15;               // float [kNHG][kQRow]
  static constexpr int kQRow = 132;  // padded row: spreads the halves' banks
  // query rows staged only for G == 1 (larger groups read them from L2 into
  // their digit table, which keeps two CTAs per SM within shared memory)
  static constexpr int kMetaBytes = (kMetaQ + (G == 1 ? F::kNHG * kQRow * 4 : 0) + 15) & ~15;

  // per query head a row of kMaxTok fp32 logits; the softmax overwrites its
  // first 3 * kMaxTok bytes with the 24-bit probability planes
  static constexpr int kOffLogit = kFastStages * kStageBytes;
  static constexpr int kOffQd = kOffLogit + F::kNHG * F::kMaxTok * 4;
  static constexpr int kOffQs = kOffQd + F::kNHG * F::kQdStride;
  static constexpr int kOffRun = kOffQs + 64;   // float2 [16]: running (m, l)
  static constexpr int kOffAB = kOffRun + 128;  // float2 [16]: (old-acc factor, chunk factor)
  static constexpr int kOffMax = kOffAB + 128;  // uint [16]: chunk logit maximum (ordered key)
  static constexpr int kOffTmp = kOffMax + 64;  // int [32] scan scratch, flag
  static constexpr int kOffMeta = kOffTmp + 144;
  static constexpr int kOffPseq = kOffMeta + 2 * kMetaBytes;
  static constexpr int kOffRed = (kOffPseq + (kStreamMaxSeqs + 1) * 4 + 15) & ~15;
  static constexpr int kRedBytes = F::kVR > 1 ? kConsumerWarps * F::kGPW * 128 * 4 : 0;
  static constexpr int kOffBar = (kOffRed + kRedBytes + 15) & ~15;
  static constexpr int kSmemBytes = kOffBar + (2 * kFastStages + 6) * 8 + 1024;
  // two CTAs per SM (228 KB of shared memory, 1 KB reserved per CTA)
  static_assert(2 * (kSmemBytes + 1024) <= 228 * 1024, "stream kernel shared memory");
  static_assert(F::kMaxPages <= 32, "one chunk page per table-warp lane");
  static_assert(kOffMeta % 16 == 0 && kMetaBytes % 16 == 0 && kMetaQ % 16 == 0 &&
                    (kQRow * 4) % 16 == 0,
                "bulk copies into the chunk table need 16-byte alignment");
};

struct StreamChunk {
  int s, g;       // unit: sequence, KV-head group
  int lp0, np;    // first page within the unit, pages in the chunk
  bool seg_first, seg_last, whole;
};

// Walks one CTA's share [pos, end) of the flattened range in chunks of at
// most max_pages pages; every thread of the CTA runs its own copy
// identically.  The range is virtual: a unit of n pages spans alpha + n
// positions, the first alpha standing for the fixed cost of one more chunk
// (its table, the K -> softmax -> V hand-offs, its partial and merge), so a
// CTA whose share starts a unit takes about alpha fewer pages.  pseq[s] is
// the virtual per-group prefix: sequence s spans ng * (alpha + pages) virtual
// positions, 0 when it has no page.  Chunk fields are in real pages.
struct StreamIter {
  long long pos, end, cta_start;
  int s, g, S, ng, max_pages, alpha;
  const int* pseq;

  __device__ void init(long long start, long long stop, const int* ps, int num_seqs, int groups,
                       int mp, int a) {
    pos = start;
    end = stop;
    cta_start = start;
    pseq = ps;
    S = num_seqs;
    ng = groups;
    max_pages = mp;
    alpha = a;
    s = 0;
    g = 0;
    if (pos >= end) return;
    int lo = 0, hi = S - 1;  // largest s with pseq[s] * ng <= pos
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((long long)pseq[mid] * ng <= pos) lo = mid; else hi = mid - 1;
    }
    s = lo;
    const int vp = pseq[s + 1] - pseq[s];
    g = (int)((pos - (long long)pseq[s] * ng) / vp);
  }

  __device__ bool next(StreamChunk& c) {
    while (pos < end) {
      const int vp = pseq[s + 1] - pseq[s];
      const long long ustart = (long long)pseq[s] * ng + (long long)g * vp;
      const long long first_page = ustart + alpha;  // virtual position of real page 0
      const long long uend = ustart + vp;
      const long long seg_hi_v = end < uend ? end : uend;
      if (pos < first_page) pos = first_page;  // the unit's overhead positions
      if (pos < seg_hi_v) {
        const long long seg_lo_v = cta_start > first_page ? cta_start : first_page;
        const int pages = vp - alpha;
        const int lp0 = (int)(pos - first_page);
        const int seg_lo = (int)(seg_lo_v - first_page);
        const int seg_hi = (int)(seg_hi_v - first_page);
        const int np = min(max_pages, seg_hi - lp0);
        c.s = s;
        c.g = g;
        c.lp0 = lp0;
        c.np = np;
        c.seg_first = lp0 == seg_lo;
        c.seg_last = lp0 + np == seg_hi;
        c.whole = seg_lo == 0 && seg_hi == pages;
        pos += np;
        if (c.seg_last && pos < end) advance();
        return true;
      }
      // nothing real of this unit in the share: on to the next unit
      pos = seg_hi_v;
      if (pos < end) advance();
    }
    return false;
  }

  __device__ void advance() {  // the next unit with pages
    if (++g == ng) {
      g = 0;
      do {
        ++s;
      } while (s < S - 1 && pseq[s + 1] == pseq[s]);
    }
  }
};

// Ordered-integer image of a float for atomicMax (NaN never reaches it).
__device__ __forceinline__ uint32_t float_max_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float float_from_max_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
constexpr uint32_t kNegInfKey = 0x007fffffu;  // float_max_key(-inf)

// First and last CTA of a C-CTA split of P flattened pages that own pages
// of [lo, lo + n).
__device__ __forceinline__ int page_owner(long long x, long long P, int C) {
  return (int)(((x + 1) * C - 1) / P);
}

// First and last CTA owning pages of unit (s, g) in the virtual layout of
// StreamIter.
__device__ __forceinline__ void unit_owners(const int* pseq, int s, int g, int ng, int alpha,
                                            long long P, int n_ctas, int& first, int& last) {
  const int vp = pseq[s + 1] - pseq[s];
  const long long page0 = (long long)pseq[s] * ng + (long long)g * vp + alpha;
  first = page_owner(page0, P, n_ctas);
  last = page_owner(page0 + (vp - alpha) - 1, P, n_ctas);
}

// A unit split across more than kMergeGroup CTAs merges in two levels: the
// last arrival of each group of kMergeGroup consecutive CTAs merges the
// group's partials into the group's first slot, and the last group merges
// those.
constexpr int kMergeGroup = 16;

// Merges n partial rows (acc relative to exp2(m), with (m, l)) of one query
// head, row j at slot slot_of(j): a = sum_j w_j acc_j and den = sum_j w_j l_j
// with w_j = exp2(m_j - M), M = max_j m_j; rows with m = -inf add nothing.
// Rows are added in index order (deterministic).  The merge runs on the
// kernel's critical path after the GPU-wide stream of page loads, where
// every L2 round trip is long: the (m, l) of the first 32 rows and the
// first kMergeBatch acc rows are requested together, so a merge of up to
// kMergeBatch partials costs one round trip.
constexpr int kMergeBatch = 8;
template <typename SlotFn>
__device__ __forceinline__ void merge_partials(const float* __restrict__ ws_acc,
                                               const float2* __restrict__ ws_ml, int n, int lane,
                                               float4& a, float& M, float& den, SlotFn slot_of) {
  auto load_ml = [&](int j) {
    return j < n ? __ldcg(&ws_ml[slot_of(j)]) : make_float2(-INFINITY, 0.0f);
  };
  auto load_rows = [&](int j0, float4 (&x)[kMergeBatch]) {
#pragma unroll
    for (int jj = 0; jj < kMergeBatch; ++jj)
      x[jj] = __ldcg(reinterpret_cast<const float4*>(ws_acc + slot_of(min(j0 + jj, n - 1)) * 128) +
                     lane);
  };
  float4 x[kMergeBatch];
  const float2 ml0 = load_ml(lane);  // the first 32 are kept for the second pass
  load_rows(0, x);
  M = ml0.x;
  for (int b = 32; b < n; b += 32) M = fmaxf(M, load_ml(b + lane).x);
  M = warp_max(M);
  den = 0.0f;
  a = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int b = 0; b < n; b += 32) {
    const float2 ml = b == 0 ? ml0 : load_ml(b + lane);
    float w = 0.0f;
    if (ml.x != -INFINITY) {
      w = exp2f(ml.x - M);
      den += w * ml.y;
    }
    const int nb = min(32, n - b);
    for (int j0 = 0; j0 < nb; j0 += kMergeBatch) {
      if (b + j0 > 0) load_rows(b + j0, x);
#pragma unroll
      for (int jj = 0; jj < kMergeBatch; ++jj) {
        const float wj = __shfl_sync(0xffffffffu, w, (j0 + jj) & 31);
        if (j0 + jj < nb && wj != 0.0f) {
          a.x += wj * x[jj].x;
          a.y += wj * x[jj].y;
          a.z += wj * x[jj].z;
          a.w += wj * x[jj].w;
        }
      }
    }
  }
  den = warp_sum(den);
}

// Arrival counters need no reset before a launch, and no CTA waits for
// another to prepare them.  A counter holds (launch tag << kArrivalBits) |
// arrivals; the arrival that completes a set writes 0 back, so a CUDA-graph
// replay of the same launch (same tag) starts from a stale counter as well.
// The caller passes a guess: the counter as it read it (relaxed) while it
// computed its last chunk, or 0.  A guess carrying this launch's tag means
// the counter keeps that tag until the set completes -- which needs this
// arrival -- so one atomic add (acquire-release, GPU scope) counts it; the
// later arrivals of a set, the completing one among them (on the kernel's
// critical path), take this single L2 round trip.  Otherwise a
// compare-and-swap replaces a counter with any other tag -- 0 after a
// completed set, or what an earlier launch or another process left -- by
// (tag, 1), or counts one more arrival on (tag, n), retrying with the value
// it found.  Returns 1 for the completing arrival, 0 otherwise, -1 if the
// swap kept failing (another kernel racing on the same workspace).
constexpr int kArrivalBits = 20;
__device__ __forceinline__ int arrive_on_unit(unsigned long long* ctr, unsigned long long tag,
                                              int nseg, unsigned long long guess) {
  constexpr unsigned long long kCount = (1ull << kArrivalBits) - 1;
  unsigned long long now = 0ull;
  if ((guess >> kArrivalBits) == tag) {
    now = atomic_add_acq_rel_gpu_u64(ctr, 1ull) + 1ull;
  } else {
    const unsigned long long fresh = (tag << kArrivalBits) | 1ull;
    unsigned long long expect = guess;
    for (int tries = 0;; ++tries) {
      if (tries == (1 << 20)) return -1;
      const unsigned long long want = (expect >> kArrivalBits) == tag ? expect + 1ull : fresh;
      const unsigned long long seen = atomic_cas_acq_rel_gpu(ctr, expect, want);
      if (seen == expect) {
        now = want;
        break;
      }
      expect = seen;
    }
  }
  const bool last = (int)(now & kCount) == nseg;
  if (last) *reinterpret_cast<volatile unsigned long long*>(ctr) = 0ull;
  return last ? 1 : 0;
}

template <int BS, int HG, int G>
__global__ void __launch_bounds__(kStreamThreads, 2)
    decode_stream_kernel(const __grid_constant__ CUtensorMap map_k,
                         const __grid_constant__ CUtensorMap map_v, const float* __restrict__ q,
                         const float* __restrict__ k_scale, const float* __restrict__ v_scale,
                         const int32_t* __restrict__ block_tables,
                         const int32_t* __restrict__ seq_lens, float* __restrict__ out,
                         float* __restrict__ ws_acc, float2* __restrict__ ws_ml,
                         unsigned long long* __restrict__ unit_arrivals, int num_seqs, int num_heads,
                         int num_kv_heads, int64_t num_blocks, int max_blocks_per_seq,
                         float qk_scale, int min_pages, int unit_cost,
                         unsigned long long launch_tag, int* err) {
  using F = FastCfg<BS, HG, G>;
  using C = StreamCfg<BS, HG, G>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* s_logit = reinterpret_cast<float*>(smem + C::kOffLogit);
  float* s_qs = reinterpret_cast<float*>(smem + C::kOffQs);
  float2* s_run = reinterpret_cast<float2*>(smem + C::kOffRun);
  float2* s_ab = reinterpret_cast<float2*>(smem + C::kOffAB);
  uint32_t* s_max = reinterpret_cast<uint32_t*>(smem + C::kOffMax);
  int* s_tmp = reinterpret_cast<int*>(smem + C::kOffTmp);
  int* s_pseq = reinterpret_cast<int*>(smem + C::kOffPseq);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + kFastStages;
  uint64_t* meta_full = empty + kFastStages;  // [2]: chunk table half published
  uint64_t* chunk_free = meta_full + 2;       // [2]: chunk table half released
  uint64_t* phys_full = chunk_free + 2;       // [2]: the half's block ids published
  const uint32_t stage_base = smem_u32(smem);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = num_seqs;
  const int ng = num_kv_heads / HG;
  const int grid_ctas = gridDim.x;

  // ---- virtual pages per sequence (unit_cost + pages, per KV-head group;
  // 0 without pages) and their prefix (every CTA, identically) -------------
  constexpr int kPer = (kStreamMaxSeqs + kStreamThreads - 1) / kStreamThreads;
  int mine[kPer];
  int sum = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int s = tid * kPer + i;
    mine[i] = 0;
    if (s < S) {
      const int L = seq_lens[s];
      const int pages = covered_pages(L, BS, max_blocks_per_seq);
      if (blockIdx.x == 0 && L > pages * BS) record_error(err, kDevSeqTooLong);
      mine[i] = pages > 0 ? pages + unit_cost : 0;
    }
    sum += mine[i];
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_tmp[warp] = incl;
  if (tid == 0) {
    for (int i = 0; i < kFastStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&meta_full[i], 1);
      mbar_init(&chunk_free[i], 2);  // consumers (softmax done) + TMA warp (pages issued)
      mbar_init(&phys_full[i], 1);
    }
    mbar_fence_init();
  }
  if (tid < F::kNHG) s_max[tid] = kNegInfKey;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < warp; ++w) before += s_tmp[w];
  int run = before + incl - sum;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int s = tid * kPer + i;
    if (s <= S) s_pseq[s] = run;  // s == S: total
    run += mine[i];
  }
  __syncthreads();
  // sequences without pages: zero output (no unit covers them)
  for (int s = blockIdx.x; s < S; s += grid_ctas) {
    if (s_pseq[s + 1] != s_pseq[s]) continue;
    float4* o = reinterpret_cast<float4*>(out + (int64_t)s * num_heads * 128);
    for (int i = tid; i < num_heads * 32; i += kStreamThreads) o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const long long P = (long long)s_pseq[S] * ng;
  // a small batch goes to fewer CTAs, at least min_pages pages each, so that
  // a unit leaves few partials to merge (every CTA derives the same count)
  const int n_ctas = (int)min((long long)grid_ctas, max(1LL, (P + min_pages - 1) / min_pages));
  if (blockIdx.x >= n_ctas) return;  // uniform
  const long long c_begin = P * blockIdx.x / n_ctas;
  const long long c_end = P * (blockIdx.x + 1) / n_ctas;
  if (c_begin >= c_end) return;  // uniform

  StreamIter it;
  it.init(c_begin, c_end, s_pseq, S, ng, F::kMaxPages, unit_cost);
  StreamChunk ch;

  // ---- table warp: chunk tables one chunk ahead ---------------------------
  if (warp == kTableWarp) {
    // block-table entry of this lane's page of chunk c (-1: none / invalid)
    auto load_phys = [&](const StreamChunk& c) {
      int phys = -1;
      if (lane < c.np) {
        const int v = block_tables[(int64_t)c.s * max_blocks_per_seq + c.lp0 + lane];
        const bool ok = v >= 0 && (int64_t)v < num_blocks;
        if (!ok) record_error(err, kDevBadBlockId);
        phys = ok ? v : -1;
      }
      return phys;
    };
    auto load_scales = [&](const StreamChunk& c, int phys, float (&ks)[HG], float (&vs)[HG]) {
      const int64_t si = (int64_t)(phys >= 0 ? phys : 0) * num_kv_heads + c.g * HG;
#pragma unroll
      for (int jj = 0; jj < HG; ++jj) {
        ks[jj] = phys >= 0 ? k_scale[si + jj] : 0.0f;
        vs[jj] = phys >= 0 ? v_scale[si + jj] : 0.0f;
      }
    };
    // Writes chunk c's block ids into half b and publishes them on
    // phys_full[b]: the TMA warp issues the pages while the scales load.
    auto publish_phys = [&](int b, const StreamChunk& c, int phys) {
      uint8_t* meta = smem + C::kOffMeta + b * C::kMetaBytes;
      if (lane < c.np) reinterpret_cast<int*>(meta + C::kMetaPhys)[lane] = phys;
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&phys_full[b]);
    };
    // Writes the rest of chunk c's table into half b and publishes it on
    // meta_full[b].
    auto publish = [&](int b, const StreamChunk& c, bool new_unit,
                       const float (&ks)[HG], const float (&vs)[HG]) {
      uint8_t* meta = smem + C::kOffMeta + b * C::kMetaBytes;
      if (lane < c.np) {
#pragma unroll
        for (int jj = 0; jj < HG; ++jj) {
          reinterpret_cast<float*>(meta + C::kMetaKs)[lane * HG + jj] = ks[jj];
          reinterpret_cast<float*>(meta + C::kMetaVs)[lane * HG + jj] = vs[jj];
        }
      }
#pragma unroll
      for (int jj = 0; jj < HG; ++jj) {
        const float v = warp_max(vs[jj]);
        if (lane == 0) reinterpret_cast<float*>(meta + C::kMetaVmax)[jj] = v;
      }
      if (lane == 0) {
        const int pages = s_pseq[c.s + 1] - s_pseq[c.s] - unit_cost;
        const int Ls = min(max(seq_lens[c.s], 0), pages * BS);
        *reinterpret_cast<int*>(meta + C::kMetaT) = min(Ls, (c.lp0 + c.np) * BS) - c.lp0 * BS;
      }
      const float* qu = q + ((int64_t)c.s * num_heads + (int64_t)c.g * F::kNHG) * 128;
      if constexpr (G == 1) {
        if (new_unit) {
          if (lane == 0) mbar_expect_tx(&meta_full[b], F::kNHG * 512);
          __syncwarp();
          if (lane < F::kNHG)
            bulk_load_g2s(meta + C::kMetaQ + lane * C::kQRow * 4, qu + lane * 128, 512,
                          &meta_full[b]);
        }
      } else {
        if (new_unit)
          for (int ln = lane; ln < F::kNHG * 4; ln += 32)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(qu + ln * 32));
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_full[b]);
    };
    StreamChunk c0, c1;
    const bool have0 = it.next(c0);
    const bool have1 = have0 && it.next(c1);
    if (!have0) return;
    {  // the first two chunks, loads interleaved
      float ks0[HG], vs0[HG], ks1[HG], vs1[HG];
      const int p0 = load_phys(c0);
      const int p1 = have1 ? load_phys(c1) : -1;
      publish_phys(0, c0, p0);
      if (have1) publish_phys(1, c1, p1);
      load_scales(c0, p0, ks0, vs0);
      if (have1) load_scales(c1, p1, ks1, vs1);
      publish(0, c0, true, ks0, vs0);
      if (have1) publish(1, c1, c1.s != c0.s || c1.g != c0.g, ks1, vs1);
    }
    int published = have1 ? 2 : 1;
    if (have1) {
      StreamChunk prev = c1, cur;
      for (; it.next(cur); ++published) {
        const int i = published, b = i & 1;
        bool ok = true;
        if (lane == 0 && !mbar_wait_bounded(&chunk_free[b], (uint32_t)((i >> 1) - 1) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          ok = false;
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        float ks[HG], vs[HG];
        const int ph = load_phys(cur);
        publish_phys(b, cur, ph);
        load_scales(cur, ph, ks, vs);
        publish(b, cur, cur.s != prev.s || cur.g != prev.g, ks, vs);
        prev = cur;
      }
    }
    if (lane == 0) drain_ring(meta_full, 2, published);  // the q-row copies have landed
    return;
  }

  // ---- TMA warp: K then V pages of each chunk -------------------------------
  if (warp == kTmaWarp) {
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
      int ns = 0;
      for (int i = 0; it.next(ch); ++i) {
        const int b = i & 1;
        if (!mbar_wait_bounded(&phys_full[b], (uint32_t)(i >> 1) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          break;
        }
        const int* m_phys =
            reinterpret_cast<const int*>(smem + C::kOffMeta + b * C::kMetaBytes + C::kMetaPhys);
        const int n_st = (ch.np + F::kPPS - 1) / F::kPPS;
        bool ok_run = true;
        for (int kind = 0; kind < 2 && ok_run; ++kind) {
          for (int st = 0; st < n_st; ++st, ++ns) {
            const int slot = ns % kFastStages;
            const uint32_t ph = (uint32_t)(ns / kFastStages) & 1u;
            if (!mbar_wait_bounded(&empty[slot], ph ^ 1u, err)) {
              record_error(err, kDevWaitTimeout);
              ok_run = false;
              break;
            }
            const int pb = st * F::kPPS;
            const int pe = min(ch.np, pb + F::kPPS);
            mbar_arrive_expect_tx(&full[slot], (uint32_t)((pe - pb) * F::kPageBytes));
            for (int pg = pb; pg < pe; ++pg)
              tma_load_3d(smem + slot * kStageBytes + (pg - pb) * F::kPageBytes,
                          kind ? &map_v : &map_k, &full[slot], 0, ch.g * HG,
                          max(m_phys[pg], 0) * BS, policy);
          }
        }
        if (!ok_run) break;
        mbar_arrive(&chunk_free[b]);  // this warp is done with the chunk's table
      }
      drain_ring(full, kFastStages, ns);  // no copy outlives the CTA
    }
    return;
  }

  // ---- consumers -------------------------------------------------------------
  const int k_line = tid >> 1;  // K phase: two threads per cache line
  const int k_half = tid & 1;
  const int k_jj = k_line % HG;
  const int unit = warp % F::kUnits;  // p.V work unit (kv head, query-head pair)
  const int v_r = warp / F::kUnits;
  const int v_jj = unit / (G / F::kGPW);
  const int g0 = (unit % (G / F::kGPW)) * F::kGPW;
  const uint32_t word_off = (uint32_t)((lane & 3) << 2);
  const int wchunk = lane >> 2;
  float acc_run[F::kGPW][4];
#pragma unroll
  for (int g = 0; g < F::kGPW; ++g) acc_run[g][0] = acc_run[g][1] = acc_run[g][2] = acc_run[g][3] = 0.0f;
  bool live = true;
  int ns = 0, cur_s = -1, cur_g = -1;
  // the first-level arrival of a split unit: its counter and count
  auto arrival_of = [&](const StreamChunk& c, int& first, int& last, int& nseg, int& ngroups,
                        int& g_lo, int& g_hi) -> unsigned long long* {
    unit_owners(s_pseq, c.s, c.g, ng, unit_cost, P, n_ctas, first, last);
    nseg = last - first + 1;
    ngroups = (nseg + kMergeGroup - 1) / kMergeGroup;
    g_lo = first + (int)(blockIdx.x - first) / kMergeGroup * kMergeGroup;
    g_hi = min(last, g_lo + kMergeGroup - 1);
    const int u = c.s * ng + c.g;
    return ngroups == 1 ? &unit_arrivals[u] : &unit_arrivals[S * ng + u + g_lo];
  };
  for (int i = 0; it.next(ch); ++i) {
    // a split unit's last chunk in this CTA: read its arrival counter now
    unsigned long long arrival_guess = 0ull;
    if (tid == 0 && ch.seg_last && !ch.whole) {
      int f, l, n, ngr, glo, ghi;
      arrival_guess = ld_relaxed_gpu_u64(arrival_of(ch, f, l, n, ngr, glo, ghi));
    }
    const uint8_t* meta = smem + C::kOffMeta + (i & 1) * C::kMetaBytes;
    const int* m_phys = reinterpret_cast<const int*>(meta + C::kMetaPhys);
    const float* m_ks = reinterpret_cast<const float*>(meta + C::kMetaKs);
    const float* m_vs = reinterpret_cast<const float*>(meta + C::kMetaVs);
    const float* m_q = reinterpret_cast<const float*>(meta + C::kMetaQ);
    if (live && !mbar_wait_bounded(&meta_full[i & 1], (uint32_t)(i >> 1) & 1u, err)) {
      record_error(err, kDevWaitTimeout);
      live = false;
    }
    const int j0 = ch.g * HG;
    const int T = live ? *reinterpret_cast<const int*>(meta + C::kMetaT) : 0;
    const int n_st = (ch.np + F::kPPS - 1) / F::kPPS;

    // every warp is past the previous chunk's V phase (which reads the
    // probability planes) before this chunk's logits overwrite them
    named_barrier(1, kConsumers);
    if (ch.s != cur_s || ch.g != cur_g) {  // a new unit: its query digits
      {
        uint8_t* s_qd = smem + C::kOffQd;
        const float* qu = q + ((int64_t)ch.s * num_heads + (int64_t)j0 * G) * 128;
        for (int hg = warp; hg < F::kNHG; hg += kConsumerWarps) {
          const float4 x = G == 1 ? reinterpret_cast<const float4*>(m_q + hg * C::kQRow)[lane]
                                  : reinterpret_cast<const float4*>(qu + hg * 128)[lane];
          float m = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
          m = warp_max(m);
          const float inv = m > 0.0f ? (float)kQFix / m : 0.0f;
          const float xs[4] = {x.x, x.y, x.z, x.w};
          int d[4][3];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            int n = __float2int_rn(xs[e] * inv);
            n = max(-kQFix, min(kQFix, n));
            to_digits(n, d[e][0], d[e][1], d[e][2]);
          }
#pragma unroll
          for (int j = 0; j < 3; ++j)
            reinterpret_cast<uint32_t*>(s_qd + hg * F::kQdStride + j * 128)[lane] =
                pack4(d[0][j], d[1][j], d[2][j], d[3][j]);
          if (lane == 0) s_qs[hg] = m > 0.0f ? m / (float)kQFix : 0.0f;
        }
        named_barrier(1, kConsumers);
      }
      cur_s = ch.s;
      cur_g = ch.g;
    }

    // ---- K phase: logits, and this thread's running maximum per head ----
    float kmax[G];
#pragma unroll
    for (int g = 0; g < G; ++g) kmax[g] = -INFINITY;
    for (int st = 0; st < n_st; ++st, ++ns) {
      const int slot = ns % kFastStages;
      const uint32_t ph = (uint32_t)(ns / kFastStages) & 1u;
      if (live && !mbar_wait_bounded(&full[slot], ph, err)) {
        record_error(err, kDevWaitTimeout);
        live = false;
      }
      if (live) {
        const int tok = st * F::kTokPerStage + k_line / HG;
        const uint32_t line_addr = stage_base + slot * kStageBytes + k_line * 128;
        int acc[G][3];
#pragma unroll
        for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = acc[g][2] = 0;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = k_half * 4 + cc;
          const uint4 kw = lds128(line_addr + ((c ^ (k_line & 7)) << 4));
#pragma unroll
          for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int j = 0; j < 3; ++j) {
              const uint4 qw = lds128(smem_u32(smem + C::kOffQd + (k_jj * G + g) * F::kQdStride +
                                               j * 128 + c * 16));
              int a = acc[g][j];
              a = __dp4a((int)kw.x, (int)qw.x, a);
              a = __dp4a((int)kw.y, (int)qw.y, a);
              a = __dp4a((int)kw.z, (int)qw.z, a);
              a = __dp4a((int)kw.w, (int)qw.w, a);
              acc[g][j] = a;
            }
          }
        }
        const int pg = min(tok / BS, F::kMaxPages - 1);
        const bool valid = tok < T && m_phys[pg] >= 0;
        const float ks = m_ks[pg * HG + k_jj];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float part =
              (float)acc[g][2] * 65536.0f + ((float)acc[g][1] * 256.0f + (float)acc[g][0]);
          part += __shfl_xor_sync(0xffffffffu, part, 1);
          const float qsv = s_qs[k_jj * G + g];
          const float logit = valid ? part * (qsv * ks * qk_scale) : -INFINITY;
          if (k_half == 0 && tok < T) {
            s_logit[(k_jj * G + g) * F::kMaxTok + tok] = logit;
            kmax[g] = fmaxf(kmax[g], logit);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    // lanes 2*HG*m apart hold the same head; lanes with (lane >> 1) < HG, even, publish
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int o = 2 * HG; o < 32; o <<= 1)
        kmax[g] = fmaxf(kmax[g], __shfl_xor_sync(0xffffffffu, kmax[g], o));
      if (k_half == 0 && (lane >> 1) < HG && kmax[g] != -INFINITY)
        atomicMax(&s_max[k_jj * G + g], float_max_key(kmax[g]));
    }
    named_barrier(1, kConsumers);

    // ---- softmax of the chunk, merged with the unit's running state ----
    for (int hg = warp; hg < F::kNHG; hg += kConsumerWarps) {
      const float4* row = reinterpret_cast<const float4*>(s_logit + hg * F::kMaxTok);
      const float m = float_from_max_key(s_max[hg]);
      const int jj = hg / G;
      const float vmax = reinterpret_cast<const float*>(meta + C::kMetaVmax)[jj];
      const float to_fix = vmax > 0.0f ? 16777215.0f / vmax : 0.0f;
      uint8_t* pd = reinterpret_cast<uint8_t*>(s_logit + hg * F::kMaxTok);
      constexpr int kIt = F::kMaxTok / 128;
      const int T4q = (T + 3) >> 2;
      float4 x[kIt];  // the whole row first: the planes overwrite it
#pragma unroll
      for (int k4 = 0; k4 < kIt; ++k4) {
        const int t4 = lane + 32 * k4;
        x[k4] = t4 < T4q ? row[t4] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      __syncwarp();
      float l = 0.0f;
#pragma unroll
      for (int k4 = 0; k4 < kIt; ++k4) {
        const int t4 = lane + 32 * k4;
        if (t4 < T4q) {
          const int t = t4 * 4;
          const float xs[4] = {x[k4].x, x[k4].y, x[k4].z, x[k4].w};
          const float vs = m_vs[(t / BS) * HG + jj];
          uint32_t n[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            n[e] = 0;
            if (t + e < T && m != -INFINITY) {
              const float p = exp2f(xs[e] - m);
              l += p;
              n[e] = __float2uint_rn(fminf(p * vs * to_fix, 16777215.0f));
            }
          }
          const uint32_t lo01 = __byte_perm(n[0], n[1], 0x5140), hi01 = __byte_perm(n[0], n[1], 0x7362);
          const uint32_t lo23 = __byte_perm(n[2], n[3], 0x5140), hi23 = __byte_perm(n[2], n[3], 0x7362);
          *reinterpret_cast<uint32_t*>(pd + t) = __byte_perm(lo01, lo23, 0x5410);
          *reinterpret_cast<uint32_t*>(pd + F::kMaxTok + t) = __byte_perm(lo01, lo23, 0x7632);
          *reinterpret_cast<uint32_t*>(pd + 2 * F::kMaxTok + t) = __byte_perm(hi01, hi23, 0x5410);
        }
      }
      l = warp_sum(l);
      if (lane == 0) {
        const float2 r = ch.seg_first ? make_float2(-INFINITY, 0.0f) : s_run[hg];
        const float mn = fmaxf(r.x, m);
        const float a = (r.x == -INFINITY) ? 0.0f : exp2f(r.x - mn);
        const float b = (m == -INFINITY) ? 0.0f : exp2f(m - mn);
        s_run[hg] = make_float2(mn, r.y * a + l * b);
        s_ab[hg] = make_float2(a, b * vmax * (1.0f / 16777215.0f));
        s_max[hg] = kNegInfKey;
      }
    }
    named_barrier(1, kConsumers);
    if (tid == 0) mbar_arrive(&chunk_free[i & 1]);  // the chunk's table half is free

    // ---- V phase: integer p.V ----
    int iacc[F::kGPW][3][4];
#pragma unroll
    for (int g = 0; g < F::kGPW; ++g)
#pragma unroll
      for (int j = 0; j < 3; ++j) iacc[g][j][0] = iacc[g][j][1] = iacc[g][j][2] = iacc[g][j][3] = 0;
    for (int st = 0; st < n_st; ++st, ++ns) {
      const int slot = ns % kFastStages;
      const uint32_t ph = (uint32_t)(ns / kFastStages) & 1u;
      if (live && !mbar_wait_bounded(&full[slot], ph, err)) {
        record_error(err, kDevWaitTimeout);
        live = false;
      }
      if (live) {
        const uint32_t base = stage_base + slot * kStageBytes;
        const int tok0 = st * F::kTokPerStage;
        const int ngroups = (min(F::kTokPerStage, T - tok0) + 3) >> 2;
#pragma unroll 2
        for (int gi = v_r; gi < ngroups; gi += F::kVR) {
          const int ts = gi * 4;
          uint32_t w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int line = (ts + u) * HG + v_jj;
            w[u] = lds32(base + line * 128 + ((wchunk ^ (line & 7)) << 4) + word_off);
          }
          const uint32_t t0 = __byte_perm(w[0], w[1], 0x5140), t1 = __byte_perm(w[0], w[1], 0x7362);
          const uint32_t t2 = __byte_perm(w[2], w[3], 0x5140), t3 = __byte_perm(w[2], w[3], 0x7362);
          const uint32_t cw[4] = {__byte_perm(t0, t2, 0x5410), __byte_perm(t0, t2, 0x7632),
                                  __byte_perm(t1, t3, 0x5410), __byte_perm(t1, t3, 0x7632)};
#pragma unroll
          for (int g = 0; g < F::kGPW; ++g) {
            const uint8_t* pd = reinterpret_cast<const uint8_t*>(s_logit + (v_jj * G + g0 + g) * F::kMaxTok) + tok0 + ts;
#pragma unroll
            for (int j = 0; j < 3; ++j) {
              const uint32_t pw = lds32(smem_u32(pd + j * F::kMaxTok));
#pragma unroll
              for (int c4 = 0; c4 < 4; ++c4) iacc[g][j][c4] = dp4a_su(cw[c4], pw, iacc[g][j][c4]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
#pragma unroll
    for (int g = 0; g < F::kGPW; ++g) {
      const float2 ab = s_ab[v_jj * G + g0 + g];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4)
        acc_run[g][c4] = acc_run[g][c4] * ab.x +
                         ab.y * ((float)iacc[g][2][c4] * 65536.0f +
                                 ((float)iacc[g][1][c4] * 256.0f + (float)iacc[g][0][c4]));
    }

    // ---- end of this CTA's part of the unit: write it ----
    if (ch.seg_last) {
      if constexpr (F::kVR > 1) {
        float* red = reinterpret_cast<float*>(smem + C::kOffRed);
#pragma unroll
        for (int g = 0; g < F::kGPW; ++g)
          reinterpret_cast<float4*>(red + ((v_r * F::kUnits + unit) * F::kGPW + g) * 128)[lane] =
              make_float4(acc_run[g][0], acc_run[g][1], acc_run[g][2], acc_run[g][3]);
        named_barrier(1, kConsumers);
        if (v_r == 0) {
#pragma unroll
          for (int g = 0; g < F::kGPW; ++g) {
            for (int r = 1; r < F::kVR; ++r) {
              const float4 o = reinterpret_cast<const float4*>(
                  red + ((r * F::kUnits + unit) * F::kGPW + g) * 128)[lane];
              acc_run[g][0] += o.x;
              acc_run[g][1] += o.y;
              acc_run[g][2] += o.z;
              acc_run[g][3] += o.w;
            }
          }
        }
      }
      const int u = ch.s * ng + ch.g;
      if (ch.whole) {
        if (v_r == 0) {
#pragma unroll
          for (int g = 0; g < F::kGPW; ++g) {
            const int hg = v_jj * G + g0 + g;
            const float2 ml = s_run[hg];
            const float inv = ml.y > 0.0f ? 1.0f / ml.y : 0.0f;
            reinterpret_cast<float4*>(out + ((int64_t)ch.s * num_heads + (int64_t)j0 * G + hg) * 128)[lane] =
                make_float4(acc_run[g][0] * inv, acc_run[g][1] * inv, acc_run[g][2] * inv,
                            acc_run[g][3] * inv);
          }
        }
      } else {
        if (v_r == 0) {
#pragma unroll
          for (int g = 0; g < F::kGPW; ++g) {
            const int hg = v_jj * G + g0 + g;
            const int64_t slot = ((int64_t)u + blockIdx.x) * F::kNHG + hg;
            reinterpret_cast<float4*>(ws_acc + slot * 128)[lane] =
                make_float4(acc_run[g][0], acc_run[g][1], acc_run[g][2], acc_run[g][3]);
            if (lane == 0) ws_ml[slot] = s_run[hg];
          }
        }
        // the unit's CTAs [first, last] in page order: every one owns pages
        // (n_ctas <= P gives each CTA at least one position)
        int first, last, nseg, ngroups, g_lo, g_hi;
        unsigned long long* ctr = arrival_of(ch, first, last, nseg, ngroups, g_lo, g_hi);
        // every partial store of this CTA is ordered before thread 0's
        // release by the barrier; the last arrival acquires all of them
        named_barrier(1, kConsumers);
        if (tid == 0) {
          const int r = arrive_on_unit(ctr, launch_tag, ngroups == 1 ? nseg : g_hi - g_lo + 1,
                                       arrival_guess);
          if (r < 0) record_error(err, kDevWaitTimeout);
          s_tmp[32] = r == 1;
        }
        named_barrier(1, kConsumers);
        // this CTA completed its group: merge it; with more than one group the
        // group's partial goes to its first slot and the last group to
        // complete merges the groups' partials (a second pass)
        int m_lo = g_lo, m_n = g_hi - g_lo + 1, m_stride = 1;
        bool final_pass = ngroups == 1;
        bool merging = s_tmp[32] != 0;
        while (merging) {
          if (v_r == 0) {
#pragma unroll 1
            for (int g = 0; g < F::kGPW; ++g) {
              const int hg = v_jj * G + g0 + g;
              float4 a;
              float M, den;
              merge_partials(ws_acc, ws_ml, m_n, lane, a, M, den, [&](int j) {
                return ((int64_t)u + m_lo + j * m_stride) * F::kNHG + hg;
              });
              if (final_pass) {
                const float inv = den > 0.0f ? 1.0f / den : 0.0f;
                reinterpret_cast<float4*>(out + ((int64_t)ch.s * num_heads + (int64_t)j0 * G + hg) * 128)[lane] =
                    make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
              } else {
                const int64_t slot = ((int64_t)u + g_lo) * F::kNHG + hg;
                reinterpret_cast<float4*>(ws_acc + slot * 128)[lane] = a;
                if (lane == 0) ws_ml[slot] = make_float2(M, den);
              }
            }
          }
          if (final_pass) break;
          named_barrier(1, kConsumers);  // the group's partial is stored
          if (tid == 0) {
            const int r = arrive_on_unit(&unit_arrivals[u], launch_tag, ngroups, 0ull);
            if (r < 0) record_error(err, kDevWaitTimeout);
            s_tmp[33] = r == 1;
          }
          named_barrier(1, kConsumers);
          merging = s_tmp[33] != 0;
          m_lo = first;
          m_n = ngroups;
          m_stride = kMergeGroup;
          final_pass = true;
        }
      }
#pragma unroll
      for (int g = 0; g < F::kGPW; ++g) acc_run[g][0] = acc_run[g][1] = acc_run[g][2] = acc_run[g][3] = 0.0f;
    }
  }
}

// ===========================================================================
// Generic kernel
// ===========================================================================

constexpr int kGenThreads = 128;
constexpr int kGenMaxTok = 2048;

__global__ void __launch_bounds__(kGenThreads)
    decode_generic_kernel(const float* __restrict__ q, const int8_t* __restrict__ k_cache,
                          const float* __restrict__ k_scale, const int8_t* __restrict__ v_cache,
                          const float* __restrict__ v_scale,
                          const int32_t* __restrict__ block_tables,
                          const int32_t* __restrict__ seq_lens, float* __restrict__ out,
                          float* __restrict__ ws_acc, float2* __restrict__ ws_ml, int num_heads,
                          int num_kv_heads, int head_dim, int bs, int64_t num_blocks,
                          int max_blocks_per_seq, float qk_scale, int pages_per_split,
                          int max_splits, int* err) {
  __shared__ float s_q[256];
  __shared__ float s_p[kGenMaxTok];
  __shared__ float s_red[kGenThreads / 32];
  const int seq = blockIdx.x;
  const int split = blockIdx.y;
  const int h = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int L_req = seq_lens[seq];
  const int n_pages = covered_pages(L_req, bs, max_blocks_per_seq);
  const int L = min(max(L_req, 0), n_pages * bs);
  if (L != max(L_req, 0) && split == 0 && h == 0 && threadIdx.x == 0)
    record_error(err, kDevSeqTooLong);
  const int p0 = split * pages_per_split;
  if (p0 >= n_pages) return;
  const int np = min(n_pages - p0, pages_per_split);
  const int t_begin = p0 * bs;
  const int T = min(L, (p0 + np) * bs) - t_begin;
  const int n_splits = (n_pages + pages_per_split - 1) / pages_per_split;
  const int kvh = h / (num_heads / num_kv_heads);
  const int32_t* bt_row = block_tables + (int64_t)seq * max_blocks_per_seq;
  const int64_t row_stride = (int64_t)num_kv_heads * head_dim;

  for (int d = tid; d < head_dim; d += kGenThreads)
    s_q[d] = q[((int64_t)seq * num_heads + h) * head_dim + d];
  __syncthreads();

  // logits: one warp per token
  for (int t = warp; t < T; t += kGenThreads / 32) {
    const int pos = t_begin + t;
    const int phys = bt_row[pos / bs];
    const bool ok = phys >= 0 && (int64_t)phys < num_blocks;
    float dot = 0.0f;
    if (ok) {
      const int8_t* kr = k_cache + ((int64_t)phys * bs + pos % bs) * row_stride +
                         (int64_t)kvh * head_dim;
      for (int d = lane; d < head_dim; d += 32) dot = fmaf(s_q[d], (float)kr[d], dot);
    }
    dot = warp_sum(dot);
    if (lane == 0) {
      if (!ok) record_error(err, kDevBadBlockId);
      s_p[t] = ok ? dot * (k_scale[(int64_t)phys * num_kv_heads + kvh] * qk_scale) : -INFINITY;
    }
  }
  __syncthreads();

  float m = -INFINITY;
  for (int t = tid; t < T; t += kGenThreads) m = fmaxf(m, s_p[t]);
  m = warp_max(m);
  if (lane == 0) s_red[warp] = m;
  __syncthreads();
  m = s_red[0];
  for (int w = 1; w < kGenThreads / 32; ++w) m = fmaxf(m, s_red[w]);
  __syncthreads();
  float l = 0.0f;
  for (int t = tid; t < T; t += kGenThreads) {
    const float p = (m == -INFINITY) ? 0.0f : exp2f(s_p[t] - m);
    s_p[t] = p;
    l += p;
  }
  l = warp_sum(l);
  if (lane == 0) s_red[warp] = l;
  __syncthreads();
  l = 0.0f;
  for (int w = 0; w < kGenThreads / 32; ++w) l += s_red[w];

  for (int d = tid; d < head_dim; d += kGenThreads) {
    float acc = 0.0f;
    for (int t = 0; t < T; ++t) {
      const int pos = t_begin + t;
      const int phys = bt_row[pos / bs];
      if (phys < 0 || (int64_t)phys >= num_blocks) continue;
      const float vs = v_scale[(int64_t)phys * num_kv_heads + kvh];
      const int8_t* vr = v_cache + ((int64_t)phys * bs + pos % bs) * row_stride +
                         (int64_t)kvh * head_dim;
      acc = fmaf(s_p[t] * vs, (float)vr[d], acc);
    }
    if (n_splits == 1) {
      out[((int64_t)seq * num_heads + h) * head_dim + d] = l > 0.0f ? acc / l : 0.0f;
    } else {
      const int64_t slot = ((int64_t)seq * max_splits + split) * num_heads + h;
      ws_acc[slot * head_dim + d] = acc;
      if (d == 0) ws_ml[slot] = make_float2(m, l);
    }
  }
}

// ===========================================================================
// Combine
// ===========================================================================

constexpr int kCombineThreads = 128;  // four (sequence, query head) pairs per CTA
constexpr int kCombineDepth = 8;      // partial rows in flight per lane

// One warp per (sequence, query head): the splits' (m, l) are read one per
// lane, M and the denominator reduced by shuffles, and each lane keeps V =
// head_dim / 32 channels (d = lane + 32 c, coalesced) with kCombineDepth
// partial rows in flight; rows are added in split order (deterministic).
template <int V>
__global__ void __launch_bounds__(kCombineThreads)
    decode_combine_kernel(const int32_t* __restrict__ seq_lens, const float* __restrict__ ws_acc,
                          const float2* __restrict__ ws_ml, float* __restrict__ out, int num_seqs,
                          int num_heads, int bs, int max_blocks_per_seq, int pages_per_split,
                          int max_splits) {
  constexpr int D = 32 * V;
  const int lane = threadIdx.x & 31;
  const int64_t pair = (int64_t)blockIdx.x * (kCombineThreads / 32) + (threadIdx.x >> 5);
  if (pair >= (int64_t)num_seqs * num_heads) return;  // whole warps
  const int seq = (int)(pair / num_heads);
  const int h = (int)(pair - (int64_t)seq * num_heads);
  const int64_t base = (int64_t)seq * max_splits * num_heads + h;
  auto slot_of = [&](int s) { return base + (int64_t)s * num_heads; };
  auto load_rows = [&](int b, int j0, int nb, float (&x)[kCombineDepth][V]) {
#pragma unroll
    for (int jj = 0; jj < kCombineDepth; ++jj) {
      const float* row = ws_acc + slot_of(b + min(j0 + jj, nb - 1)) * D + lane;
#pragma unroll
      for (int c = 0; c < V; ++c) x[jj][c] = __ldcg(row + 32 * c);
    }
  };
  // The (m, l) of the first 32 split slots and the first kCombineDepth
  // partial rows are requested together with the sequence length, before
  // the split count is known: one L2 round trip before the first adds.
  // Slots past the count hold older contents; they are masked out below and
  // never added.  (With one split per sequence there is no workspace.)
  float2 ml_first = make_float2(-INFINITY, 0.0f);
  float x[kCombineDepth][V];
  if (max_splits > 1) {
    ml_first = __ldcg(&ws_ml[slot_of(min(lane, max_splits - 1))]);
    load_rows(0, 0, min(32, max_splits), x);
  }
  const int n_pages = covered_pages(seq_lens[seq], bs, max_blocks_per_seq);
  const int n = (n_pages + pages_per_split - 1) / pages_per_split;
  float* o = out + ((int64_t)seq * num_heads + h) * D;
  if (n == 0) {
#pragma unroll
    for (int c = 0; c < V; ++c) o[lane + 32 * c] = 0.0f;
    return;
  }
  if (n == 1) return;  // written by the split kernel
  auto load_ml = [&](int s) {
    return s < n ? __ldcg(&ws_ml[slot_of(s)]) : make_float2(-INFINITY, 0.0f);
  };
  const float2 ml0 = lane < n ? ml_first : make_float2(-INFINITY, 0.0f);
  float M = ml0.x;
  for (int b = 32; b < n; b += 32) M = fmaxf(M, load_ml(b + lane).x);
  M = warp_max(M);
  float den = 0.0f;
  float acc[V];
#pragma unroll
  for (int c = 0; c < V; ++c) acc[c] = 0.0f;
  for (int b = 0; b < n; b += 32) {
    const float2 ml = b == 0 ? ml0 : load_ml(b + lane);
    float w = 0.0f;
    if (ml.x != -INFINITY) {
      w = exp2f(ml.x - M);
      den += w * ml.y;
    }
    const int nb = min(32, n - b);
    for (int j0 = 0; j0 < nb; j0 += kCombineDepth) {
      if (b + j0 > 0) load_rows(b, j0, nb, x);
#pragma unroll
      for (int jj = 0; jj < kCombineDepth; ++jj) {
        const float wj = __shfl_sync(0xffffffffu, w, (j0 + jj) & 31);
        if (j0 + jj < nb && wj != 0.0f) {  // rows of empty splits are not added
#pragma unroll
          for (int c = 0; c < V; ++c) acc[c] += wj * x[jj][c];
        }
      }
    }
  }
  den = warp_sum(den);
  const float inv = den > 0.0f ? 1.0f / den : 0.0f;
#pragma unroll
  for (int c = 0; c < V; ++c) o[lane + 32 * c] = acc[c] * inv;
}

// ===========================================================================
// Tensor-core kernel for GQA groups (tcgen05, int8, accumulators in TMEM)
// ===========================================================================
//
// With G = 2..8 query heads per KV head the CUDA-core kernels spend G x 12
// dp4a and G x 3 shared-memory digit loads per 16 bytes of K, and fall to
// ~1 TB/s.  Here one CTA owns (sequence, KV head, split of <= 512 tokens)
// and the products run on the tensor cores:
//
//   q.K  D1[t, n] = sum_d K[t, d] * Qd[n, d]   M = 128 tokens (8 pages), N = G x 3
//        query digit planes (padded to 8/16/32), K-major A (the TMA page
//        rows) and B (the digit planes), s8 x s8 -> s32 in TMEM;
//   p.V  D2[d, n] = sum_t V[t, d] * Pd[n, t]   M = 128 channels, N = G x 3
//        probability planes, A = the V page rows read MN-major, B = the
//        planes written K-major by the softmax warps, s8 x u8 -> s32.
//
// The integer formats are the CUDA-core path's (query as three signed
// base-256 digits of a 24-bit integer, p * v_scale as a 24-bit fixed point
// relative to the split's largest V scale), so results match it to fp32
// rounding.  Warp 0 issues the TMA page loads (one (128, 1, 16) box per
// page: one head, so a tile is 128 consecutive 128-byte rows), warp 1 owns
// tensor memory and issues the MMAs, warps 4-7 (one per 32-lane TMEM
// quarter) turn logits into probabilities and read the results; partials
// go through decode_combine_kernel.

// STAGES page-tile stages per CTA; MINB CTAs per SM (launch bound); splits
// of at most MAXTILES 128-token tiles.  Several small CTAs per SM (2 stages
// each: the bytes in flight per SM of 2 CTAs with 4) overlap each other's
// prologue, softmax and epilogue.  Groups of 8 take 2-tile splits, so that
// 3 CTAs fit the SM's registers and tensor memory.
template <int G, int STAGES = 2, int MINB = (G <= 4 ? 4 : 3), int MAXTILES = (G <= 4 ? 4 : 2)>
struct TcCfg {
  static constexpr int kNQ = G * 3 <= 8 ? 8 : (G * 3 <= 16 ? 16 : 32);  // MMA N
  static constexpr int kTileTok = 128;
  static constexpr int kPagesPerTile = 8;
  static constexpr int kMaxTiles = MAXTILES;
  static constexpr int kMaxTok = kMaxTiles * kTileTok;
  static constexpr int kMaxPages = kMaxTiles * kPagesPerTile;
  static constexpr int kStages = STAGES;
  static constexpr int kMinBlocks = MINB;
  static constexpr int kThreads = 256;
  static constexpr int kRowBytes = ((kNQ * 128 + 1023) / 1024) * 1024;  // one operand tile
  static constexpr int kOffQ = kStages * kStageBytes;
  static constexpr int kOffP = kOffQ + kRowBytes;
  static constexpr int kOffLogit = kOffP + kMaxTiles * kRowBytes;
  static constexpr int kOffPhys = kOffLogit + G * kMaxTok * 4;
  static constexpr int kOffKs = kOffPhys + kMaxPages * 4;
  static constexpr int kOffVs = kOffKs + kMaxPages * 4;
  static constexpr int kOffQs = kOffVs + kMaxPages * 4;
  static constexpr int kOffRed = kOffQs + 32;
  static constexpr int kOffTmem = kOffRed + 2 * 4 * 8 * 4;
  static constexpr int kOffBar = kOffTmem + 16;
  static constexpr int kNumBars = 2 * kStages + 3;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 1024;
  // D1: one kNQ-column slice per K tile, then D2
  static constexpr int kD2Col = kMaxTiles * kNQ;
  static constexpr int kTmemCols = (kD2Col + kNQ) <= 64 ? 64 : ((kD2Col + kNQ) <= 128 ? 128 : 256);
  static_assert(kMinBlocks * (kSmemBytes + 1024) <= 228 * 1024, "CTAs per SM by shared memory");
  static_assert((kMinBlocks + 1) * kTmemCols <= 512 ||
                    (kMinBlocks + 1) * (kSmemBytes + 1024) > 228 * 1024,
                "every CTA that fits on an SM must fit in its tensor memory");
  static_assert(kMinBlocks * kTmemCols <= 512, "tensor memory for kMinBlocks CTAs");
};

// Calls f(g, v) for each query head g of a TMEM accumulator row holding the
// three digit / plane columns 3g, 3g + 1, 3g + 2 (v = c2 * 65536 + c1 * 256
// + c0 as float).  Rows wider than 16 columns are read in two 16-aligned
// loads; the group straddling them (columns 15-17) is assembled from both.
template <int G, int NQ, typename F>
__device__ __forceinline__ void tmem_row_groups(uint32_t taddr, F f) {
  auto combine = [](uint32_t c0, uint32_t c1, uint32_t c2) {
    return (float)(int)c2 * 65536.0f + ((float)(int)c1 * 256.0f + (float)(int)c0);
  };
  if constexpr (NQ <= 16) {
    uint32_t r[NQ];
    tmem_load<NQ>(taddr, r);
    tmem_wait_load();
#pragma unroll
    for (int g = 0; g < G; ++g) f(g, combine(r[3 * g], r[3 * g + 1], r[3 * g + 2]));
  } else {
    static_assert(NQ == 32 && G >= 6 && G <= 10, "two-slice rows");
    uint32_t a[16];
    tmem_load<16>(taddr, a);
    tmem_wait_load();
#pragma unroll
    for (int g = 0; g < 5; ++g) f(g, combine(a[3 * g], a[3 * g + 1], a[3 * g + 2]));
    const uint32_t c15 = a[15];
    uint32_t b[16];
    tmem_load<16>(taddr + 16, b);
    tmem_wait_load();
    f(5, combine(c15, b[0], b[1]));
#pragma unroll
    for (int g = 6; g < G; ++g) f(g, combine(b[3 * g - 16], b[3 * g - 15], b[3 * g - 14]));
  }
}

template <int G>
__global__ void __launch_bounds__(256, TcCfg<G>::kMinBlocks)
    decode_tc_kernel(const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const float* __restrict__ q,
                     const float* __restrict__ k_scale, const float* __restrict__ v_scale,
                     const int32_t* __restrict__ block_tables, const int32_t* __restrict__ seq_lens,
                     float* __restrict__ out, float* __restrict__ ws_acc,
                     float2* __restrict__ ws_ml, int num_heads, int num_kv_heads,
                     int64_t num_blocks, int max_blocks_per_seq, float qk_scale,
                     int pages_per_split, int max_splits, int* err) {
  using C = TcCfg<G>;
  constexpr int NQ = C::kNQ;
  constexpr int BS = 16;
  const int seq = blockIdx.x, split = blockIdx.y, j = blockIdx.z;
  const int L = max(seq_lens[seq], 0);
  const int n_pages = covered_pages(L, BS, max_blocks_per_seq);
  if (split == 0 && j == 0 && threadIdx.x == 0 && L > n_pages * BS) record_error(err, kDevSeqTooLong);
  const int n_splits = (n_pages + pages_per_split - 1) / pages_per_split;
  if (split >= n_splits) return;  // uniform, before any barrier or TMEM use
  const int p0 = split * pages_per_split;
  const int np = min(pages_per_split, n_pages - p0);
  const int T = min(L, (p0 + np) * BS) - p0 * BS;
  const int n_tiles = (np + C::kPagesPerTile - 1) / C::kPagesPerTile;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* s_q = smem + C::kOffQ;
  uint8_t* s_p = smem + C::kOffP;
  float* s_logit = reinterpret_cast<float*>(smem + C::kOffLogit);
  int* s_phys = reinterpret_cast<int*>(smem + C::kOffPhys);
  float* s_ks = reinterpret_cast<float*>(smem + C::kOffKs);
  float* s_vs = reinterpret_cast<float*>(smem + C::kOffVs);
  float* s_qs = reinterpret_cast<float*>(smem + C::kOffQs);
  float* s_red = reinterpret_cast<float*>(smem + C::kOffRed);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffTmem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + C::kStages;
  uint64_t* k_done = empty + C::kStages;
  uint64_t* p_ready = k_done + 1;
  uint64_t* pv_done = p_ready + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(k_done, 1);
    mbar_init(p_ready, 1);
    mbar_init(pv_done, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(s_tmem, C::kTmemCols);
  if (warp == 0) {  // the split's block ids: all the page loads need
    for (int pg = lane; pg < np; pg += 32) {
      const int phys = block_tables[(int64_t)seq * max_blocks_per_seq + p0 + pg];
      const bool ok = phys >= 0 && (int64_t)phys < num_blocks;
      if (!ok) record_error(err, kDevBadBlockId);
      s_phys[pg] = ok ? phys : -1;
    }
  }
  tmem_fence_before_sync();
  __syncthreads();  // barriers initialized, block ids and TMEM base published
  tmem_fence_after_sync();
  // The page loads start now; scales and query digits load meanwhile and are
  // published to the MMA and epilogue warps (1-7) by named barrier 2.
  if (warp == 2 || warp == 3) {
    for (int pg = tid - 64; pg < np; pg += 64) {
      const int phys = s_phys[pg];
      const int64_t si = (int64_t)(phys >= 0 ? phys : 0) * num_kv_heads + j;
      s_ks[pg] = phys >= 0 ? k_scale[si] : 0.0f;
      s_vs[pg] = phys >= 0 ? v_scale[si] : 0.0f;
    }
  }
  if (warp >= 4) {  // query digit planes: row 3g + plane of the B operand
    const int w4 = warp - 4;
    for (int g = w4; g < G; g += 4) {
      const float4 x = reinterpret_cast<const float4*>(
          q + ((int64_t)seq * num_heads + (int64_t)j * G + g) * 128)[lane];
      float m = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
      m = warp_max(m);
      const float inv = m > 0.0f ? (float)kQFix / m : 0.0f;
      const float xs[4] = {x.x, x.y, x.z, x.w};
      int d[4][3];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int n = __float2int_rn(xs[e] * inv);
        n = max(-kQFix, min(kQFix, n));
        to_digits(n, d[e][0], d[e][1], d[e][2]);
      }
#pragma unroll
      for (int pl = 0; pl < 3; ++pl)
        *reinterpret_cast<uint32_t*>(s_q + sw128_offset(3 * g + pl, 4 * lane)) =
            pack4(d[0][pl], d[1][pl], d[2][pl], d[3][pl]);
      if (lane == 0) s_qs[g] = m > 0.0f ? m / (float)kQFix : 0.0f;
    }
    for (int r = 3 * G + w4; r < NQ; r += 4)  // padding rows
      *reinterpret_cast<uint32_t*>(s_q + sw128_offset(r, 4 * lane)) = 0u;
    fence_proxy_async_smem();  // the digit planes are an MMA operand
  }
  if (warp >= 1) named_barrier(2, C::kThreads - 32);
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ---- TMA: K tiles of the split, then its V tiles -------------------------
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
      int ns = 0;
      bool ok_run = true;
      for (int kind = 0; kind < 2 && ok_run; ++kind) {
        for (int ti = 0; ti < n_tiles; ++ti, ++ns) {
          const int st = ns % C::kStages;
          const uint32_t ph = (uint32_t)(ns / C::kStages) & 1u;
          if (!mbar_wait_bounded(&empty[st], ph ^ 1u, err)) {
            record_error(err, kDevWaitTimeout);
            ok_run = false;
            break;
          }
          const int pb = ti * C::kPagesPerTile;
          const int pe = min(np, pb + C::kPagesPerTile);
          mbar_arrive_expect_tx(&full[st], (uint32_t)((pe - pb) * BS * 128));
          for (int pg = pb; pg < pe; ++pg)
            tma_load_3d(smem + st * kStageBytes + (pg - pb) * BS * 128, kind ? &map_v : &map_k,
                        &full[st], 0, j, max(s_phys[pg], 0) * BS, policy);
        }
      }
      drain_ring(full, C::kStages, ns);  // no copy outlives the CTA
    }
  } else if (warp == 1) {
    // ---- MMA issue: one thread ---------------------------------------------
    if (lane == 0) {
      constexpr uint32_t kIdQK = umma_i8_idesc(1, 1, 0, 0, 128, NQ);
      constexpr uint32_t kIdPV = umma_i8_idesc(1, 0, 1, 0, 128, NQ);
      const uint32_t stage0 = smem_u32(smem);
      const uint32_t qaddr = smem_u32(s_q);
      const uint32_t paddr = smem_u32(s_p);
      int ns = 0;
      bool ok_run = true;
      for (int ti = 0; ti < n_tiles && ok_run; ++ti, ++ns) {
        const int st = ns % C::kStages;
        if (!mbar_wait_bounded(&full[st], (uint32_t)(ns / C::kStages) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          ok_run = false;
          break;
        }
        tmem_fence_after_sync();
        const uint32_t a = stage0 + st * kStageBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_i8(tmem + ti * NQ, umma_sw128_desc(a + k * 32, 16, 1024),
                  umma_sw128_desc(qaddr + k * 32, 16, 1024), kIdQK, k > 0);
        // frees the stage once these MMAs complete -- only when a later tile of
        // this CTA reuses it: an arrival nobody waits for could land after the
        // CTA has exited, in shared memory that belongs to the next CTA
        if (ns + C::kStages < 2 * n_tiles) umma_commit(&empty[st]);
      }
      umma_commit(k_done);
      if (ok_run && !mbar_wait_bounded(p_ready, 0, err)) {
        record_error(err, kDevWaitTimeout);
        ok_run = false;
      }
      tmem_fence_after_sync();
      for (int ti = 0; ti < n_tiles && ok_run; ++ti, ++ns) {
        const int st = ns % C::kStages;
        if (!mbar_wait_bounded(&full[st], (uint32_t)(ns / C::kStages) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          ok_run = false;
          break;
        }
        tmem_fence_after_sync();
        const uint32_t a = stage0 + st * kStageBytes;
        const uint32_t b = paddr + ti * C::kRowBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_i8(tmem + C::kD2Col, umma_sw128_desc(a + k * 4096, 16, 1024),
                  umma_sw128_desc(b + k * 32, 16, 1024), kIdPV, (ti > 0 || k > 0) ? 1u : 0u);
        if (ns + C::kStages < 2 * n_tiles) umma_commit(&empty[st]);
      }
      umma_commit(pv_done);  // the last arrival: the epilogue waits for it
      mbar_drain(pv_done, 0);  // every MMA of this thread is done before TMEM is freed
    }
  } else if (warp >= 4) {
    // ---- logits, softmax, probability planes, output -----------------------
    const int w4 = warp - 4;
    const int e = tid - 128;  // TMEM lane: token of a tile, then channel
    const uint32_t lane_base = (uint32_t)(32 * w4) << 16;
    bool live = mbar_wait_bounded(k_done, 0, err);
    if (!live) record_error(err, kDevWaitTimeout);
    tmem_fence_after_sync();
    float kmax[G];
#pragma unroll
    for (int g = 0; g < G; ++g) kmax[g] = -INFINITY;
    for (int ti = 0; ti < n_tiles; ++ti) {
      const int tok = ti * C::kTileTok + e;
      const int pg = min(tok / BS, C::kMaxPages - 1);
      const bool valid = live && tok < T && s_phys[pg] >= 0;
      const float ks = s_ks[pg];
      tmem_row_groups<G, NQ>(tmem + lane_base + ti * NQ, [&](int g, float v) {
        const float logit = valid ? v * (s_qs[g] * ks * qk_scale) : -INFINITY;
        s_logit[g * C::kMaxTok + tok] = logit;
        kmax[g] = fmaxf(kmax[g], logit);
      });
    }
    float* red_m = s_red;
    float* red_l = s_red + 32;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float m = warp_max(kmax[g]);
      if (lane == 0) red_m[w4 * 8 + g] = m;
    }
    float vmax = 0.0f;
    for (int pg = 0; pg < np; ++pg) vmax = fmaxf(vmax, s_vs[pg]);
    const float to_fix = vmax > 0.0f ? 16777215.0f / vmax : 0.0f;
    named_barrier(1, 128);
    float m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m[g] = fmaxf(fmaxf(red_m[g], red_m[8 + g]), fmaxf(red_m[16 + g], red_m[24 + g]));
      l[g] = 0.0f;
    }
    for (int ti = 0; ti < n_tiles; ++ti) {
      const int tok = ti * C::kTileTok + e;
      const float vs = s_vs[min(tok / BS, C::kMaxPages - 1)];
      uint8_t* pt = s_p + ti * C::kRowBytes;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        uint32_t n = 0;
        if (tok < T && m[g] != -INFINITY) {
          const float p = exp2f(s_logit[g * C::kMaxTok + tok] - m[g]);
          l[g] += p;
          n = __float2uint_rn(fminf(p * vs * to_fix, 16777215.0f));
        }
        pt[sw128_offset(3 * g, e)] = (uint8_t)(n & 255u);
        pt[sw128_offset(3 * g + 1, e)] = (uint8_t)((n >> 8) & 255u);
        pt[sw128_offset(3 * g + 2, e)] = (uint8_t)(n >> 16);
      }
      for (int rw = 3 * G; rw < NQ; ++rw) pt[sw128_offset(rw, e)] = 0;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float s = warp_sum(l[g]);
      if (lane == 0) red_l[w4 * 8 + g] = s;
    }
    fence_proxy_async_smem();
    named_barrier(1, 128);
    if (e == 0) mbar_arrive(p_ready);
#pragma unroll
    for (int g = 0; g < G; ++g)
      l[g] = (red_l[g] + red_l[8 + g]) + (red_l[16 + g] + red_l[24 + g]);
    if (live && !mbar_wait_bounded(pv_done, 0, err)) {
      record_error(err, kDevWaitTimeout);
      live = false;
    }
    tmem_fence_after_sync();
    const float back = vmax * (1.0f / 16777215.0f);
    tmem_row_groups<G, NQ>(tmem + lane_base + C::kD2Col, [&](int g, float v) {
      const float acc = v * back;
      const int hq = j * G + g;
      if (n_splits == 1) {
        out[((int64_t)seq * num_heads + hq) * 128 + e] = l[g] > 0.0f ? acc / l[g] : 0.0f;
      } else {
        const int64_t slot = ((int64_t)seq * max_splits + split) * num_heads + hq;
        ws_acc[slot * 128 + e] = acc;
        if (e == 0) ws_ml[slot] = make_float2(m[g], l[g]);
      }
    });
  }
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// ---------------------------------------------------------------------------
// Persistent form: CTAs walk their share of the (sequence, KV head, split)
// units, so the page ring stays busy from one unit to the next.
// ---------------------------------------------------------------------------
//
// Unit k of a CTA is its k-th non-empty unit of c, c + C, c + 2C, ...  Two
// table warps fill the unit's half of a double-buffered table (block ids,
// scales, token count and the query digit planes) and publish it on
// meta_full[k & 1]; the half is released on meta_free[k & 1] by the TMA
// warp (its loads issued), the MMA lane (a commit: its q.K MMAs completed)
// and the epilogue (softmax done).  Per unit the MMA lane runs q.K into D1
// (after the epilogue has read the previous unit's D1: d1_free), then p.V
// into D2 (after p_ready); the epilogue reads D1 (k_done), writes the
// probability planes, reads D2 (pv_done).  Each of those barriers completes
// once per unit and its waiters are at most one phase behind, so parity
// waits cannot alias.  Asynchronous (commit) arrivals target only stages
// and table halves that a later tile or unit of the same CTA reuses.

template <int G>
struct TcsCfg {
  static constexpr int kNQ = G * 3 <= 8 ? 8 : (G * 3 <= 16 ? 16 : 32);
  static constexpr int kTileTok = 128;
  static constexpr int kPagesPerTile = 8;
  static constexpr int kMaxTiles = G <= 4 ? 4 : 2;
  static constexpr int kMaxTok = kMaxTiles * kTileTok;
  static constexpr int kMaxPages = kMaxTiles * kPagesPerTile;
  // four CTAs per SM with 2-stage rings beat three with 3-stage rings (one
  // more unit chain per SM); groups of 8 do not fit four CTAs' shared memory
  static constexpr int kStages = G <= 4 ? 2 : 3;
  static constexpr int kMinBlocks = G <= 4 ? 4 : 3;
  static constexpr int kThreads = 256;
  static constexpr int kRowBytes = ((kNQ * 128 + 1023) / 1024) * 1024;
  // table halves: the query digit tiles (1 KB aligned, an MMA operand), and
  // apart from them block ids, scales, per-head q scale, token count and
  // largest V scale
  static constexpr int kOffQ = kStages * kStageBytes;
  static constexpr int kMetaPhys = 0;
  static constexpr int kMetaKs = kMetaPhys + kMaxPages * 4;
  static constexpr int kMetaVs = kMetaKs + kMaxPages * 4;
  static constexpr int kMetaQs = kMetaVs + kMaxPages * 4;
  static constexpr int kMetaT = kMetaQs + 32;
  static constexpr int kMetaBytes = (kMetaT + 16 + 15) & ~15;
  static constexpr int kOffMeta = kOffQ + 2 * kRowBytes;
  static constexpr int kOffP = ((kOffMeta + 2 * kMetaBytes + 1023) / 1024) * 1024;
  static constexpr int kOffLogit = kOffP + kMaxTiles * kRowBytes;
  static constexpr int kOffRed = kOffLogit + G * kMaxTok * 4;
  static constexpr int kOffTmem = kOffRed + 2 * 4 * 8 * 4;
  static constexpr int kOffBar = kOffTmem + 16;
  // full[S], empty[S], meta_full[2], meta_free[2], k_done, d1_free, p_ready, pv_done
  static constexpr int kNumBars = 2 * kStages + 8;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 1024;
  static constexpr int kD2Col = kMaxTiles * kNQ;
  static constexpr int kTmemCols = (kD2Col + kNQ) <= 64 ? 64 : ((kD2Col + kNQ) <= 128 ? 128 : 256);
  static_assert(kMinBlocks * (kSmemBytes + 1024) <= 228 * 1024, "CTAs per SM by shared memory");
  static_assert((kMinBlocks + 1) * kTmemCols <= 512 ||
                    (kMinBlocks + 1) * (kSmemBytes + 1024) > 228 * 1024,
                "every CTA that fits on an SM must fit in its tensor memory");
  static_assert(kMinBlocks * kTmemCols <= 512, "tensor memory");
};

// Unit u -> (sequence, KV head, split) and its page range; false if empty.
struct TcsUnit {
  int seq, j, split, p0, np, T, n_splits, n_tiles;
};
__device__ __forceinline__ bool tcs_unit(int64_t u, int hkv, int max_splits, int pps,
                                         const int32_t* seq_lens, int max_blocks_per_seq,
                                         TcsUnit& r) {
  const int64_t per_seq = (int64_t)hkv * max_splits;
  r.seq = (int)(u / per_seq);
  const int rem = (int)(u - (int64_t)r.seq * per_seq);
  r.j = rem / max_splits;
  r.split = rem % max_splits;
  const int L = max(seq_lens[r.seq], 0);
  const int n_pages = covered_pages(L, 16, max_blocks_per_seq);
  r.n_splits = (n_pages + pps - 1) / pps;
  if (r.split >= r.n_splits) return false;
  r.p0 = r.split * pps;
  r.np = min(pps, n_pages - r.p0);
  r.T = min(L, (r.p0 + r.np) * 16) - r.p0 * 16;
  r.n_tiles = (r.np + 7) / 8;
  return true;
}

template <int G>
__global__ void __launch_bounds__(256, TcsCfg<G>::kMinBlocks)
    decode_tc_stream_kernel(const __grid_constant__ CUtensorMap map_k,
                            const __grid_constant__ CUtensorMap map_v, const float* __restrict__ q,
                            const float* __restrict__ k_scale, const float* __restrict__ v_scale,
                            const int32_t* __restrict__ block_tables,
                            const int32_t* __restrict__ seq_lens, float* __restrict__ out,
                            float* __restrict__ ws_acc, float2* __restrict__ ws_ml, int num_seqs,
                            int num_heads, int num_kv_heads, int64_t num_blocks,
                            int max_blocks_per_seq, float qk_scale, int pages_per_split,
                            int max_splits, int* err) {
  using C = TcsCfg<G>;
  constexpr int NQ = C::kNQ;
  constexpr int BS = 16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* s_p = smem + C::kOffP;
  float* s_logit = reinterpret_cast<float*>(smem + C::kOffLogit);
  float* s_red = reinterpret_cast<float*>(smem + C::kOffRed);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffTmem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + C::kStages;
  uint64_t* meta_full = empty + C::kStages;
  uint64_t* meta_free = meta_full + 2;
  uint64_t* k_done = meta_free + 2;
  uint64_t* d1_free = k_done + 1;
  uint64_t* p_ready = d1_free + 1;
  uint64_t* pv_done = p_ready + 1;
  auto meta = [&](int b) { return smem + C::kOffMeta + b * C::kMetaBytes; };
  auto qtile = [&](int b) { return smem + C::kOffQ + b * C::kRowBytes; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n_units = (int64_t)num_seqs * num_kv_heads * max_splits;
  const int64_t stride = gridDim.x;
  if (blockIdx.x == 0)  // lengths beyond the table width, checked by all threads of CTA 0
    for (int s = tid; s < num_seqs; s += C::kThreads)
      if (max(seq_lens[s], 0) > covered_pages(seq_lens[s], BS, max_blocks_per_seq) * BS)
        record_error(err, kDevSeqTooLong);
  // probability tiles: rows 3G..NQ-1 (MMA padding) are never written again
  for (int i = tid; i < C::kMaxTiles * C::kRowBytes / 4; i += C::kThreads)
    reinterpret_cast<uint32_t*>(s_p)[i] = 0u;
  fence_proxy_async_smem();  // an MMA operand
  if (tid == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&meta_full[i], 2);  // the two table warps
      mbar_init(&meta_free[i], 3);  // TMA warp, MMA lane (commit), epilogue
    }
    mbar_init(k_done, 1);
    mbar_init(d1_free, 1);
    mbar_init(p_ready, 1);
    mbar_init(pv_done, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(s_tmem, C::kTmemCols);
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tmem = *s_tmem;

  if (warp == 2 || warp == 3) {
    // ---- chunk tables: warp 2 block ids / scales / counts, warp 3 query digits
    TcsUnit un;
    int k = 0;
    for (int64_t u = blockIdx.x; u < n_units; u += stride) {
      if (!tcs_unit(u, num_kv_heads, max_splits, pages_per_split, seq_lens, max_blocks_per_seq, un))
        continue;
      const int b = k & 1;
      if (k >= 2) {
        bool ok = true;
        if (lane == 0 && !mbar_wait_bounded(&meta_free[b], (uint32_t)((k >> 1) - 1) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          ok = false;
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
      uint8_t* m = meta(b);
      if (warp == 2) {
        int* phys_t = reinterpret_cast<int*>(m + C::kMetaPhys);
        float* ks_t = reinterpret_cast<float*>(m + C::kMetaKs);
        float* vs_t = reinterpret_cast<float*>(m + C::kMetaVs);
        float vmax = 0.0f;
        for (int pg = lane; pg < un.np; pg += 32) {
          const int phys = block_tables[(int64_t)un.seq * max_blocks_per_seq + un.p0 + pg];
          const bool okb = phys >= 0 && (int64_t)phys < num_blocks;
          if (!okb) record_error(err, kDevBadBlockId);
          phys_t[pg] = okb ? phys : -1;
          const int64_t si = (int64_t)(okb ? phys : 0) * num_kv_heads + un.j;
          ks_t[pg] = okb ? k_scale[si] : 0.0f;
          const float vs = okb ? v_scale[si] : 0.0f;
          vs_t[pg] = vs;
          vmax = fmaxf(vmax, vs);
        }
        vmax = warp_max(vmax);
        if (lane == 0) {
          reinterpret_cast<int*>(m + C::kMetaT)[0] = un.T;
          reinterpret_cast<float*>(m + C::kMetaT)[1] = vmax;
        }
      } else {
        uint8_t* sq = qtile(b);
        float* qs_t = reinterpret_cast<float*>(m + C::kMetaQs);
        for (int g = 0; g < G; ++g) {
          const float4 x = reinterpret_cast<const float4*>(
              q + ((int64_t)un.seq * num_heads + (int64_t)un.j * G + g) * 128)[lane];
          float mx = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
          mx = warp_max(mx);
          const float inv = mx > 0.0f ? (float)kQFix / mx : 0.0f;
          const float xs[4] = {x.x, x.y, x.z, x.w};
          int d[4][3];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            int n = __float2int_rn(xs[e] * inv);
            n = max(-kQFix, min(kQFix, n));
            to_digits(n, d[e][0], d[e][1], d[e][2]);
          }
#pragma unroll
          for (int pl = 0; pl < 3; ++pl)
            *reinterpret_cast<uint32_t*>(sq + sw128_offset(3 * g + pl, 4 * lane)) =
                pack4(d[0][pl], d[1][pl], d[2][pl], d[3][pl]);
          if (lane == 0) qs_t[g] = mx > 0.0f ? mx / (float)kQFix : 0.0f;
        }
        for (int r = 3 * G; r < NQ; ++r)
          *reinterpret_cast<uint32_t*>(sq + sw128_offset(r, 4 * lane)) = 0u;
        fence_proxy_async_smem();  // an MMA operand
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_full[b]);
      ++k;
    }
  } else if (warp == 0) {
    // ---- TMA: per unit its K tiles, then its V tiles.  The whole warp
    // issues: lane 0 waits for a stage and arms its barrier, then lane i
    // issues page i of the tile (one 2 KB box per page and KV head; one
    // issuing thread managed ~one box per 85 ns).
    const uint64_t policy = l2_policy_evict_first();
    if (lane == 0) {
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
    }
    TcsUnit un;
    int k = 0, ns = 0;
    bool ok_run = true;
    for (int64_t u = blockIdx.x; u < n_units && ok_run; u += stride) {
      if (!tcs_unit(u, num_kv_heads, max_splits, pages_per_split, seq_lens, max_blocks_per_seq, un))
        continue;
      const int b = k & 1;
      bool ok = true;
      if (lane == 0 && !mbar_wait_bounded(&meta_full[b], (uint32_t)(k >> 1) & 1u, err)) {
        record_error(err, kDevWaitTimeout);
        ok = false;
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      const int* phys_t = reinterpret_cast<const int*>(meta(b) + C::kMetaPhys);
      for (int kind = 0; kind < 2 && ok_run; ++kind) {
        for (int ti = 0; ti < un.n_tiles; ++ti, ++ns) {
          const int st = ns % C::kStages;
          const int pb = ti * 8, pe = min(un.np, pb + 8);
          bool oks = true;
          if (lane == 0) {
            if (!mbar_wait_bounded(&empty[st], ((uint32_t)(ns / C::kStages) & 1u) ^ 1u, err)) {
              record_error(err, kDevWaitTimeout);
              oks = false;
            } else {
              mbar_arrive_expect_tx(&full[st], (uint32_t)((pe - pb) * BS * 128));
            }
          }
          oks = __shfl_sync(0xffffffffu, oks, 0);
          __syncwarp();  // the stage is armed before any of its copies is issued
          if (!oks) {
            ok_run = false;
            break;
          }
          if (lane < pe - pb)
            tma_load_3d(smem + st * kStageBytes + lane * BS * 128, kind ? &map_v : &map_k,
                        &full[st], 0, un.j, max(phys_t[pb + lane], 0) * BS, policy);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_free[b]);
      ++k;
    }
    if (lane == 0) drain_ring(full, C::kStages, ns);  // no copy outlives the CTA
  } else if (warp == 1) {
    // ---- MMA issue ---------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t kIdQK = umma_i8_idesc(1, 1, 0, 0, 128, NQ);
      constexpr uint32_t kIdPV = umma_i8_idesc(1, 0, 1, 0, 128, NQ);
      const uint32_t stage0 = smem_u32(smem);
      const uint32_t paddr = smem_u32(s_p);
      TcsUnit un;
      // this CTA's units and page tiles, for the reuse tests below
      int total_units = 0, total_ns = 0;
      for (int64_t u = blockIdx.x; u < n_units; u += stride)
        if (tcs_unit(u, num_kv_heads, max_splits, pages_per_split, seq_lens, max_blocks_per_seq, un)) {
          ++total_units;
          total_ns += 2 * un.n_tiles;
        }
      int k = 0, ns = 0;
      bool ok_run = true;
      for (int64_t u = blockIdx.x; u < n_units && ok_run; u += stride) {
        if (!tcs_unit(u, num_kv_heads, max_splits, pages_per_split, seq_lens, max_blocks_per_seq, un))
          continue;
        const int b = k & 1;
        const uint32_t qaddr = smem_u32(qtile(b));
        if (!mbar_wait_bounded(&meta_full[b], (uint32_t)(k >> 1) & 1u, err) ||
            (k > 0 && !mbar_wait_bounded(d1_free, (uint32_t)(k - 1) & 1u, err))) {
          record_error(err, kDevWaitTimeout);
          break;
        }
        tmem_fence_after_sync();
        for (int ti = 0; ti < un.n_tiles && ok_run; ++ti, ++ns) {
          const int st = ns % C::kStages;
          if (!mbar_wait_bounded(&full[st], (uint32_t)(ns / C::kStages) & 1u, err)) {
            record_error(err, kDevWaitTimeout);
            ok_run = false;
            break;
          }
          tmem_fence_after_sync();
          const uint32_t a = stage0 + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8(tmem + ti * NQ, umma_sw128_desc(a + kk * 32, 16, 1024),
                    umma_sw128_desc(qaddr + kk * 32, 16, 1024), kIdQK, kk > 0);
          if (ns + C::kStages < total_ns) umma_commit(&empty[st]);
        }
        umma_commit(k_done);
        if (k + 2 < total_units) umma_commit(&meta_free[b]);  // q digits read
        if (ok_run && !mbar_wait_bounded(p_ready, (uint32_t)k & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          ok_run = false;
        }
        tmem_fence_after_sync();
        for (int ti = 0; ti < un.n_tiles && ok_run; ++ti, ++ns) {
          const int st = ns % C::kStages;
          if (!mbar_wait_bounded(&full[st], (uint32_t)(ns / C::kStages) & 1u, err)) {
            record_error(err, kDevWaitTimeout);
            ok_run = false;
            break;
          }
          tmem_fence_after_sync();
          const uint32_t a = stage0 + st * kStageBytes;
          const uint32_t pb = paddr + ti * C::kRowBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8(tmem + C::kD2Col, umma_sw128_desc(a + kk * 4096, 16, 1024),
                    umma_sw128_desc(pb + kk * 32, 16, 1024), kIdPV, (ti > 0 || kk > 0) ? 1u : 0u);
          if (ns + C::kStages < total_ns) umma_commit(&empty[st]);
        }
        umma_commit(pv_done);
        ++k;
      }
      // every MMA of this thread is done before TMEM is freed
      if (k > 0) mbar_drain(pv_done, (uint32_t)(k - 1) & 1u);
    }
  } else {
    // ---- epilogue: logits, softmax, probability planes, output ------------------
    const int w4 = warp - 4;
    const int e = tid - 128;
    const uint32_t lane_base = (uint32_t)(32 * w4) << 16;
    float* red_m = s_red;
    float* red_l = s_red + 32;
    TcsUnit un;
    int k = 0;
    bool live = true;
    for (int64_t u = blockIdx.x; u < n_units; u += stride) {
      if (!tcs_unit(u, num_kv_heads, max_splits, pages_per_split, seq_lens, max_blocks_per_seq, un))
        continue;
      const int b = k & 1;
      const uint8_t* m = meta(b);
      const int* phys_t = reinterpret_cast<const int*>(m + C::kMetaPhys);
      const float* ks_t = reinterpret_cast<const float*>(m + C::kMetaKs);
      const float* vs_t = reinterpret_cast<const float*>(m + C::kMetaVs);
      const float* qs_t = reinterpret_cast<const float*>(m + C::kMetaQs);
      if (live && (!mbar_wait_bounded(&meta_full[b], (uint32_t)(k >> 1) & 1u, err) ||
                   !mbar_wait_bounded(k_done, (uint32_t)k & 1u, err))) {
        record_error(err, kDevWaitTimeout);
        live = false;
      }
      tmem_fence_after_sync();
      const int T = un.T;
      const float vmax = reinterpret_cast<const float*>(m + C::kMetaT)[1];
      float kmax[G];
#pragma unroll
      for (int g = 0; g < G; ++g) kmax[g] = -INFINITY;
      for (int ti = 0; ti < un.n_tiles; ++ti) {
        const int tok = ti * C::kTileTok + e;
        const int pg = min(tok / BS, C::kMaxPages - 1);
        const bool valid = live && tok < T && phys_t[pg] >= 0;
        const float ks = ks_t[pg];
        tmem_row_groups<G, NQ>(tmem + lane_base + ti * NQ, [&](int g, float v) {
          const float logit = valid ? v * (qs_t[g] * ks * qk_scale) : -INFINITY;
          s_logit[g * C::kMaxTok + tok] = logit;
          kmax[g] = fmaxf(kmax[g], logit);
        });
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float mm = warp_max(kmax[g]);
        if (lane == 0) red_m[w4 * 8 + g] = mm;
      }
      tmem_fence_before_sync();
      named_barrier(1, 128);  // maxima published; D1 read by all four warps
      if (e == 0) mbar_arrive(d1_free);
      const float to_fix = vmax > 0.0f ? 16777215.0f / vmax : 0.0f;
      float mh[G], l[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        mh[g] = fmaxf(fmaxf(red_m[g], red_m[8 + g]), fmaxf(red_m[16 + g], red_m[24 + g]));
        l[g] = 0.0f;
      }
      for (int ti = 0; ti < un.n_tiles; ++ti) {
        const int tok = ti * C::kTileTok + e;
        const float vs = vs_t[min(tok / BS, C::kMaxPages - 1)];
        uint8_t* pt = s_p + ti * C::kRowBytes;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          uint32_t n = 0;
          if (tok < T && mh[g] != -INFINITY) {
            const float p = exp2f(s_logit[g * C::kMaxTok + tok] - mh[g]);
            l[g] += p;
            n = __float2uint_rn(fminf(p * vs * to_fix, 16777215.0f));
          }
          pt[sw128_offset(3 * g, e)] = (uint8_t)(n & 255u);
          pt[sw128_offset(3 * g + 1, e)] = (uint8_t)((n >> 8) & 255u);
          pt[sw128_offset(3 * g + 2, e)] = (uint8_t)(n >> 16);
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float s = warp_sum(l[g]);
        if (lane == 0) red_l[w4 * 8 + g] = s;
      }
      fence_proxy_async_smem();
      named_barrier(1, 128);
      if (e == 0) {
        mbar_arrive(p_ready);
        mbar_arrive(&meta_free[b]);  // the epilogue is done with this table half
      }
#pragma unroll
      for (int g = 0; g < G; ++g)
        l[g] = (red_l[g] + red_l[8 + g]) + (red_l[16 + g] + red_l[24 + g]);
      if (live && !mbar_wait_bounded(pv_done, (uint32_t)k & 1u, err)) {
        record_error(err, kDevWaitTimeout);
        live = false;
      }
      tmem_fence_after_sync();
      const float back = vmax * (1.0f / 16777215.0f);
      tmem_row_groups<G, NQ>(tmem + lane_base + C::kD2Col, [&](int g, float v) {
        const float acc = v * back;
        const int hq = un.j * G + g;
        if (un.n_splits == 1) {
          out[((int64_t)un.seq * num_heads + hq) * 128 + e] = l[g] > 0.0f ? acc / l[g] : 0.0f;
        } else {
          const int64_t slot = ((int64_t)un.seq * max_splits + un.split) * num_heads + hq;
          ws_acc[slot * 128 + e] = acc;
          if (e == 0) ws_ml[slot] = make_float2(mh[g], l[g]);
        }
      });
      tmem_fence_before_sync();
      // every epilogue thread has read D2 before the next unit's p_ready
      // (which lets the MMA lane overwrite it) -- the first named barrier of
      // the next unit orders that
      ++k;
    }
  }
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// ===========================================================================
// Tensor-core decode over whole pages (GQA groups of 2/4/8, bs 16, D 128)
// ===========================================================================
//
// The per-head tensor-core kernels above copy one 2 KB box per (page, KV
// head): on the paged layout such a stream needs ~200 KB in flight per SM to
// reach the HBM peak (a TMA-only probe: 5.1 TB/s at one CTA per SM with a
// 10-stage ring, against 6.3 TB/s for whole 16 KB pages).  This kernel copies
// whole pages, one box per page, through a 4-D tensor map ordered (D, token,
// head, block), so a page lands as [head][token][128 B]: a 128-row stage
// holds 8 / Hkv pages, row r = (page, head, token) with head = (r / 16) % Hkv.
//
//   q.K  D1[128 rows][NQ] = stage (K-major, 128 rows x 128 B) x Qd^T, where
//        Qd holds the 3 digit planes of every (KV head h, query head g):
//        column n = 3 (h G + g) + plane.  Row r only needs the 3G columns of
//        its own head; the rest of the product is discarded (the tensor pipe
//        has the room: ~30 % busy at the HBM rate).
//   p.V  D2[128 dims][NQ] += stage^T (MN-major) x P^T, where P is
//        block-diagonal: P[n][r] is the probability plane n of row r if the
//        head of column n is the head of row r, else 0.
//
// Scheduling is the MHA stream kernel's: one unit per sequence (all KV
// heads), the units' pages flattened into one virtual range split evenly
// over the CTAs (one per SM), chunks of at most 256 tokens, a running
// (m, l, acc) per query head across the chunks of a unit, partials and
// arrival counters where a unit straddles CTAs.  Roles: warp 0 issues the
// page copies, warp 1 the MMAs, warps 2-3 fill the chunk tables (block ids
// and scales; query digits), warps 4-7 (one per TMEM lane quarter) turn
// logits into probability tiles and read the results.
template <int HKV, int G>
struct TcpCfg {
  static constexpr int kHeads = HKV * G;  // query heads of a unit
  // columns per KV head (its G query heads x 3 digit planes, padded so that
  // a warp's two heads start on a 16-column boundary of tensor memory)
  static constexpr int kCS = G == 2 ? 8 : (G == 4 ? 16 : 24);
  static constexpr int kNQ = ((HKV * kCS + 15) / 16) * 16;
  static_assert(kNQ <= 128, "three accumulators of kNQ columns in 512");
  static constexpr int kPPS = 8 / HKV;  // pages per 128-row stage
  static constexpr int kMaxTok = 128;
  static constexpr int kMaxPages = kMaxTok / 16;
  static constexpr int kThreads = 256;
  static constexpr int kRowBytes = ((kNQ * 128 + 1023) / 1024) * 1024;  // q digit / P tile
  static constexpr int kMetaPhys = 0;                                  // int [kMaxPages]
  static constexpr int kMetaKs = kMetaPhys + kMaxPages * 4;            // float [page][HKV]
  static constexpr int kMetaVs = kMetaKs + kMaxPages * HKV * 4;        // float [page][HKV]
  static constexpr int kMetaVmax = kMetaVs + kMaxPages * HKV * 4;      // float [HKV]
  static constexpr int kMetaT = kMetaVmax + 32;                        // int
  static constexpr int kMetaBytes = (kMetaT + 16 + 15) & ~15;
  // chunk tables in flight: the table warp runs this many chunks ahead of the
  // copies, so its loads (which queue behind the SM's page stream) stay off
  // the critical path
  static constexpr int kMetaRing = 4;
  static constexpr int kNumBars = 2 * 10 + 2 * kMetaRing + 2 * 2 + 2 * 2 + 2 * 2 + 2;
  static constexpr int kFixed = 4 * kRowBytes + kHeads * kMaxTok * 4 + kMetaRing * kMetaBytes +
                                2 * 32 * 4 + 3 * kHeads * 8 + 2 * 8 * G * 4 + (kStreamMaxSeqs + 1) * 4 + 64 + 16 +
                                kNumBars * 8;
  static constexpr int kMaxDynSmem = 227 * 1024;
  static constexpr int kStagesFit = (kMaxDynSmem - 1024 - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesFit < 10 ? kStagesFit : 10;
  static_assert(kStages >= 4, "ring stages");
  static constexpr int kOffQ = kStages * kStageBytes;               // [2] digit tiles
  static constexpr int kOffP = kOffQ + 2 * kRowBytes;               // [2] probability tiles
  static constexpr int kOffLogit = kOffP + 2 * kRowBytes;           // [kHeads][kMaxTok]
  static constexpr int kOffMeta = kOffLogit + kHeads * kMaxTok * 4; // [kMetaRing] chunk tables
  static constexpr int kOffQs = kOffMeta + kMetaRing * kMetaBytes;  // float [2][32] query scales
  static constexpr int kOffRun = kOffQs + 2 * 32 * 4;               // float2 [kHeads] running (m, l)
  static constexpr int kOffChunk = kOffRun + kHeads * 8;            // float2 [kHeads] chunk (m, l)
  static constexpr int kOffAB = kOffChunk + kHeads * 8;             // float2 [kHeads] merge factors
  static constexpr int kOffHalf = kOffAB + kHeads * 8;              // float [2][8][G] half-warp max / sum
  static constexpr int kOffPseq = kOffHalf + 2 * 8 * G * 4;         // int [kStreamMaxSeqs + 1]
  static constexpr int kOffTmp = kOffPseq + (kStreamMaxSeqs + 1) * 4;  // int [16]
  static constexpr int kOffTmem = ((kOffTmp + 64) + 15) & ~15;
  static constexpr int kOffBar = kOffTmem + 16;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 1024;
  static_assert(kSmemBytes <= kMaxDynSmem, "shared memory");
  static_assert(kOffQ % 1024 == 0 && kOffP % 1024 == 0, "MMA operand tiles: 1 KB alignment");
  static_assert(kOffMeta % 16 == 0 && kOffBar % 8 == 0, "alignment");
  // tensor memory: D1 double-buffered, then D2
  static constexpr int kD2Col = 2 * kNQ;
  static constexpr int kCols = 3 * kNQ;
  static constexpr int kTmemCols = kCols <= 128 ? 128 : (kCols <= 256 ? 256 : 512);
  static_assert(kCols <= 512, "tensor memory");
};

// Loads W consecutive TMEM columns (W in 8, 16, 24, 32, 48; taddr 16-column
// aligned) of this warp's 32 lanes.
template <int W>
__device__ __forceinline__ void tmem_cols(uint32_t taddr, uint32_t (&r)[W]) {
  if constexpr (W == 8 || W == 16 || W == 32) {
    tmem_load<W>(taddr, r);
  } else if constexpr (W == 24) {
    uint32_t a[16], b[8];
    tmem_load<16>(taddr, a);
    tmem_load<8>(taddr + 16, b);
#pragma unroll
    for (int i = 0; i < 16; ++i) r[i] = a[i];
#pragma unroll
    for (int i = 0; i < 8; ++i) r[16 + i] = b[i];
  } else {
    static_assert(W == 48, "TMEM load width");
    uint32_t a[32], b[16];
    tmem_load<32>(taddr, a);
    tmem_load<16>(taddr + 32, b);
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = a[i];
#pragma unroll
    for (int i = 0; i < 16; ++i) r[32 + i] = b[i];
  }
}

__device__ __forceinline__ float digits_value(uint32_t c0, uint32_t c1, uint32_t c2) {
  return (float)(int)c2 * 65536.0f + ((float)(int)c1 * 256.0f + (float)(int)c0);
}

template <int HKV, int G>
__global__ void __launch_bounds__(256, 1)
    decode_tcp_kernel(const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v, const float* __restrict__ q,
                      const float* __restrict__ k_scale, const float* __restrict__ v_scale,
                      const int32_t* __restrict__ block_tables,
                      const int32_t* __restrict__ seq_lens, float* __restrict__ out,
                      float* __restrict__ ws_acc, float2* __restrict__ ws_ml,
                      unsigned long long* __restrict__ unit_arrivals, int num_seqs,
                      int num_heads, int64_t num_blocks, int max_blocks_per_seq, float qk_scale,
                      int min_pages, int unit_cost, unsigned long long launch_tag, int* err) {
  using C = TcpCfg<HKV, G>;
  constexpr int NQ = C::kNQ;
  constexpr int S = C::kStages;
  constexpr int BS = 16;
  constexpr int NH = C::kHeads;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* s_logit = reinterpret_cast<float*>(smem + C::kOffLogit);
  float2* s_run = reinterpret_cast<float2*>(smem + C::kOffRun);
  float2* s_chunk = reinterpret_cast<float2*>(smem + C::kOffChunk);
  float2* s_ab = reinterpret_cast<float2*>(smem + C::kOffAB);
  float* s_half = reinterpret_cast<float*>(smem + C::kOffHalf);  // [2][8][G]
  int* s_pseq = reinterpret_cast<int*>(smem + C::kOffPseq);
  int* s_tmp = reinterpret_cast<int*>(smem + C::kOffTmp);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffTmem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + S;
  constexpr int R = C::kMetaRing;
  uint64_t* meta_full = empty + S;      // [R] chunk table filled (warp 2)
  uint64_t* meta_free = meta_full + R;  // [R] TMA and epilogue done with it
  uint64_t* q_full = meta_free + R;     // [2] a sequence's query digits and scales (warp 3)
  uint64_t* q_free = q_full + 2;        // [2] MMA (commit) and epilogue done with them
  uint64_t* d1_full = q_free + 2;       // [2] q.K of a stage committed
  uint64_t* d1_free = d1_full + 2;      // [2] the epilogue has read that D1
  uint64_t* p_full = d1_free + 2;       // [2] a probability tile written
  uint64_t* p_free = p_full + 2;        // [2] p.V of that tile committed
  uint64_t* d2_full = p_free + 2;       // p.V of a chunk committed
  uint64_t* d2_free = d2_full + 1;      // the epilogue has read D2
  auto meta = [&](int b) { return smem + C::kOffMeta + b * C::kMetaBytes; };
  float* s_qs = reinterpret_cast<float*>(smem + C::kOffQs);  // [2][32]
  auto qtile = [&](int b) { return smem + C::kOffQ + b * C::kRowBytes; };
  auto ptile = [&](int b) { return smem + C::kOffP + b * C::kRowBytes; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S_ = num_seqs;
  const int grid_ctas = gridDim.x;

  // ---- virtual pages per sequence and their prefix (every CTA, identically)
  constexpr int kPer = (kStreamMaxSeqs + C::kThreads - 1) / C::kThreads;
  int mine[kPer];
  int sum = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int s = tid * kPer + i;
    mine[i] = 0;
    if (s < S_) {
      const int L = seq_lens[s];
      const int pages = covered_pages(L, BS, max_blocks_per_seq);
      if (blockIdx.x == 0 && L > pages * BS) record_error(err, kDevSeqTooLong);
      mine[i] = pages > 0 ? pages + unit_cost : 0;
    }
    sum += mine[i];
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_tmp[warp] = incl;
  // query digit and probability tiles: padding rows, and the probability
  // entries off the block diagonal, stay zero; each chunk rewrites only the
  // digit rows and its rows' own diagonal probability bytes
  for (int i = tid; i < 4 * C::kRowBytes / 4; i += C::kThreads)
    reinterpret_cast<uint32_t*>(smem + C::kOffQ)[i] = 0u;
  fence_proxy_async_smem();
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < R; ++i) {
      mbar_init(&meta_full[i], 1);
      mbar_init(&meta_free[i], 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_free[i], 2);
      mbar_init(&d1_full[i], 1);
      mbar_init(&d1_free[i], 1);
      mbar_init(&p_full[i], 1);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(d2_full, 1);
    mbar_init(d2_free, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(s_tmem, C::kTmemCols);
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tmem = *s_tmem;
  int before = 0;
  for (int w = 0; w < warp; ++w) before += s_tmp[w];
  int run = before + incl - sum;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int s = tid * kPer + i;
    if (s <= S_) s_pseq[s] = run;
    run += mine[i];
  }
  __syncthreads();
  for (int s = blockIdx.x; s < S_; s += grid_ctas) {  // sequences without pages: zeros
    if (s_pseq[s + 1] != s_pseq[s]) continue;
    float4* o = reinterpret_cast<float4*>(out + (int64_t)s * num_heads * 128);
    for (int i = tid; i < num_heads * 32; i += C::kThreads) o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const long long P = (long long)s_pseq[S_];  // one unit (group) per sequence
  const int n_ctas = (int)min((long long)grid_ctas, max(1LL, (P + min_pages - 1) / min_pages));
  const long long c_begin = P * blockIdx.x / n_ctas;
  const long long c_end = P * (blockIdx.x + 1) / n_ctas;
  const bool active = blockIdx.x < n_ctas && c_begin < c_end;
  StreamIter it;
  it.init(active ? c_begin : 0, active ? c_end : 0, s_pseq, S_, 1, C::kMaxPages, unit_cost);
  StreamChunk ch;

  if (warp == 2) {
    // ---- chunk tables (block ids, scales, token count), up to R chunks ahead
    // of the copies.  Under the full page stream an L2 round trip takes
    // microseconds (responses queue behind the SM's copies), so the loads are
    // pipelined: the block ids of the next chunk go out with the scales of
    // this one, and both are in flight while the warp waits for a free table.
    StreamIter ahead = it;  // one chunk ahead: block ids
    StreamChunk nx;
    int v_next = -1, L_next = 0;
    if (ahead.next(nx)) {
      if (lane < nx.np) v_next = block_tables[(int64_t)nx.s * max_blocks_per_seq + nx.lp0 + lane];
      if (lane == 0) L_next = seq_lens[nx.s];
    }
    int i = 0;
    while (it.next(ch)) {
      const int m = i % R;
      int phys = -1;
      if (lane < ch.np) {
        const bool okb = v_next >= 0 && (int64_t)v_next < num_blocks;
        if (!okb) record_error(err, kDevBadBlockId);
        phys = okb ? v_next : -1;
      }
      const int Ls = L_next;
      float ks[HKV], vs[HKV];
#pragma unroll
      for (int h = 0; h < HKV; ++h) {
        ks[h] = phys >= 0 ? k_scale[(int64_t)phys * HKV + h] : 0.0f;
        vs[h] = phys >= 0 ? v_scale[(int64_t)phys * HKV + h] : 0.0f;
      }
      v_next = -1;
      L_next = 0;
      if (ahead.next(nx)) {
        if (lane < nx.np)
          v_next = block_tables[(int64_t)nx.s * max_blocks_per_seq + nx.lp0 + lane];
        if (lane == 0) L_next = seq_lens[nx.s];
      }
      if (i >= R) {
        bool ok = true;
        if (lane == 0 && !mbar_wait_bounded(&meta_free[m], (uint32_t)((i / R) - 1) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          ok = false;
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
      uint8_t* mt = meta(m);
      if (lane < ch.np) reinterpret_cast<int*>(mt + C::kMetaPhys)[lane] = phys;
#pragma unroll
      for (int h = 0; h < HKV; ++h) {
        if (lane < ch.np) {
          reinterpret_cast<float*>(mt + C::kMetaKs)[lane * HKV + h] = ks[h];
          reinterpret_cast<float*>(mt + C::kMetaVs)[lane * HKV + h] = vs[h];
        }
        const float vm = warp_max(vs[h]);
        if (lane == 0) reinterpret_cast<float*>(mt + C::kMetaVmax)[h] = vm;
      }
      if (lane == 0) {
        const int pages = s_pseq[ch.s + 1] - s_pseq[ch.s] - unit_cost;
        const int L = min(max(Ls, 0), pages * BS);
        *reinterpret_cast<int*>(mt + C::kMetaT) = min(L, (ch.lp0 + ch.np) * BS) - ch.lp0 * BS;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_full[m]);
      ++i;
    }
  } else if (warp == 3) {
    // ---- query digit tiles, one per sequence (its chunks are consecutive),
    // in a ring of two: the digits are computed into registers before the
    // warp waits for a free tile, so only the shared-memory stores follow it
    constexpr int kBatch = NH < 8 ? NH : 8;  // query rows in flight per lane
    int j = -1, prev_s = -1;
    while (it.next(ch)) {
      if (ch.s == prev_s) continue;
      prev_s = ch.s;
      ++j;
      const int qb = j & 1;
      uint32_t dg[NH][3];
      float my_qs = 0.0f;  // lane hq: the scale of query head hq
#pragma unroll
      for (int h0 = 0; h0 < NH; h0 += kBatch) {
        float4 xq[kBatch];
#pragma unroll
        for (int t = 0; t < kBatch; ++t)
          xq[t] = reinterpret_cast<const float4*>(
              q + ((int64_t)ch.s * num_heads + h0 + t) * 128)[lane];
#pragma unroll
        for (int t = 0; t < kBatch; ++t) {
          const float4 x = xq[t];
          float mx = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
          mx = warp_max(mx);
          const float inv = mx > 0.0f ? (float)kQFix / mx : 0.0f;
          const float xs[4] = {x.x, x.y, x.z, x.w};
          int d[4][3];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            int n = __float2int_rn(xs[e] * inv);
            n = max(-kQFix, min(kQFix, n));
            to_digits(n, d[e][0], d[e][1], d[e][2]);
          }
#pragma unroll
          for (int pl = 0; pl < 3; ++pl) dg[h0 + t][pl] = pack4(d[0][pl], d[1][pl], d[2][pl], d[3][pl]);
          if (lane == h0 + t) my_qs = mx > 0.0f ? mx / (float)kQFix : 0.0f;
        }
      }
      if (j >= 2) {
        bool ok = true;
        if (lane == 0 && !mbar_wait_bounded(&q_free[qb], (uint32_t)((j >> 1) - 1) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          ok = false;
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
      uint8_t* sq = qtile(qb);
#pragma unroll
      for (int hq = 0; hq < NH; ++hq)
#pragma unroll
        for (int pl = 0; pl < 3; ++pl)
          *reinterpret_cast<uint32_t*>(
              sq + sw128_offset((hq / G) * C::kCS + 3 * (hq % G) + pl, 4 * lane)) = dg[hq][pl];
      if (lane < NH) s_qs[qb * 32 + lane] = my_qs;
      fence_proxy_async_smem();  // an MMA operand
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_full[qb]);
    }
  } else if (warp == 0) {
    // ---- TMA: the chunk's K stages, then its V stages; lane 0 arms each
    // stage, lane j issues page j of it (one box per page)
    const uint64_t policy = l2_policy_evict_first();
    if (lane == 0) {
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
    }
    int i = 0, ns = 0;
    bool ok_run = true;
    while (ok_run && it.next(ch)) {
      const int m = i % R;
      bool ok = true;
      if (lane == 0 && !mbar_wait_bounded(&meta_full[m], (uint32_t)(i / R) & 1u, err)) {
        record_error(err, kDevWaitTimeout);
        ok = false;
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      const int* phys_t = reinterpret_cast<const int*>(meta(m) + C::kMetaPhys);
      const int n_st = (ch.np + C::kPPS - 1) / C::kPPS;
      for (int kind = 0; kind < 2 && ok_run; ++kind) {
        for (int st = 0; st < n_st; ++st, ++ns) {
          const int slot = ns % S;
          const int pb = st * C::kPPS, pe = min(ch.np, pb + C::kPPS);
          bool oks = true;
          if (lane == 0) {
            if (!mbar_wait_bounded(&empty[slot], ((uint32_t)(ns / S) & 1u) ^ 1u, err)) {
              record_error(err, kDevWaitTimeout);
              oks = false;
            } else {
              mbar_arrive_expect_tx(&full[slot], (uint32_t)((pe - pb) * BS * HKV * 128));
            }
          }
          oks = __shfl_sync(0xffffffffu, oks, 0);
          __syncwarp();  // the stage is armed before any of its copies is issued
          if (!oks) {
            ok_run = false;
            break;
          }
          if (lane < pe - pb)
            tma_load_4d(smem + slot * kStageBytes + lane * BS * HKV * 128, kind ? &map_v : &map_k,
                        &full[slot], 0, 0, 0, max(phys_t[pb + lane], 0), policy);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_free[m]);
      ++i;
    }
    if (lane == 0) drain_ring(full, S, ns);  // no copy outlives the CTA
  } else if (warp == 1) {
    // ---- MMA issue: per chunk q.K of each K stage into D1 (alternating
    // buffers), then p.V of each V stage into D2 ----------------------------
    if (lane == 0) {
      constexpr uint32_t kIdQK = umma_i8_idesc(1, 1, 0, 0, 128, NQ);
      constexpr uint32_t kIdPV = umma_i8_idesc(1, 0, 1, 0, 128, NQ);
      const uint32_t stage0 = smem_u32(smem);
      int i = 0, ns = 0, kd = 0, pv = 0, j = -1, prev_s = -1;
      uint64_t* last_bar = nullptr;  // the last d1_full / d2_full commit, drained at exit
      uint32_t last_par = 0;
      bool ok_run = true;
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        if (!mbar_wait_bounded(bar, parity, err)) {
          record_error(err, kDevWaitTimeout);
          ok_run = false;
          return false;
        }
        tmem_fence_after_sync();
        return true;
      };
      while (ok_run && it.next(ch)) {
        const int n_st = (ch.np + C::kPPS - 1) / C::kPPS;
        if (ch.s != prev_s) {  // a new sequence: release the last digit tile, take the next
          if (j >= 0) umma_commit(&q_free[j & 1]);
          prev_s = ch.s;
          ++j;
          if (!wait(&q_full[j & 1], (uint32_t)(j >> 1) & 1u)) break;
        }
        const uint32_t qaddr = smem_u32(qtile(j & 1));
        for (int st = 0; st < n_st && ok_run; ++st, ++ns, ++kd) {
          const int slot = ns % S, db = kd & 1;
          if (!wait(&full[slot], (uint32_t)(ns / S) & 1u)) break;
          if (kd >= 2 && !wait(&d1_free[db], (uint32_t)((kd >> 1) - 1) & 1u)) break;
          const uint32_t a = stage0 + slot * kStageBytes;
#pragma unroll
          for (int kq = 0; kq < 4; ++kq)
            umma_i8(tmem + db * NQ, umma_sw128_desc(a + kq * 32, 16, 1024),
                    umma_sw128_desc(qaddr + kq * 32, 16, 1024), kIdQK, kq > 0);
          umma_commit(&empty[slot]);
          umma_commit(&d1_full[db]);
          last_bar = &d1_full[db];
          last_par = (uint32_t)(kd >> 1) & 1u;
        }
        if (!ok_run) break;
        if (i >= 1 && !wait(d2_free, (uint32_t)(i - 1) & 1u)) break;
        for (int st = 0; st < n_st && ok_run; ++st, ++ns, ++pv) {
          const int slot = ns % S, pb = pv & 1;
          if (!wait(&full[slot], (uint32_t)(ns / S) & 1u)) break;
          if (!wait(&p_full[pb], (uint32_t)(pv >> 1) & 1u)) break;
          const uint32_t a = stage0 + slot * kStageBytes;
          const uint32_t paddr = smem_u32(ptile(pb));
#pragma unroll
          for (int kq = 0; kq < 4; ++kq)
            umma_i8(tmem + C::kD2Col, umma_sw128_desc(a + kq * 4096, 16, 1024),
                    umma_sw128_desc(paddr + kq * 32, 16, 1024), kIdPV,
                    (st > 0 || kq > 0) ? 1u : 0u);
          umma_commit(&empty[slot]);
          umma_commit(&p_free[pb]);
        }
        if (!ok_run) break;
        umma_commit(d2_full);
        last_bar = d2_full;
        last_par = (uint32_t)i & 1u;
        ++i;
      }
      // every MMA of this thread is done before TMEM is freed
      if (last_bar != nullptr) mbar_drain(last_bar, last_par);
    }
  } else if (warp >= 4) {
    // ---- epilogue: TMEM lane e is a stage row for D1 and a head dimension
    // for D2 -------------------------------------------------------------------
    constexpr int CS = C::kCS;
    constexpr int W1 = HKV >= 2 ? 2 * CS : CS;  // D1 columns a warp reads (its two heads)
    const int e = tid - 128;
    const int w4 = warp - 4;
    const uint32_t lane_base = (uint32_t)(32 * w4) << 16;
    const int h_e = (e >> 4) % HKV;   // the row's KV head
    const int pp_e = e / (16 * HKV);  // its page within the stage
    const int t_e = e & 15;           // its token within the page
    const int hw = e >> 4;            // half-warp 0..7 (head hw % HKV)
    const bool upper = HKV >= 2 && (lane >> 4) != 0;
    const int hcol = HKV >= 2 ? (2 * w4) % HKV : 0;  // the warp's first head
    float acc_run[NH];
#pragma unroll
    for (int hq = 0; hq < NH; ++hq) acc_run[hq] = 0.0f;
    int i = 0, kd = 0, pv = 0, j = -1, prev_s = -1;
    bool live = true;
    while (it.next(ch)) {
      const int b = i % R;
      const uint8_t* m = meta(b);
      const int* phys_t = reinterpret_cast<const int*>(m + C::kMetaPhys);
      const float* ks_t = reinterpret_cast<const float*>(m + C::kMetaKs);
      const float* vs_t = reinterpret_cast<const float*>(m + C::kMetaVs);
      const float* vmax_t = reinterpret_cast<const float*>(m + C::kMetaVmax);
      if (ch.s != prev_s) {
        // a new sequence: every thread finished the last one's query scales
        // at the barriers that ended its chunk
        if (j >= 0 && e == 0) mbar_arrive(&q_free[j & 1]);
        prev_s = ch.s;
        ++j;
        if (live && !mbar_wait_bounded(&q_full[j & 1], (uint32_t)(j >> 1) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          live = false;
        }
      }
      const float* qs_t = s_qs + (j & 1) * 32;
      if (live && !mbar_wait_bounded(&meta_full[b], (uint32_t)(i / R) & 1u, err)) {
        record_error(err, kDevWaitTimeout);
        live = false;
      }
      const int T = live ? *reinterpret_cast<const int*>(m + C::kMetaT) : 0;
      const int n_st = (ch.np + C::kPPS - 1) / C::kPPS;

      // ---- K phase: logits of this row's query heads, running maxima
      float kmax[G];
#pragma unroll
      for (int g = 0; g < G; ++g) kmax[g] = -INFINITY;
      for (int st = 0; st < n_st; ++st, ++kd) {
        const int db = kd & 1;
        if (live && !mbar_wait_bounded(&d1_full[db], (uint32_t)(kd >> 1) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          live = false;
        }
        tmem_fence_after_sync();
        const int pg = st * C::kPPS + pp_e;
        const int tok = pg * 16 + t_e;
        const bool valid = live && pg < ch.np && tok < T && phys_t[pg] >= 0;
        const float ksc = pg < ch.np ? ks_t[pg * HKV + h_e] : 0.0f;
        uint32_t r[W1];
        tmem_cols<W1>(tmem + lane_base + db * NQ + hcol * CS, r);
        tmem_wait_load();
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float v = digits_value(r[3 * g], r[3 * g + 1], r[3 * g + 2]);
          if constexpr (HKV >= 2) {
            const float hi = digits_value(r[CS + 3 * g], r[CS + 3 * g + 1], r[CS + 3 * g + 2]);
            v = upper ? hi : v;
          }
          const float logit = valid ? v * (qs_t[h_e * G + g] * ksc * qk_scale) : -INFINITY;
          s_logit[(h_e * G + g) * C::kMaxTok + tok] = logit;
          kmax[g] = fmaxf(kmax[g], logit);
        }
        tmem_fence_before_sync();
        named_barrier(1, 128);  // every row of D1 read
        if (e == 0) mbar_arrive(&d1_free[db]);
      }
      // ---- the chunk's maximum per (KV head, query head): half-warps hold
      // 16 rows of one head; heads repeat over the stage's pages
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float mm = kmax[g];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        if ((lane & 15) == 0) s_half[hw * G + g] = mm;
      }
      named_barrier(1, 128);
      if (e < NH) {
        float mm = -INFINITY;
        for (int j = e / G; j < 8; j += HKV) mm = fmaxf(mm, s_half[j * G + e % G]);
        s_chunk[e].x = mm;
      }
      named_barrier(1, 128);

      // ---- V phase: one block-diagonal probability tile per V stage
      const float vmax_e = vmax_t[h_e];
      const float to_fix = vmax_e > 0.0f ? 16777215.0f / vmax_e : 0.0f;
      float mh[G], lsum[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        mh[g] = s_chunk[h_e * G + g].x;
        lsum[g] = 0.0f;
      }
      for (int st = 0; st < n_st; ++st, ++pv) {
        const int pb = pv & 1;
        if (pv >= 2 && live &&
            !mbar_wait_bounded(&p_free[pb], (uint32_t)((pv >> 1) - 1) & 1u, err)) {
          record_error(err, kDevWaitTimeout);
          live = false;
        }
        const int pg = st * C::kPPS + pp_e;
        const int tok = pg * 16 + t_e;
        const bool valid = pg < ch.np && tok < T;
        const float vs = pg < ch.np ? vs_t[pg * HKV + h_e] : 0.0f;
        uint8_t* pt = ptile(pb);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          uint32_t n = 0;
          if (valid && mh[g] != -INFINITY) {
            const float p = exp2f(s_logit[(h_e * G + g) * C::kMaxTok + tok] - mh[g]);
            lsum[g] += p;
            n = __float2uint_rn(fminf(p * vs * to_fix, 16777215.0f));
          }
          const int row = h_e * CS + 3 * g;
          pt[sw128_offset(row, e)] = (uint8_t)(n & 255u);
          pt[sw128_offset(row + 1, e)] = (uint8_t)((n >> 8) & 255u);
          pt[sw128_offset(row + 2, e)] = (uint8_t)(n >> 16);
        }
        fence_proxy_async_smem();
        named_barrier(1, 128);
        if (e == 0) mbar_arrive(&p_full[pb]);
      }
      // ---- the chunk's sums, then the merge factors with the running (m, l)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float ls = lsum[g];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
        if ((lane & 15) == 0) s_half[8 * G + hw * G + g] = ls;
      }
      named_barrier(1, 128);
      if (e < NH) {
        float l = 0.0f;
        for (int j = e / G; j < 8; j += HKV) l += s_half[8 * G + j * G + e % G];
        const float mc = s_chunk[e].x;
        if (ch.seg_first) {
          s_ab[e] = make_float2(0.0f, 1.0f);
          s_run[e] = make_float2(mc, l);
        } else {
          const float2 rr = s_run[e];
          const float M = fmaxf(rr.x, mc);
          const float a = rr.x == -INFINITY ? 0.0f : exp2f(rr.x - M);
          const float bb = mc == -INFINITY ? 0.0f : exp2f(mc - M);
          s_ab[e] = make_float2(a, bb);
          s_run[e] = make_float2(M, rr.y * a + l * bb);
        }
      }
      if (live && !mbar_wait_bounded(d2_full, (uint32_t)i & 1u, err)) {
        record_error(err, kDevWaitTimeout);
        live = false;
      }
      tmem_fence_after_sync();
      named_barrier(1, 128);  // s_ab, s_run published
      // ---- D2: this thread's dimension e of every query head's result
#pragma unroll
      for (int hp = 0; hp < (HKV >= 2 ? HKV / 2 : 1); ++hp) {
        uint32_t r[W1];
        tmem_cols<W1>(tmem + lane_base + C::kD2Col + hp * W1, r);
        tmem_wait_load();
#pragma unroll
        for (int hh = 0; hh < (HKV >= 2 ? 2 : 1); ++hh) {
          const int h = hp * 2 + hh;
          const float back = vmax_t[h] * (1.0f / 16777215.0f);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const int hq = h * G + g;
            const float accc =
                digits_value(r[hh * CS + 3 * g], r[hh * CS + 3 * g + 1], r[hh * CS + 3 * g + 2]) *
                back;
            const float2 ab = s_ab[hq];
            acc_run[hq] = acc_run[hq] * ab.x + ab.y * accc;
          }
        }
      }
      tmem_fence_before_sync();
      named_barrier(1, 128);  // D2 and the table half read
      if (e == 0) {
        mbar_arrive(d2_free);
        mbar_arrive(&meta_free[b]);
      }

      // ---- end of this CTA's part of the unit: write it
      if (ch.seg_last) {
        const int u = ch.s;  // one unit per sequence
        if (ch.whole) {
#pragma unroll
          for (int hq = 0; hq < NH; ++hq) {
            const float l = s_run[hq].y;
            out[((int64_t)ch.s * num_heads + hq) * 128 + e] = l > 0.0f ? acc_run[hq] / l : 0.0f;
          }
        } else {
#pragma unroll
          for (int hq = 0; hq < NH; ++hq) {
            const int64_t slot = ((int64_t)u + blockIdx.x) * NH + hq;
            ws_acc[slot * 128 + e] = acc_run[hq];
            if (e == 0) ws_ml[slot] = s_run[hq];
          }
          int first, last;
          unit_owners(s_pseq, ch.s, 0, 1, unit_cost, P, n_ctas, first, last);
          const int nseg = last - first + 1;
          const int ngroups = (nseg + kMergeGroup - 1) / kMergeGroup;
          const int g_lo = first + (int)(blockIdx.x - first) / kMergeGroup * kMergeGroup;
          const int g_hi = min(last, g_lo + kMergeGroup - 1);
          // every partial store of this CTA is ordered before thread e == 0's
          // release by the barrier; the last arrival acquires all of them
          named_barrier(1, 128);
          if (e == 0) {
            const int r = ngroups == 1
                              ? arrive_on_unit(&unit_arrivals[u], launch_tag, nseg, 0ull)
                              : arrive_on_unit(&unit_arrivals[S_ + u + g_lo], launch_tag,
                                               g_hi - g_lo + 1, 0ull);
            if (r < 0) record_error(err, kDevWaitTimeout);
            s_tmp[8] = r == 1;
          }
          named_barrier(1, 128);
          int m_lo = g_lo, m_n = g_hi - g_lo + 1, m_stride = 1;
          bool final_pass = ngroups == 1;
          bool merging = s_tmp[8] != 0;
          while (merging) {
#pragma unroll 1
            for (int hq = w4; hq < NH; hq += 4) {
              float4 a;
              float M, den;
              merge_partials(ws_acc, ws_ml, m_n, lane, a, M, den, [&](int j) {
                return ((int64_t)u + m_lo + j * m_stride) * NH + hq;
              });
              if (final_pass) {
                const float inv = den > 0.0f ? 1.0f / den : 0.0f;
                reinterpret_cast<float4*>(out + ((int64_t)ch.s * num_heads + hq) * 128)[lane] =
                    make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
              } else {
                const int64_t slot = ((int64_t)u + g_lo) * NH + hq;
                reinterpret_cast<float4*>(ws_acc + slot * 128)[lane] = a;
                if (lane == 0) ws_ml[slot] = make_float2(M, den);
              }
            }
            if (final_pass) break;
            named_barrier(1, 128);  // the group's partial is stored
            if (e == 0) {
              const int r = arrive_on_unit(&unit_arrivals[u], launch_tag, ngroups, 0ull);
              if (r < 0) record_error(err, kDevWaitTimeout);
              s_tmp[9] = r == 1;
            }
            named_barrier(1, 128);
            merging = s_tmp[9] != 0;
            m_lo = first;
            m_n = ngroups;
            m_stride = kMergeGroup;
            final_pass = true;
          }
        }
#pragma unroll
        for (int hq = 0; hq < NH; ++hq) acc_run[hq] = 0.0f;
      }
      ++i;
    }
  }
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// ===========================================================================
// Planning and dispatch
// ===========================================================================

struct Plan {
  bool fast = false;
  bool tc = false;      // tensor-core GQA kernel (bs 16, group 2/4/8)
  bool stream = false;  // persistent balanced kernel (fast shapes, S <= 1024)
  bool tcp = false;     // whole-page tensor-core stream kernel (a stream plan too)
  int hg = 1, g = 1;
  int pages_per_split = 1;
  int max_splits = 1;
  int n_ctas = 0;     // stream kernel grid
  int min_pages = 1;  // stream kernel: fewest pages a CTA takes
  int unit_cost = 0;  // stream kernel: a unit's fixed cost, in pages
};

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

int largest_pow2_divisor_upto(int n, int cap) {
  int r = 1;
  while (r * 2 <= cap && n % (r * 2) == 0) r *= 2;
  return r;
}

Plan make_plan(const DecodeArgs& a) {
  Plan p;
  const int group = a.num_heads / a.num_kv_heads;
  const bool g_ok = group >= 1 && group <= 8 && (group & (group - 1)) == 0;
  const bool aligned = (reinterpret_cast<uintptr_t>(a.k_cache) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(a.v_cache) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(a.q) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(a.out) % 16 == 0);
  p.fast = a.head_dim == 128 && (a.block_size == 16 || a.block_size == 32) && g_ok && aligned &&
           (int64_t)a.num_blocks * a.block_size < (int64_t)1 << 31 && env_int("PKV_DECODE_GENERIC", 0) == 0;
  const int M = a.max_blocks_per_seq;
  if (p.fast) {
    p.g = group;
    const int cap = std::min(128 / a.block_size, 16 / group);
    p.hg = largest_pow2_divisor_upto(a.num_kv_heads, std::min(8, cap));
    if (a.block_size * p.hg < 8) p.fast = false;
  }
  if (p.fast) {
    const int pps_stage = 128 / (a.block_size * p.hg);
    const int max_pages = (p.hg * p.g <= 8 ? 512 : 256) / a.block_size;
    const int groups = a.num_kv_heads / p.hg;
    int pps = max_pages;
    const int64_t target = env_int("PKV_DECODE_TARGET_CTAS", 888);
    while (pps > pps_stage && (int64_t)a.num_seqs * groups * ((M + pps - 1) / pps) < target)
      pps /= 2;
    const int forced = env_int("PKV_DECODE_SPLIT_PAGES", 0);
    if (forced > 0) pps = std::max(pps_stage, std::min(max_pages, forced / pps_stage * pps_stage));
    p.pages_per_split = std::max(pps, pps_stage);
  } else {
    const int max_pages = std::max(1, kGenMaxTok / a.block_size);
    int pps = max_pages;
    while (pps > 1 && (int64_t)a.num_seqs * a.num_heads * ((M + pps - 1) / pps) < 888) pps /= 2;
    p.pages_per_split = pps;
  }
  if (p.fast && a.block_size == 16 && (group == 2 || group == 4 || group == 8) &&
      env_int("PKV_DECODE_TC", 1) != 0) {
    const int hkv = a.num_kv_heads;
    const int cs = group == 2 ? 8 : (group == 4 ? 16 : 24);
    if ((hkv == 1 || hkv == 2 || hkv == 4 || hkv == 8) && hkv * cs <= 128 &&
        a.num_seqs <= kStreamMaxSeqs && env_int("PKV_DECODE_TC_PAGES", 0) != 0 &&
        env_int("PKV_DECODE_TC_SPLIT", 0) == 0) {
      // whole pages on the tensor cores, the stream kernel's scheduling (on
      // request: measured slower than the per-head kernel below, since one
      // CTA per SM keeps at most 8 pages of 16 KB in flight)
      p.tcp = true;
      p.stream = true;
      p.hg = hkv;
      p.g = group;
      const int forced = env_int("PKV_DECODE_CTAS", 0);
      p.n_ctas = forced > 0 ? forced : sm_count();
      p.min_pages = std::max(1, env_int("PKV_STREAM_MIN_PAGES", 4));
      p.unit_cost = std::max(0, env_int("PKV_STREAM_UNIT_COST", 4));
      p.max_splits = 1;
      return p;
    }
    // one CTA per (sequence, KV head, split of 8..32 pages)
    p.tc = true;
    int pps = group <= 4 ? TcCfg<4>::kMaxPages : TcCfg<8>::kMaxPages;
    while (pps > 8 && (int64_t)a.num_seqs * a.num_kv_heads * ((M + pps - 1) / pps) <
                          env_int("PKV_DECODE_TARGET_CTAS", 888))
      pps /= 2;
    const int forced = env_int("PKV_DECODE_SPLIT_PAGES", 0);
    if (forced > 0)
      pps = std::max(8, std::min(group <= 4 ? TcCfg<4>::kMaxPages : TcCfg<8>::kMaxPages,
                                 forced / 8 * 8));
    p.pages_per_split = pps;
    p.max_splits = std::max(1, (M + pps - 1) / pps);
    return p;
  }
  p.max_splits = std::max(1, (M + p.pages_per_split - 1) / p.pages_per_split);
  if (p.fast && a.num_seqs <= kStreamMaxSeqs && env_int("PKV_DECODE_SPLIT", 0) == 0) {
    p.stream = true;
    const int forced = env_int("PKV_DECODE_CTAS", 0);
    p.n_ctas = forced > 0 ? forced : 2 * sm_count();
    p.min_pages = std::max(1, env_int("PKV_STREAM_MIN_PAGES", 4));
    p.unit_cost = std::max(0, env_int("PKV_STREAM_UNIT_COST", 4));
  }
  return p;
}

// A fresh tag per stream-kernel launch for its arrival counters: 44 bits
// (the counters keep 20 for the count), never 0, starting at a random point
// so that counters another process left behind do not match.
unsigned long long next_launch_tag() {
  static std::atomic<unsigned long long> tag{[] {
    std::random_device rd;
    return ((unsigned long long)rd() << 32) ^ (unsigned long long)rd();
  }()};
  constexpr unsigned long long kMask = (1ull << (64 - kArrivalBits)) - 1;
  for (;;) {
    const unsigned long long t = tag.fetch_add(1) & kMask;
    if (t != 0) return t;
  }
}

// Workspace of the stream kernel: partial slots (units + CTAs) x query
// heads per unit, then (m, l) per slot, then one arrival counter per unit.
struct StreamWs {
  size_t acc_off, ml_off, cnt_off, units, bytes;
};

StreamWs stream_ws_layout(const DecodeArgs& a, const Plan& p) {
  const size_t units = (size_t)a.num_seqs * (a.num_kv_heads / p.hg);
  const size_t slots = (units + p.n_ctas) * (size_t)(p.hg * p.g);
  StreamWs w;
  w.units = units;
  w.acc_off = 0;
  w.ml_off = (slots * 128 * sizeof(float) + 255) & ~(size_t)255;
  w.cnt_off = (w.ml_off + slots * sizeof(float2) + 255) & ~(size_t)255;
  // arrival counters: one per unit, then one per (unit + CTA) for two-level merges
  w.bytes = w.cnt_off + (2 * units + p.n_ctas) * sizeof(unsigned long long) + 256;
  return w;
}

template <int BS, int HG, int G>
int launch_fast_t(const DecodeArgs& a, const Plan& p, float* ws_acc, float2* ws_ml,
                  cudaStream_t stream) {
  using C = FastCfg<BS, HG, G>;
  CUtensorMap mk, mv;
  if (!cached_cache_map(&mk, a.k_cache, a.num_blocks, BS, a.num_kv_heads, HG) ||
      !cached_cache_map(&mv, a.v_cache, a.num_blocks, BS, a.num_kv_heads, HG)) {
    set_error("cuTensorMapEncodeTiled failed for the paged cache");
    return kCudaError;
  }
  if (p.stream) {
    using SC = StreamCfg<BS, HG, G>;
    auto skern = decode_stream_kernel<BS, HG, G>;
    cudaFuncSetAttribute(skern, cudaFuncAttributeMaxDynamicSharedMemorySize, SC::kSmemBytes);
    const StreamWs w = stream_ws_layout(a, p);
    uint8_t* base = reinterpret_cast<uint8_t*>(ws_acc);
    float* sacc = reinterpret_cast<float*>(base + w.acc_off);
    float2* sml = reinterpret_cast<float2*>(base + w.ml_off);
    auto* scnt = reinterpret_cast<unsigned long long*>(base + w.cnt_off);
    skern<<<p.n_ctas, kStreamThreads, SC::kSmemBytes, stream>>>(
        mk, mv, a.q, a.k_scale, a.v_scale, a.block_tables, a.seq_lens, a.out, sacc, sml, scnt,
        a.num_seqs, a.num_heads, a.num_kv_heads, a.num_blocks, a.max_blocks_per_seq,
        a.sm_scale * kLog2e, std::max(1, p.min_pages), std::max(0, p.unit_cost), next_launch_tag(),
        device_error_word());
    return kOk;
  }
  auto kern = decode_fast_kernel<BS, HG, G>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  dim3 grid(a.num_seqs, p.max_splits, a.num_kv_heads / HG);
  kern<<<grid, kFastThreads, C::kSmemBytes, stream>>>(
      mk, mv, a.q, a.k_scale, a.v_scale, a.block_tables, a.seq_lens, a.out, ws_acc, ws_ml,
      a.num_heads, a.num_kv_heads, a.num_blocks, a.max_blocks_per_seq, a.sm_scale * kLog2e,
      p.pages_per_split, p.max_splits, device_error_word());
  return kOk;
}

template <int G>
int launch_tc_t(const DecodeArgs& a, const Plan& p, float* ws_acc, float2* ws_ml,
                cudaStream_t stream) {
  using C = TcCfg<G>;
  CUtensorMap mk, mv;
  if (!cached_cache_map(&mk, a.k_cache, a.num_blocks, 16, a.num_kv_heads, 1) ||
      !cached_cache_map(&mv, a.v_cache, a.num_blocks, 16, a.num_kv_heads, 1)) {
    set_error("cuTensorMapEncodeTiled failed for the paged cache");
    return kCudaError;
  }
  if (env_int("PKV_DECODE_TC_SPLIT", 0) == 0) {  // persistent form
    using CS = TcsCfg<G>;
    auto skern = decode_tc_stream_kernel<G>;
    cudaFuncSetAttribute(skern, cudaFuncAttributeMaxDynamicSharedMemorySize, CS::kSmemBytes);
    const int64_t units = (int64_t)a.num_seqs * a.num_kv_heads * p.max_splits;
    const int64_t ctas = std::max<int64_t>(
        1, std::min<int64_t>(units, (int64_t)CS::kMinBlocks * sm_count()));
    skern<<<(unsigned)ctas, CS::kThreads, CS::kSmemBytes, stream>>>(
        mk, mv, a.q, a.k_scale, a.v_scale, a.block_tables, a.seq_lens, a.out, ws_acc, ws_ml,
        a.num_seqs, a.num_heads, a.num_kv_heads, a.num_blocks, a.max_blocks_per_seq,
        a.sm_scale * kLog2e, p.pages_per_split, p.max_splits, device_error_word());
    return kOk;
  }
  auto kern = decode_tc_kernel<G>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  dim3 grid(a.num_seqs, p.max_splits, a.num_kv_heads);
  kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(
      mk, mv, a.q, a.k_scale, a.v_scale, a.block_tables, a.seq_lens, a.out, ws_acc, ws_ml,
      a.num_heads, a.num_kv_heads, a.num_blocks, a.max_blocks_per_seq, a.sm_scale * kLog2e,
      p.pages_per_split, p.max_splits, device_error_word());
  return kOk;
}

template <int HKV, int G>
int launch_tcp_t(const DecodeArgs& a, const Plan& p, float* ws_base, cudaStream_t stream) {
  using C = TcpCfg<HKV, G>;
  CUtensorMap mk, mv;
  if (!cached_cache_map(&mk, a.k_cache, a.num_blocks, 16, HKV, -1) ||
      !cached_cache_map(&mv, a.v_cache, a.num_blocks, 16, HKV, -1)) {
    set_error("cuTensorMapEncodeTiled failed for the paged cache (page map)");
    return kCudaError;
  }
  auto kern = decode_tcp_kernel<HKV, G>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  const StreamWs w = stream_ws_layout(a, p);
  uint8_t* base = reinterpret_cast<uint8_t*>(ws_base);
  kern<<<p.n_ctas, C::kThreads, C::kSmemBytes, stream>>>(
      mk, mv, a.q, a.k_scale, a.v_scale, a.block_tables, a.seq_lens, a.out,
      reinterpret_cast<float*>(base + w.acc_off), reinterpret_cast<float2*>(base + w.ml_off),
      reinterpret_cast<unsigned long long*>(base + w.cnt_off), a.num_seqs, a.num_heads,
      a.num_blocks, a.max_blocks_per_seq, a.sm_scale * kLog2e, std::max(1, p.min_pages),
      std::max(0, p.unit_cost), next_launch_tag(), device_error_word());
  return kOk;
}

int launch_tcp(const DecodeArgs& a, const Plan& p, float* ws_base, cudaStream_t stream) {
  const int g = a.num_heads / a.num_kv_heads;
#define PKV_TCP(H, GG) \
  if (a.num_kv_heads == H && g == GG) return launch_tcp_t<H, GG>(a, p, ws_base, stream);
  PKV_TCP(8, 2) PKV_TCP(8, 4)
  PKV_TCP(4, 2) PKV_TCP(4, 4) PKV_TCP(4, 8)
  PKV_TCP(2, 2) PKV_TCP(2, 4) PKV_TCP(2, 8)
  PKV_TCP(1, 2) PKV_TCP(1, 4) PKV_TCP(1, 8)
#undef PKV_TCP
  set_error("internal: no whole-page tensor-core instantiation for this head layout");
  return kUnsupported;
}

int launch_tc(const DecodeArgs& a, const Plan& p, float* ws_acc, float2* ws_ml,
              cudaStream_t stream) {
  switch (a.num_heads / a.num_kv_heads) {
    case 2: return launch_tc_t<2>(a, p, ws_acc, ws_ml, stream);
    case 4: return launch_tc_t<4>(a, p, ws_acc, ws_ml, stream);
    case 8: return launch_tc_t<8>(a, p, ws_acc, ws_ml, stream);
  }
  set_error("internal: no tensor-core decode instantiation for this group size");
  return kUnsupported;
}

template <int BS, int HG>
int dispatch_g(const DecodeArgs& a, const Plan& p, float* wa, float2* wm, cudaStream_t s) {
  switch (p.g) {
    case 1: return launch_fast_t<BS, HG, 1>(a, p, wa, wm, s);
    case 2: if constexpr (HG * 2 <= 16) return launch_fast_t<BS, HG, 2>(a, p, wa, wm, s); break;
    case 4: if constexpr (HG * 4 <= 16) return launch_fast_t<BS, HG, 4>(a, p, wa, wm, s); break;
    case 8: if constexpr (HG * 8 <= 16) return launch_fast_t<BS, HG, 8>(a, p, wa, wm, s); break;
  }
  set_error("internal: no fast decode instantiation for this group size");
  return kUnsupported;
}

template <int BS>
int dispatch_hg(const DecodeArgs& a, const Plan& p, float* wa, float2* wm, cudaStream_t s) {
  switch (p.hg) {
    case 1: return dispatch_g<BS, 1>(a, p, wa, wm, s);
    case 2: return dispatch_g<BS, 2>(a, p, wa, wm, s);
    case 4: return dispatch_g<BS, 4>(a, p, wa, wm, s);
    case 8: if constexpr (BS * 8 <= 128) return dispatch_g<BS, 8>(a, p, wa, wm, s); break;
  }
  set_error("internal: no fast decode instantiation for this head grouping");
  return kUnsupported;
}

// Launched right after the split kernel on the same stream.  (As a
// programmatic dependent launch, whose CTAs wait in griddepcontrol.wait
// until the split kernel is done, it measured 1-4% slower on B200.)
cudaError_t launch_combine(const DecodeArgs& a, const Plan& p, const float* ws_acc,
                           const float2* ws_ml, cudaStream_t stream) {
  const int64_t pairs = (int64_t)a.num_seqs * a.num_heads;
  const unsigned grid = (unsigned)((pairs + kCombineThreads / 32 - 1) / (kCombineThreads / 32));
#define PKV_COMBINE_V(V)                                                                        \
  case V:                                                                                      \
    decode_combine_kernel<V><<<grid, kCombineThreads, 0, stream>>>(                            \
        a.seq_lens, ws_acc, ws_ml, a.out, a.num_seqs, a.num_heads, a.block_size,               \
        a.max_blocks_per_seq, p.pages_per_split, p.max_splits);                                \
    return cudaGetLastError();
  switch (a.head_dim / 32) {  // head_dim % 32 == 0 and <= 256 (launch checks)
    PKV_COMBINE_V(1) PKV_COMBINE_V(2) PKV_COMBINE_V(3) PKV_COMBINE_V(4)
    PKV_COMBINE_V(5) PKV_COMBINE_V(6) PKV_COMBINE_V(7) PKV_COMBINE_V(8)
  }
#undef PKV_COMBINE_V
  return cudaErrorInvalidValue;
}

}  // namespace

size_t decode_workspace_size(const DecodeArgs& a) {
  const Plan p = make_plan(a);
  if (p.stream) return stream_ws_layout(a, p).bytes;
  if (p.max_splits <= 1) return 0;
  const size_t slots = (size_t)a.num_seqs * p.max_splits * a.num_heads;
  return slots * a.head_dim * sizeof(float) + slots * sizeof(float2) + 256;
}

int decode_kernel_launches(const DecodeArgs& a) {
  if (a.num_seqs <= 0) return 0;
  return make_plan(a).stream ? 1 : 2;  // stream kernel | split kernel + combine
}

int launch_decode(const DecodeArgs& a, void* workspace, size_t workspace_bytes,
                  cudaStream_t stream) {
  if (a.num_seqs == 0) return kOk;
  const Plan p = make_plan(a);
  float* ws_acc = nullptr;
  float2* ws_ml = nullptr;
  if (p.stream) {
    const size_t need = stream_ws_layout(a, p).bytes;
    if (workspace == nullptr || workspace_bytes < need) {
      set_error("workspace too small for decode: need " + std::to_string(need) + " bytes");
      return kWorkspace;
    }
    ws_acc = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) &
                                      ~(uintptr_t)255);
    const int rc = p.tcp ? launch_tcp(a, p, ws_acc, stream)
                   : a.block_size == 16 ? dispatch_hg<16>(a, p, ws_acc, nullptr, stream)
                                        : dispatch_hg<32>(a, p, ws_acc, nullptr, stream);
    if (rc != kOk) return rc;
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      set_error(std::string("decode launch failed: ") + cudaGetErrorString(e));
      return kCudaError;
    }
    return kOk;
  }
  if (p.max_splits > 1) {
    const size_t need = decode_workspace_size(a);
    if (workspace == nullptr || workspace_bytes < need) {
      set_error("workspace too small for split-K decode: need " + std::to_string(need) +
                " bytes");
      return kWorkspace;
    }
    uintptr_t base = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~(uintptr_t)255;
    const size_t slots = (size_t)a.num_seqs * p.max_splits * a.num_heads;
    ws_acc = reinterpret_cast<float*>(base);
    ws_ml = reinterpret_cast<float2*>(base + slots * a.head_dim * sizeof(float));
  }
  int rc = kOk;
  if (p.tc) {
    rc = launch_tc(a, p, ws_acc, ws_ml, stream);
  } else if (p.fast) {
    rc = a.block_size == 16 ? dispatch_hg<16>(a, p, ws_acc, ws_ml, stream)
                            : dispatch_hg<32>(a, p, ws_acc, ws_ml, stream);
  } else {
    dim3 grid(a.num_seqs, p.max_splits, a.num_heads);
    decode_generic_kernel<<<grid, kGenThreads, 0, stream>>>(
        a.q, a.k_cache, a.k_scale, a.v_cache, a.v_scale, a.block_tables, a.seq_lens, a.out,
        ws_acc, ws_ml, a.num_heads, a.num_kv_heads, a.head_dim, a.block_size, a.num_blocks,
        a.max_blocks_per_seq, a.sm_scale * kLog2e, p.pages_per_split, p.max_splits,
        device_error_word());
  }
  if (rc != kOk) return rc;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("decode launch failed: ") + cudaGetErrorString(e));
    return kCudaError;
  }
  // Splits > 1 and empty sequences are finished by the combine.
  e = launch_combine(a, p, ws_acc, ws_ml, stream);
  if (e != cudaSuccess) {
    set_error(std::string("combine launch failed: ") + cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

}  // namespace pkv
