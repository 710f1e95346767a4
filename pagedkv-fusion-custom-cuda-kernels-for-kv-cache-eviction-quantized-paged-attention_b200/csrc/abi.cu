// extern "C" entry points of libpagedkv_sm100.so (declared in
// include/pagedkv_fusion.h): argument checks with the reference launcher's
// messages (csrc/eviction_score.cu:105-110, csrc/quant_paged_attention.cu:
// 181-197), then dispatch to the kernel launchers.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/pagedkv_fusion.h"
#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

namespace {
thread_local std::string g_last_error;
constexpr int kMaxDevices = 64;
}  // namespace

// One error word per device: a file-scope __device__ variable exists once
// in every device context that loads this library.
__device__ int g_device_error = 0;

void set_error(const std::string& msg) { g_last_error = msg; }

int* device_error_word() {
  static int* ptrs[kMaxDevices] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

}  // namespace pkv

using pkv::set_error;

namespace {

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

inline int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

inline void clear_error() { set_error(""); }

}  // namespace

extern "C" {

const char* pkv_last_error_string(void) { return pkv::g_last_error.c_str(); }

int pkv_version(void) { return 10000; }

int pkv_read_device_error(int32_t* code, int reset) {
  clear_error();
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess)
    return fail(PKV_ERR_CUDA, std::string("device synchronize failed: ") + cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, pkv::g_device_error, sizeof(int));
  if (e != cudaSuccess)
    return fail(PKV_ERR_CUDA, std::string("reading the device error word failed: ") +
                                  cudaGetErrorString(e));
  if (reset && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(pkv::g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess)
      return fail(PKV_ERR_CUDA, std::string("clearing the device error word failed: ") +
                                    cudaGetErrorString(e));
  }
  if (code) *code = v;
  if (v != 0) return fail(PKV_ERR_DEVICE_INPUT, "a kernel recorded device error code " +
                                                    std::to_string(v));
  return PKV_OK;
}

int pkv_eviction_scores(const float* recency, const float* frequency, const float* attn_weights,
                        const uint8_t* valid_mask, float* scores, int64_t num_blocks,
                        int32_t block_size, float w_recency, float w_frequency,
                        float w_attention, void* stream) {
  clear_error();
  if (num_blocks < 0 || block_size < 0)
    return fail(PKV_ERR_INVALID_ARGUMENT, "attn_weights must be [num_blocks, block_size]");
  if (num_blocks > 0 && (!recency || !frequency || !scores ||
                         (block_size > 0 && (!attn_weights || !valid_mask))))
    return fail(PKV_ERR_INVALID_ARGUMENT, "all inputs must be CUDA tensors");
  return pkv::launch_eviction_scores(recency, frequency, attn_weights, valid_mask, scores,
                                     num_blocks, block_size, w_recency, w_frequency, w_attention,
                                     as_stream(stream));
}

size_t pkv_eviction_select_workspace_size(int64_t num_blocks, int64_t k) {
  return pkv::scores_select_workspace_size(num_blocks, k);
}

static int check_select(int64_t n, int64_t k, const void* in, const void* out) {
  if (k < 0) return fail(PKV_ERR_INVALID_ARGUMENT, "k must be non-negative");
  if (n < 0) return fail(PKV_ERR_INVALID_ARGUMENT, "num_blocks must be non-negative");
  if (n > ((int64_t)1 << 31))
    return fail(PKV_ERR_UNSUPPORTED, "more than 2^31 blocks per selection");
  if (n > 0 && k > 0 && (!in || !out))
    return fail(PKV_ERR_INVALID_ARGUMENT, "null input or output pointer");
  return PKV_OK;
}

int pkv_eviction_select(const float* scores, int64_t num_blocks, int64_t k, int64_t* out_indices,
                        void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  int rc = check_select(num_blocks, k, scores, out_indices);
  if (rc != PKV_OK) return rc;
  return pkv::launch_select(scores, nullptr, num_blocks, k, 0, out_indices, nullptr, workspace,
                            workspace_bytes, as_stream(stream));
}

size_t pkv_eviction_scores_select_workspace_size(int64_t num_blocks, int64_t k) {
  return pkv::fused_select_workspace_size(num_blocks, k);
}

int pkv_eviction_scores_select(const float* recency, const float* frequency,
                               const float* attn_weights, const uint8_t* valid_mask,
                               float* scores, int64_t num_blocks, int32_t block_size,
                               float w_recency, float w_frequency, float w_attention, int64_t k,
                               int64_t* out_indices, void* workspace, size_t workspace_bytes,
                               void* stream) {
  clear_error();
  if (num_blocks < 0 || block_size < 0)
    return fail(PKV_ERR_INVALID_ARGUMENT, "attn_weights must be [num_blocks, block_size]");
  int rc = check_select(num_blocks, k, recency, out_indices);
  if (rc != PKV_OK) return rc;
  if (num_blocks > 0 &&
      (!recency || !frequency || (block_size > 0 && (!attn_weights || !valid_mask))))
    return fail(PKV_ERR_INVALID_ARGUMENT, "all inputs must be CUDA tensors");
  return pkv::launch_scores_select(recency, frequency, attn_weights, valid_mask, scores,
                                   num_blocks, block_size, w_recency, w_frequency, w_attention,
                                   k, out_indices, workspace, workspace_bytes,
                                   as_stream(stream));
}

int pkv_eviction_local_candidates(const float* scores, int64_t num_blocks, int64_t k,
                                  int64_t id_offset, uint64_t* out_keys, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  clear_error();
  int rc = check_select(num_blocks, k, scores, out_keys);
  if (rc != PKV_OK) return rc;
  if (id_offset < 0 || id_offset + num_blocks > ((int64_t)1 << 32))
    return fail(PKV_ERR_INVALID_ARGUMENT, "global block ids must lie in [0, 2^32)");
  return pkv::launch_select(scores, nullptr, num_blocks, k, id_offset, nullptr, out_keys,
                            workspace, workspace_bytes, as_stream(stream));
}

size_t pkv_eviction_merge_workspace_size(int64_t num_keys, int64_t k) {
  return pkv::select_workspace_size(num_keys, k);
}

int pkv_eviction_merge(const uint64_t* keys, int64_t num_keys, int64_t k, int64_t* out_indices,
                       void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  int rc = check_select(num_keys, k, keys, out_indices);
  if (rc != PKV_OK) return rc;
  return pkv::launch_select(nullptr, keys, num_keys, k, 0, out_indices, nullptr, workspace,
                            workspace_bytes, as_stream(stream));
}

static int quantize_checked(const void* kv, int32_t kv_dtype, int8_t* q, float* scale,
                            int64_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                            int32_t head_dim, const uint8_t* skip, void* stream) {
  if (num_blocks < 0 || block_size < 0 || num_kv_heads < 0 || head_dim < 0)
    return fail(PKV_ERR_INVALID_ARGUMENT, "expected 4D [nb, bs, nkv, hd]");
  if (kv_dtype < 0 || kv_dtype > 2)
    return fail(PKV_ERR_INVALID_ARGUMENT, "kv must be float32, float16 or bfloat16");
  if (num_blocks > 0 && num_kv_heads > 0 && (!kv || !q || !scale))
    return fail(PKV_ERR_INVALID_ARGUMENT, "null input or output pointer");
  if (num_blocks > 0x7fffffffLL)
    return fail(PKV_ERR_UNSUPPORTED, "more than 2^31 - 1 blocks in one call");
  if ((int64_t)num_kv_heads * 4 > 48 * 1024)
    return fail(PKV_ERR_UNSUPPORTED, "num_kv_heads too large");
  if (num_kv_heads == 0) return PKV_OK;
  return pkv::launch_quantize(kv, kv_dtype, q, scale, num_blocks, block_size, num_kv_heads,
                              head_dim, skip, as_stream(stream));
}

int pkv_quantize_kv_per_block(const void* kv, int32_t kv_dtype, int8_t* q, float* scale,
                              int64_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                              int32_t head_dim, void* stream) {
  clear_error();
  return quantize_checked(kv, kv_dtype, q, scale, num_blocks, block_size, num_kv_heads, head_dim,
                          nullptr, stream);
}

int pkv_quantize_kv_per_block_except(const void* kv, int32_t kv_dtype, const uint8_t* skip,
                                     int8_t* q, float* scale, int64_t num_blocks,
                                     int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                                     void* stream) {
  clear_error();
  if (num_blocks > 0 && !skip) return fail(PKV_ERR_INVALID_ARGUMENT, "null skip mask");
  return quantize_checked(kv, kv_dtype, q, scale, num_blocks, block_size, num_kv_heads, head_dim,
                          skip, stream);
}

size_t pkv_attention_stats_workspace_size(int64_t num_blocks, int32_t block_size,
                                          int32_t num_kv_heads) {
  if (num_blocks <= 0 || block_size <= 0 || num_kv_heads <= 0) return 0;
  return pkv::attention_stats_workspace_size(num_blocks, block_size, num_kv_heads);
}

int pkv_attention_stats(const void* k, int32_t k_dtype, const float* q, float* attn,
                        int64_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                        int32_t head_dim, float sm_scale, void* workspace, size_t workspace_bytes,
                        void* stream) {
  clear_error();
  if (num_blocks < 0 || num_kv_heads <= 0)
    return fail(PKV_ERR_INVALID_ARGUMENT, "expected K [nb, bs, nkv, 128] and q [nkv, 128]");
  if (head_dim != 128) return fail(PKV_ERR_UNSUPPORTED, "attention statistics need head_dim 128");
  if (block_size != 16 && block_size != 32)
    return fail(PKV_ERR_UNSUPPORTED, "attention statistics need block_size 16 or 32");
  if (k_dtype < 0 || k_dtype > 2)
    return fail(PKV_ERR_INVALID_ARGUMENT, "k must be float32, float16 or bfloat16");
  if (num_blocks > 0 && (!k || !q || !attn))
    return fail(PKV_ERR_INVALID_ARGUMENT, "null input or output pointer");
  const size_t elem = k_dtype == 0 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(k) % (4 * elem) != 0 || reinterpret_cast<uintptr_t>(q) % 16 != 0)
    return fail(PKV_ERR_INVALID_ARGUMENT, "k and q must be aligned to 4 elements / 16 bytes");
  return pkv::launch_attention_stats(k, k_dtype, q, attn, num_blocks, block_size, num_kv_heads,
                                     sm_scale, workspace, workspace_bytes, as_stream(stream));
}

int pkv_mark_blocks(const int64_t* ids, int64_t num_ids, int64_t id_offset, int64_t num_blocks,
                    uint8_t* mask, void* stream) {
  clear_error();
  if (num_ids < 0 || num_blocks < 0) return fail(PKV_ERR_INVALID_ARGUMENT, "negative size");
  if ((num_ids > 0 && !ids) || (num_blocks > 0 && !mask))
    return fail(PKV_ERR_INVALID_ARGUMENT, "null input or output pointer");
  return pkv::launch_mark_blocks(ids, num_ids, id_offset, num_blocks, mask, as_stream(stream));
}

int pkv_compact_block_tables(const int32_t* block_tables, const int32_t* seq_lens,
                             const uint8_t* evicted, int32_t* tables_out, int32_t* lens_out,
                             int32_t num_seqs, int32_t max_blocks_per_seq, int32_t block_size,
                             int64_t num_blocks, void* stream) {
  clear_error();
  if (num_seqs < 0 || max_blocks_per_seq < 0 || block_size <= 0 || num_blocks < 0)
    return fail(PKV_ERR_INVALID_ARGUMENT, "invalid table shape");
  if (num_seqs > 0 && (!block_tables || !seq_lens || !evicted || !tables_out || !lens_out))
    return fail(PKV_ERR_INVALID_ARGUMENT, "null input or output pointer");
  return pkv::launch_compact_tables(block_tables, seq_lens, evicted, tables_out, lens_out,
                                    num_seqs, max_blocks_per_seq, block_size, num_blocks,
                                    as_stream(stream));
}

static int check_decode(const pkv::DecodeArgs& a) {
  if (a.num_seqs < 0 || a.num_heads <= 0 || a.num_kv_heads <= 0 || a.head_dim <= 0 ||
      a.block_size <= 0 || a.num_blocks < 0 || a.max_blocks_per_seq < 0)
    return fail(PKV_ERR_INVALID_ARGUMENT, "invalid decode shape");
  if (a.head_dim % 32 != 0 || a.head_dim > 256)
    return fail(PKV_ERR_INVALID_ARGUMENT, "supports head_dim % 32 == 0, <= 256");
  if (a.block_size > 64) return fail(PKV_ERR_INVALID_ARGUMENT, "supports block_size <= 64");
  if (a.num_heads % a.num_kv_heads != 0)
    return fail(PKV_ERR_INVALID_ARGUMENT, "GQA requires num_heads % num_kv_heads == 0");
  if (a.num_seqs > 0 && (!a.q || !a.k_cache || !a.k_scale || !a.v_cache || !a.v_scale ||
                         !a.seq_lens || !a.out || (a.max_blocks_per_seq > 0 && !a.block_tables)))
    return fail(PKV_ERR_INVALID_ARGUMENT, "null input or output pointer");
  if (a.num_heads > 65535) return fail(PKV_ERR_UNSUPPORTED, "num_heads > 65535");
  return PKV_OK;
}

static pkv::DecodeArgs decode_args(const float* q, const int8_t* k_cache, const float* k_scale,
                                   const int8_t* v_cache, const float* v_scale,
                                   const int32_t* block_tables, const int32_t* seq_lens,
                                   float* out, int32_t num_seqs, int32_t num_heads,
                                   int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                   int64_t num_blocks, int32_t max_blocks_per_seq,
                                   float sm_scale) {
  pkv::DecodeArgs a;
  a.q = q;
  a.k_cache = k_cache;
  a.k_scale = k_scale;
  a.v_cache = v_cache;
  a.v_scale = v_scale;
  a.block_tables = block_tables;
  a.seq_lens = seq_lens;
  a.out = out;
  a.num_seqs = num_seqs;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.num_blocks = num_blocks;
  a.max_blocks_per_seq = max_blocks_per_seq;
  a.sm_scale = sm_scale;
  return a;
}

size_t pkv_quant_paged_attention_workspace_size(int32_t num_seqs, int32_t num_heads,
                                                int32_t num_kv_heads, int32_t head_dim,
                                                int32_t block_size,
                                                int32_t max_blocks_per_seq) {
  // Pointers are unknown here; size for the largest plan (16-byte aligned
  // pointers take the same or fewer splits).
  pkv::DecodeArgs a = decode_args(reinterpret_cast<const float*>(16),
                                  reinterpret_cast<const int8_t*>(16), nullptr,
                                  reinterpret_cast<const int8_t*>(16), nullptr, nullptr, nullptr,
                                  reinterpret_cast<float*>(16), num_seqs, num_heads, num_kv_heads,
                                  head_dim, block_size, 1, max_blocks_per_seq, 1.0f);
  if (num_seqs <= 0 || num_heads <= 0 || num_kv_heads <= 0 || block_size <= 0) return 0;
  size_t fast = pkv::decode_workspace_size(a);
  a.q = reinterpret_cast<const float*>(4);  // force the generic plan
  size_t gen = pkv::decode_workspace_size(a);
  return fast > gen ? fast : gen;
}

int pkv_quant_paged_attention_kernel_launches(int32_t num_seqs, int32_t num_heads,
                                              int32_t num_kv_heads, int32_t head_dim,
                                              int32_t block_size, int32_t max_blocks_per_seq) {
  if (num_seqs <= 0 || num_heads <= 0 || num_kv_heads <= 0 || block_size <= 0) return 0;
  const pkv::DecodeArgs a = decode_args(
      reinterpret_cast<const float*>(16), reinterpret_cast<const int8_t*>(16), nullptr,
      reinterpret_cast<const int8_t*>(16), nullptr, nullptr, nullptr, reinterpret_cast<float*>(16),
      num_seqs, num_heads, num_kv_heads, head_dim, block_size, 1, max_blocks_per_seq, 1.0f);
  return pkv::decode_kernel_launches(a);
}

int pkv_quant_paged_attention(const float* q, const int8_t* k_cache, const float* k_scale,
                              const int8_t* v_cache, const float* v_scale,
                              const int32_t* block_tables, const int32_t* seq_lens, float* out,
                              int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                              int32_t head_dim, int32_t block_size, int64_t num_blocks,
                              int32_t max_blocks_per_seq, float sm_scale, void* workspace,
                              size_t workspace_bytes, void* stream) {
  clear_error();
  pkv::DecodeArgs a = decode_args(q, k_cache, k_scale, v_cache, v_scale, block_tables, seq_lens,
                                  out, num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                                  num_blocks, max_blocks_per_seq, sm_scale);
  int rc = check_decode(a);
  if (rc != PKV_OK) return rc;
  return pkv::launch_decode(a, workspace, workspace_bytes, as_stream(stream));
}

size_t pkv_write_to_cache_workspace_size(int64_t num_tokens, int32_t num_kv_heads) {
  return pkv::write_to_cache_workspace_size(num_tokens, num_kv_heads);
}

int pkv_write_to_cache(const void* key, const void* value, int32_t dtype, int8_t* kv_cache,
                       float* scale_cache, const int64_t* slot_mapping, int64_t num_tokens,
                       int64_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                       int32_t head_dim, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (num_tokens < 0 || num_blocks < 0 || block_size <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return fail(PKV_ERR_INVALID_ARGUMENT, "invalid write_to_cache shape");
  if (dtype < 0 || dtype > 2)
    return fail(PKV_ERR_INVALID_ARGUMENT, "key/value must be float32, float16 or bfloat16");
  if (num_tokens > 0 && (!key || !value || !kv_cache || !scale_cache || !slot_mapping))
    return fail(PKV_ERR_INVALID_ARGUMENT, "null input or output pointer");
  if (num_tokens > 0x7fffffffLL)
    return fail(PKV_ERR_UNSUPPORTED, "more than 2^31 - 1 tokens in one call");
  return pkv::launch_write_to_cache(key, value, dtype, kv_cache, scale_cache, slot_mapping,
                                    num_tokens, num_blocks, block_size, num_kv_heads, head_dim,
                                    workspace, workspace_bytes, as_stream(stream));
}

}  // extern "C"
