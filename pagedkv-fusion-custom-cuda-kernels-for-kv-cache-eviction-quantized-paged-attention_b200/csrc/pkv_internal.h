// Internal launcher interface shared by the C-ABI layer (abi.cu) and the
// kernel translation units.  Every launcher enqueues work on `stream` and
// returns a pkv::Status; none of them synchronizes.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

namespace pkv {

// Per-device error word (abi.cu).  Kernels record the first bad-input or
// timeout event here instead of trapping.
int* device_error_word();

// Thread-local message for the last failing call (abi.cu).
void set_error(const std::string& msg);

// ---- quantize.cu ----------------------------------------------------------
// skip (nullable): blocks with a nonzero byte are neither read nor written.
int launch_quantize(const void* kv, int dtype, int8_t* q, float* scale, int64_t num_blocks,
                    int block_size, int num_kv_heads, int head_dim, const uint8_t* skip,
                    cudaStream_t stream);

// ---- attn_stats.cu ------------------------------------------------------------
size_t attention_stats_workspace_size(int64_t num_blocks, int block_size, int num_kv_heads);
int launch_attention_stats(const void* k, int dtype, const float* q, float* attn,
                           int64_t num_blocks, int block_size, int num_kv_heads, float sm_scale,
                           void* workspace, size_t workspace_bytes, cudaStream_t stream);

// ---- compose.cu -------------------------------------------------------------
int launch_mark_blocks(const int64_t* ids, int64_t n, int64_t id_offset, int64_t num_blocks,
                       uint8_t* mask, cudaStream_t stream);
int launch_compact_tables(const int32_t* block_tables, const int32_t* seq_lens,
                          const uint8_t* evicted, int32_t* tables_out, int32_t* lens_out,
                          int num_seqs, int max_blocks_per_seq, int block_size,
                          int64_t num_blocks, cudaStream_t stream);

int launch_write_to_cache(const void* key, const void* value, int dtype, int8_t* kv_cache,
                          float* scale_cache, const int64_t* slot_mapping, int64_t num_tokens,
                          int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                          void* workspace, size_t workspace_bytes, cudaStream_t stream);
size_t write_to_cache_workspace_size(int64_t num_tokens, int num_kv_heads);

// ---- eviction.cu ----------------------------------------------------------
int launch_eviction_scores(const float* recency, const float* frequency, const float* attn,
                           const uint8_t* valid, float* scores, int64_t num_blocks,
                           int block_size, float w_r, float w_f, float w_a,
                           cudaStream_t stream);

size_t select_workspace_size(int64_t n, int64_t k);
// Sorts (orderable(score) << 32 | id) keys; emits the first k ids (out_ids)
// and/or the first k keys with `id_offset` added to the id (out_keys).
int launch_select(const float* scores, const uint64_t* keys_in, int64_t n, int64_t k,
                  int64_t id_offset, int64_t* out_ids, uint64_t* out_keys, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream);

// Single-launch cluster path (eviction_cluster.cu) for n <= 16,384: scores
// from the statistics (scores_in == nullptr) or given scores; writes the k
// selected ids.  Returns kUnsupported without launching when it cannot run.
int launch_cluster_select(const float* rec, const float* freq, const float* attn,
                          const uint8_t* valid, const float* scores_in, float* scores_out,
                          int64_t n, int bs, float wr, float wf, float wa, int64_t k,
                          int64_t* out_ids, cudaStream_t stream);
int cluster_select_max_blocks();
// True when the current device can schedule the selection cluster.
bool cluster_select_available();
// Workspace bytes for pkv_eviction_select: 0 when the cluster path runs.
size_t scores_select_workspace_size(int64_t n, int64_t k);

size_t fused_select_workspace_size(int64_t n, int64_t k);
int launch_scores_select(const float* recency, const float* frequency, const float* attn,
                         const uint8_t* valid, float* scores, int64_t num_blocks,
                         int block_size, float w_r, float w_f, float w_a, int64_t k,
                         int64_t* out_ids, void* workspace, size_t workspace_bytes,
                         cudaStream_t stream);

// ---- decode.cu ------------------------------------------------------------
struct DecodeArgs {
  const float* q;
  const int8_t* k_cache;
  const float* k_scale;
  const int8_t* v_cache;
  const float* v_scale;
  const int32_t* block_tables;
  const int32_t* seq_lens;
  float* out;
  int num_seqs, num_heads, num_kv_heads, head_dim, block_size;
  int64_t num_blocks;
  int max_blocks_per_seq;
  float sm_scale;
};

size_t decode_workspace_size(const DecodeArgs& a);
// Kernels one launch_decode call issues for these arguments.
int decode_kernel_launches(const DecodeArgs& a);
int launch_decode(const DecodeArgs& a, void* workspace, size_t workspace_bytes,
                  cudaStream_t stream);

}  // namespace pkv
