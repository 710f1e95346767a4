/*
 * PagedKV-Fusion for NVIDIA B200 (sm_100a) -- C ABI of libpagedkv_sm100.so.
 *
 * This is the drop-in boundary that replaces the reference's pybind11
 * module (csrc/bindings.cpp:14-26, module pagedkv_fusion._C) and the torch /
 * library calls around it.  Every entry point takes plain device pointers
 * and sizes, enqueues its kernels on `stream` (a cudaStream_t; NULL is the
 * legacy default stream), never synchronizes, and returns a status code.
 * On failure the message of the last error on the calling thread is
 * available from pkv_last_error_string().
 *
 * Layouts (unchanged from the reference, csrc/quant_paged_attention.cu:4-8):
 *   paged cache   int8  [num_blocks, block_size, num_kv_heads, head_dim]
 *   scales        fp32  [num_blocks, num_kv_heads]
 *   block_tables  int32 [num_seqs, max_blocks_per_seq]  (-1 = unused)
 *   seq_lens      int32 [num_seqs]
 * All arrays are C-contiguous.  Kernels that find bad data on the device (a
 * block id outside [0, num_blocks), a slot outside the cache) skip it and
 * record a code in a per-device error word read by pkv_read_device_error();
 * they never trap.
 */
#ifndef PAGEDKV_FUSION_H
#define PAGEDKV_FUSION_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
#define PKV_OK 0
#define PKV_ERR_INVALID_ARGUMENT 1 /* shape / dtype / pointer precondition */
#define PKV_ERR_UNSUPPORTED 2      /* valid but outside this build's envelope */
#define PKV_ERR_WORKSPACE 3        /* workspace missing or too small */
#define PKV_ERR_CUDA 4             /* a CUDA runtime call or launch failed */
#define PKV_ERR_DEVICE_INPUT 5     /* pkv_read_device_error found bad input */

/* Device error codes recorded by kernels. */
#define PKV_DEVERR_NONE 0
#define PKV_DEVERR_BAD_BLOCK_ID 1
#define PKV_DEVERR_WAIT_TIMEOUT 2
#define PKV_DEVERR_BAD_SLOT 3
#define PKV_DEVERR_SEQ_TOO_LONG 4 /* seq_len beyond the block-table width */

/* Element types of floating-point KV inputs. */
#define PKV_DTYPE_F32 0
#define PKV_DTYPE_F16 1
#define PKV_DTYPE_BF16 2

/* Message of the last failing call on this thread ("" if none). */
const char *pkv_last_error_string(void);

/* ABI version: major * 10000 + minor * 100 + patch. */
int pkv_version(void);

/*
 * Reads (and, if `reset` != 0, clears) the error word of the current
 * device.  Synchronizes the device.  *code receives a PKV_DEVERR_* value.
 * Returns PKV_ERR_DEVICE_INPUT when the word was non-zero.
 */
int pkv_read_device_error(int32_t *code, int reset);

/*
 * Fused eviction score per KV block (lower = evict first):
 *   score[b] = w_recency*recency[b] + w_frequency*frequency[b]
 *            + w_attention*mean(attn_weights[b, t] over valid t)
 * bit-identical to pagedkv_fusion/reference.py:38-71 (NumPy float32).
 * valid_mask holds one byte per token (non-zero = valid).
 * Replaces eviction_scores_cuda (csrc/eviction_score.cu:97-136) bound at
 * csrc/bindings.cpp:16-20.
 */
int pkv_eviction_scores(const float *recency, const float *frequency,
                        const float *attn_weights, const uint8_t *valid_mask,
                        float *scores, int64_t num_blocks, int32_t block_size,
                        float w_recency, float w_frequency, float w_attention,
                        void *stream);

/*
 * Indices of the k lowest scores, ascending by (score, block id), -0.0 ==
 * +0.0, NaN last; min(k, num_blocks) int64 entries are written.  Matches
 * select_eviction_candidates_ref (pagedkv_fusion/reference.py:74-81) and
 * replaces torch.topk in pagedkv_fusion/ops.py:97-98.
 */
size_t pkv_eviction_select_workspace_size(int64_t num_blocks, int64_t k);
int pkv_eviction_select(const float *scores, int64_t num_blocks, int64_t k,
                        int64_t *out_indices, void *workspace,
                        size_t workspace_bytes, void *stream);

/*
 * Score and select in one call: writes scores (if non-NULL) and the
 * min(k, num_blocks) selected block ids.  Composition of
 * ops.eviction_scores + ops.select_eviction_candidates
 * (pagedkv_fusion/ops.py:63-98).
 */
size_t pkv_eviction_scores_select_workspace_size(int64_t num_blocks, int64_t k);
int pkv_eviction_scores_select(const float *recency, const float *frequency,
                               const float *attn_weights,
                               const uint8_t *valid_mask, float *scores,
                               int64_t num_blocks, int32_t block_size,
                               float w_recency, float w_frequency,
                               float w_attention, int64_t k,
                               int64_t *out_indices, void *workspace,
                               size_t workspace_bytes, void *stream);

/*
 * Sharded eviction (one rank's block range [id_offset, id_offset +
 * num_blocks)): the min(k, num_blocks) smallest candidate keys
 * (orderable(score) << 32 | (id_offset + i)), ascending.  No reference
 * counterpart: the reference is single-GPU (integration/vllm/
 * pagedkv_fusion_backend.py:23); these keys are what ranks exchange.
 */
int pkv_eviction_local_candidates(const float *scores, int64_t num_blocks,
                                  int64_t k, int64_t id_offset,
                                  uint64_t *out_keys, void *workspace,
                                  size_t workspace_bytes, void *stream);

/*
 * Global selection from gathered candidate keys: the block ids of the k
 * smallest keys, ascending.  Identical on every rank for identical input.
 */
size_t pkv_eviction_merge_workspace_size(int64_t num_keys, int64_t k);
int pkv_eviction_merge(const uint64_t *keys, int64_t num_keys, int64_t k,
                       int64_t *out_indices, void *workspace,
                       size_t workspace_bytes, void *stream);

/*
 * Symmetric per-(block, head) INT8 quantization of kv [num_blocks,
 * block_size, num_kv_heads, head_dim] (PKV_DTYPE_*): q int8 of the same
 * shape, scale fp32 [num_blocks, num_kv_heads].  Codes bit-identical to
 * quantize_kv_per_block_ref (pagedkv_fusion/reference.py:88-105); replaces
 * the torch ops of pagedkv_fusion/quantize.py:15-31.
 */
int pkv_quantize_kv_per_block(const void *kv, int32_t kv_dtype, int8_t *q,
                              float *scale, int64_t num_blocks,
                              int32_t block_size, int32_t num_kv_heads,
                              int32_t head_dim, void *stream);

/*
 * Per-token attention statistics derived from the keys, the input the
 * eviction score's attention term reads: for a K pool [num_blocks,
 * block_size, num_kv_heads, 128] (float32 / float16 / bfloat16, dtype codes
 * as for quantization) and one query vector per KV head q [num_kv_heads,
 * 128] float32,
 *   s_h[b, t]  = sm_scale * (q_h . K[b, t, h, :])
 *   attn[b, t] = mean_h exp(s_h[b, t] - max over the pool of s_h)
 * written to attn [num_blocks, block_size] float32, in (0, 1].  block_size
 * 16 or 32.  The workspace holds the logits and the per-head maxima.  No
 * counterpart in the reference, whose eviction statistics are given arrays
 * (pagedkv_fusion/reference.py:38-71); the definition is this library's.
 */
size_t pkv_attention_stats_workspace_size(int64_t num_blocks,
                                          int32_t block_size,
                                          int32_t num_kv_heads);
int pkv_attention_stats(const void *k, int32_t k_dtype, const float *q,
                        float *attn, int64_t num_blocks, int32_t block_size,
                        int32_t num_kv_heads, int32_t head_dim, float sm_scale,
                        void *workspace, size_t workspace_bytes, void *stream);

/*
 * pkv_quantize_kv_per_block for the blocks whose skip[b] byte is zero;
 * blocks with a nonzero byte are neither read nor written (their codes and
 * scale keep whatever they held).  Quantizes the blocks that survive an
 * eviction without touching the evicted ones.  No counterpart in the
 * reference: its end-to-end demo (scripts/run_end_to_end_demo.py:74-116)
 * scores and selects, then quantizes every block and decodes over the
 * unchanged tables.
 */
int pkv_quantize_kv_per_block_except(const void *kv, int32_t kv_dtype,
                                     const uint8_t *skip, int8_t *q,
                                     float *scale, int64_t num_blocks,
                                     int32_t block_size, int32_t num_kv_heads,
                                     int32_t head_dim, void *stream);

/*
 * mask[0 .. num_blocks) = 0, then mask[id - id_offset] = 1 for every id in
 * ids[0 .. num_ids) that falls in [id_offset, id_offset + num_blocks): the
 * local eviction mask of a rank holding blocks id_offset.. from the global
 * ids a (sharded) selection returned.  No counterpart in the reference.
 */
int pkv_mark_blocks(const int64_t *ids, int64_t num_ids, int64_t id_offset,
                    int64_t num_blocks, uint8_t *mask, void *stream);

/*
 * Removes evicted blocks from block tables.  For sequence s the first
 * ceil(seq_lens[s] / block_size) entries (clamped to the table width;
 * PKV_DEVERR_SEQ_TOO_LONG beyond it) are its pages, the last holding the
 * remainder; pages whose block has evicted[id] != 0 are dropped, the rest
 * are written in order to tables_out (row padded with -1) and lens_out[s]
 * is the number of tokens they hold.  Every kept page but the last is full,
 * so (tables_out, lens_out) is a valid input to pkv_quant_paged_attention.
 * Ids outside [0, num_blocks) are kept.  No counterpart in the reference.
 */
int pkv_compact_block_tables(const int32_t *block_tables,
                             const int32_t *seq_lens, const uint8_t *evicted,
                             int32_t *tables_out, int32_t *lens_out,
                             int32_t num_seqs, int32_t max_blocks_per_seq,
                             int32_t block_size, int64_t num_blocks,
                             void *stream);

/*
 * Decode-step attention over the INT8 paged cache: out[s, h, :] =
 * softmax(q[s, h] . K^T * sm_scale) V over the seq_lens[s] tokens reached
 * through block_tables[s], dequantized with the per-(block, head) scales;
 * GQA maps head h to kv head h / (num_heads / num_kv_heads).  A sequence of
 * length 0 yields zeros.  Replaces quant_paged_attention_cuda
 * (csrc/quant_paged_attention.cu:172-225) bound at csrc/bindings.cpp:21-25.
 * Envelope: head_dim % 32 == 0 and <= 256, block_size <= 64,
 * num_heads % num_kv_heads == 0.  The workspace holds the partial results
 * of sequences whose pages are split across CTAs, and one arrival counter
 * per (sequence, KV-head group); it needs no initialisation (the counters
 * carry a per-launch tag) and the call issues no memset.
 */
size_t pkv_quant_paged_attention_workspace_size(
    int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
    int32_t block_size, int32_t max_blocks_per_seq);
int pkv_quant_paged_attention(const float *q, const int8_t *k_cache,
                              const float *k_scale, const int8_t *v_cache,
                              const float *v_scale, const int32_t *block_tables,
                              const int32_t *seq_lens, float *out,
                              int32_t num_seqs, int32_t num_heads,
                              int32_t num_kv_heads, int32_t head_dim,
                              int32_t block_size, int64_t num_blocks,
                              int32_t max_blocks_per_seq, float sm_scale,
                              void *workspace, size_t workspace_bytes,
                              void *stream);

/*
 * Number of kernels one pkv_quant_paged_attention call with these shapes
 * launches on its stream (16-byte aligned pointers): 1 for the persistent
 * stream kernel (up to 1,024 sequences with head_dim 128, block_size 16 or
 * 32 and a GQA group of 1, or 2/4/8 at block_size 32), 2 for the
 * tensor-core GQA kernel (block_size 16, groups of 2/4/8) or the split-K
 * kernel, each with its combine.  Lets a caller account for launches
 * without a profiler.  No counterpart in the reference.
 */
int pkv_quant_paged_attention_kernel_launches(int32_t num_seqs, int32_t num_heads,
                                              int32_t num_kv_heads, int32_t head_dim,
                                              int32_t block_size,
                                              int32_t max_blocks_per_seq);

/*
 * pkv_quant_paged_attention without a workspace argument, for callers that
 * cannot allocate device memory (a plugin whose host framework hands it
 * only input/output pointers and forbids allocation, or a serving path that
 * must not pay cudaMalloc's implicit synchronization).  Identical results.
 * The split-K partials live in a fixed pkv_noalloc_scratch_bytes() (32 MiB)
 * array inside the library, held on every GPU that loads the library until
 * exit; calls needing more are rejected with PKV_ERR_UNSUPPORTED.  The
 * first call on a device looks up the array's address (make it before any
 * stream capture).  Calls share the array: calls overlapping on the GPU
 * race.  No counterpart in the reference.
 */
size_t pkv_noalloc_scratch_bytes(void);
int pkv_quant_paged_attention_noalloc(const float *q, const int8_t *k_cache,
                                      const float *k_scale,
                                      const int8_t *v_cache,
                                      const float *v_scale,
                                      const int32_t *block_tables,
                                      const int32_t *seq_lens, float *out,
                                      int32_t num_seqs, int32_t num_heads,
                                      int32_t num_kv_heads, int32_t head_dim,
                                      int32_t block_size, int64_t num_blocks,
                                      int32_t max_blocks_per_seq,
                                      float sm_scale, void *stream);

/*
 * Quantize new K/V tokens and scatter them into the vLLM-shaped cache
 * kv_cache int8 [2, num_blocks, block_size, num_kv_heads, head_dim] and
 * scale_cache fp32 [2, num_blocks, num_kv_heads].  The tokens of one call
 * that land in the same block are quantized together and their scale
 * overwrites that block's scale, as PagedKVFusionBackend.write_to_cache
 * (integration/vllm/pagedkv_fusion_backend.py:63-95) does.
 */
size_t pkv_write_to_cache_workspace_size(int64_t num_tokens,
                                         int32_t num_kv_heads);
int pkv_write_to_cache(const void *key, const void *value, int32_t dtype,
                       int8_t *kv_cache, float *scale_cache,
                       const int64_t *slot_mapping, int64_t num_tokens,
                       int64_t num_blocks, int32_t block_size,
                       int32_t num_kv_heads, int32_t head_dim, void *workspace,
                       size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGEDKV_FUSION_H */
