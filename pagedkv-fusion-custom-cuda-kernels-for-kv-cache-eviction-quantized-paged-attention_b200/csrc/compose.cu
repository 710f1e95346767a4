// Pieces of the evict -> quantize -> decode composition: marking the
// selected blocks, and compacting block tables so that decode skips them.
//
// The reference composes these steps only in a demo that scores and
// selects, then quantizes every block and decodes over the unchanged tables
// (scripts/run_end_to_end_demo.py:74-116); the composition here is: score every block, select the globally lowest
// fraction, quantize the surviving blocks (pkv_quantize_kv_per_block_except
// with this mask), and decode over tables from which the evicted blocks are
// removed, each sequence keeping the tokens of its surviving blocks in order.

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {
namespace {

// mask[id - id_offset] = 1 for every id in [id_offset, id_offset + num_blocks).
__global__ void mark_blocks_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t id_offset,
                                   int64_t num_blocks, uint8_t* __restrict__ mask) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t local = ids[i] - id_offset;
    if (local >= 0 && local < num_blocks) mask[local] = 1;
  }
}

// One warp per sequence.  Page p of the first ceil(L/bs) (clamped to the
// table width) holds bs tokens, the last one L - (pages-1)*bs.  Pages whose
// block is marked are dropped; the kept ones are written in order (a ballot
// and prefix count per 32 pages), the rest of the row becomes -1, and the
// new length is the kept tokens.  Every kept page but the last is full, so
// the compacted row is a valid table for L'.  Block ids outside
// [0, num_blocks) are kept as they are (decode reports them); a length
// beyond the table width is clamped to it and reported like decode does.
__global__ void compact_tables_kernel(const int32_t* __restrict__ bt, const int32_t* __restrict__ sl,
                                      const uint8_t* __restrict__ evicted,
                                      int32_t* __restrict__ bt_out, int32_t* __restrict__ sl_out,
                                      int S, int M, int bs, int64_t nb, int* err) {
  const int lane = threadIdx.x & 31;
  const int s = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (s >= S) return;  // whole warp
  const int L = max(sl[s], 0);
  const int pages = covered_pages(L, bs, M);
  if (lane == 0 && L > pages * bs) record_error(err, kDevSeqTooLong);
  const int32_t* row = bt + (int64_t)s * M;
  int32_t* orow = bt_out + (int64_t)s * M;
  int kept = 0, tokens = 0;
  for (int p0 = 0; p0 < pages; p0 += 32) {
    const int p = p0 + lane;
    bool keep = false;
    int32_t id = -1;
    int tok = 0;
    if (p < pages) {
      id = row[p];
      keep = !(id >= 0 && (int64_t)id < nb && evicted[id]);
      tok = p == pages - 1 ? min(L, pages * bs) - p * bs : bs;
    }
    const uint32_t ball = __ballot_sync(0xffffffffu, keep);
    if (keep) orow[kept + __popc(ball & ((1u << lane) - 1u))] = id;
    int t = keep ? tok : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    tokens += t;
    kept += __popc(ball);
  }
  for (int p = kept + lane; p < M; p += 32) orow[p] = -1;
  if (lane == 0) sl_out[s] = tokens;
}

}  // namespace

int launch_mark_blocks(const int64_t* ids, int64_t n, int64_t id_offset, int64_t num_blocks,
                       uint8_t* mask, cudaStream_t stream) {
  if (num_blocks > 0) {
    const cudaError_t e = cudaMemsetAsync(mask, 0, (size_t)num_blocks, stream);
    if (e != cudaSuccess) {
      set_error(std::string("mask reset failed: ") + cudaGetErrorString(e));
      return kCudaError;
    }
  }
  if (n > 0) {
    const int64_t blocks = (n + 255) / 256;
    mark_blocks_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, stream>>>(
        ids, n, id_offset, num_blocks, mask);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("mark launch failed: ") + cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

int launch_compact_tables(const int32_t* block_tables, const int32_t* seq_lens,
                          const uint8_t* evicted, int32_t* tables_out, int32_t* lens_out,
                          int num_seqs, int max_blocks_per_seq, int block_size,
                          int64_t num_blocks, cudaStream_t stream) {
  if (num_seqs == 0) return kOk;
  compact_tables_kernel<<<(unsigned)((num_seqs + 7) / 8), 256, 0, stream>>>(
      block_tables, seq_lens, evicted, tables_out, lens_out, num_seqs, max_blocks_per_seq,
      block_size, num_blocks, device_error_word());
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("compact launch failed: ") + cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

}  // namespace pkv
