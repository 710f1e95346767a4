// Decode attention for callers that cannot allocate device memory.
//
// pkv_quant_paged_attention needs a workspace for its split-K partials,
// which the caller allocates.  Some callers have no way to do that: a
// plugin that its host framework hands only input and output device
// pointers (the framework budgets all device memory up front and forbids
// allocation afterwards), or a latency-critical serving path that must not
// pay cudaMalloc's implicit device synchronization.  For them,
// pkv_quant_paged_attention_noalloc runs the same kernels with the
// partials in a fixed scratch array that lives in this library's device
// image: every GPU that loads the library holds kNoAllocScratchBytes of
// device memory for it until the process exits.
//
// Host code cannot pass `g_noalloc_scratch` itself to a kernel: in host
// code that name is only a host-side stand-in for the symbol.  The device
// address is looked up once per device, with that device current, by
// cudaGetSymbolAddress on the first call on that device; that first call
// should therefore be made before any stream capture begins.
//
// All calls on a device share the one scratch array: two calls whose
// kernels overlap on the GPU (different streams without ordering between
// them) race on it and may produce wrong outputs.  Serialize them, e.g. by
// issuing every call on one stream.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/pagedkv_fusion.h"
#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace {

// 32 MiB: room for the split-K partials of, e.g., 64 sequences of 2,048
// tokens with 8 heads (4.3 MB).  A call that needs more (the 512-sequence,
// 40-head decode needs ~170 MB) is rejected with PKV_ERR_UNSUPPORTED.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;

// Device address of g_noalloc_scratch on the current device, looked up on
// first use with that device current.  Returns nullptr on failure (the
// caller reports the CUDA error).
void* scratch_on_current_device(cudaError_t* why) {
  static void* ptrs[kMaxDevices] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *why = e != cudaSuccess ? e : cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      *why = e;
      return nullptr;
    }
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace

extern "C" {

size_t pkv_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int pkv_quant_paged_attention_noalloc(const float* q, const int8_t* k_cache,
                                      const float* k_scale, const int8_t* v_cache,
                                      const float* v_scale, const int32_t* block_tables,
                                      const int32_t* seq_lens, float* out, int32_t num_seqs,
                                      int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                      int32_t block_size, int64_t num_blocks,
                                      int32_t max_blocks_per_seq, float sm_scale, void* stream) {
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
  // Shape checks first (the envelope violations are reported by the
  // allocating entry point, which rejects them before launching anything),
  // then the scratch requirement.
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks < 0 || max_blocks_per_seq < 0) {
    pkv::set_error("invalid decode shape");
    return PKV_ERR_INVALID_ARGUMENT;
  }
  if (head_dim % 32 != 0 || head_dim > 256 || block_size > 64 || num_heads % num_kv_heads != 0) {
    // let the allocating entry point produce its exact message
    return pkv_quant_paged_attention(q, k_cache, k_scale, v_cache, v_scale, block_tables,
                                     seq_lens, out, num_seqs, num_heads, num_kv_heads, head_dim,
                                     block_size, num_blocks, max_blocks_per_seq, sm_scale,
                                     nullptr, 0, stream);
  }
  const size_t need = pkv::decode_workspace_size(a);
  if (need > kNoAllocScratchBytes) {
    pkv::set_error("decode needs " + std::to_string(need) +
                   " bytes of split-K scratch; the no-allocation entry point has " +
                   std::to_string(kNoAllocScratchBytes) +
                   " (use pkv_quant_paged_attention with a caller-provided workspace)");
    return PKV_ERR_UNSUPPORTED;
  }
  void* scratch = nullptr;
  if (need > 0) {
    cudaError_t why = cudaSuccess;
    scratch = scratch_on_current_device(&why);
    if (scratch == nullptr) {
      pkv::set_error(std::string("cudaGetSymbolAddress for the decode scratch failed: ") +
                     cudaGetErrorString(why));
      return PKV_ERR_CUDA;
    }
  }
  // The scratch holds split-K partials, each written by its split before it
  // is merged within the same call, and the persistent decode kernel's
  // arrival counters, which carry a per-launch tag (a counter left by an
  // earlier call never matches).  Nothing in it has to start at zero, and
  // the previous call's contents are harmless.
  return pkv_quant_paged_attention(q, k_cache, k_scale, v_cache, v_scale, block_tables,
                                   seq_lens, out, num_seqs, num_heads, num_kv_heads, head_dim,
                                   block_size, num_blocks, max_blocks_per_seq, sm_scale, scratch,
                                   need > 0 ? kNoAllocScratchBytes : 0, stream);
}

}  // extern "C"
