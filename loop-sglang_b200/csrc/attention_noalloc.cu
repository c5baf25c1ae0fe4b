// Paged attention without any device allocation: the split-KV scratch lives in a
// file-scope device array instead of a caller-provided workspace.
//
// Some callers cannot call cudaMalloc: a plugin whose host framework owns all
// device memory and hands it only the input and output tensors (no workspace
// argument), or a latency-critical loop that must not pay cudaMalloc's implicit
// device-wide synchronisation. They call lsb_paged_attention_noalloc, which runs
// the same kernel as lsb_paged_attention with this array as its workspace.
//
// Limits and sharing rules:
//  * the array holds LSB_NOALLOC_ATTENTION_SCRATCH_BYTES bytes on every GPU that
//    loads the library, until the process exits; calls whose scratch would not
//    fit are rejected with LSB_ERR_INVALID;
//  * every call on a device shares the one array, which keeps the last call's
//    contents: calls that overlap on the GPU (different streams, or different
//    host threads without ordering) race on it and must be serialised by the
//    caller;
//  * every call looks up the array's device address on the current device with
//    cudaGetSymbolAddress (host code cannot use the array's name as a device
//    address) and clears the arrival-counter region with an asynchronous memset
//    on the caller's stream before the kernel, so a call whose bounded wait gave
//    up (LSB_DEVERR_TIMEOUT) cannot leave stale counters for the next one. The
//    first call on a device may load the module: make it before any stream
//    capture.
#include "common.cuh"

namespace {

constexpr int64_t kScratchBytes = LSB_NOALLOC_ATTENTION_SCRATCH_BYTES;
static_assert(kScratchBytes > lsb::kAttnCounterBytes,
              "the static scratch must hold the attention counter region");

__device__ __align__(256) unsigned char g_attention_scratch[kScratchBytes];

// Device address of the array on the current device, with its counters cleared on
// `stream`. Allocates nothing.
int scratch_for_current_device(void** out, cudaStream_t stream) {
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_attention_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    cudaGetLastError();
    return lsb::fail(LSB_ERR_CUDA, "paged_attention_noalloc: cudaGetSymbolAddress failed: %s",
                     cudaGetErrorString(e));
  }
  LSB_CUDA(cudaMemsetAsync(ptr, 0, lsb::kAttnCounterBytes, stream));
  *out = ptr;
  return LSB_OK;
}

}  // namespace

extern "C" int lsb_paged_attention_noalloc(void* out, int64_t out_stride, const void* q,
                                           int64_t q_stride, const void* k_cache,
                                           const void* v_cache, int64_t slot_stride,
                                           int64_t num_slots, const int32_t* page_table,
                                           int64_t pt_stride, const int32_t* cache_seqlens,
                                           const int32_t* cu_seqlens_q, int64_t num_reqs,
                                           int64_t rows, int32_t hq, int32_t hkv,
                                           int32_t head_dim, int32_t page_size,
                                           int64_t max_seqlen, float scale, void* stream) {
  const int64_t need = lsb_paged_attention_workspace_size(rows, hq, head_dim, max_seqlen);
  LSB_REQUIRE(need <= kScratchBytes,
              "paged_attention_noalloc: this call needs %lld bytes of scratch; the static "
              "array holds %lld (fewer rows or a smaller max_seqlen fit)",
              (long long)need, (long long)kScratchBytes);
  void* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch, lsb::as_stream(stream))) return rc;
  return lsb_paged_attention(out, out_stride, q, q_stride, k_cache, v_cache, slot_stride,
                             num_slots, page_table, pt_stride, cache_seqlens, cu_seqlens_q,
                             num_reqs, rows, hq, hkv, head_dim, page_size, max_seqlen, scale,
                             scratch, kScratchBytes, stream);
}
