// nvkv_paged_attention_noalloc: the paged attention entry point for callers
// that cannot allocate device memory on the call path.
//
// Why some callers cannot allocate: nanovllm_rs-style engines hand almost all
// free GPU memory to the KV pool at start-up (gpu_memory_utilization, 0.9 by
// default), so a per-call cudaMalloc of split-KV scratch can fail at any
// step; other hosts run attention inside code that must not allocate at all
// (a stream being captured into a CUDA graph that may not contain allocation
// nodes, a runtime whose allocator is not reachable from the kernel binding).
// This entry point takes the same inputs and outputs as nvkv_paged_attention
// but no workspace: the split-KV scratch is a file-scope __device__ array.
//
// Limits and sharing rules:
//  * the scratch is NVKV_NOALLOC_SCRATCH_BYTES (4 MiB); a batch whose
//    split-KV plan needs more is rejected with NVKV_ERR_WORKSPACE;
//  * every GPU that loads the library holds the array until the process
//    exits;
//  * all calls on a device share the one array, which keeps the last call's
//    contents; nothing in it has to start at zero (each partial is written
//    before the combine reads it), but calls that overlap on the GPU (other
//    streams, other threads) race on it -- serialise them;
//  * the first call on a device looks the array's device address up
//    (cudaGetSymbolAddress, once per device, with that device current); with
//    CUDA's lazy module loading that lookup is also when the 4 MiB are taken
//    from the device.  Make that first call before any stream capture and
//    before sizing the KV pool from free memory (nvkv_kv_pool_probe); a call
//    with num_seqs == 0 does only this set-up;
//  * the address is kept for the life of the process: a cudaDeviceReset
//    after the first call is not supported.
#include <mutex>

#include "common.cuh"

namespace nvkv {
namespace {

constexpr size_t kNoAllocScratchBytes = NVKV_NOALLOC_SCRATCH_BYTES;
static_assert(kNoAllocScratchBytes % 256 == 0, "scratch size must keep 256-byte alignment");

// In host code this name is only a stand-in for the symbol, never a device
// address: kernels receive the address that cudaGetSymbolAddress returns.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDev = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDev] = {nullptr};

int noalloc_scratch(void** out) {
  int dev = -1;
  int rc = check_cuda(cudaGetDevice(&dev), "paged_attention_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDev)
    return set_error(NVKV_ERR_UNSUPPORTED, "paged_attention_noalloc: device index above 63");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                    "paged_attention_noalloc: cudaGetSymbolAddress(scratch)");
    if (rc) return rc;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return NVKV_OK;
}

}  // namespace
}  // namespace nvkv

extern "C" int nvkv_paged_attention_noalloc(
    const void* q, int64_t q_stride, int64_t num_q_tokens, const void* k_cache,
    const void* v_cache, int64_t num_blocks, int64_t kv_stride, void* out,
    const uint32_t* cu_seqlens_q, const uint32_t* cu_seqlens_k, const uint32_t* block_tables,
    int64_t block_table_stride, int num_seqs, int max_seqlen_q, int max_seqlen_k,
    int num_q_heads, int num_kv_heads, int head_dim, int page_size, float softmax_scale,
    int causal, int dtype, nvkv_stream_t stream) {
  using namespace nvkv;
  clear_error();
  size_t need = 0;
  int rc = nvkv_paged_attention_workspace_size(num_seqs, num_q_heads, num_kv_heads, head_dim,
                                               max_seqlen_q, max_seqlen_k, &need);
  if (rc) return rc;
  if (need > kNoAllocScratchBytes)
    return set_error(NVKV_ERR_WORKSPACE,
                     "paged_attention_noalloc: this batch needs " + std::to_string(need) +
                         " bytes of split-KV scratch, above the fixed " +
                         std::to_string(kNoAllocScratchBytes) +
                         "-byte static scratch; call nvkv_paged_attention with a workspace");
  void* ws = nullptr;
  rc = noalloc_scratch(&ws);  // every call, so an empty first call is the set-up
  if (rc) return rc;
  return nvkv_paged_attention(q, q_stride, num_q_tokens, k_cache, v_cache, num_blocks, kv_stride,
                              out, cu_seqlens_q, cu_seqlens_k, block_tables, block_table_stride,
                              num_seqs, max_seqlen_q, max_seqlen_k, num_q_heads, num_kv_heads,
                              head_dim, page_size, softmax_scale, causal, ws, kNoAllocScratchBytes,
                              dtype, stream);
}
