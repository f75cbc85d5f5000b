// KV-pool sizing: ModelRunner::probe_num_kvcache_blocks
// (nanovllm_rs/src/engine/model_runner.rs:264-284).
//   block_bytes = 2 * layers * block_size * kv_heads_per_rank * head_dim * dtype_bytes
//   budget      = (i64)(total * gpu_memory_utilization) - (total - free)
//   num_blocks  = max(budget / block_bytes, 0), and 0 is an error (the
//                 reference asserts "not enough GPU memory left")
// Integer arithmetic as the reference's (the f64 product truncated toward 0,
// i64 floor division of a non-negative budget).  Under tensor parallelism
// each rank probes its own device and the caller takes the minimum.
#include "common.cuh"

extern "C" {

int nvkv_kv_pool_blocks(int64_t free_bytes, int64_t total_bytes, double gpu_memory_utilization,
                        int num_layers, int block_size, int num_kv_heads, int head_dim,
                        int dtype_bytes, int64_t* num_blocks) {
  using namespace nvkv;
  clear_error();
  if (!num_blocks || free_bytes < 0 || total_bytes <= 0 || free_bytes > total_bytes ||
      !(gpu_memory_utilization > 0.0 && gpu_memory_utilization <= 1.0) || num_layers <= 0 ||
      block_size <= 0 || num_kv_heads <= 0 || head_dim <= 0 || dtype_bytes <= 0)
    return set_error(NVKV_ERR_INVALID_ARG, "kv_pool_blocks: bad arguments");
  const int64_t block_bytes = 2 * (int64_t)num_layers * block_size * num_kv_heads * head_dim *
                              (int64_t)dtype_bytes;
  const int64_t budget =
      (int64_t)((double)total_bytes * gpu_memory_utilization) - (total_bytes - free_bytes);
  const int64_t n = budget > 0 ? budget / block_bytes : 0;
  *num_blocks = n;
  if (n <= 0)
    return set_error(NVKV_ERR_INVALID_ARG,
                     "kv_pool_blocks: not enough GPU memory left to allocate the KV cache");
  return NVKV_OK;
}

int nvkv_kv_pool_probe(double gpu_memory_utilization, int num_layers, int block_size,
                       int num_kv_heads, int head_dim, int dtype_bytes, int64_t* num_blocks) {
  NVKV_RANGE("nvkv_kv_pool_probe");
  using namespace nvkv;
  clear_error();
  if (!num_blocks) return set_error(NVKV_ERR_INVALID_ARG, "kv_pool_probe: null output");
  size_t free_b = 0, total_b = 0;
  int rc = check_cuda(cudaMemGetInfo(&free_b, &total_b), "kv_pool_probe: cudaMemGetInfo");
  if (rc) return rc;
  return nvkv_kv_pool_blocks((int64_t)free_b, (int64_t)total_b, gpu_memory_utilization,
                             num_layers, block_size, num_kv_heads, head_dim, dtype_bytes,
                             num_blocks);
}

}  // extern "C"
