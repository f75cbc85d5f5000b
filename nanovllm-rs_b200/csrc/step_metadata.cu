// Device-side step metadata for pure decode steps.
//
// Replaces, for steps where every sequence decodes one token, the host work
// of nanovllm_rs/src/engine/model_runner.rs:69-160 (prepare_model_input:
// positions, slot_mapping, cu_seqlens_q/k, context_lens; its decode case)
// after Sequence::append (src/engine/sequence.rs) added last step's token,
// and the H2D upload of those tensors (model_runner.rs:134-146).  With the
// lengths and block tables resident, consecutive decode steps need no host
// round trip; the block manager only has to have appended the page a
// sequence grows into before the step (block_manager.rs may_append).
//
// One CTA of up to 1024 threads walks the batch in chunks, with a block-wide
// inclusive scan of the new lengths (warp shuffles, then the per-warp totals)
// and a running carry between chunks.  Integer arithmetic only: the outputs
// are bit-exact with the host computation.
#include "common.cuh"

namespace nvkv {

constexpr int kMetaThreads = 1024;

__global__ void __launch_bounds__(kMetaThreads)
    decode_advance_kernel(int num_seqs, int page_size, int64_t* seq_lens,
                          const uint32_t* block_tables, int64_t bt_stride, int64_t num_blocks,
                          int64_t* positions, int64_t* slot_mapping, uint32_t* cu_q,
                          uint32_t* cu_k, int* err) {
  __shared__ uint32_t warp_tot[kMetaThreads / 32];
  __shared__ uint32_t carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    carry = 0;
    cu_q[0] = 0;
    cu_k[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < num_seqs; base += kMetaThreads) {
    const int b = base + tid;
    uint32_t len = 0;
    if (b < num_seqs) {
      const int64_t n = seq_lens[b] + 1;  // last step's token is appended
      seq_lens[b] = n;
      len = (uint32_t)n;
      const int64_t pos = n - 1;
      positions[b] = pos;
      const int64_t blk = pos / page_size;
      int64_t slot = -1;
      if (blk < bt_stride) {
        const uint32_t page = block_tables[(int64_t)b * bt_stride + blk];
        if ((int64_t)page < num_blocks) slot = (int64_t)page * page_size + pos % page_size;
        else record_error(err, NVKV_DEVERR_BLOCK_RANGE);
      } else {
        record_error(err, NVKV_DEVERR_BLOCK_RANGE);  // the page was not appended
      }
      slot_mapping[b] = slot;
      cu_q[b + 1] = (uint32_t)(b + 1);
    }
    uint32_t incl = len;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    uint32_t before = carry;
    for (int w = 0; w < warp; ++w) before += warp_tot[w];
    if (b < num_seqs) cu_k[b + 1] = before + incl;
    __syncthreads();
    if (tid == kMetaThreads - 1) carry = before + incl;  // last thread: chunk total
    __syncthreads();
  }
}

}  // namespace nvkv

extern "C" int nvkv_decode_advance(int num_seqs, int page_size, int64_t* seq_lens,
                                   const uint32_t* block_tables, int64_t block_table_stride,
                                   int64_t num_blocks, int64_t* positions,
                                   int64_t* slot_mapping, uint32_t* cu_seqlens_q,
                                   uint32_t* cu_seqlens_k, nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_decode_advance");
  using namespace nvkv;
  clear_error();
  if (num_seqs < 0 || page_size <= 0 || block_table_stride <= 0 || num_blocks <= 0)
    return set_error(NVKV_ERR_INVALID_ARG, "decode_advance: bad sizes");
  if (num_seqs == 0) return NVKV_OK;
  if (!seq_lens || !block_tables || !positions || !slot_mapping || !cu_seqlens_q ||
      !cu_seqlens_k)
    return set_error(NVKV_ERR_INVALID_ARG, "decode_advance: null pointer");
  decode_advance_kernel<<<1, kMetaThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      num_seqs, page_size, seq_lens, block_tables, block_table_stride, num_blocks, positions,
      slot_mapping, cu_seqlens_q, cu_seqlens_k, device_error_word());
  return check_cuda(cudaGetLastError(), "decode_advance launch");
}
