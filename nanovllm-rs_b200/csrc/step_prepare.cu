// Host-side step metadata: ModelRunner::prepare_model_input and
// prepare_block_tables (nanovllm_rs/src/engine/model_runner.rs:53-160)
// for any step (prefill, decode, mixed, prefix-cache hits), into caller-owned
// buffers (pinned host memory, so one copy each takes them to the GPU).
// Integer bookkeeping only: the outputs are bit-exact with the reference's.
// nvkv_decode_advance covers pure decode steps on the device; this covers
// the rest, from the same nvkv_block_seq views the block manager updates.
#include <algorithm>

#include "common.cuh"

extern "C" {

int nvkv_prepare_step(const nvkv_block_seq* seqs, int64_t num_seqs, int64_t block_size,
                      int64_t* input_ids, int64_t* positions, uint32_t* cu_seqlens_q,
                      uint32_t* cu_seqlens_k, int64_t* slot_mapping, int64_t* context_lens,
                      int64_t* need_logits, uint32_t* block_tables, int64_t capacity_tokens,
                      int64_t capacity_slots, int64_t capacity_table, nvkv_step_sizes* sizes) {
  NVKV_RANGE("nvkv_prepare_step");
  using namespace nvkv;
  clear_error();
  if (!sizes || num_seqs < 0 || block_size <= 0 || (num_seqs > 0 && !seqs))
    return set_error(NVKV_ERR_INVALID_ARG, "prepare_step: bad arguments");
  // pass 1: sizes and validation (model_runner.rs:82-131 counts)
  nvkv_step_sizes z = {};
  int64_t sum_q = 0, sum_k = 0;
  for (int64_t b = 0; b < num_seqs; ++b) {
    const nvkv_block_seq& s = seqs[b];
    const int64_t ctx = s.num_cached_tokens + s.num_new_tokens;  // num_context_tokens
    if (s.num_cached_tokens < 0 || s.num_new_tokens < 0 || ctx > s.num_tokens ||
        s.block_table_len < 0 || (s.num_tokens > 0 && !s.token_ids) ||
        (s.block_table_len > 0 && !s.block_table))
      return set_error(NVKV_ERR_INVALID_ARG, "prepare_step: inconsistent sequence " +
                                                 std::to_string(b));
    z.num_tokens += s.num_new_tokens;
    z.max_seqlen_q = std::max<int64_t>(z.max_seqlen_q, s.num_new_tokens);
    z.max_seqlen_k = std::max<int64_t>(z.max_seqlen_k, ctx);
    z.block_table_width = std::max<int64_t>(z.block_table_width, s.block_table_len);
    sum_q += s.num_new_tokens;
    sum_k += ctx;
    if (s.num_tokens == ctx && s.block_table_len > 0) ++z.num_need_logits;
    if (s.block_table_len == 0) continue;  // warm-up: no slots (:103-106)
    const int64_t first = s.num_cached_tokens / block_size;
    for (int64_t i = first; i < s.block_table_len; ++i) {
      const int64_t page = s.block_table[i];
      const int64_t start = page * block_size + (i == first ? s.num_cached_tokens % block_size : 0);
      const int64_t end = (i == s.block_table_len - 1 && ctx % block_size != 0)
                              ? page * block_size + ctx % block_size
                              : (page + 1) * block_size;
      z.num_slots += std::max<int64_t>(end - start, 0);
    }
  }
  if (sum_q > 0xffffffffLL || sum_k > 0xffffffffLL)
    return set_error(NVKV_ERR_UNSUPPORTED, "prepare_step: cu_seqlens exceed uint32");
  z.has_block_tables = sum_k > sum_q ? 1 : 0;  // :127-131
  *sizes = z;
  if (!input_ids && !positions && !cu_seqlens_q && !cu_seqlens_k && !slot_mapping &&
      !context_lens && !need_logits && !block_tables)
    return NVKV_OK;  // a size query
  if (!cu_seqlens_q || !cu_seqlens_k || (num_seqs > 0 && !context_lens) ||
      (z.num_tokens > 0 && (!input_ids || !positions)) ||
      (z.num_need_logits > 0 && !need_logits) || (z.num_slots > 0 && !slot_mapping) ||
      (z.has_block_tables && z.block_table_width > 0 && !block_tables))
    return set_error(NVKV_ERR_INVALID_ARG, "prepare_step: null output buffer");
  if (capacity_tokens < z.num_tokens || capacity_slots < z.num_slots ||
      (z.has_block_tables && capacity_table < num_seqs * z.block_table_width))
    return set_error(NVKV_ERR_INVALID_ARG, "prepare_step: output buffers too small (sizes "
                                           "returned in *sizes)");
  // pass 2: fill (model_runner.rs:82-124, prepare_block_tables :53-67)
  int64_t t = 0, sl = 0, nl = 0;
  cu_seqlens_q[0] = 0;
  cu_seqlens_k[0] = 0;
  for (int64_t b = 0; b < num_seqs; ++b) {
    const nvkv_block_seq& s = seqs[b];
    const int64_t ctx = s.num_cached_tokens + s.num_new_tokens;
    if (s.num_tokens == ctx && s.block_table_len > 0) need_logits[nl++] = b;
    context_lens[b] = ctx;
    for (int64_t p = s.num_cached_tokens; p < ctx; ++p, ++t) {
      input_ids[t] = (int64_t)s.token_ids[p];
      positions[t] = p;
    }
    cu_seqlens_q[b + 1] = cu_seqlens_q[b] + (uint32_t)s.num_new_tokens;
    cu_seqlens_k[b + 1] = cu_seqlens_k[b] + (uint32_t)ctx;
    if (s.block_table_len == 0) continue;
    const int64_t first = s.num_cached_tokens / block_size;
    for (int64_t i = first; i < s.block_table_len; ++i) {
      const int64_t page = s.block_table[i];
      const int64_t start = page * block_size + (i == first ? s.num_cached_tokens % block_size : 0);
      const int64_t end = (i == s.block_table_len - 1 && ctx % block_size != 0)
                              ? page * block_size + ctx % block_size
                              : (page + 1) * block_size;
      for (int64_t v = start; v < end; ++v) slot_mapping[sl++] = v;
    }
  }
  if (z.has_block_tables) {
    const int64_t w = z.block_table_width;
    for (int64_t b = 0; b < num_seqs; ++b) {
      const nvkv_block_seq& s = seqs[b];
      uint32_t* row = block_tables + b * w;
      std::copy(s.block_table, s.block_table + s.block_table_len, row);
      std::fill(row + s.block_table_len, row + w, 0u);  // padding, never read (:60-62)
    }
  }
  return NVKV_OK;
}

}  // extern "C"
