// C-ABI attention entry points and the host-side mirror of the reference's
// operator surface (Context side channel + Attention object).
//
// nvkv_paged_attention validates everything on the host, then launches the
// split-KV decode kernel for q_len == 1 sequences and the tcgen05 prefill
// kernel for the rest (each kernel skips the other's sequences on the device,
// so no host synchronisation is needed to split a mixed batch).
#include <new>

#include "common.cuh"

namespace nvkv {

int validate_shapes(int num_seqs, int max_q, int max_k, int hq, int hkv, int d) {
  if (num_seqs < 0 || max_q < 0 || max_k < 0)
    return set_error(NVKV_ERR_INVALID_ARG, "paged_attention: negative size");
  if (d != 128) return set_error(NVKV_ERR_UNSUPPORTED, "paged_attention: head_dim must be 128");
  if (hq <= 0 || hkv <= 0 || hq % hkv != 0)
    return set_error(NVKV_ERR_INVALID_ARG,
                     "paged_attention: num_q_heads must be a positive multiple of num_kv_heads");
  if (hq / hkv > 16)
    return set_error(NVKV_ERR_UNSUPPORTED, "paged_attention: GQA group (Hq/Hkv) above 16");
  if (num_seqs > 65535) return set_error(NVKV_ERR_UNSUPPORTED, "paged_attention: > 65535 seqs");
  return NVKV_OK;
}

// Split-KV decode scratch, then (for max_seqlen_q > 1) the prefill work plan.
size_t attention_workspace_bytes(int num_seqs, int hq, int hkv, int max_q, int max_k, bool fp8) {
  if (num_seqs <= 0) return 0;
  const size_t dec = decode_workspace_bytes(num_seqs, hq, hkv, max_k, fp8);
  const size_t plan = prefill_plan_bytes(num_seqs, max_q);
  return plan ? attention_plan_offset(dec) + plan : dec;
}

static int run_attention(const AttnArgs& a) {
  int rc = launch_paged_decode(a);
  if (rc) return rc;
  if (a.max_q > 1) rc = launch_paged_prefill(a);
  return rc;
}

// ---------------------------------------------------------------------------
// Host mirror: Context (utils/context.rs:4-54)
// ---------------------------------------------------------------------------
struct Context {
  bool set = false;
  const uint32_t* cu_seqlens_q = nullptr;
  const uint32_t* cu_seqlens_k = nullptr;
  int num_seqs = 0;
  int max_seqlen_q = 0;
  int max_seqlen_k = 0;
  const int64_t* slot_mapping = nullptr;
  int64_t num_slot_entries = 0;
  const int64_t* context_lens = nullptr;
  const uint32_t* block_tables = nullptr;
  int64_t block_table_stride = 0;
};

// Thread-local like the reference: each tensor-parallel rank drives its own
// device from its own thread (utils/context.rs:16-21).
thread_local Context g_ctx;

}  // namespace nvkv

// Attention (layers/attention.rs:7-21): scale + this layer's KV cache.
struct nvkv_attention {
  float scale = 1.f;
  void* k_cache = nullptr;
  void* v_cache = nullptr;
  int64_t num_blocks = 0;
  int page_size = 0;
  int num_kv_heads = 0;
  int head_dim = 0;
  int dtype = NVKV_DTYPE_BF16;
  // split-KV scratch owned by the layer, grown on demand
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int ws_device = -1;
};

namespace nvkv {
static int ensure_workspace(nvkv_attention* attn, size_t need) {
  if (need <= attn->ws_bytes) return NVKV_OK;
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "attention_forward: cudaGetDevice");
  if (rc) return rc;
  if (attn->ws) cudaFree(attn->ws);
  attn->ws = nullptr;
  attn->ws_bytes = 0;
  rc = check_cuda(cudaMalloc(&attn->ws, need), "attention_forward: workspace alloc");
  if (rc) return rc;
  attn->ws_bytes = need;
  attn->ws_device = dev;
  return NVKV_OK;
}
}  // namespace nvkv

extern "C" {

int nvkv_paged_attention_workspace_size(int num_seqs, int num_q_heads, int num_kv_heads,
                                        int head_dim, int max_seqlen_q, int max_seqlen_k,
                                        size_t* bytes) {
  using namespace nvkv;
  clear_error();
  if (!bytes) return set_error(NVKV_ERR_INVALID_ARG, "workspace_size: null output");
  int rc = validate_shapes(num_seqs, max_seqlen_q, max_seqlen_k, num_q_heads, num_kv_heads,
                           head_dim);
  if (rc) return rc;
  *bytes = attention_workspace_bytes(num_seqs, num_q_heads, num_kv_heads, max_seqlen_q,
                                     max_seqlen_k);
  return NVKV_OK;
}

int nvkv_paged_attention(const void* q, int64_t q_stride, int64_t num_q_tokens,
                         const void* k_cache, const void* v_cache, int64_t num_blocks,
                         int64_t kv_stride, void* out, const uint32_t* cu_seqlens_q,
                         const uint32_t* cu_seqlens_k, const uint32_t* block_tables,
                         int64_t block_table_stride, int num_seqs, int max_seqlen_q,
                         int max_seqlen_k, int num_q_heads, int num_kv_heads, int head_dim,
                         int page_size, float softmax_scale, int causal, void* workspace,
                         size_t workspace_bytes, int dtype, nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_paged_attention");
  using namespace nvkv;
  clear_error();
  if (dtype != NVKV_DTYPE_BF16 && dtype != NVKV_DTYPE_F16)
    return set_error(NVKV_ERR_UNSUPPORTED, "paged_attention: unsupported dtype (bf16/f16 only)");
  int rc = validate_shapes(num_seqs, max_seqlen_q, max_seqlen_k, num_q_heads, num_kv_heads,
                           head_dim);
  if (rc) return rc;
  if (num_seqs == 0 || max_seqlen_q == 0 || num_q_tokens == 0) return NVKV_OK;
  if (num_q_tokens < 0 || num_q_tokens > 0x7fffffffLL)
    return set_error(NVKV_ERR_INVALID_ARG, "paged_attention: bad num_q_tokens");
  if (!q || !k_cache || !v_cache || !out || !cu_seqlens_q || !cu_seqlens_k)
    return set_error(NVKV_ERR_INVALID_ARG, "paged_attention: null pointer");
  if (num_blocks <= 0) return set_error(NVKV_ERR_INVALID_ARG, "paged_attention: num_blocks <= 0");
  if (kv_stride == 0) kv_stride = (int64_t)num_kv_heads * head_dim;
  if (kv_stride < (int64_t)num_kv_heads * head_dim || kv_stride % 8 != 0)
    return set_error(NVKV_ERR_INVALID_ARG,
                     "paged_attention: kv_stride must be >= Hkv*D and a multiple of 8");
  if (block_tables) {
    if (page_size <= 0 || page_size % 128 != 0)
      return set_error(NVKV_ERR_UNSUPPORTED,
                       "paged_attention: page_size must be a positive multiple of 128");
    if (block_table_stride < (max_seqlen_k + page_size - 1) / page_size)
      return set_error(NVKV_ERR_INVALID_ARG,
                       "paged_attention: block_table_stride < blocks needed by max_seqlen_k");
    if (num_blocks * (int64_t)page_size > 0x7fffffffLL)
      return set_error(NVKV_ERR_UNSUPPORTED, "paged_attention: more than 2^31 cache rows");
  } else if (num_blocks > 0x7fffffffLL) {
    return set_error(NVKV_ERR_UNSUPPORTED, "paged_attention: more than 2^31 K/V rows");
  }
  if (q_stride < (int64_t)num_q_heads * head_dim)
    return set_error(NVKV_ERR_INVALID_ARG, "paged_attention: q_stride smaller than a row");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out) ||
      (q_stride * 2) % 16 != 0)
    return set_error(NVKV_ERR_ALIGNMENT,
                     "paged_attention: q/k_cache/v_cache/out and q_stride must be 16-byte aligned");
  if (!(softmax_scale > 0.f))
    return set_error(NVKV_ERR_INVALID_ARG, "paged_attention: softmax_scale must be > 0");
  const size_t need =
      attention_workspace_bytes(num_seqs, num_q_heads, num_kv_heads, max_seqlen_q, max_seqlen_k);
  if (need > 0 && (!workspace || workspace_bytes < need || !aligned16(workspace)))
    return set_error(NVKV_ERR_WORKSPACE, "paged_attention: workspace missing or too small (need " +
                                             std::to_string(need) + " bytes)");
  AttnArgs a;
  a.q = q;
  a.q_stride = q_stride;
  a.num_q_rows = num_q_tokens;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.num_blocks = num_blocks;
  a.kv_stride = kv_stride;
  a.out = out;
  a.cu_q = cu_seqlens_q;
  a.cu_k = cu_seqlens_k;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.num_seqs = num_seqs;
  a.max_q = max_seqlen_q;
  a.max_k = max_seqlen_k;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.d = head_dim;
  a.page = page_size;
  a.scale = softmax_scale;
  a.causal = causal ? 1 : 0;
  a.ws = workspace;
  a.ws_bytes = workspace_bytes;
  a.dtype = dtype;
  a.stream = (cudaStream_t)stream;
  return run_attention(a);
}

int nvkv_context_set(const uint32_t* cu_seqlens_q, const uint32_t* cu_seqlens_k, int num_seqs,
                     int max_seqlen_q, int max_seqlen_k, const int64_t* slot_mapping,
                     int64_t num_slot_entries, const int64_t* context_lens,
                     const uint32_t* block_tables, int64_t block_table_stride) {
  using namespace nvkv;
  clear_error();
  if (!cu_seqlens_q || !cu_seqlens_k || num_seqs < 0)
    return set_error(NVKV_ERR_INVALID_ARG, "context_set: cu_seqlens_q/k must be set");
  Context c;
  c.set = true;
  c.cu_seqlens_q = cu_seqlens_q;
  c.cu_seqlens_k = cu_seqlens_k;
  c.num_seqs = num_seqs;
  c.max_seqlen_q = max_seqlen_q;
  c.max_seqlen_k = max_seqlen_k;
  c.slot_mapping = slot_mapping;
  c.num_slot_entries = num_slot_entries;
  c.context_lens = context_lens;
  c.block_tables = block_tables;
  c.block_table_stride = block_table_stride;
  g_ctx = c;
  return NVKV_OK;
}

int nvkv_context_reset(void) {
  nvkv::g_ctx = nvkv::Context();
  return NVKV_OK;
}

int nvkv_attention_create(float scale, nvkv_attention_t* out) {
  using namespace nvkv;
  clear_error();
  if (!out) return set_error(NVKV_ERR_INVALID_ARG, "attention_create: null output");
  *out = new (std::nothrow) nvkv_attention();
  if (!*out) return set_error(NVKV_ERR_INVALID_ARG, "attention_create: out of host memory");
  (*out)->scale = scale;
  return NVKV_OK;
}

int nvkv_attention_destroy(nvkv_attention_t attn) {
  if (!attn) return NVKV_OK;
  if (attn->ws) {
    int prev = -1;
    cudaGetDevice(&prev);
    if (attn->ws_device >= 0) cudaSetDevice(attn->ws_device);
    cudaFree(attn->ws);
    if (prev >= 0) cudaSetDevice(prev);
  }
  delete attn;
  return NVKV_OK;
}

int nvkv_attention_set_kv_cache(nvkv_attention_t attn, void* k_cache, void* v_cache,
                                int64_t num_blocks, int page_size, int num_kv_heads,
                                int head_dim, int dtype) {
  using namespace nvkv;
  clear_error();
  if (!attn || !k_cache || !v_cache || num_blocks <= 0 || page_size <= 0 || num_kv_heads <= 0)
    return set_error(NVKV_ERR_INVALID_ARG, "set_kv_cache: bad arguments");
  if (head_dim != 128) return set_error(NVKV_ERR_UNSUPPORTED, "set_kv_cache: head_dim must be 128");
  attn->k_cache = k_cache;
  attn->v_cache = v_cache;
  attn->num_blocks = num_blocks;
  attn->page_size = page_size;
  attn->num_kv_heads = num_kv_heads;
  attn->head_dim = head_dim;
  attn->dtype = dtype;
  return NVKV_OK;
}

int nvkv_attention_forward(nvkv_attention_t attn, const void* q, int64_t q_stride, const void* k,
                           int64_t k_stride, const void* v, int64_t v_stride,
                           int64_t num_tokens, int num_q_heads, int num_kv_heads, void* out,
                           int dtype, nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_attention_forward");
  using namespace nvkv;
  clear_error();
  if (!attn) return set_error(NVKV_ERR_INVALID_ARG, "attention_forward: null attention");
  const Context& c = g_ctx;
  // get_context().cu_seqlens_q.expect(...) (attention.rs:25-27)
  if (!c.set) return set_error(NVKV_ERR_INVALID_ARG, "attention_forward: cu_seqlens_q must be set");
  const bool has_cache = attn->k_cache && attn->v_cache;
  const int head_dim = 128;
  if (has_cache) {
    // store_kv_cache (attention.rs:29-35, kv_cache.rs:168-190)
    if (!c.slot_mapping)
      return set_error(NVKV_ERR_INVALID_ARG,
                       "attention_forward: slot_mapping must be set when a kv cache is present");
    if (attn->dtype != dtype)
      return set_error(NVKV_ERR_INVALID_ARG, "attention_forward: cache dtype mismatch");
    if (attn->num_kv_heads != num_kv_heads)
      return set_error(NVKV_ERR_INVALID_ARG, "attention_forward: kv head count != cache's");
    if (c.num_slot_entries != num_tokens)
      return set_error(NVKV_ERR_INVALID_ARG,
                       "attention_forward: slot_mapping length differs from the token count");
    if (num_tokens > 0) {
      if (!k || !v) return set_error(NVKV_ERR_INVALID_ARG, "attention_forward: null k/v");
      if (num_tokens > 1 && (k_stride < (int64_t)num_kv_heads * head_dim ||
                             v_stride < (int64_t)num_kv_heads * head_dim))
        return set_error(NVKV_ERR_INVALID_ARG, "attention_forward: k/v stride below a row");
      int rc = launch_store_kvcache(k, v, attn->k_cache, attn->v_cache, c.slot_mapping,
                                    num_tokens, (int64_t)num_kv_heads * head_dim, k_stride,
                                    v_stride, attn->num_blocks * attn->page_size,
                                    (cudaStream_t)stream);
      if (rc) return rc;
    }
  }
  size_t need = 0;
  int rc = nvkv_paged_attention_workspace_size(c.num_seqs, num_q_heads, num_kv_heads, head_dim,
                                               c.max_seqlen_q, c.max_seqlen_k, &need);
  if (rc) return rc;
  rc = ensure_workspace(attn, need);
  if (rc) return rc;
  if (c.block_tables) {
    // flash_attn_varlen_paged_windowed over the cache (attention.rs:38-59)
    if (!has_cache)
      return set_error(NVKV_ERR_INVALID_ARG,
                       "attention_forward: kv cache must be set for prefix caching");
    return nvkv_paged_attention(q, q_stride, num_tokens, attn->k_cache, attn->v_cache,
                                attn->num_blocks, 0, out, c.cu_seqlens_q, c.cu_seqlens_k,
                                c.block_tables, c.block_table_stride, c.num_seqs, c.max_seqlen_q,
                                c.max_seqlen_k, num_q_heads, num_kv_heads, head_dim,
                                attn->page_size, attn->scale, 1, attn->ws, attn->ws_bytes, dtype,
                                stream);
  }
  // flash_attn_varlen on the fresh K/V (attention.rs:60-74), read in place.
  if (!k || !v) return set_error(NVKV_ERR_INVALID_ARG, "attention_forward: null k/v");
  if (k_stride != v_stride)
    return set_error(NVKV_ERR_INVALID_ARG, "attention_forward: k and v strides must match");
  return nvkv_paged_attention(q, q_stride, num_tokens, k, v, num_tokens, k_stride, out,
                              c.cu_seqlens_q, c.cu_seqlens_k, nullptr, 0, c.num_seqs,
                              c.max_seqlen_q, c.max_seqlen_k, num_q_heads, num_kv_heads,
                              head_dim, 0, attn->scale, 1, attn->ws, attn->ws_bytes, dtype,
                              stream);
}

}  // extern "C"
