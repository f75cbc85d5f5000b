// FP8 (e4m3) KV-cache format: the store that quantises K/V rows into the
// pool, and the attention entry point over such a pool.
//
// No counterpart in the reference: its KV pool is in the model dtype
// (nanovllm_rs/src/engine/model_runner.rs:286-303) and its store copies rows
// (layers/kv_cache.rs:13-37).  This is the optional "KV pool format" of the
// hot-path table's next row; bf16/f16 stays the default everywhere.
//
// Format.  k_cache / v_cache: [num_blocks, page, Hkv, 128] e4m3 codes (one
// byte each), the same page / slot addressing as the dtype pool.  Each
// (slot, kv head) row has its own f32 scale, laid out [num_blocks, Hkv, page]
// so a 64-row tile of one head reads 256 contiguous bytes of scales:
//   scale = amax / 448,  code = e4m3_rn_satfinite(x * (448 / amax)),
//   value = code * scale        (amax = max |x| of the row; 0 for a zero row)
// A row scale, not a page scale, because decode appends one row at a time:
// a page-wide scale fixed by its first rows would clip later ones.
//
// Attention.  Decode rows (q_len == 1) run on the decode kernel's fp8 form:
// half the K/V bytes from HBM, converted to the dtype in shared memory by two
// converter warps, the per-tile arithmetic unchanged.  Prompt rows (q_len >
// 1): their keys are dequantised into a contiguous dtype buffer in the
// workspace (one row per key, sequence by sequence), and the tcgen05 prefill
// kernel runs on it in its contiguous mode -- compute-bound work, for which
// the extra read and write of the keys is small.
#include "common.cuh"

namespace nvkv {
namespace {

constexpr int kF8Row = 128;  // head_dim

// e4m3 codes of (a, b) packed low byte = a (cvt.rn.satfinite: nearest, ties
// to even, magnitudes above 448 saturate).
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}

// One warp per (token, kv head, K|V) row of 128 values: lane l holds values
// 4l .. 4l + 3.
template <typename T>
__global__ void __launch_bounds__(256)
    store_kvcache_fp8_kernel(const T* __restrict__ key, const T* __restrict__ value,
                             uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                             float* __restrict__ k_scale, float* __restrict__ v_scale,
                             const int64_t* __restrict__ slots, int64_t num_tokens, int hkv,
                             int64_t key_stride, int64_t value_stride, int64_t num_slots,
                             int page, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t nrows = num_tokens * hkv * 2;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < nrows;
       w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int kv = (int)(w & 1);
    const int64_t th = w >> 1;
    const int h = (int)(th % hkv);
    const int64_t t = th / hkv;
    const int64_t slot = slots[t];
    if (slot < 0) continue;  // padding / warm-up rows (kv_cache.rs:19-20)
    if (slot >= num_slots) {
      if (lane == 0) record_error(err, NVKV_DEVERR_SLOT_RANGE);
      continue;
    }
    const T* src = (kv ? value + t * value_stride : key + t * key_stride) + h * kF8Row + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const float2 x01 = DT<T>::to_f2(raw.x), x23 = DT<T>::to_f2(raw.y);
    float amax = fmaxf(fmaxf(fabsf(x01.x), fabsf(x01.y)), fmaxf(fabsf(x23.x), fabsf(x23.y)));
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    const float inv = amax > 0.f ? __fdiv_rn(448.f, amax) : 0.f;
    const uint32_t codes = (uint32_t)f32x2_to_e4m3x2(__fmul_rn(x01.x, inv), __fmul_rn(x01.y, inv)) |
                           ((uint32_t)f32x2_to_e4m3x2(__fmul_rn(x23.x, inv),
                                                      __fmul_rn(x23.y, inv)) << 16);
    uint8_t* cache = kv ? v_cache : k_cache;
    *reinterpret_cast<uint32_t*>(cache + (slot * hkv + h) * kF8Row + lane * 4) = codes;
    if (lane == 0) {
      float* sc = kv ? v_scale : k_scale;
      sc[((slot / page) * hkv + h) * page + slot % page] = __fdiv_rn(amax, 448.f);
    }
  }
}

// Four e4m3 codes (lowest byte first) -> four floats (exact).
__device__ __forceinline__ void e4m3x4_to_f32_(uint32_t w, float* f) {
  uint32_t lo, hi;
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
  const float2 a = __half22float2(*reinterpret_cast<__half2*>(&lo));
  const float2 b = __half22float2(*reinterpret_cast<__half2*>(&hi));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

// Key offsets of the prompts' dequantised rows: cu_kd[b + 1] - cu_kd[b] =
// k_len of sequence b if it is a well-formed prompt (q_len > 1, q_len <= k_len
// <= max_k) whose rows fit the `capacity` rows after those of the prompts
// before it, else 0 (the prefill kernel then skips and reports it).  One CTA:
// a block scan per 1024 sequences, then the ends past the capacity are set to
// the last end within it.
__global__ void __launch_bounds__(1024)
    fp8_prompt_rows_kernel(const uint32_t* __restrict__ cu_q, const uint32_t* __restrict__ cu_k,
                           int num_seqs, int max_k, int64_t capacity, uint32_t* cu_kd, int* err) {
  __shared__ uint64_t warp_tot[32];
  __shared__ uint64_t carry;
  __shared__ uint32_t last_fit;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint64_t cap = (uint64_t)capacity;
  if (tid == 0) {
    carry = 0;
    last_fit = 0;
    cu_kd[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < num_seqs; base += 1024) {
    const int b = base + tid;
    uint64_t len = 0;
    if (b < num_seqs) {
      const int q_len = (int)(cu_q[b + 1] - cu_q[b]);
      const int k_len = (int)(cu_k[b + 1] - cu_k[b]);
      if (q_len > 1 && k_len >= q_len && k_len <= max_k) len = (uint64_t)k_len;
    }
    uint64_t incl = len;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint64_t v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const uint64_t v = warp_tot[lane];
      uint64_t s = v;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const uint64_t u = __shfl_up_sync(0xffffffffu, s, d);
        if (lane >= d) s += u;
      }
      warp_tot[lane] = s - v;  // exclusive prefix of the warp totals
    }
    __syncthreads();
    const uint64_t end = carry + warp_tot[warp] + incl;
    if (b < num_seqs) {
      cu_kd[b + 1] = (uint32_t)(end <= cap ? end : cap + 1);  // marked, fixed below
      if (end <= cap) atomicMax(&last_fit, (uint32_t)end);
      else if (len > 0) record_error(err, NVKV_DEVERR_SEQLEN);  // does not fit: no rows
    }
    __syncthreads();
    if (tid == 1023) carry = end;
    __syncthreads();
  }
  const uint32_t fit = last_fit;
  for (int b = tid; b < num_seqs; b += 1024)
    if ((uint64_t)cu_kd[b + 1] > cap) cu_kd[b + 1] = fit;
}

// Dequantises 64 keys of prompt b (blockIdx.x) from the paged fp8 pool into
// rows cu_kd[b] + j of kbuf / vbuf ([rows, Hkv, 128] in the dtype).
template <typename T>
__global__ void __launch_bounds__(256)
    fp8_dequant_prompt_kernel(const uint8_t* __restrict__ k_cache,
                              const uint8_t* __restrict__ v_cache,
                              const float* __restrict__ k_scale, const float* __restrict__ v_scale,
                              const uint32_t* __restrict__ cu_kd,
                              const uint32_t* __restrict__ block_tables, int64_t bt_stride,
                              int64_t num_blocks, int page, int hkv, T* kbuf, T* vbuf, int* err) {
  const int b = blockIdx.x;
  const int j0 = blockIdx.y * 64;
  const uint32_t ks = cu_kd[b];
  const int len = (int)(cu_kd[b + 1] - ks);
  if (j0 >= len) return;
  const int n = min(64, len - j0);
  const int chunks = hkv * 8;  // 16-byte code chunks per row
  for (int i = threadIdx.x; i < n * chunks * 2; i += blockDim.x) {
    const int kv = i & 1;
    const int rest = i >> 1;
    const int j = j0 + rest / chunks;
    const int hc = rest % chunks, h = hc >> 3, c = hc & 7;
    uint32_t pg = block_tables[(int64_t)b * bt_stride + j / page];
    if ((int64_t)pg >= num_blocks) {
      record_error(err, NVKV_DEVERR_BLOCK_RANGE);
      pg = 0;
    }
    const int64_t slot = (int64_t)pg * page + j % page;
    const uint8_t* src = (kv ? v_cache : k_cache) + (slot * hkv + h) * kF8Row + c * 16;
    const float sc = (kv ? v_scale : k_scale)[((int64_t)pg * hkv + h) * page + j % page];
    const uint4 w = *reinterpret_cast<const uint4*>(src);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float f[4];
      e4m3x4_to_f32_(ws[k], f);
      o[2 * k] = DT<T>::from_f2(__fmul_rn(f[0], sc), __fmul_rn(f[1], sc));
      o[2 * k + 1] = DT<T>::from_f2(__fmul_rn(f[2], sc), __fmul_rn(f[3], sc));
    }
    T* dst = (kv ? vbuf : kbuf) + ((int64_t)(ks + j) * hkv + h) * kF8Row + c * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(dst + 8) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// fp8 workspace: the attention workspace (split-KV scratch, prefill plan),
// then cu_kd [num_seqs + 1], then the prompts' dequantised K and V rows.
struct F8Layout {
  size_t base, cu_kd, kbuf, vbuf, total;
};
F8Layout f8_layout(int num_seqs, int hq, int hkv, int max_q, int max_k, int64_t prompt_rows) {
  F8Layout L;
  L.base = attention_workspace_bytes(num_seqs, hq, hkv, max_q, max_k, true);
  if (max_q <= 1 || num_seqs <= 0) {
    L.cu_kd = L.kbuf = L.vbuf = L.total = L.base;
    return L;
  }
  L.cu_kd = align256(L.base);
  L.kbuf = align256(L.cu_kd + ((size_t)num_seqs + 1) * 4);
  const size_t rows = (size_t)prompt_rows * hkv * kF8Row * 2;
  L.vbuf = align256(L.kbuf + rows);
  L.total = L.vbuf + rows;
  return L;
}

}  // namespace
}  // namespace nvkv

extern "C" int nvkv_store_kvcache_fp8(const void* key, const void* value, void* k_cache,
                                      void* v_cache, float* k_scale, float* v_scale,
                                      const int64_t* slot_mapping, int64_t num_tokens,
                                      int num_kv_heads, int head_dim, int64_t key_stride,
                                      int64_t value_stride, int64_t num_blocks, int page_size,
                                      int dtype, nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_store_kvcache_fp8");
  using namespace nvkv;
  clear_error();
  if (dtype != NVKV_DTYPE_BF16 && dtype != NVKV_DTYPE_F16)
    return set_error(NVKV_ERR_UNSUPPORTED, "store_kvcache_fp8: source dtype must be bf16/f16");
  if (head_dim != kF8Row) return set_error(NVKV_ERR_UNSUPPORTED, "store_kvcache_fp8: head_dim 128");
  if (num_tokens < 0 || num_kv_heads <= 0 || num_blocks <= 0 || page_size <= 0)
    return set_error(NVKV_ERR_INVALID_ARG, "store_kvcache_fp8: bad sizes");
  if (num_tokens == 0) return NVKV_OK;
  if (!key || !value || !k_cache || !v_cache || !k_scale || !v_scale || !slot_mapping)
    return set_error(NVKV_ERR_INVALID_ARG, "store_kvcache_fp8: null pointer");
  if (key_stride < (int64_t)num_kv_heads * kF8Row || value_stride < (int64_t)num_kv_heads * kF8Row ||
      key_stride % 4 || value_stride % 4 || (reinterpret_cast<uintptr_t>(key) & 7) ||
      (reinterpret_cast<uintptr_t>(value) & 7) || !aligned16(k_cache) || !aligned16(v_cache))
    return set_error(NVKV_ERR_ALIGNMENT,
                     "store_kvcache_fp8: rows must be 8-byte aligned, caches 16-byte aligned");
  const int64_t rows = num_tokens * num_kv_heads * 2;
  const int64_t blocks = std::min<int64_t>((rows + 7) / 8, 148 * 16);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t num_slots = num_blocks * page_size;
  if (dtype == NVKV_DTYPE_BF16)
    store_kvcache_fp8_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(key), static_cast<const __nv_bfloat16*>(value),
        static_cast<uint8_t*>(k_cache), static_cast<uint8_t*>(v_cache), k_scale, v_scale,
        slot_mapping, num_tokens, num_kv_heads, key_stride, value_stride, num_slots, page_size,
        device_error_word());
  else
    store_kvcache_fp8_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(
        static_cast<const __half*>(key), static_cast<const __half*>(value),
        static_cast<uint8_t*>(k_cache), static_cast<uint8_t*>(v_cache), k_scale, v_scale,
        slot_mapping, num_tokens, num_kv_heads, key_stride, value_stride, num_slots, page_size,
        device_error_word());
  return check_cuda(cudaGetLastError(), "store_kvcache_fp8 launch");
}

extern "C" int nvkv_paged_attention_fp8_workspace_size(int num_seqs, int num_q_heads,
                                                       int num_kv_heads, int head_dim,
                                                       int max_seqlen_q, int max_seqlen_k,
                                                       int64_t prompt_kv_tokens, size_t* bytes) {
  using namespace nvkv;
  clear_error();
  if (!bytes) return set_error(NVKV_ERR_INVALID_ARG, "fp8 workspace_size: null output");
  int rc = validate_shapes(num_seqs, max_seqlen_q, max_seqlen_k, num_q_heads, num_kv_heads,
                           head_dim);
  if (rc) return rc;
  if (prompt_kv_tokens < 0)
    return set_error(NVKV_ERR_INVALID_ARG, "fp8 workspace_size: negative prompt_kv_tokens");
  *bytes = f8_layout(num_seqs, num_q_heads, num_kv_heads, max_seqlen_q, max_seqlen_k,
                     prompt_kv_tokens)
               .total;
  return NVKV_OK;
}

extern "C" int nvkv_paged_attention_fp8(
    const void* q, int64_t q_stride, int64_t num_q_tokens, const void* k_cache,
    const void* v_cache, const float* k_scale, const float* v_scale, int64_t num_blocks, void* out,
    const uint32_t* cu_seqlens_q, const uint32_t* cu_seqlens_k, const uint32_t* block_tables,
    int64_t block_table_stride, int num_seqs, int max_seqlen_q, int max_seqlen_k,
    int num_q_heads, int num_kv_heads, int head_dim, int page_size, float softmax_scale,
    int causal, int64_t prompt_kv_tokens, void* workspace, size_t workspace_bytes, int dtype,
    nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_paged_attention_fp8");
  using namespace nvkv;
  clear_error();
  if (dtype != NVKV_DTYPE_BF16 && dtype != NVKV_DTYPE_F16)
    return set_error(NVKV_ERR_UNSUPPORTED, "paged_attention_fp8: q/out dtype must be bf16/f16");
  int rc = validate_shapes(num_seqs, max_seqlen_q, max_seqlen_k, num_q_heads, num_kv_heads,
                           head_dim);
  if (rc) return rc;
  if (num_seqs == 0 || max_seqlen_q == 0 || num_q_tokens == 0) return NVKV_OK;
  if (num_q_tokens < 0 || num_q_tokens > 0x7fffffffLL || prompt_kv_tokens < 0 ||
      prompt_kv_tokens > 0x7fffffffLL)
    return set_error(NVKV_ERR_INVALID_ARG, "paged_attention_fp8: bad num_q_tokens / prompt rows");
  if (!q || !k_cache || !v_cache || !k_scale || !v_scale || !out || !cu_seqlens_q ||
      !cu_seqlens_k || !block_tables)
    return set_error(NVKV_ERR_INVALID_ARG,
                     "paged_attention_fp8: null pointer (the fp8 pool is paged: block_tables)");
  if (num_blocks <= 0 || page_size <= 0 || page_size % 128 != 0)
    return set_error(NVKV_ERR_UNSUPPORTED,
                     "paged_attention_fp8: page_size must be a positive multiple of 128");
  if (block_table_stride < (max_seqlen_k + page_size - 1) / page_size)
    return set_error(NVKV_ERR_INVALID_ARG,
                     "paged_attention_fp8: block_table_stride < blocks needed by max_seqlen_k");
  if (num_blocks * (int64_t)page_size > 0x7fffffffLL)
    return set_error(NVKV_ERR_UNSUPPORTED, "paged_attention_fp8: more than 2^31 cache rows");
  if (q_stride < (int64_t)num_q_heads * head_dim || (q_stride * 2) % 16 != 0 || !aligned16(q) ||
      !aligned16(out) || !aligned16(k_cache) || !aligned16(v_cache) ||
      !aligned16(k_scale) || !aligned16(v_scale))
    return set_error(NVKV_ERR_ALIGNMENT, "paged_attention_fp8: misaligned buffer or stride");
  if (!(softmax_scale > 0.f))
    return set_error(NVKV_ERR_INVALID_ARG, "paged_attention_fp8: softmax_scale must be > 0");
  const F8Layout L = f8_layout(num_seqs, num_q_heads, num_kv_heads, max_seqlen_q, max_seqlen_k,
                               prompt_kv_tokens);
  if (L.total > 0 && (!workspace || workspace_bytes < L.total || !aligned16(workspace)))
    return set_error(NVKV_ERR_WORKSPACE, "paged_attention_fp8: workspace missing or too small "
                                         "(need " + std::to_string(L.total) + " bytes)");
  AttnArgs a;
  a.q = q;
  a.q_stride = q_stride;
  a.num_q_rows = num_q_tokens;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.num_blocks = num_blocks;
  a.kv_stride = (int64_t)num_kv_heads * head_dim;  // one byte per code
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
  a.stream = reinterpret_cast<cudaStream_t>(stream);
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.fp8_layout = true;
  if (max_seqlen_q > 1 && prompt_kv_tokens == 0)
    return set_error(NVKV_ERR_INVALID_ARG,
                     "paged_attention_fp8: max_seqlen_q > 1 needs prompt_kv_tokens >= the "
                     "prompts' total k_len");
  rc = launch_paged_decode(a);  // q_len == 1 rows, straight from the fp8 pool
  if (rc || max_seqlen_q <= 1) return rc;
  // q_len > 1 rows: dequantise the prompts' keys, then the contiguous prefill
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* cu_kd = reinterpret_cast<uint32_t*>(ws + L.cu_kd);
  int* err = device_error_word();
  fp8_prompt_rows_kernel<<<1, 1024, 0, a.stream>>>(cu_seqlens_q, cu_seqlens_k, num_seqs,
                                                    max_seqlen_k, prompt_kv_tokens, cu_kd, err);
  rc = check_cuda(cudaGetLastError(), "fp8 prompt rows launch");
  if (rc) return rc;
  const dim3 grid((unsigned)num_seqs, (unsigned)((max_seqlen_k + 63) / 64));
  if (dtype == NVKV_DTYPE_BF16)
    fp8_dequant_prompt_kernel<__nv_bfloat16><<<grid, 256, 0, a.stream>>>(
        static_cast<const uint8_t*>(k_cache), static_cast<const uint8_t*>(v_cache), k_scale,
        v_scale, cu_kd, block_tables, block_table_stride, num_blocks, page_size, num_kv_heads,
        reinterpret_cast<__nv_bfloat16*>(ws + L.kbuf), reinterpret_cast<__nv_bfloat16*>(ws + L.vbuf),
        err);
  else
    fp8_dequant_prompt_kernel<__half><<<grid, 256, 0, a.stream>>>(
        static_cast<const uint8_t*>(k_cache), static_cast<const uint8_t*>(v_cache), k_scale,
        v_scale, cu_kd, block_tables, block_table_stride, num_blocks, page_size, num_kv_heads,
        reinterpret_cast<__half*>(ws + L.kbuf), reinterpret_cast<__half*>(ws + L.vbuf), err);
  rc = check_cuda(cudaGetLastError(), "fp8 dequant launch");
  if (rc) return rc;
  AttnArgs c = a;  // the contiguous route over the dequantised rows
  c.k_cache = ws + L.kbuf;
  c.v_cache = ws + L.vbuf;
  c.k_scale = c.v_scale = nullptr;
  c.block_tables = nullptr;
  c.bt_stride = 0;
  c.num_blocks = prompt_kv_tokens;
  c.kv_stride = (int64_t)num_kv_heads * head_dim;
  c.cu_k = cu_kd;
  return launch_paged_prefill(c);
}
