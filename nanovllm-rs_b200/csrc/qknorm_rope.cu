// Kernel 4: fused qk-RMSNorm + RoPE prologue (nvkv_qknorm_rope), optionally
// fused with the KV-cache scatter of kernel 1.
//
// Replaces the ~20 small candle launches per layer of
// nanovllm_rs/src/models/qwen3.rs:128-141 (split_qkv, q_norm/k_norm of
// layers/layernorm.rs:18-25, RotaryEmbedding::forward of
// layers/rotary_embedding.rs:11-26,59-70) and the two store launches of
// layers/kv_cache.rs:187-188 with ONE pass over the fused qkv buffer.
//
// Arithmetic follows the reference's rounding points exactly: the norm is
// f32 (mean of squares, rsqrt via sqrt then reciprocal), rounded to the
// activation dtype, multiplied by the weight and rounded again; cos/sin are
// f32 (inv_freq = 1/exp((2i/D)*ln theta), freq = pos*inv_freq) rounded to the
// activation dtype, and every product / sum of the rotation is rounded to the
// activation dtype.  Computing in f32 then rounding once reproduces a native
// bf16/f16 op because the operands are dtype values (products are exact in
// f32; sums round at most below half a dtype ulp).
//
// Layout: one CTA per token, 8 warps.  cos/sin for the token's 64 frequency
// pairs are computed once into shared memory; each warp then owns whole head
// rows (128 elements): lane l holds elements {2l, 2l+1} and {64+2l, 64+2l+1},
// so both halves of each rotation pair sit in the same lane and every warp
// load/store covers 128 contiguous bytes.
#include "common.cuh"

namespace nvkv {

constexpr int kRopeD = 128;

template <typename T>
__global__ void __launch_bounds__(256) qknorm_rope_kernel(
    const T* __restrict__ qkv, int64_t qkv_stride, int num_q_heads, int num_kv_heads,
    const int64_t* __restrict__ positions, const T* __restrict__ q_w, const T* __restrict__ k_w,
    float eps, float ln_theta, int64_t max_position, T* __restrict__ q_out,
    T* __restrict__ k_out, T* __restrict__ v_out, T* __restrict__ k_cache,
    T* __restrict__ v_cache, const int64_t* __restrict__ slot_mapping, int64_t num_slots,
    int* err) {
  __shared__ float s_cos[kRopeD / 2];
  __shared__ float s_sin[kRopeD / 2];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;

  const int64_t pos = positions[t];
  // the warp's first kPre rows are loaded before the RoPE table is built, so
  // their latency overlaps the trigonometry and the barrier (8B TP1 layer,
  // 256 tokens: 5.29 -> 5.03 us)
  constexpr int kPre = 12;
  const int i0 = 2 * lane;  // this lane's two rotation pairs: i0, i0+1
  const int rows = num_q_heads + 2 * num_kv_heads;
  const T* src_tok = qkv + t * qkv_stride;
  uint32_t pa[kPre], pb[kPre];
#pragma unroll
  for (int k = 0; k < kPre; ++k) {
    const int r = warp + 8 * k;
    if (r < rows) {
      pa[k] = *reinterpret_cast<const uint32_t*>(src_tok + (int64_t)r * kRopeD + i0);
      pb[k] = *reinterpret_cast<const uint32_t*>(src_tok + (int64_t)r * kRopeD + 64 + i0);
    }
  }
  const bool do_norm = (q_w != nullptr);
  float wq[4], wk[4];
  if (do_norm) {
    float2 a = DT<T>::to_f2(*reinterpret_cast<const uint32_t*>(q_w + i0));
    float2 b = DT<T>::to_f2(*reinterpret_cast<const uint32_t*>(q_w + 64 + i0));
    wq[0] = a.x; wq[1] = a.y; wq[2] = b.x; wq[3] = b.y;
    a = DT<T>::to_f2(*reinterpret_cast<const uint32_t*>(k_w + i0));
    b = DT<T>::to_f2(*reinterpret_cast<const uint32_t*>(k_w + 64 + i0));
    wk[0] = a.x; wk[1] = a.y; wk[2] = b.x; wk[3] = b.y;
  }
  if (tid < kRopeD / 2) {
    if (tid == 0 && (pos < 0 || pos >= max_position)) record_error(err, NVKV_DEVERR_POSITION_RANGE);
    // rotary_embedding.rs:31-49 in f32, then the cast of :60
    const float expo = (float)(2 * tid) * (1.0f / (float)kRopeD);
    const float inv = 1.0f / expf(expo * ln_theta);
    const float f = (float)pos * inv;
    s_cos[tid] = rnd<T>(cosf(f));
    s_sin[tid] = rnd<T>(sinf(f));
  }
  int64_t slot = -1;
  if (slot_mapping) {
    slot = slot_mapping[t];
    if (slot >= num_slots) {
      if (tid == 0) record_error(err, NVKV_DEVERR_SLOT_RANGE);
      slot = -1;
    }
  }
  __syncthreads();

  const float c0 = s_cos[i0], c1 = s_cos[i0 + 1];
  const float sn0 = s_sin[i0], sn1 = s_sin[i0 + 1];
  const int64_t kv_row = (int64_t)num_kv_heads * kRopeD;
  auto row_out = [&](int r, uint32_t ua, uint32_t ub) {
    if (r >= num_q_heads + num_kv_heads) {  // V head: plain copy
      const int h = r - num_q_heads - num_kv_heads;
      if (v_out) {
        T* d = v_out + t * kv_row + (int64_t)h * kRopeD;
        *reinterpret_cast<uint32_t*>(d + i0) = ua;
        *reinterpret_cast<uint32_t*>(d + 64 + i0) = ub;
      }
      if (slot >= 0 && v_cache) {
        T* d = v_cache + slot * kv_row + (int64_t)h * kRopeD;
        *reinterpret_cast<uint32_t*>(d + i0) = ua;
        *reinterpret_cast<uint32_t*>(d + 64 + i0) = ub;
      }
      return;
    }
    const bool is_q = r < num_q_heads;
    const float2 fa = DT<T>::to_f2(ua), fb = DT<T>::to_f2(ub);
    float x1a = fa.x, x1b = fa.y, x2a = fb.x, x2b = fb.y;  // x1 = first half, x2 = second
    if (do_norm) {
      // x.sqr() rounds each square to f32, then the row is summed
      float ss = __fadd_rn(__fadd_rn(__fmul_rn(x1a, x1a), __fmul_rn(x1b, x1b)),
                           __fadd_rn(__fmul_rn(x2a, x2a), __fmul_rn(x2b, x2b)));
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
      const float var = ss * (1.0f / (float)kRopeD);
      const float inv = 1.0f / sqrtf(var + eps);
      x1a = rnd<T>(rnd<T>(x1a * inv) * (is_q ? wq[0] : wk[0]));
      x1b = rnd<T>(rnd<T>(x1b * inv) * (is_q ? wq[1] : wk[1]));
      x2a = rnd<T>(rnd<T>(x2a * inv) * (is_q ? wq[2] : wk[2]));
      x2b = rnd<T>(rnd<T>(x2b * inv) * (is_q ? wq[3] : wk[3]));
    }
    // y1 = x1*cos - x2*sin ; y2 = x2*cos + x1*sin (rotary_embedding.rs:148-149)
    const float y1a = rnd<T>(rnd<T>(x1a * c0) - rnd<T>(x2a * sn0));
    const float y1b = rnd<T>(rnd<T>(x1b * c1) - rnd<T>(x2b * sn1));
    const float y2a = rnd<T>(rnd<T>(x2a * c0) + rnd<T>(x1a * sn0));
    const float y2b = rnd<T>(rnd<T>(x2b * c1) + rnd<T>(x1b * sn1));
    const uint32_t oa = DT<T>::from_f2(y1a, y1b);
    const uint32_t ob = DT<T>::from_f2(y2a, y2b);
    if (is_q) {
      T* d = q_out + (t * num_q_heads + r) * (int64_t)kRopeD;
      *reinterpret_cast<uint32_t*>(d + i0) = oa;
      *reinterpret_cast<uint32_t*>(d + 64 + i0) = ob;
    } else {
      const int h = r - num_q_heads;
      if (k_out) {
        T* d = k_out + t * kv_row + (int64_t)h * kRopeD;
        *reinterpret_cast<uint32_t*>(d + i0) = oa;
        *reinterpret_cast<uint32_t*>(d + 64 + i0) = ob;
      }
      if (slot >= 0 && k_cache) {
        T* d = k_cache + slot * kv_row + (int64_t)h * kRopeD;
        *reinterpret_cast<uint32_t*>(d + i0) = oa;
        *reinterpret_cast<uint32_t*>(d + 64 + i0) = ob;
      }
    }
  };
#pragma unroll
  for (int k = 0; k < kPre; ++k) {
    const int r = warp + 8 * k;
    if (r < rows) row_out(r, pa[k], pb[k]);
  }
  for (int r = warp + 8 * kPre; r < rows; r += 8) {  // rows beyond the preloaded ones
    const T* src = src_tok + (int64_t)r * kRopeD;
    row_out(r, *reinterpret_cast<const uint32_t*>(src + i0),
            *reinterpret_cast<const uint32_t*>(src + 64 + i0));
  }
}


}  // namespace nvkv

extern "C" int nvkv_qknorm_rope(const void* qkv, int64_t qkv_stride, int64_t num_tokens,
                                int num_q_heads, int num_kv_heads, int head_dim,
                                const int64_t* positions, const void* q_norm_w,
                                const void* k_norm_w, float eps, float rope_theta,
                                int64_t max_position, void* q_out, void* k_out, void* v_out,
                                void* k_cache, void* v_cache, const int64_t* slot_mapping,
                                int64_t num_slots, int dtype, nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_qknorm_rope");
  using namespace nvkv;
  clear_error();
  if (dtype != NVKV_DTYPE_BF16 && dtype != NVKV_DTYPE_F16)
    return set_error(NVKV_ERR_UNSUPPORTED, "qknorm_rope: unsupported dtype (bf16/f16 only)");
  if (head_dim != kRopeD)
    return set_error(NVKV_ERR_UNSUPPORTED, "qknorm_rope: head_dim must be 128");
  if (num_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_position <= 0)
    return set_error(NVKV_ERR_INVALID_ARG, "qknorm_rope: bad sizes");
  if (num_tokens == 0) return NVKV_OK;
  if (!qkv || !positions || !q_out)
    return set_error(NVKV_ERR_INVALID_ARG, "qknorm_rope: null qkv/positions/q_out");
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
    return set_error(NVKV_ERR_INVALID_ARG, "qknorm_rope: pass both norm weights or neither");
  const bool any_cache = k_cache || v_cache || slot_mapping;
  if (any_cache && !(k_cache && v_cache && slot_mapping))
    return set_error(NVKV_ERR_INVALID_ARG,
                     "qknorm_rope: k_cache, v_cache and slot_mapping go together");
  if (qkv_stride < (int64_t)(num_q_heads + 2 * num_kv_heads) * head_dim)
    return set_error(NVKV_ERR_INVALID_ARG, "qknorm_rope: qkv_stride smaller than a row");
  if (num_tokens > 0x7fffffffLL)
    return set_error(NVKV_ERR_INVALID_ARG, "qknorm_rope: too many tokens");
  // 4-byte accesses: every base pointer and the row stride must be even-element aligned
  uintptr_t m = (uintptr_t)qkv | (uintptr_t)q_out | (uintptr_t)k_out | (uintptr_t)v_out |
                (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)q_norm_w |
                (uintptr_t)k_norm_w | (uintptr_t)(qkv_stride * 2);
  if (m & 3u) return set_error(NVKV_ERR_ALIGNMENT, "qknorm_rope: pointers must be 4-byte aligned");
  const float ln_theta = (float)log((double)rope_theta);
  int* err = device_error_word();
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == NVKV_DTYPE_BF16) {
    using T = __nv_bfloat16;
    qknorm_rope_kernel<T><<<(unsigned)num_tokens, 256, 0, s>>>(
        (const T*)qkv, qkv_stride, num_q_heads, num_kv_heads, positions, (const T*)q_norm_w,
        (const T*)k_norm_w, eps, ln_theta, max_position, (T*)q_out, (T*)k_out, (T*)v_out,
        (T*)k_cache, (T*)v_cache, slot_mapping, num_slots, err);
  } else {
    using T = __half;
    qknorm_rope_kernel<T><<<(unsigned)num_tokens, 256, 0, s>>>(
        (const T*)qkv, qkv_stride, num_q_heads, num_kv_heads, positions, (const T*)q_norm_w,
        (const T*)k_norm_w, eps, ln_theta, max_position, (T*)q_out, (T*)k_out, (T*)v_out,
        (T*)k_cache, (T*)v_cache, slot_mapping, num_slots, err);
  }
  return check_cuda(cudaGetLastError(), "qknorm_rope launch");
}
