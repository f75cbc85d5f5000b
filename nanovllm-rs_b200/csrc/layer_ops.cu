// Fused epilogues around the attention path: RMSNorm (optionally with the
// residual add) and SiLU*mul.
//
// Replace the per-layer candle op chains of nanovllm_rs/src/layers/
// layernorm.rs:18-42 (RMSNorm::forward / residual_forward, ~8 launches each)
// and layers/activation.rs:5-17 (SiluAndMul::forward, 3 launches) with one
// HBM-bound launch each, at the reference's rounding points:
//   residual_forward: s = x + r (f32); r' = dtype(s); y = dtype(dtype(s *
//                     1/sqrt(mean(s^2) + eps)) * w)
//   forward:          the same with s = x and no residual output
//   silu_and_mul:     y = dtype(dtype(silu(g)) * u), silu in f32
// Layout: one CTA (256 threads) per token row for the norm, every thread
// holding up to 32 elements in registers (16-byte loads), a block reduction of
// the f32 sum of squares; a grid-stride 16-byte loop for SiLU*mul.
#include "norm_row.cuh"

namespace nvkv {

template <typename T>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(
    const T* __restrict__ x, int64_t x_stride, T* residual, int64_t res_stride,
    const T* __restrict__ w, float eps, T* __restrict__ out, int64_t out_stride, int H) {
  __shared__ float red[kNormThreads / 32];
  const int64_t t = blockIdx.x;
  T* r = residual ? residual + t * res_stride : nullptr;
  norm_row<T>(x + t * x_stride, r, r, w, eps, out + t * out_stride, H, red);
}

template <typename T>
__global__ void __launch_bounds__(256) silu_mul_kernel(const T* __restrict__ gu, int64_t gu_stride,
                                                       T* __restrict__ out, int64_t out_stride,
                                                       int64_t T_, int F) {
  const int nvec = F / 8;
  const int64_t total = T_ * nvec;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / nvec;
    const int c = (int)(i - t * nvec);
    const uint4 g = *reinterpret_cast<const uint4*>(gu + t * gu_stride + c * 8);
    const uint4 u = *reinterpret_cast<const uint4*>(gu + t * gu_stride + F + c * 8);
    const uint32_t* gp = reinterpret_cast<const uint32_t*>(&g);
    const uint32_t* up = reinterpret_cast<const uint32_t*>(&u);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 gf = DT<T>::to_f2(gp[e]);
      const float2 uf = DT<T>::to_f2(up[e]);
      const float s0 = rnd<T>(gf.x / (1.0f + expf(-gf.x)));
      const float s1 = rnd<T>(gf.y / (1.0f + expf(-gf.y)));
      op[e] = DT<T>::from_f2(s0 * uf.x, s1 * uf.y);
    }
    *reinterpret_cast<uint4*>(out + t * out_stride + c * 8) = o;
  }
}

}  // namespace nvkv

extern "C" int nvkv_rms_norm(const void* x, int64_t x_stride, void* residual, int64_t res_stride,
                             const void* weight, float eps, void* out, int64_t out_stride,
                             int64_t num_tokens, int hidden, int dtype, nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_rms_norm");
  using namespace nvkv;
  clear_error();
  if (dtype != NVKV_DTYPE_BF16 && dtype != NVKV_DTYPE_F16)
    return set_error(NVKV_ERR_UNSUPPORTED, "rms_norm: unsupported dtype (bf16/f16 only)");
  if (num_tokens < 0 || hidden <= 0 || hidden % 8 != 0 ||
      hidden > kNormThreads * 8 * kNormMaxVec)
    return set_error(NVKV_ERR_UNSUPPORTED, "rms_norm: hidden must be a multiple of 8, <= 8192");
  if (num_tokens == 0) return NVKV_OK;
  if (!x || !weight || !out) return set_error(NVKV_ERR_INVALID_ARG, "rms_norm: null pointer");
  if (num_tokens > 0x7fffffffLL) return set_error(NVKV_ERR_INVALID_ARG, "rms_norm: too many rows");
  uintptr_t m = (uintptr_t)x | (uintptr_t)residual | (uintptr_t)weight | (uintptr_t)out |
                (uintptr_t)(x_stride * 2) | (uintptr_t)(res_stride * 2) |
                (uintptr_t)(out_stride * 2);
  if (m & 15u) return set_error(NVKV_ERR_ALIGNMENT, "rms_norm: rows must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == NVKV_DTYPE_BF16) {
    using T = __nv_bfloat16;
    rms_norm_kernel<T><<<(unsigned)num_tokens, kNormThreads, 0, s>>>(
        (const T*)x, x_stride, (T*)residual, res_stride, (const T*)weight, eps, (T*)out,
        out_stride, hidden);
  } else {
    using T = __half;
    rms_norm_kernel<T><<<(unsigned)num_tokens, kNormThreads, 0, s>>>(
        (const T*)x, x_stride, (T*)residual, res_stride, (const T*)weight, eps, (T*)out,
        out_stride, hidden);
  }
  return check_cuda(cudaGetLastError(), "rms_norm launch");
}

extern "C" int nvkv_silu_and_mul(const void* gate_up, int64_t gu_stride, void* out,
                                 int64_t out_stride, int64_t num_tokens, int inter, int dtype,
                                 nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_silu_and_mul");
  using namespace nvkv;
  clear_error();
  if (dtype != NVKV_DTYPE_BF16 && dtype != NVKV_DTYPE_F16)
    return set_error(NVKV_ERR_UNSUPPORTED, "silu_and_mul: unsupported dtype (bf16/f16 only)");
  if (num_tokens < 0 || inter <= 0 || inter % 8 != 0)
    return set_error(NVKV_ERR_UNSUPPORTED, "silu_and_mul: width must be a multiple of 8");
  if (num_tokens == 0) return NVKV_OK;
  if (!gate_up || !out) return set_error(NVKV_ERR_INVALID_ARG, "silu_and_mul: null pointer");
  uintptr_t m = (uintptr_t)gate_up | (uintptr_t)out | (uintptr_t)(gu_stride * 2) |
                (uintptr_t)(out_stride * 2);
  if (m & 15u) return set_error(NVKV_ERR_ALIGNMENT, "silu_and_mul: rows must be 16-byte aligned");
  const int64_t total = num_tokens * (inter / 8);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == NVKV_DTYPE_BF16) {
    using T = __nv_bfloat16;
    silu_mul_kernel<T><<<(unsigned)blocks, 256, 0, s>>>((const T*)gate_up, gu_stride, (T*)out,
                                                       out_stride, num_tokens, inter);
  } else {
    using T = __half;
    silu_mul_kernel<T><<<(unsigned)blocks, 256, 0, s>>>((const T*)gate_up, gu_stride, (T*)out,
                                                       out_stride, num_tokens, inter);
  }
  return check_cuda(cudaGetLastError(), "silu_and_mul launch");
}
