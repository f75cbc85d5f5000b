// One token row of RMSNorm at the reference's rounding points
// (layers/layernorm.rs:18-42), shared by nvkv_rms_norm and the fused
// all-reduce epilogue so both produce the same bits for the same input:
//   s = x (+ residual_in), f32;  residual_out = dtype(s)
//   y = dtype(dtype(s * 1/sqrt(mean(s^2) + eps)) * w), mean = sum(s^2) * (1/H)
// kNormThreads threads per row, each holding up to kNormMaxVec 8-element
// vectors in registers; the f32 sum of rounded squares is reduced with warp
// shuffles and then across the 8 warps in a fixed order.
#pragma once

#include "common.cuh"

namespace nvkv {

constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 4;  // 8-element vectors per thread: H <= 256 * 8 * 4 = 8192

// load(c) returns the row's 8-element vector c (8 dtype values in a uint4).
// residual_in / residual_out may be null and may alias.  red: shared
// [kNormThreads / 32].  Ends with a barrier, so calls may follow each other.
template <typename T, typename Load>
__device__ __forceinline__ void norm_row_load(Load load, const T* residual_in, T* residual_out,
                                              const T* __restrict__ w, float eps,
                                              T* __restrict__ out, int H, float* red) {
  const int tid = threadIdx.x;
  const int nvec = H / 8;
  float v[kNormMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = tid + i * kNormThreads;
    if (c < nvec) {
      const uint4 a = load(c);
      const uint32_t* ap = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = DT<T>::to_f2(ap[e]);
        v[i][2 * e] = f.x;
        v[i][2 * e + 1] = f.y;
      }
      if (residual_in) {
        const uint4 b = *reinterpret_cast<const uint4*>(residual_in + c * 8);
        const uint32_t* bp = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = DT<T>::to_f2(bp[e]);
          v[i][2 * e] += f.x;
          v[i][2 * e + 1] += f.y;
        }
      }
      if (residual_out) {
        uint4 nr;
        uint32_t* np = reinterpret_cast<uint32_t*>(&nr);
#pragma unroll
        for (int e = 0; e < 4; ++e) np[e] = DT<T>::from_f2(v[i][2 * e], v[i][2 * e + 1]);
        *reinterpret_cast<uint4*>(residual_out + c * 8) = nr;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += __fmul_rn(v[i][e], v[i][e]);  // rounded squares (x.sqr())
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot * (1.0f / (float)H) + eps);
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = tid + i * kNormThreads;
    if (c < nvec) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + c * 8);
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wv);
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 wf = DT<T>::to_f2(wp[e]);
        op[e] = DT<T>::from_f2(rnd<T>(v[i][2 * e] * inv) * wf.x,
                               rnd<T>(v[i][2 * e + 1] * inv) * wf.y);
      }
      *reinterpret_cast<uint4*>(out + c * 8) = o;
    }
  }
  __syncthreads();  // red[] may be rewritten by the next row
}

// The row at x (read with L1-bypassing loads: other GPUs may have written it).
template <typename T>
__device__ __forceinline__ void norm_row(const T* __restrict__ x, const T* residual_in,
                                         T* residual_out, const T* __restrict__ w, float eps,
                                         T* __restrict__ out, int H, float* red) {
  norm_row_load<T>([x](int c) { return __ldcg(reinterpret_cast<const uint4*>(x + c * 8)); },
                   residual_in, residual_out, w, eps, out, H, red);
}

}  // namespace nvkv
