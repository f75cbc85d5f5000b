// On-device sampling of the next token: replaces Sampler::forward
// (nanovllm_rs/src/layers/sampler.rs:7-21), which divides the last-token
// logits by each sequence's temperature, takes the softmax p, draws
// E = max(-log U, 1e-10) per element with U uniform, and picks
// argmax(p / E).  Since log is monotonic and softmax only subtracts the
// row's log-sum-exp, argmax(p / E) = argmax(logit / T - log E): the
// Gumbel-max form, which needs no softmax pass and no normalisation, and
// which a vocab-parallel shard can evaluate on its own slice -- each rank's
// (value, global index) candidate is all-gathered exactly like the greedy
// pick's.
//
// Noise: Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011), a counter-based generator, keyed by
// the 64-bit seed, with counter (global vocab index / 4, row, step low,
// step high): one call gives the four uniforms of vocab entries 4k .. 4k + 3.
// The noise of an element therefore depends only on (seed, step, row, global
// vocab index), so a sharded vocabulary draws the same noise as the whole one
// and the same seed reproduces the same tokens.  u = ((bits >> 9) + 1/2)
// 2^-23, exact in f32 and inside (0, 1): 2^-24 <= u <= 1 - 2^-24.
//
// One CTA per row; 8 logits per thread per iteration (16-byte loads of
// bf16/f16), two Philox calls; a block arg-max reduction, ties to the lowest
// index (candle's argmax takes the first maximum too).  Temperatures <= 0
// select the plain arg-max of the logits (greedy; the reference requires
// T > 1e-10, so such rows never come from it).
#include "common.cuh"

namespace nvkv {

constexpr int kSampThreads = 1024;  // one row per CTA: enough warps to hide the Philox chains

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

__device__ __forceinline__ float uniform23(uint32_t bits) {
  return ((float)(bits >> 9) + 0.5f) * 1.1920928955078125e-07f;  // 2^-23
}

// logit / T - log(max(-log u, 1e-10)); the logit itself when T <= 0
__device__ __forceinline__ float gumbel_score(float logit, float temp, uint32_t bits) {
  if (!(temp > 0.f)) return logit;
  const float e = fmaxf(-logf(uniform23(bits)), 1e-10f);
  return logit / temp - logf(e);
}

__device__ __forceinline__ void better(float& bv, int64_t& bi, float v, int64_t i) {
  // the larger value wins, ties (and NaN-free equal values) to the lower index
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 x = DT<T>::to_f2(w[k]);
    f[2 * k] = x.x;
    f[2 * k + 1] = x.y;
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* f) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
}
template <typename T>
__device__ __forceinline__ float to_float(T x) {
  return DT<T>::to_f(x);
}
template <>
__device__ __forceinline__ float to_float<float>(float x) {
  return x;
}

template <typename T>
__global__ void __launch_bounds__(kSampThreads)
    sample_kernel(const T* __restrict__ logits, int64_t vocab, int64_t row_stride,
                  int64_t vocab_offset, const float* __restrict__ temps, uint32_t k0, uint32_t k1,
                  uint64_t step0, const int64_t* __restrict__ step_ptr,
                  float* __restrict__ out_value, int64_t* __restrict__ out_index) {
  __shared__ float sv[kSampThreads / 32];
  __shared__ int64_t si[kSampThreads / 32];
  const int64_t b = blockIdx.x;
  const T* row = logits + b * row_stride;
  const float temp = temps[b];
  const uint64_t step = step0 + (step_ptr ? (uint64_t)*step_ptr : 0ull);
  const uint32_t step_lo = (uint32_t)step, step_hi = (uint32_t)(step >> 32);
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  // vectors of 8 where the row allows them (16-byte aligned row, offset a
  // multiple of 4 so that each Philox call covers whole groups of 4)
  const bool vec = (vocab_offset & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const int64_t nvec = vec ? vocab / 8 : 0;
  for (int64_t j = threadIdx.x; j < nvec; j += kSampThreads) {
    float f[8];
    load8<T>(row + j * 8, f);
    const int64_t g0 = vocab_offset + j * 8;  // global index of f[0], a multiple of 4
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t ctr = (uint32_t)(g0 / 4 + h);
      const uint4 r = philox4x32_10(make_uint4(ctr, (uint32_t)b, step_lo, step_hi), k0, k1);
      const uint32_t bits[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int k = 0; k < 4; ++k)
        better(bv, bi, gumbel_score(f[4 * h + k], temp, bits[k]), g0 + 4 * h + k);
    }
  }
  for (int64_t v = nvec * 8 + threadIdx.x; v < vocab; v += kSampThreads) {  // the rest, one by one
    const int64_t g = vocab_offset + v;
    const uint4 r =
        philox4x32_10(make_uint4((uint32_t)(g / 4), (uint32_t)b, step_lo, step_hi), k0, k1);
    const uint32_t bits[4] = {r.x, r.y, r.z, r.w};
    better(bv, bi, gumbel_score(to_float<T>(row[v]), temp, bits[g & 3]), g);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kSampThreads / 32; ++w) better(bv, bi, sv[w], si[w]);
    out_value[b] = bv;
    out_index[b] = bi;
  }
}

}  // namespace nvkv

extern "C" int nvkv_sample(const void* logits, int64_t num_rows, int64_t vocab,
                           int64_t row_stride, int64_t vocab_offset, const float* temperatures,
                           uint64_t seed, uint64_t step, const int64_t* step_device,
                           float* out_value, int64_t* out_index, int dtype,
                           nvkv_stream_t stream) {
  NVKV_RANGE("nvkv_sample");
  using namespace nvkv;
  clear_error();
  if (num_rows < 0 || vocab < 0 || vocab_offset < 0 || row_stride < vocab)
    return set_error(NVKV_ERR_INVALID_ARG, "sample: negative size or row_stride < vocab");
  if (num_rows > 0x7fffffffLL || vocab_offset + vocab > ((int64_t)1 << 34))
    return set_error(NVKV_ERR_UNSUPPORTED, "sample: more than 2^31 rows or 2^34 vocab entries");
  if (num_rows == 0) return NVKV_OK;
  if (vocab == 0) return set_error(NVKV_ERR_INVALID_ARG, "sample: empty vocabulary");
  if (!logits || !temperatures || !out_value || !out_index)
    return set_error(NVKV_ERR_INVALID_ARG, "sample: null pointer");
  if (dtype != NVKV_DTYPE_BF16 && dtype != NVKV_DTYPE_F16 && dtype != NVKV_DTYPE_F32)
    return set_error(NVKV_ERR_UNSUPPORTED, "sample: logits must be bf16, f16 or f32");
  const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)num_rows);
  if (dtype == NVKV_DTYPE_BF16)
    sample_kernel<__nv_bfloat16><<<grid, kSampThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(logits), vocab, row_stride, vocab_offset, temperatures,
        k0, k1, step, step_device, out_value, out_index);
  else if (dtype == NVKV_DTYPE_F16)
    sample_kernel<__half><<<grid, kSampThreads, 0, s>>>(static_cast<const __half*>(logits), vocab,
                                                        row_stride, vocab_offset, temperatures, k0,
                                                        k1, step, step_device, out_value, out_index);
  else
    sample_kernel<float><<<grid, kSampThreads, 0, s>>>(static_cast<const float*>(logits), vocab,
                                                       row_stride, vocab_offset, temperatures, k0,
                                                       k1, step, step_device, out_value, out_index);
  return check_cuda(cudaGetLastError(), "sample launch");
}
