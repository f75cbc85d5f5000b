// Kernel 1: KV-cache scatter (nvkv_store_kvcache).
//
// Restates nanovllm_rs/src/layers/kv_cache.rs:13-24 (one row copy per token,
// skipping slot < 0) for sm_100a: K and V go out in ONE launch, every thread
// moves 16 bytes (narrower only when a pointer or stride is not 16-byte
// aligned), rows are read through their token stride (so the K/V slices of a
// fused qkv buffer need no contiguous copy), and a slot past the end of the
// cache is skipped and recorded in the device error word instead of writing
// out of bounds.  Pure HBM traffic: 2 * T_valid * row_bytes read + the same
// written + 8 * T bytes of slots.
#include "common.cuh"

namespace nvkv {

template <int VEC>
struct VecT;
template <>
struct VecT<16> { using type = uint4; };
template <>
struct VecT<8> { using type = uint2; };
template <>
struct VecT<4> { using type = uint32_t; };
template <>
struct VecT<2> { using type = uint16_t; };

template <int VEC>
__global__ void __launch_bounds__(256) store_kvcache_kernel(
    const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
    uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
    const int64_t* __restrict__ slot_mapping, int64_t num_tokens, int64_t chunks_per_row,
    int64_t key_stride_b, int64_t value_stride_b, int64_t row_bytes, int64_t num_slots,
    int* err) {
  using V = typename VecT<VEC>::type;
  const int64_t per_tok = 2 * chunks_per_row;
  const int64_t total = num_tokens * per_tok;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / per_tok;
    const int64_t r = idx - t * per_tok;
    const bool is_v = r >= chunks_per_row;
    const int64_t c = is_v ? r - chunks_per_row : r;
    const int64_t slot = __ldg(slot_mapping + t);
    if (slot < 0) continue;  // padded / warm-up token
    if (slot >= num_slots) {
      record_error(err, NVKV_DEVERR_SLOT_RANGE);
      continue;
    }
    const uint8_t* src = is_v ? value + t * value_stride_b : key + t * key_stride_b;
    uint8_t* dst = (is_v ? v_cache : k_cache) + slot * row_bytes;
    V x = __ldg(reinterpret_cast<const V*>(src) + c);
    reinterpret_cast<V*>(dst)[c] = x;
  }
}

int launch_store_kvcache(const void* key, const void* value, void* k_cache, void* v_cache,
                         const int64_t* slot_mapping, int64_t num_tokens, int64_t row_elems,
                         int64_t key_stride, int64_t value_stride, int64_t num_slots,
                         cudaStream_t stream) {
  const int64_t row_bytes = row_elems * 2;
  const int64_t ks = key_stride * 2, vs = value_stride * 2;
  auto fits = [&](int64_t v) {
    uintptr_t m = (uintptr_t)key | (uintptr_t)value | (uintptr_t)k_cache | (uintptr_t)v_cache |
                  (uintptr_t)row_bytes | (uintptr_t)ks | (uintptr_t)vs;
    return (m % (uintptr_t)v) == 0;
  };
  const int vec = fits(16) ? 16 : fits(8) ? 8 : fits(4) ? 4 : 2;
  const int64_t cpr = row_bytes / vec;
  const int64_t total = num_tokens * 2 * cpr;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  int* err = device_error_word();
  auto k = reinterpret_cast<const uint8_t*>(key);
  auto v = reinterpret_cast<const uint8_t*>(value);
  auto kc = reinterpret_cast<uint8_t*>(k_cache);
  auto vc = reinterpret_cast<uint8_t*>(v_cache);
  switch (vec) {
    case 16:
      store_kvcache_kernel<16><<<(unsigned)blocks, 256, 0, stream>>>(
          k, v, kc, vc, slot_mapping, num_tokens, cpr, ks, vs, row_bytes, num_slots, err);
      break;
    case 8:
      store_kvcache_kernel<8><<<(unsigned)blocks, 256, 0, stream>>>(
          k, v, kc, vc, slot_mapping, num_tokens, cpr, ks, vs, row_bytes, num_slots, err);
      break;
    case 4:
      store_kvcache_kernel<4><<<(unsigned)blocks, 256, 0, stream>>>(
          k, v, kc, vc, slot_mapping, num_tokens, cpr, ks, vs, row_bytes, num_slots, err);
      break;
    default:
      store_kvcache_kernel<2><<<(unsigned)blocks, 256, 0, stream>>>(
          k, v, kc, vc, slot_mapping, num_tokens, cpr, ks, vs, row_bytes, num_slots, err);
      break;
  }
  return check_cuda(cudaGetLastError(), "store_kvcache launch");
}

}  // namespace nvkv

extern "C" int nvkv_store_kvcache(const void* key, const void* value, void* k_cache,
                                  void* v_cache, const int64_t* slot_mapping, int64_t num_tokens,
                                  int64_t row_elems, int64_t key_stride, int64_t value_stride,
                                  int64_t num_slots, int dtype, nvkv_stream_t stream) {
  using namespace nvkv;
  clear_error();
  if (dtype != NVKV_DTYPE_BF16 && dtype != NVKV_DTYPE_F16)
    return set_error(NVKV_ERR_UNSUPPORTED, "store_kvcache: unsupported dtype (bf16/f16 only)");
  if (num_tokens < 0 || row_elems <= 0 || num_slots < 0)
    return set_error(NVKV_ERR_INVALID_ARG, "store_kvcache: negative size");
  if (num_tokens == 0) return NVKV_OK;  // kv_cache.rs:128-130
  if (!key || !value || !k_cache || !v_cache || !slot_mapping)
    return set_error(NVKV_ERR_INVALID_ARG, "store_kvcache: null pointer");
  if (num_tokens > 1 && (key_stride < row_elems || value_stride < row_elems))
    return set_error(NVKV_ERR_INVALID_ARG,
                     "store_kvcache: token stride smaller than the per-slot width");
  return launch_store_kvcache(key, value, k_cache, v_cache, slot_mapping, num_tokens, row_elems,
                              key_stride, value_stride, num_slots, (cudaStream_t)stream);
}
