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

// A block walks kStoreTok tokens at a time; thread i moves chunks i, i + 256,
// ... of the token's K row then V row (2 * chunks_per_row per token, no
// division).  The row loads do not depend on the slot (the source row always
// exists), so all kStoreTok loads and their slots are in flight together
// before the slot checks decide which stores happen.
constexpr int kStoreTok = 4;

template <int VEC>
__global__ void __launch_bounds__(256) store_kvcache_kernel(
    const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
    uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
    const int64_t* __restrict__ slot_mapping, int64_t num_tokens, int64_t chunks_per_row,
    int64_t key_stride_b, int64_t value_stride_b, int64_t row_bytes, int64_t num_slots,
    int* err) {
  using V = typename VecT<VEC>::type;
  const int per_tok = (int)(2 * chunks_per_row);
  for (int64_t t0 = (int64_t)blockIdx.x * kStoreTok; t0 < num_tokens;
       t0 += (int64_t)gridDim.x * kStoreTok) {
    for (int r = threadIdx.x; r < per_tok; r += blockDim.x) {
      const bool is_v = r >= chunks_per_row;
      const int c = is_v ? r - (int)chunks_per_row : r;
      const uint8_t* base = is_v ? value : key;
      const int64_t stride = is_v ? value_stride_b : key_stride_b;
      uint8_t* cache = is_v ? v_cache : k_cache;
      V x[kStoreTok];
      int64_t slot[kStoreTok];
#pragma unroll
      for (int u = 0; u < kStoreTok; ++u) {
        const int64_t t = t0 + u;
        if (t < num_tokens) {
          slot[u] = __ldg(slot_mapping + t);
          x[u] = __ldg(reinterpret_cast<const V*>(base + t * stride) + c);
        } else {
          slot[u] = -1;
        }
      }
#pragma unroll
      for (int u = 0; u < kStoreTok; ++u) {
        if (slot[u] < 0) continue;  // padded / warm-up token (or past the batch)
        if (slot[u] >= num_slots) {
          record_error(err, NVKV_DEVERR_SLOT_RANGE);
          continue;
        }
        reinterpret_cast<V*>(cache + slot[u] * row_bytes)[c] = x[u];
      }
    }
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
  if (2 * cpr > 0x7fffffffLL)
    return set_error(NVKV_ERR_UNSUPPORTED, "store_kvcache: row too wide");
  int64_t blocks = (num_tokens + kStoreTok - 1) / kStoreTok;
  if (blocks > 148 * 8) blocks = 148 * 8;  // 8 resident blocks of 256 threads per SM
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
  NVKV_RANGE("nvkv_store_kvcache");
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
