// Shared helpers for the nvkv kernels (sm_100a only).
//
// * host-side status/error plumbing behind the C ABI (thread-local message);
// * the device error word that bounds checks write instead of faulting;
// * thin inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor, no
//   cluster-wide variants anywhere in this library), ldmatrix and mma.sync;
// * tensor-map encoding through the driver entry point (no -lcuda needed).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/nvkv.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "nvkv is written for sm_100a only"
#endif

#include <nvtx3/nvToolsExt.h>

namespace nvkv {

// NVTX range for the lifetime of a host call (a profiler shows one range per
// C-ABI call, named after the entry point; without one attached the NVTX3
// calls return at once).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
#define NVKV_RANGE(name) ::nvkv::NvtxRange nvkv_nvtx_range_(name)


// ---------------------------------------------------------------------------
// Host status plumbing
// ---------------------------------------------------------------------------
int set_error(int code, const std::string& msg);  // records msg, returns code
void clear_error();
int check_cuda(cudaError_t e, const char* what);  // NVKV_OK or NVKV_ERR_CUDA

// Device address of the per-device error word (file-scope __device__ array
// in errors.cu, looked up with cudaGetSymbolAddress once per device).
int* device_error_word();

// Tensor maps: encodes a rank-3 bf16/f16 tiled map over a
// [rows][heads][head_dim] array (strides in bytes for dims 1 and 2).
int encode_kv_tensor_map(CUtensorMap* map, const void* base, int64_t head_dim,
                         int64_t num_heads, int64_t num_rows, int64_t row_stride_bytes,
                         int box_inner, int box_rows, bool swizzle128);

// The same for an fp8 (1-byte) pool: box = one head's row_bytes (128) x
// box_rows rows, SWIZZLE_128B.
int encode_kv_tensor_map_u8(CUtensorMap* map, const void* base, int64_t row_bytes,
                            int64_t num_heads, int64_t num_rows, int64_t row_stride_bytes,
                            int box_rows);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Raises a kernel's dynamic shared-memory limit once per device (first call
// outside any stream capture), so later launches -- captured or not -- do no
// attribute calls.  `done` is a per-kernel bitmask of devices.
int ensure_smem_attr(const void* kernel, int bytes, unsigned long long* done);

// Validated arguments of one nvkv_paged_attention call.
struct AttnArgs {
  const void* q;
  int64_t q_stride;     // elements between query tokens
  int64_t num_q_rows;   // rows of q (bounds the Q tensor map)
  const void* k_cache;
  const void* v_cache;
  int64_t num_blocks;   // pages (paged) or K/V rows (contiguous)
  int64_t kv_stride;    // elements between K/V rows
  void* out;
  const uint32_t* cu_q;
  const uint32_t* cu_k;
  const uint32_t* block_tables;
  int64_t bt_stride;
  int num_seqs, max_q, max_k, hq, hkv, d, page;
  float scale;
  int causal;
  void* ws;
  size_t ws_bytes;
  int dtype;
  cudaStream_t stream;
  // fp8 (e4m3) pool: per (page, kv head, row) f32 scales [num_blocks, Hkv,
  // page]; null for a bf16/f16 pool
  const float* k_scale = nullptr;
  const float* v_scale = nullptr;
  // the workspace's split-KV scratch is sized for the fp8 decode plan (the
  // prefill work plan follows it)
  bool fp8_layout = false;
};

// Shared by the attention entry points (api.cu): shape checks, and the
// workspace of split-KV scratch + prefill work plan.
int validate_shapes(int num_seqs, int max_q, int max_k, int hq, int hkv, int d);
size_t attention_workspace_bytes(int num_seqs, int hq, int hkv, int max_q, int max_k,
                                 bool fp8 = false);
int launch_paged_decode(const AttnArgs& a);
size_t decode_workspace_bytes(int num_seqs, int num_q_heads, int num_kv_heads, int max_seqlen_k,
                              bool fp8);
void decode_plan(int num_seqs, int num_kv_heads, int max_seqlen_k, bool fp8, int* chunk_tokens,
                 int* max_splits);
int launch_paged_prefill(const AttnArgs& a);
// Bytes of the prefill work plan (0 when max_seqlen_q <= 1); it sits in the
// attention workspace after the decode scratch, at attention_plan_offset().
size_t prefill_plan_bytes(int num_seqs, int max_seqlen_q);
inline size_t attention_plan_offset(size_t decode_bytes) { return (decode_bytes + 255) & ~size_t(255); }
constexpr int kPfMaxQTiles = 12000;  // plan histogram in 48 KB of shared memory
int launch_store_kvcache(const void* key, const void* value, void* k_cache, void* v_cache,
                         const int64_t* slot_mapping, int64_t num_tokens, int64_t row_elems,
                         int64_t key_stride, int64_t value_stride, int64_t num_slots,
                         cudaStream_t stream);

// Launch as a programmatic dependent of the previous kernel in the stream
// (PDL): the grid may be scheduled while that kernel drains, and the kernel
// must execute griddepcontrol.wait (pdl_wait below) before it reads any
// input.  After a non-kernel stream operation the attribute has no effect.
#ifdef __CUDACC__
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), what);
}
#endif

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
#ifdef __CUDACC__

// Waits until the grid this one programmatically depends on has completed and
// its memory is visible (no-op for a normally launched grid).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the dependent grid of this one be scheduled (it still waits for this
// grid's completion in its own pdl_wait).
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

template <typename T>
struct DT;
template <>
struct DT<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float2 to_f2(uint32_t u) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(h);
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <>
struct DT<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ float2 to_f2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// round-trip through the storage dtype (the reference rounds after each op)
template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return DT<T>::to_f(DT<T>::from_f(x));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: every spin in this library gives up after a fixed number of
// try_wait rounds (each round itself blocks for a hardware time slice), sets
// the error word and returns false, so a logic error can never hang a GPU.
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kDevErrTimeout = 99;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  record_error(err, kDevErrTimeout);
  return false;
}

// ---- TMA (single-CTA destination only) ------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---- warp-level MMA (legacy path, used by the HBM-bound decode kernel) ------
__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                            uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1);
template <>
__device__ __forceinline__ void mma_16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4],
                                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma_16816<__half>(float (&c)[4], const uint32_t (&a)[4],
                                                  uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a tile that
// TMA wrote with CU_TENSOR_MAP_SWIZZLE_128B (128-byte rows, 1024-byte aligned).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ float warp_max_xor(float v, int mask) {
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, mask));
}

#endif  // __CUDACC__

}  // namespace nvkv
