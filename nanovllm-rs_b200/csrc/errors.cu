// Host-side status plumbing, the per-device error word and tensor-map
// encoding shared by every nvkv entry point.
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace nvkv {

namespace {
thread_local std::string g_last_error;

// One error word per device: the module holding this array is loaded once
// per device context, so each GPU gets its own copy.  Kernels receive its
// device address (never the host-side symbol) as an argument.
__device__ int g_device_error_word[4];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_err_ptr[kMaxDevices] = {nullptr};

// Looked up once; published with release/acquire so callers on other threads
// see a complete pointer without taking the lock.
std::atomic<PFN_cuTensorMapEncodeTiled_v12000> g_encode{nullptr};
}  // namespace

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

void clear_error() { g_last_error.clear(); }

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return NVKV_OK;
  return set_error(NVKV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

int ensure_smem_attr(const void* kernel, int bytes, unsigned long long* done) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  const unsigned long long bit = 1ull << (dev & 63);
  std::lock_guard<std::mutex> lk(g_mu);
  if (*done & bit) return NVKV_OK;
  rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                  "cudaFuncSetAttribute(max dynamic smem)");
  if (rc) return rc;
  *done |= bit;
  return NVKV_OK;
}

static int get_encoder(PFN_cuTensorMapEncodeTiled_v12000* out) {
  *out = g_encode.load(std::memory_order_acquire);
  if (*out) return NVKV_OK;
  std::lock_guard<std::mutex> lk(g_mu);
  *out = g_encode.load(std::memory_order_relaxed);
  if (*out) return NVKV_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                   cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return set_error(NVKV_ERR_CUDA, "cuTensorMapEncodeTiled entry point not available");
  *out = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  g_encode.store(*out, std::memory_order_release);
  return NVKV_OK;
}

int encode_kv_tensor_map(CUtensorMap* map, const void* base, int64_t head_dim, int64_t num_heads,
                         int64_t num_rows, int64_t row_stride_bytes, int box_inner, int box_rows,
                         bool swizzle128) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  int rc = get_encoder(&encode);
  if (rc) return rc;
  // dim0 = head_dim (contiguous), dim1 = heads, dim2 = rows (tokens / slots)
  cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)num_heads, (cuuint64_t)num_rows};
  cuuint64_t strides[2] = {(cuuint64_t)(head_dim * 2), (cuuint64_t)row_stride_bytes};
  cuuint32_t box[3] = {(cuuint32_t)box_inner, 1u, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NVKV_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " +
                                        std::to_string((int)r) + ")");
  return NVKV_OK;
}

int encode_kv_tensor_map_u8(CUtensorMap* map, const void* base, int64_t row_bytes,
                            int64_t num_heads, int64_t num_rows, int64_t row_stride_bytes,
                            int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  int rc = get_encoder(&encode);
  if (rc) return rc;
  // dim0 = the head's bytes (contiguous), dim1 = heads, dim2 = rows (slots)
  cuuint64_t dims[3] = {(cuuint64_t)row_bytes, (cuuint64_t)num_heads, (cuuint64_t)num_rows};
  cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)row_stride_bytes};
  cuuint32_t box[3] = {(cuuint32_t)row_bytes, 1u, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NVKV_ERR_CUDA, "cuTensorMapEncodeTiled (u8) failed (code " +
                                        std::to_string((int)r) + ")");
  return NVKV_OK;
}

}  // namespace nvkv

extern "C" {

int nvkv_version(void) {
  nvkv::clear_error();
  return 100;
}

const char* nvkv_last_error(void) { return nvkv::g_last_error.c_str(); }

int nvkv_device_error(int* code, int clear) {
  if (!code) return nvkv::set_error(NVKV_ERR_INVALID_ARG, "nvkv_device_error: null code");
  int* p = nvkv::device_error_word();
  if (!p) return nvkv::set_error(NVKV_ERR_CUDA, "device error word unavailable");
  int v = 0;
  int rc = nvkv::check_cuda(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost),
                            "nvkv_device_error: read");
  if (rc) return rc;
  *code = v;
  if (clear && v) {
    int z = 0;
    rc = nvkv::check_cuda(cudaMemcpy(p, &z, sizeof(int), cudaMemcpyHostToDevice),
                          "nvkv_device_error: clear");
    if (rc) return rc;
  }
  return NVKV_OK;
}

}  // extern "C"
