// Library-wide C-ABI entry points and host helpers: status strings, the
// thread-local error message, device error bits, SM counts and TMA
// descriptor encoding.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "cie_common.cuh"
#include "cie_host.h"

namespace cie {

namespace {
thread_local char t_message[512] = "";

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_err = cudaSuccess;

constexpr int kMaxSmemSlots = 16;
bool g_smem_set[kMaxDevices][kMaxSmemSlots] = {};
std::mutex g_smem_mu;
}  // namespace

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_message, sizeof(t_message), fmt, ap);
  va_end(ap);
  return status;
}

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return dev;
}

int sm_count() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  });
  if (g_encode == nullptr)
    return fail(CIE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)",
                cudaGetErrorString(g_encode_err));
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, static_cast<cuuint32_t>(rank), base,
                        reinterpret_cast<const cuuint64_t*>(dims),
                        reinterpret_cast<const cuuint64_t*>(strides_bytes),
                        reinterpret_cast<const cuuint32_t*>(box), elem_strides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CIE_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CIE_OK;
}

int ensure_smem_attribute(const void* func, int bytes, int slot) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices || slot < 0 || slot >= kMaxSmemSlots) {
    cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    return e == cudaSuccess ? CIE_OK : fail(CIE_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  std::lock_guard<std::mutex> lk(g_smem_mu);
  if (!g_smem_set[dev][slot]) {
    cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    g_smem_set[dev][slot] = true;
  }
  return CIE_OK;
}

}  // namespace cie

extern "C" {

int cie_version(void) { return 1; }

const char* cie_status_string(int status) {
  switch (status) {
    case CIE_OK: return "ok";
    case CIE_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CIE_ERR_UNSUPPORTED: return "unsupported shape";
    case CIE_ERR_OVERFLOW: return "index overflow";
    case CIE_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case CIE_ERR_WORKSPACE: return "workspace missing or too small";
    case CIE_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* cie_last_error_message(void) { return cie::t_message; }

int cie_read_device_errors(int device, unsigned int* bits, int clear) {
  if (bits == nullptr) return cie::fail(CIE_ERR_INVALID_ARGUMENT, "bits is NULL");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  unsigned int v = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, cie::g_device_errors, sizeof(v));
  if (e == cudaSuccess && clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(cie::g_device_errors, &zero, sizeof(zero));
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cie::fail(CIE_ERR_CUDA, "reading device errors: %s", cudaGetErrorString(e));
  *bits = v;
  return CIE_OK;
}

}  // extern "C"
