// Library-wide state of the C ABI: last-error strings, the device error word,
// SM count, and the tensor-map encoder obtained from the driver.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "tmap.h"

namespace mirai {

static thread_local char t_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

// Kernels this library has enqueued since it was loaded (all devices and streams).
static std::atomic<unsigned long long> g_launches{0};

int check_launch(const char* what, int kernels) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  g_launches.fetch_add((unsigned long long)kernels, std::memory_order_relaxed);
  return MIRAI_OK;
}

// Upper bound on the SMs the persistent GEMMs occupy (0 = all).  Read at each
// launch; set by mirai_b200_set_gemm_sm_limit.
static int g_gemm_sm_limit = 0;

int gemm_sm_limit() { return g_gemm_sm_limit; }

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void* base,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encoder();
  if (!fn) return set_error(MIRAI_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "TMA base address %p is not 16-byte aligned", base);
  if (row_stride_bytes % 16 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "TMA row stride %llu is not a multiple of 16 bytes",
                     (unsigned long long)row_stride_bytes);
  if ((uint64_t)box_inner * elem_bytes % 16 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "TMA box inner extent is not a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(MIRAI_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for a [%llu x %llu] tensor", (int)r,
                     (unsigned long long)outer, (unsigned long long)inner);
  return MIRAI_OK;
}

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static AddressRangeFn address_range() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}

}  // namespace mirai

extern "C" {

const char* mirai_b200_last_error(void) { return mirai::t_last_error; }

int mirai_b200_version(void) { return 100; }

uint64_t mirai_b200_launch_count(void) { return mirai::g_launches.load(std::memory_order_relaxed); }

int mirai_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  if (!ptr || !handle || !offset) return mirai::set_error(MIRAI_ERR_INVALID_ARG, "ipc_export: null pointer");
  mirai::AddressRangeFn range = mirai::address_range();
  if (!range) return mirai::set_error(MIRAI_ERR_CUDA, "ipc_export: cuMemGetAddressRange is not available");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return mirai::set_error(MIRAI_ERR_INVALID_ARG, "ipc_export: %p is not device memory", ptr);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return mirai::set_error(MIRAI_ERR_CUDA, "ipc_export: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  *offset = (uint64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return MIRAI_OK;
}

int mirai_ipc_import(const void* handle, uint64_t offset, void** ptr, void** base) {
  if (!handle || !ptr || !base) return mirai::set_error(MIRAI_ERR_INVALID_ARG, "ipc_import: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return mirai::set_error(MIRAI_ERR_CUDA, "ipc_import: %s", cudaGetErrorString(e));
  *base = b;
  *ptr = static_cast<uint8_t*>(b) + offset;
  return MIRAI_OK;
}

int mirai_ipc_release(void* base) {
  if (!base) return MIRAI_OK;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return mirai::set_error(MIRAI_ERR_CUDA, "ipc_release: %s", cudaGetErrorString(e));
  return MIRAI_OK;
}

int mirai_copy_async(void* dst, const void* src, uint64_t bytes, mirai_stream_t stream) {
  if (bytes == 0) return MIRAI_OK;
  if (!dst || !src) return mirai::set_error(MIRAI_ERR_INVALID_ARG, "copy_async: null pointer");
  cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return mirai::set_error(MIRAI_ERR_CUDA, "copy_async: %s", cudaGetErrorString(e));
  return MIRAI_OK;
}

int mirai_copy_blocks(int32_t count, const uint64_t* dst, const uint64_t* src, const uint64_t* bytes,
                      mirai_stream_t stream) {
  if (count < 0 || (count > 0 && (!dst || !src || !bytes)))
    return mirai::set_error(MIRAI_ERR_INVALID_ARG, "copy_blocks: bad block list");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int32_t i = 0; i < count; ++i) {
    if (bytes[i] == 0) continue;
    if (!dst[i] || !src[i]) return mirai::set_error(MIRAI_ERR_INVALID_ARG, "copy_blocks: null address in block %d", i);
    cudaError_t e = cudaMemcpyAsync(reinterpret_cast<void*>(dst[i]), reinterpret_cast<const void*>(src[i]),
                                    (size_t)bytes[i], cudaMemcpyDefault, s);
    if (e != cudaSuccess)
      return mirai::set_error(MIRAI_ERR_CUDA, "copy_blocks: block %d: %s", i, cudaGetErrorString(e));
  }
  return MIRAI_OK;
}

int mirai_b200_set_gemm_sm_limit(int32_t max_sms) {
  if (max_sms < 0 || max_sms == 1)
    return mirai::set_error(MIRAI_ERR_INVALID_ARG, "set_gemm_sm_limit: %d (use 0 for no limit, or >= 2)", max_sms);
  mirai::g_gemm_sm_limit = max_sms;
  return MIRAI_OK;
}

int mirai_b200_device_status(mirai_stream_t stream, int* code, int* info) {
  if (!code || !info) return mirai::set_error(MIRAI_ERR_INVALID_ARG, "device_status: null output pointer");
  cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return mirai::set_error(MIRAI_ERR_CUDA, "device_status: %s", cudaGetErrorString(e));
  int zero = 0;
  e = cudaMemcpyFromSymbol(code, mirai::g_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(info, mirai::g_device_error_info, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(mirai::g_device_error, &zero, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(mirai::g_device_error_info, &zero, sizeof(int));
  if (e != cudaSuccess) return mirai::set_error(MIRAI_ERR_CUDA, "device_status: %s", cudaGetErrorString(e));
  return MIRAI_OK;
}

}  // extern "C"
