// Dispatch plan without caller-provided scratch.
//
// mirai_dispatch_plan needs a device workspace (per-chunk expert counts) that
// the caller allocates.  Some callers cannot allocate at the moment they plan:
// a host binding that is handed only the routing tensors and the output
// buffers (a C/Go/JNI caller with no device allocator of its own), or code that
// must not grow device memory between a memory-budget check and the launch.
// mirai_dispatch_plan_static serves them: the scratch is one fixed array in
// the library's device image, sized kPlanStaticScratchBytes, and the same plan
// kernels run on it.  Nothing here calls cudaMalloc / cudaFree or any library
// that allocates.
//
// Rules that follow from one shared array per device:
//  * nothing in it has to start at zero: every entry a call reads was written
//    earlier by the same call (the histogram pass writes all chunk x expert
//    counts before the scan reads them);
//  * two calls that can run at the same time on one device (different streams
//    or threads without ordering) race on the array and corrupt each other's
//    plans; calls on one stream are ordered and safe;
//  * the first call on each device looks the array's address up
//    (cudaGetSymbolAddress, which can load the module); make that first call
//    outside any stream capture;
//  * with lazy module loading (the CUDA default) the library's device image,
//    this 1 MiB array included, is loaded by the first library call on a
//    device, which can grow device memory once: make one library call on each
//    device before a memory-budget check that must stay true until the launch.
#include <mutex>

#include "common.cuh"

namespace mirai {

// chunks x experts int32 counts: 1 MiB covers e.g. E = 128 experts up to
// 4,194,304 routes (T*k), or E = 32 up to 16,777,216.
constexpr size_t kPlanStaticScratchBytes = (size_t)1 << 20;
constexpr int kPlanStaticMaxDevices = 64;

static __device__ __align__(256) int g_plan_static_scratch[kPlanStaticScratchBytes / sizeof(int)];

// Device address of g_plan_static_scratch in the current device's context,
// looked up once per device.
static int plan_static_scratch(void** out) {
  static std::mutex mu;
  static void* addr[kPlanStaticMaxDevices] = {};
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "dispatch_plan_static: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kPlanStaticMaxDevices)
    return set_error(MIRAI_ERR_UNSUPPORTED, "dispatch_plan_static: device ordinal %d >= %d", dev,
                     kPlanStaticMaxDevices);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_plan_static_scratch);
    if (e != cudaSuccess || !p)
      return set_error(MIRAI_ERR_CUDA, "dispatch_plan_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return MIRAI_OK;
}

}  // namespace mirai

extern "C" {

size_t mirai_dispatch_plan_static_scratch_bytes(void) { return mirai::kPlanStaticScratchBytes; }

int mirai_dispatch_plan_static(const int64_t* top_indices, int64_t num_tokens, int32_t top_k, int32_t num_experts,
                               int64_t* counts, int64_t* starts, int32_t* offsets, int64_t* sort_positions,
                               int64_t* sorted_token_indices, int64_t* inverse_order, mirai_stream_t stream) {
  // arguments first, so that an unusable plan is reported as such and not as a scratch shortfall
  if (const char* why = mirai::plan_sizes_problem(num_tokens, top_k, num_experts))
    return mirai::set_error(MIRAI_ERR_INVALID_ARG, "dispatch_plan_static: %s (T=%lld, k=%d, E=%d)", why,
                            (long long)num_tokens, top_k, num_experts);
  const size_t need = mirai_dispatch_plan_workspace_bytes(num_tokens, top_k, num_experts);
  if (need > mirai::kPlanStaticScratchBytes)
    return mirai::set_error(MIRAI_ERR_WORKSPACE,
                            "dispatch_plan_static: %lld routes x %d experts need %zu bytes of scratch, the fixed "
                            "array holds %zu; use mirai_dispatch_plan with a workspace",
                            (long long)num_tokens * top_k, num_experts, need, mirai::kPlanStaticScratchBytes);
  void* scratch = nullptr;
  const int rc = mirai::plan_static_scratch(&scratch);
  if (rc != MIRAI_OK) return rc;
  return mirai_dispatch_plan(top_indices, num_tokens, top_k, num_experts, counts, starts, offsets, sort_positions,
                             sorted_token_indices, inverse_order, scratch, mirai::kPlanStaticScratchBytes, stream);
}

}  // extern "C"
