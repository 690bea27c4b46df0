/*
 * mirai_b200_noalloc.h -- dispatch plan for callers that cannot allocate.
 *
 * No counterpart in the reference: its dispatch plan (build_dispatch_plan,
 * dispatch_preprocess.py:128-179) is torch code that allocates as it goes.
 *
 * mirai_dispatch_plan (mirai_b200.h) needs a device workspace of
 * mirai_dispatch_plan_workspace_bytes() that the caller provides.  A caller
 * with no device allocator at hand when it plans -- a C / Go / JNI binding
 * that is given only the routing tensors and the output buffers, or code that
 * must not grow device memory between a memory-budget check and the launch --
 * uses mirai_dispatch_plan_static instead.  It produces exactly the same six
 * outputs; its scratch is one fixed array of
 * mirai_dispatch_plan_static_scratch_bytes() (1 MiB) inside the library's
 * device image, one per device, and it allocates nothing.
 *
 * Limits and rules:
 *   - a plan whose mirai_dispatch_plan_workspace_bytes() exceeds the fixed
 *     array (1 MiB: e.g. more than 4,194,304 routes T*k at 128 experts, or
 *     16,777,216 at 32) is rejected with MIRAI_ERR_WORKSPACE and a message
 *     naming both sizes; nothing is launched;
 *   - nothing in the array has to start at zero: each call writes every entry
 *     it later reads;
 *   - calls that may run at the same time on one device (different streams or
 *     threads without ordering between them) share the array and race; calls
 *     on one stream are ordered and safe;
 *   - the first call on each device looks up the array's address
 *     (cudaGetSymbolAddress, which can load the module): make that first call
 *     outside any stream capture;
 *   - under lazy module loading (the CUDA default) the first call into this
 *     library on a device loads its device image, the 1 MiB array included,
 *     which can grow device memory once: make one library call on each device
 *     before a memory-budget check that must hold until the launch;
 *   - arguments are range-checked before any size is derived from them: a bad
 *     T, k or E is MIRAI_ERR_INVALID_ARG, never MIRAI_ERR_WORKSPACE.
 */
#ifndef MIRAI_B200_NOALLOC_H_
#define MIRAI_B200_NOALLOC_H_

#include "mirai_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Size in bytes of the fixed scratch array (the largest plan workspace
 * mirai_dispatch_plan_static accepts). */
size_t mirai_dispatch_plan_static_scratch_bytes(void);

/* Same arguments and outputs as mirai_dispatch_plan, minus the workspace. */
int mirai_dispatch_plan_static(const int64_t* top_indices, int64_t num_tokens, int32_t top_k,
                               int32_t num_experts, int64_t* counts, int64_t* starts, int32_t* offsets,
                               int64_t* sort_positions, int64_t* sorted_token_indices,
                               int64_t* inverse_order, mirai_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MIRAI_B200_NOALLOC_H_ */
