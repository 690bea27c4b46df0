/*
 * mirai_b200.h -- C ABI of the B200 (sm_100a) sparse-MoE expert FFN path.
 *
 * This library replaces the routed expert FFN of seruva19/mirai: fp32 router
 * top-k, expert-contiguous token permute, SwiGLU gate/up and down grouped GEMMs
 * over frozen bf16 / NF4 / INT8 expert weights, the weighted un-permute
 * (combine), and the input-gradient (dX) path through the frozen experts.
 *
 * Conventions shared by every entry point:
 *   - all data pointers are CUDA device pointers, except where noted;
 *   - every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *     default stream) and never synchronises the host;
 *   - nothing in this library allocates device memory: callers pass outputs
 *     and, where needed, a workspace sized by the matching *_workspace_bytes();
 *   - the return value is MIRAI_OK (0) or a MIRAI_ERR_* code; the message of
 *     the last failure on the calling thread is mirai_b200_last_error();
 *   - kernels never trap.  A device-side bound check or a bounded wait that
 *     gives up records a code that mirai_b200_device_status() returns.
 *
 * Weight layouts are the reference's (w1/w3 [E, I, H], w2 [E, H, I], out x in,
 * transformer_lingbot_video.py:1143-1145), stored as the reference's
 * CompressedGroupedExperts buffers (experts.py:998-1031, 1382-1470).
 */
#ifndef MIRAI_B200_H_
#define MIRAI_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* mirai_stream_t; /* identical to cudaStream_t */

enum {
  MIRAI_OK = 0,
  MIRAI_ERR_INVALID_ARG = 1,    /* bad pointer, size, dtype or alignment */
  MIRAI_ERR_UNSUPPORTED = 2,    /* shape outside what the kernels tile */
  MIRAI_ERR_CUDA = 3,           /* a CUDA runtime / driver call failed */
  MIRAI_ERR_DEVICE_TIMEOUT = 4, /* a device-side wait reached its time limit */
  MIRAI_ERR_DEVICE_BOUNDS = 5,  /* a device-side index check failed */
  MIRAI_ERR_WORKSPACE = 6       /* workspace missing or too small */
};

/* Score function and renormalisation of mirai_route_topk. */
enum { MIRAI_SCORE_SOFTMAX = 0, MIRAI_SCORE_SIGMOID = 1 };
enum {
  MIRAI_NORM_NONE = 0,  /* weights = gathered scores * route_scale                     */
  MIRAI_NORM_CLAMP = 1, /* w / clamp_min(sum w, 1e-20)       (routers.py:248)          */
  MIRAI_NORM_EPS = 2,   /* w / (sum w + 1e-20) if k > 1, then * route_scale
                           (transformer_lingbot_video.py:1031-1033)                   */
  MIRAI_NORM_L1 = 3     /* w / max(sum |w|, 1e-12), then * route_scale (MAGI-2:
                           F.normalize(p=1), flash_mh_moe/route.py:144-145, and the
                           route_scale of magi2_preview.py:2742)                      */
};

/* Output element type selector.  MIRAI_COMBINE_BF16_ACCUM (combine only):
 * bf16 output summed in bf16, out = bf16(out + bf16(y * bf16(w))) route by
 * route in ascending sorted position -- MAGI-2's weighted index_add on bf16
 * tensors (grouped_moe.py:751-756). */
enum { MIRAI_DTYPE_BF16 = 0, MIRAI_DTYPE_F32 = 1, MIRAI_COMBINE_BF16_ACCUM = 2 };

/* Expert weight layouts of the *_ex GEMMs: [G, out, in] (the compressed
 * experts', w1/w3 [E, I, H], w2 [E, H, I]) or [G, in, out] (MAGI-2's W_gate /
 * W_up [heads*E, d_head, d_expert], W_down [heads*E, d_expert, d_head],
 * magi2_preview.py:2686-2709; NF4 blocks along each stored row). */
enum { MIRAI_LAYOUT_OUT_IN = 0, MIRAI_LAYOUT_IN_OUT = 1 };
/* Gate/up activations: SwiGLU silu(g) * u (experts.py:301-317), or MAGI-2's
 * swiglu7 min(g,7) sigmoid(1.702 min(g,7)) (clamp(u,-7,7) + 1) computed in fp32
 * on the bf16 gate/up (grouped_moe.py:287-335). */
enum { MIRAI_ACT_SWIGLU = 0, MIRAI_ACT_SWIGLU7 = 1 };

/* Frozen NF4 expert tensor as stored by the reference for one key
 * (CompressedGroupedExperts._store_nf4_grouped, experts.py:998-1031;
 * load_nf4_packed_weight, experts.py:1424-1470).  Blocks of `blocksize`
 * consecutive elements of each expert's row-major [out, in] matrix share one
 * scale; two codes per byte, the first element in the high nibble. */
typedef struct mirai_nf4_weight {
  const uint8_t* packed;      /* {key}_nf4          [E, out*in/2]                     */
  const uint8_t* absmax;      /* {key}_nf4_absmax   [E, out*in/blocksize] 8-bit codes */
  const float* nested_absmax; /* {key}_nf4_nabsmax  [E, n_nested] fp32                */
  const float* offset;        /* {key}_nf4_offset   [E] fp32                          */
  const float* code;          /* {key}_nf4_code     [16] fp32 NF4 values              */
  const float* nested_code;   /* {key}_nf4_ncode    [256] fp32 absmax code map         */
  int32_t blocksize;          /* 64                                                   */
  int32_t nested_blocksize;   /* 256                                                  */
} mirai_nf4_weight;

/* Frozen INT8 expert tensor (quant.py:189-235 with group_size = 0, i.e. plain
 * per-output-channel symmetric; load_quantized_weight, experts.py:1382-1422). */
typedef struct mirai_int8_weight {
  const int8_t* q;    /* {key}_int8  [E, out, in]  */
  const float* scale; /* {key}_scale [E, out, 1]   */
} mirai_int8_weight;

/* ----------------------------------------------------------------- library */
const char* mirai_b200_last_error(void);
int mirai_b200_version(void);
/* Kernels this library has enqueued since it was loaded (every entry point,
 * all devices and streams): lets a caller count the launches of a region. */
uint64_t mirai_b200_launch_count(void);
/* Synchronises `stream`, then returns (and clears) the device error word:
 * *code = 0 or a MIRAI_ERR_DEVICE_* code, *info = where it was raised. */
int mirai_b200_device_status(mirai_stream_t stream, int* code, int* info);
/* Caps the SMs the persistent grouped GEMMs occupy (0 = all SMs, the default),
 * process-wide, for launches made after the call.  A GEMM otherwise holds
 * every SM for its whole duration; leaving a few free lets communication
 * kernels on another stream (an expert-parallel all-to-all) run alongside it.
 * No reference counterpart: the reference has no expert parallelism. */
int mirai_b200_set_gemm_sm_limit(int32_t max_sms);

/* Peer buffers for the expert-parallel exchange (one process per GPU).  No
 * reference counterpart.  mirai_ipc_export gives the 64-byte CUDA IPC handle of
 * the allocation holding `ptr` and ptr's byte offset in it; another process
 * maps it into its own device's context with mirai_ipc_import (peer access
 * over NVLink, no context on the exporting GPU) and unmaps it with
 * mirai_ipc_release(base).  mirai_copy_async is one cudaMemcpyAsync (a
 * copy-engine transfer, also between a local and a mapped peer pointer) on
 * `stream`.  The exporter keeps the memory alive while peers map it. */
int mirai_ipc_export(const void* ptr, void* handle, uint64_t* offset);
int mirai_ipc_import(const void* handle, uint64_t offset, void** ptr, void** base);
int mirai_ipc_release(void* base);
int mirai_copy_async(void* dst, const void* src, uint64_t bytes, mirai_stream_t stream);
/* `count` such copies, block i from src[i] to dst[i] of bytes[i] bytes (host
 * arrays of device addresses), issued in order on `stream`, one
 * cudaMemcpyAsync each; zero-byte blocks are skipped. */
int mirai_copy_blocks(int32_t count, const uint64_t* dst, const uint64_t* src, const uint64_t* bytes,
                      mirai_stream_t stream);
/* Arrival flags of that exchange: mirai_ep_signal stores `epoch` (release,
 * system scope) into each of `count` 8-byte slots given by device pointers
 * (a rank's slot in every peer's flag array; NULL entries skipped), after the
 * work already on `stream`; mirai_ep_wait holds `stream` until flags[i] >=
 * epoch for every i < count except `skip`.  The wait gives up after 2 s and
 * records MIRAI_ERR_DEVICE_TIMEOUT (mirai_b200_device_status). */
int mirai_ep_signal(void* const* peer_slots, int32_t count, uint64_t epoch, mirai_stream_t stream);
int mirai_ep_wait(const uint64_t* flags, int32_t count, int32_t skip, uint64_t epoch, mirai_stream_t stream);

/* ------------------------------------------------------------ a1: router top-k
 * Replaces TokenChoiceRouter.forward's selection (routers.py:241-249) and the
 * LingBot router's (transformer_lingbot_video.py:1002-1033) on fp32 logits
 * [T, E] (E <= 1024, 1 <= k <= min(E, 16)).  Choice scores are
 * `score + choice_bias` (bias may be NULL); slots come out in descending choice
 * order, ties to the lower expert id.  Weights are fp32 [T, k]. */
int mirai_route_topk(const float* logits, int64_t num_tokens, int32_t num_experts, int32_t top_k,
                     int32_t score_func, const float* choice_bias, int32_t norm_mode,
                     float route_scale, int64_t* top_indices, float* top_weights,
                     mirai_stream_t stream);

/* The same with one bias row per `bias_period` consecutive tokens: token t
 * ranks score + bias_rows[(t / bias_period) * E + e].  MAGI-2 routes every
 * head over its own experts with its own expert_bias row
 * (compute_topk_probs_and_indices, flash_mh_moe/route.py:157-199; logits
 * [heads, S, E] as heads * S rows, bias [heads, E], bias_period = S). */
int mirai_route_topk_rows(const float* logits, int64_t num_tokens, int32_t num_experts, int32_t top_k,
                          int32_t score_func, const float* bias_rows, int64_t bias_period, int32_t norm_mode,
                          float route_scale, int64_t* top_indices, float* top_weights, mirai_stream_t stream);

/* -------------------------------------------------------- a2: dispatch plan
 * Replaces build_dispatch_plan (dispatch_preprocess.py:128-179): stable sort of
 * the flat [T*k] expert ids, bincount, cumsum, inverse permutation.  Outputs:
 * counts/starts int64 [E], offsets int32 [E] (inclusive), sort_positions,
 * sorted_token_indices, inverse_order int64 [T*k].  Deterministic.
 * E <= 4096 (MAGI-2's flattened heads x experts groups included). */
size_t mirai_dispatch_plan_workspace_bytes(int64_t num_tokens, int32_t top_k, int32_t num_experts);
int mirai_dispatch_plan(const int64_t* top_indices, int64_t num_tokens, int32_t top_k,
                        int32_t num_experts, int64_t* counts, int64_t* starts, int32_t* offsets,
                        int64_t* sort_positions, int64_t* sorted_token_indices,
                        int64_t* inverse_order, void* workspace, size_t workspace_bytes,
                        mirai_stream_t stream);

/* ------------------------------------------------------------- a3: permute
 * routed[s, :] = tokens[sorted_token_indices[s], :] for bf16 rows, tokens
 * [num_tokens, hidden] (permute_routed_tokens, dispatch_ops.py:8-20;
 * experts.py:2399-2421). */
int mirai_permute_rows_bf16(const void* tokens, int64_t num_tokens, const int64_t* sorted_token_indices,
                            int64_t num_rows, int32_t hidden, void* routed, mirai_stream_t stream);

/* --------------------------------------- a6: gate/up grouped GEMM + SwiGLU
 * For every expert segment of the expert-contiguous rows x_sorted [S, H]
 * (segment e = rows [offsets[e-1], offsets[e])):
 *   h = silu(x W1[e]^T) * (x W3[e]^T)                       -> h [S, I] bf16
 * Replaces _FrozenDequantBatchedLinearPair.forward + silu*up (linear.py:166-189,
 * experts.py:301-317).  `gate_up` (nullable) receives the pre-activation
 * [S, 2I] bf16 (gate | up) that the dX path consumes.  Requires H % 64 == 0,
 * I % 64 == 0. */
int mirai_moe_gateup_swiglu_bf16(const void* x_sorted, const int32_t* offsets, int32_t num_experts,
                                 int64_t num_rows, int32_t hidden, int32_t inter, const void* w1,
                                 const void* w3, void* h, void* gate_up, mirai_stream_t stream);
int mirai_moe_gateup_swiglu_nf4(const void* x_sorted, const int32_t* offsets, int32_t num_experts,
                                int64_t num_rows, int32_t hidden, int32_t inter,
                                const mirai_nf4_weight* w1, const mirai_nf4_weight* w3, void* h,
                                void* gate_up, mirai_stream_t stream);
int mirai_moe_gateup_swiglu_int8(const void* x_sorted, const int32_t* offsets, int32_t num_experts,
                                 int64_t num_rows, int32_t hidden, int32_t inter,
                                 const mirai_int8_weight* w1, const mirai_int8_weight* w3, void* h,
                                 void* gate_up, mirai_stream_t stream);

/* ------------------------------------------------- a7: down grouped GEMM
 * y[s, :] = h[s, :] W2[e]^T for the rows of segment e -> y [S, H] bf16
 * (_FrozenDequantBatchedLinear.forward, linear.py:95-114).  Requires
 * I % 64 == 0, H % 64 == 0. */
int mirai_moe_down_bf16(const void* h, const int32_t* offsets, int32_t num_experts,
                        int64_t num_rows, int32_t inter, int32_t hidden, const void* w2, void* y,
                        mirai_stream_t stream);
int mirai_moe_down_nf4(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                       int32_t inter, int32_t hidden, const mirai_nf4_weight* w2, void* y,
                       mirai_stream_t stream);
int mirai_moe_down_int8(const void* h, const int32_t* offsets, int32_t num_experts,
                        int64_t num_rows, int32_t inter, int32_t hidden,
                        const mirai_int8_weight* w2, void* y, mirai_stream_t stream);

/* --------------------------- a6 / a7 over source-major segments (expert parallel)
 * The same two GEMMs when the rows of each expert come in num_sources separate
 * runs, as an expert owner receives them from its peers: `offsets` holds the
 * inclusive ends of num_sources * num_experts segments in memory order, segment
 * s * num_experts + e being source s's rows for (weight) expert e.  Each
 * segment is cut into 128-row blocks and an expert's blocks, of any sources, are
 * paired into 256-row tiles (one per SM of a CTA pair), so a source boundary
 * wastes at most part of a block; tiles visit the experts in order, so the
 * weights of one expert stay hot in L2.  No
 * reference counterpart (the reference has no expert parallelism); with
 * num_sources = 1 these equal the entry points above. */
int mirai_moe_gateup_swiglu_src_bf16(const void* x, const int32_t* offsets, int32_t num_sources,
                                     int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter,
                                     const void* w1, const void* w3, void* h, void* gate_up,
                                     mirai_stream_t stream);
int mirai_moe_gateup_swiglu_src_nf4(const void* x, const int32_t* offsets, int32_t num_sources,
                                    int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter,
                                    const mirai_nf4_weight* w1, const mirai_nf4_weight* w3, void* h,
                                    void* gate_up, mirai_stream_t stream);
int mirai_moe_gateup_swiglu_src_int8(const void* x, const int32_t* offsets, int32_t num_sources,
                                     int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter,
                                     const mirai_int8_weight* w1, const mirai_int8_weight* w3, void* h,
                                     void* gate_up, mirai_stream_t stream);
int mirai_moe_down_src_bf16(const void* h, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                            int64_t num_rows, int32_t inter, int32_t hidden, const void* w2, void* y,
                            mirai_stream_t stream);
int mirai_moe_down_src_nf4(const void* h, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                           int64_t num_rows, int32_t inter, int32_t hidden, const mirai_nf4_weight* w2, void* y,
                           mirai_stream_t stream);
int mirai_moe_down_src_int8(const void* h, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                            int64_t num_rows, int32_t inter, int32_t hidden, const mirai_int8_weight* w2,
                            void* y, mirai_stream_t stream);

/* The dX GEMMs over source-major segments (an expert owner's share of the
 * expert-parallel backward: gradient rows arrive as the forward's rows did).
 * down_dx_src with gate_up == NULL writes dh = dy W2 [S, I] (no SwiGLU
 * backward; the block-Hadamard INT8 format rotates dh first). */
int mirai_moe_down_dx_src_bf16(const void* grad_y, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                               int64_t num_rows, int32_t hidden, int32_t inter, const void* w2, const void* gate_up,
                               void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_down_dx_src_nf4(const void* grad_y, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                              int64_t num_rows, int32_t hidden, int32_t inter, const mirai_nf4_weight* w2,
                              const void* gate_up, void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_down_dx_src_int8(const void* grad_y, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                               int64_t num_rows, int32_t hidden, int32_t inter, const mirai_int8_weight* w2,
                               const void* gate_up, void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_gateup_dx_src_bf16(const void* grad_gate_up, const int32_t* offsets, int32_t num_sources,
                                 int32_t num_experts, int64_t num_rows, int32_t inter, int32_t hidden,
                                 const void* w1, const void* w3, void* dx_sorted, mirai_stream_t stream);
int mirai_moe_gateup_dx_src_nf4(const void* grad_gate_up, const int32_t* offsets, int32_t num_sources,
                                int32_t num_experts, int64_t num_rows, int32_t inter, int32_t hidden,
                                const mirai_nf4_weight* w1, const mirai_nf4_weight* w3, void* dx_sorted,
                                mirai_stream_t stream);
int mirai_moe_gateup_dx_src_int8(const void* grad_gate_up, const int32_t* offsets, int32_t num_sources,
                                 int32_t num_experts, int64_t num_rows, int32_t inter, int32_t hidden,
                                 const mirai_int8_weight* w1, const mirai_int8_weight* w3, void* dx_sorted,
                                 mirai_stream_t stream);

/* ------------------------------------------------------------- a8: combine
 * out[t, :] = sum_j top_weights[t, j] * y[inverse_order[t*k + j], :], summed in
 * fp32 in ascending sorted position (the order of the reference's
 * output.index_add_, experts.py:2433-2437), then cast to out_dtype.
 * (combine_routed_tokens, dispatch_ops.py:23-44.)  With top_weights == NULL
 * every weight is 1: the un-permute sum that is the permute backward
 * (_PermuteRoutedTokens.backward, dispatch_ops.py:15-20). */
int mirai_moe_combine(const void* y_sorted, const int64_t* inverse_order, const float* top_weights,
                      int64_t num_tokens, int32_t top_k, int32_t hidden, void* out,
                      int32_t out_dtype, mirai_stream_t stream);

/* ---------------------------------------------------- a8 backward: combine
 * _CombineRoutedTokens.backward (dispatch_ops.py:36-44) for the bf16 path:
 *   grad_y[s, :]     = bf16( grad_out[t, :] * w[t, j] )     s = inverse_order[t*k + j]
 *   grad_weights[t,j] = sum_h grad_out[t, h] * y[s, h]      (fp32)
 * grad_out is bf16 [T, H]; y_sorted / grad_y_sorted bf16 [S, H]. */
int mirai_moe_combine_backward(const void* grad_out, const void* y_sorted, const int64_t* inverse_order,
                               const float* top_weights, int64_t num_tokens, int32_t top_k, int32_t hidden,
                               void* grad_y_sorted, float* grad_weights, mirai_stream_t stream);

/* ------------------------------------ a9: dX through the frozen experts
 * Down projection backward fused with the SwiGLU backward
 * (_FrozenDequantBatchedLinear.backward, linear.py:116-125, then autograd of
 * silu(gate) * up, experts.py:301-317):
 *   dh = bf16(grad_y W2[e])                                 (K = H, N = I)
 *   dgate = bf16(silu'(gate) * bf16(dh * up)), dup = bf16(dh * bf16(silu(gate)))
 * gate_up is the [S, 2I] bf16 (gate | up) saved by the forward; the result
 * grad_gate_up is [S, 2I] bf16 (dgate | dup).  Requires H, I % 64 == 0. */
int mirai_moe_down_dx_bf16(const void* grad_y, const int32_t* offsets, int32_t num_experts,
                           int64_t num_rows, int32_t hidden, int32_t inter, const void* w2,
                           const void* gate_up, void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_down_dx_nf4(const void* grad_y, const int32_t* offsets, int32_t num_experts,
                          int64_t num_rows, int32_t hidden, int32_t inter, const mirai_nf4_weight* w2,
                          const void* gate_up, void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_down_dx_int8(const void* grad_y, const int32_t* offsets, int32_t num_experts,
                           int64_t num_rows, int32_t hidden, int32_t inter, const mirai_int8_weight* w2,
                           const void* gate_up, void* grad_gate_up, mirai_stream_t stream);

/* Gate/up projection backward (_FrozenDequantBatchedLinearPair.backward,
 * linear.py:191-203): dx_sorted = dgate W1[e] + dup W3[e], one fp32
 * accumulation over K = 2I, rounded once to bf16 [S, H]. */
int mirai_moe_gateup_dx_bf16(const void* grad_gate_up, const int32_t* offsets, int32_t num_experts,
                             int64_t num_rows, int32_t inter, int32_t hidden, const void* w1,
                             const void* w3, void* dx_sorted, mirai_stream_t stream);
int mirai_moe_gateup_dx_nf4(const void* grad_gate_up, const int32_t* offsets, int32_t num_experts,
                            int64_t num_rows, int32_t inter, int32_t hidden, const mirai_nf4_weight* w1,
                            const mirai_nf4_weight* w3, void* dx_sorted, mirai_stream_t stream);
int mirai_moe_gateup_dx_int8(const void* grad_gate_up, const int32_t* offsets, int32_t num_experts,
                             int64_t num_rows, int32_t inter, int32_t hidden, const mirai_int8_weight* w1,
                             const mirai_int8_weight* w3, void* dx_sorted, mirai_stream_t stream);

/* ------------------------------------------- a10: LoRA on the down projection
 * ActiveExpertLoRA.batched_subset_forward (active_expert_lora.py:434-478):
 * y += scale * (h A_e^T) B_e^T with A [E, r, I], B [E, H, r] (r <= 32), fused
 * into the down GEMMs as one extra 64-wide k-block.
 *
 * mirai_moe_lora_project writes the rank-block operand
 *   out[s, j] = bf16(scale * sum_k x[s, k] * F_e[j, k])  (j < rank; 0 for rank <= j < 64)
 * as [S, 64] bf16 for the rows s of every expert segment e, from the adapter
 * factor zero-padded to 64 ranks (bf16) in one of two layouts:
 *   MIRAI_LORA_FACTOR_ROWS: [E*64, K], F_e[j, k] at row e*64+j (A padded: the
 *     forward projection, x = h, K = I);
 *   MIRAI_LORA_FACTOR_COLS: [E*K, 64], F_e[j, k] at row e*K+k (B padded, the
 *     operand mirai_moe_down_lora_* takes: the dX projection, x = grad_y, K = H).
 * K % 8 == 0, out 16-byte aligned. */
#define MIRAI_LORA_FACTOR_ROWS 0
#define MIRAI_LORA_FACTOR_COLS 1
int mirai_moe_lora_project(const void* x, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                           int32_t k_dim, const void* factor, int32_t factor_layout, int32_t rank, float scale,
                           void* out, mirai_stream_t stream);

/* Adapter-factor gradient (the LoRA weight gradients of bmm's backward in
 * batched_subset_forward): grad[e][j][k] = sum over the rows s of segment e of
 * g_rank[s, j] * x[s, k], fp32 (tensor cores, one accumulator per expert and
 * 128 columns, rows summed in order: deterministic).
 * g_rank is a [S, 64] bf16 rank-block operand (already scaled); grad element
 * (e, j, k) is stored at grad[e*stride_e + j*stride_r + k*stride_k]:
 * dA = lora_grad(h, grad-side rank block) into [E, r, I];
 * dB = lora_grad(grad_y, forward rank block) into [E, H, r]. */
int mirai_moe_lora_grad(const void* x, const void* g_rank, const int32_t* offsets, int32_t num_experts,
                        int64_t num_rows, int32_t k_dim, int32_t rank, float* grad, int64_t stride_e,
                        int64_t stride_r, int64_t stride_k, mirai_stream_t stream);

/* Down GEMM plus the rank block: y = h W2^T + rank_a rank_b_e^T, with rank_a the
 * [S, 64] projection of h and rank_b = B zero-padded to [E*H, 64] bf16. */
int mirai_moe_down_lora_bf16(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                             int32_t inter, int32_t hidden, const void* w2, const void* rank_a,
                             const void* rank_b, void* y, mirai_stream_t stream);
int mirai_moe_down_lora_nf4(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                            int32_t inter, int32_t hidden, const mirai_nf4_weight* w2, const void* rank_a,
                            const void* rank_b, void* y, mirai_stream_t stream);
int mirai_moe_down_lora_int8(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                             int32_t inter, int32_t hidden, const mirai_int8_weight* w2, const void* rank_a,
                             const void* rank_b, void* y, mirai_stream_t stream);

/* Down dX plus the rank block: dh = grad_y W2 + rank_a rank_b_e, with rank_a the
 * [S, 64] projection of grad_y through B (times scale) and rank_b = A
 * zero-padded to [E*64, I] bf16; the SwiGLU backward is fused as in
 * mirai_moe_down_dx_*. */
int mirai_moe_down_dx_lora_bf16(const void* grad_y, const int32_t* offsets, int32_t num_experts,
                                int64_t num_rows, int32_t hidden, int32_t inter, const void* w2,
                                const void* gate_up, const void* rank_a, const void* rank_b,
                                void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_down_dx_lora_nf4(const void* grad_y, const int32_t* offsets, int32_t num_experts,
                               int64_t num_rows, int32_t hidden, int32_t inter, const mirai_nf4_weight* w2,
                               const void* gate_up, const void* rank_a, const void* rank_b,
                               void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_down_dx_lora_int8(const void* grad_y, const int32_t* offsets, int32_t num_experts,
                                int64_t num_rows, int32_t hidden, int32_t inter, const mirai_int8_weight* w2,
                                const void* gate_up, const void* rank_a, const void* rank_b,
                                void* grad_gate_up, mirai_stream_t stream);

/* The LoRA kernels and the fused rank-block GEMMs over source-major segments
 * (no counterpart: the reference has no expert parallelism).  offsets holds
 * num_sources * num_experts running ends, segment s*E + e = source s's rows of
 * expert e (the layout an expert owner receives); num_sources = 1 is the
 * entry point without _src.  At most 1024 segments and 64 sources.  A factor
 * gradient sums each expert's segments in source order. */
int mirai_moe_lora_project_src(const void* x, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                               int64_t num_rows, int32_t k_dim, const void* factor, int32_t factor_layout,
                               int32_t rank, float scale, void* out, mirai_stream_t stream);
int mirai_moe_lora_grad_src(const void* x, const void* g_rank, const int32_t* offsets, int32_t num_sources,
                            int32_t num_experts, int64_t num_rows, int32_t k_dim, int32_t rank, float* grad,
                            int64_t stride_e, int64_t stride_r, int64_t stride_k, mirai_stream_t stream);
int mirai_moe_down_lora_src_bf16(const void* h, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                                 int64_t num_rows, int32_t inter, int32_t hidden, const void* w2,
                                 const void* rank_a, const void* rank_b, void* y, mirai_stream_t stream);
int mirai_moe_down_lora_src_nf4(const void* h, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                                int64_t num_rows, int32_t inter, int32_t hidden, const mirai_nf4_weight* w2,
                                const void* rank_a, const void* rank_b, void* y, mirai_stream_t stream);
int mirai_moe_down_lora_src_int8(const void* h, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                                 int64_t num_rows, int32_t inter, int32_t hidden, const mirai_int8_weight* w2,
                                 const void* rank_a, const void* rank_b, void* y, mirai_stream_t stream);
/* gate_up == NULL: dh = grad_y W2 + the rank block, [S, I], without the SwiGLU backward */
int mirai_moe_down_dx_lora_src_bf16(const void* grad_y, const int32_t* offsets, int32_t num_sources,
                                    int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter,
                                    const void* w2, const void* gate_up, const void* rank_a, const void* rank_b,
                                    void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_down_dx_lora_src_nf4(const void* grad_y, const int32_t* offsets, int32_t num_sources,
                                   int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter,
                                   const mirai_nf4_weight* w2, const void* gate_up, const void* rank_a,
                                   const void* rank_b, void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_down_dx_lora_src_int8(const void* grad_y, const int32_t* offsets, int32_t num_sources,
                                    int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter,
                                    const mirai_int8_weight* w2, const void* gate_up, const void* rank_a,
                                    const void* rank_b, void* grad_gate_up, mirai_stream_t stream);

/* ------------------------------- f4: any weight layout, activation, group count
 * The four grouped GEMMs (gate/up + activation, down, down dX with the
 * activation's backward, gate/up dX) for weights in either layout above and
 * any number of groups (more than 1024 run as consecutive launches of 1024
 * groups).  MAGI-2's multi-head grouped MoE (grouped_moe.py:583-757) flattens
 * (head, expert) into heads * E groups over (token, head) rows of d_head
 * features: hidden = d_head, inter = d_expert.  Replaces its grouped matmul
 * roles (_grouped_linear / _grouped_linear_dx, grouped_moe.py:206-284, over
 * gemm.py:359-367,433-482 segments) and the swiglu7 forward / backward.
 * bf16 and NF4 weights; the [G, in, out] layout needs CTA pairs (the default). */
int mirai_moe_gateup_ex_bf16(const void* x_sorted, const int32_t* offsets, int32_t num_groups, int64_t num_rows,
                             int32_t hidden, int32_t inter, const void* w1, const void* w3, int32_t layout,
                             int32_t activation, void* h, void* gate_up, mirai_stream_t stream);
int mirai_moe_gateup_ex_nf4(const void* x_sorted, const int32_t* offsets, int32_t num_groups, int64_t num_rows,
                            int32_t hidden, int32_t inter, const mirai_nf4_weight* w1, const mirai_nf4_weight* w3,
                            int32_t layout, int32_t activation, void* h, void* gate_up, mirai_stream_t stream);
int mirai_moe_down_ex_bf16(const void* h, const int32_t* offsets, int32_t num_groups, int64_t num_rows,
                           int32_t inter, int32_t hidden, const void* w2, int32_t layout, void* y,
                           mirai_stream_t stream);
int mirai_moe_down_ex_nf4(const void* h, const int32_t* offsets, int32_t num_groups, int64_t num_rows,
                          int32_t inter, int32_t hidden, const mirai_nf4_weight* w2, int32_t layout, void* y,
                          mirai_stream_t stream);
int mirai_moe_down_dx_ex_bf16(const void* grad_y, const int32_t* offsets, int32_t num_groups, int64_t num_rows,
                              int32_t hidden, int32_t inter, const void* w2, int32_t layout, int32_t activation,
                              const void* gate_up, void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_down_dx_ex_nf4(const void* grad_y, const int32_t* offsets, int32_t num_groups, int64_t num_rows,
                             int32_t hidden, int32_t inter, const mirai_nf4_weight* w2, int32_t layout,
                             int32_t activation, const void* gate_up, void* grad_gate_up, mirai_stream_t stream);
int mirai_moe_gateup_dx_ex_bf16(const void* grad_gate_up, const int32_t* offsets, int32_t num_groups,
                                int64_t num_rows, int32_t inter, int32_t hidden, const void* w1, const void* w3,
                                int32_t layout, void* dx_sorted, mirai_stream_t stream);
int mirai_moe_gateup_dx_ex_nf4(const void* grad_gate_up, const int32_t* offsets, int32_t num_groups,
                               int64_t num_rows, int32_t inter, int32_t hidden, const mirai_nf4_weight* w1,
                               const mirai_nf4_weight* w3, int32_t layout, void* dx_sorted, mirai_stream_t stream);

/* --------------------------------------------------- a4 / a5: weight ingest
 * NF4 quantisation of a bf16 [E, out, in] expert stack into the reference's
 * per-expert buffers (CompressedGroupedExperts._store_nf4_grouped,
 * experts.py:998-1031, which calls bitsandbytes quantize_4bit with
 * blocksize 64 and compress_statistics=True, quant.py:315-358):
 * packed [E, out*in/2], absmax codes [E, out*in/64], nested_absmax
 * [E, ceil(out*in/64/nested_blocksize)], offset [E].  `code` (16) and
 * `nested_code` (256) are the NF4 and dynamic-map tables to quantise against.
 * The workspace holds the fp32 block absmax (size from the query). */
size_t mirai_nf4_quantize_workspace_bytes(int32_t num_experts, int64_t out_features, int64_t in_features);
int mirai_nf4_quantize(const void* weight_bf16, int32_t num_experts, int64_t out_features, int64_t in_features,
                       const float* code, const float* nested_code, int32_t blocksize, int32_t nested_blocksize,
                       uint8_t* packed, uint8_t* absmax, float* nested_absmax, float* offset, void* workspace,
                       size_t workspace_bytes, mirai_stream_t stream);

/* Per-output-channel symmetric INT8 of `rows` rows of `in_features`
 * (quant.py:189-235 with group_size 0): scale = max(amax/127, 1e-30),
 * q = clamp(round_half_even(x / scale), -127, 127).  weight_dtype is
 * MIRAI_DTYPE_F32 or MIRAI_DTYPE_BF16.  The block-Hadamard format
 * (group_size > 0) quantises rows rotated first by mirai_rotate_rows. */
/* NF4 buffers of one key -> bf16 [E, out, in] (nf4_dequantize_stack, quant.py:380-434; the
 * chunked_dequant runner's per-chunk dequantisation, experts.py:2148-2240), bit-identical to
 * the grouped GEMMs' in-loop decode.  packed and out 16-byte aligned. */
int mirai_nf4_dequantize(const uint8_t* packed, const uint8_t* absmax, const float* nested_absmax,
                         const float* offset, const float* code, const float* nested_code, int32_t num_experts,
                         int64_t out_features, int64_t in_features, int32_t blocksize, int32_t nested_blocksize,
                         void* out_bf16, mirai_stream_t stream);
int mirai_int8_quantize_rows(const void* weight, int32_t weight_dtype, int64_t rows, int64_t in_features,
                             int8_t* q, float* scale, mirai_stream_t stream);

/* ------------------------------------- a5: the block-Hadamard INT8 format
 * The reference's default INT8 storage rotates each weight row's groups of g
 * input features (g = 4^m, the largest of 256/64/16 dividing in_features,
 * quant.py:87-91) by H = h4 (x) ... (x) h4 / sqrt(g) before quantising
 * (quant.py:103-122, 189-235), so q * s = W H, and de-rotates the weight before
 * each matmul (_dequantize_weight, quant.py:238-260).  H is symmetric and
 * orthogonal, so this library rotates activations instead
 * (rotated_int8.py:7-21) and runs the plain INT8 GEMMs on the stored codes:
 *   forward  y  = (x H) (q s)^T         rotate x (and h, for w2) first
 *   dX       dx = (dy (q s)) H          rotate the GEMM result after
 *
 * mirai_rotate_rows: out = in H along every g-wide group of the last dimension
 * of a row-major [rows, cols] matrix (cols % g == 0, cols % 16 == 0, g a power
 * of 4 in [4, 4096]), in fp32; in/out dtypes MIRAI_DTYPE_BF16 or _F32, 16-byte
 * aligned; out may equal in.  Replaces _rotate_last_dim (quant.py:152-182). */
int mirai_rotate_rows(const void* in, int32_t in_dtype, int64_t rows, int32_t cols, int32_t group, void* out,
                      int32_t out_dtype, mirai_stream_t stream);

/* The down projection's dX for the block-Hadamard format, in two steps:
 * mirai_moe_down_dh_int8[_lora] computes dh_raw = bf16(grad_y (q s))
 * [S, I] (+ rank_a rank_b_e, rank_b = A zero-padded to [E*64, I] AND rotated
 * by H, so that rotating the sum gives the adapter's exact contribution); then
 * mirai_swiglu_backward_rotated rotates dh_raw into dh = bf16(dh_raw H) and
 * applies the SwiGLU backward of mirai_moe_down_dx_* to the saved gate_up,
 * writing grad_gate_up [S, 2I].  (linear.py:116-125 with the de-rotated weight
 * of quant.py:238-260, then experts.py:301-317 autograd.) */
int mirai_moe_down_dh_int8(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                           int32_t hidden, int32_t inter, const mirai_int8_weight* w2, void* dh,
                           mirai_stream_t stream);
int mirai_moe_down_dh_lora_int8(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                int32_t hidden, int32_t inter, const mirai_int8_weight* w2, const void* rank_a,
                                const void* rank_b, void* dh, mirai_stream_t stream);
int mirai_swiglu_backward_rotated(const void* dh, const void* gate_up, int64_t rows, int32_t inter, int32_t group,
                                  void* grad_gate_up, mirai_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MIRAI_B200_H_ */
