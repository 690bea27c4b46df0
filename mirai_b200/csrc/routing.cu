// a1 router top-k, a2 dispatch plan, a3 permute, a8 combine.
//
// These are HBM-bound integer / byte-movement kernels: coalesced 16-byte row
// traffic, warp-level reductions, no tensor cores.
#include "common.cuh"

namespace mirai {

// ============================================================================
// a1: router top-k, one warp per token.  Lane l holds experts l, l+32, ...
// ============================================================================
constexpr int kRouteMaxPerLane = 32;  // E <= 1024

template <int PER_LANE>
__global__ void __launch_bounds__(256) route_topk_kernel(const float* __restrict__ logits, int64_t T, int E,
                                                         int k, int score_func,
                                                         const float* __restrict__ bias_rows, int64_t bias_period,
                                                         int norm_mode, float route_scale,
                                                         int64_t* __restrict__ out_idx, float* __restrict__ out_w) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (t >= T) return;
  const float* row = logits + t * E;
  // bias row of this token: rows of `bias_period` tokens share one (MAGI-2: one per head)
  const float* bias = bias_rows ? bias_rows + (t / bias_period) * E : nullptr;
  float lg[PER_LANE], sc[PER_LANE], ch[PER_LANE];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = lane + 32 * i;
    lg[i] = e < E ? row[e] : -INFINITY;
    mx = fmaxf(mx, lg[i]);
  }
  if (score_func == MIRAI_SCORE_SOFTMAX) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      const int e = lane + 32 * i;
      sc[i] = e < E ? expf(lg[i] - mx) : 0.f;
      sum += sc[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) sc[i] = sc[i] / sum;
  } else {
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) sc[i] = 1.f / (1.f + expf(-lg[i]));
  }
  // Choice key: with a bias the reference ranks score + bias; without one,
  // softmax ranks the logits (same order, free of exp rounding ties) and
  // sigmoid ranks the scores.
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = lane + 32 * i;
    float c;
    if (bias) c = sc[i] + bias[e < E ? e : 0];
    else c = score_func == MIRAI_SCORE_SOFTMAX ? lg[i] : sc[i];
    // a NaN key ranks last (as -inf, lowest id first), so every slot gets a
    // valid expert id even for a row of NaN logits
    ch[i] = (e < E && !isnan(c)) ? c : -INFINITY;
  }
  float wsel[16];
  int isel[16];
  float wsum = 0.f;
  uint32_t taken = 0;  // bit i: expert lane + 32 i already selected
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((taken >> i) & 1u) && (ch[i] > best || (ch[i] == best && e < bi))) {
        best = ch[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    // owner lane removes the winner and publishes its score
    float w = 0.f;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      if (lane + 32 * i == bi) {
        w = sc[i];
        taken |= 1u << i;
      }
    }
    w = __shfl_sync(0xffffffffu, w, bi & 31);
    wsel[j] = w;
    isel[j] = bi;
    wsum += w;
  }
  if (lane == 0) {
    float scale = 1.f;
    bool divide = false;
    float den = 1.f;
    if (norm_mode == MIRAI_NORM_CLAMP) {
      den = fmaxf(wsum, 1e-20f);
      divide = true;
    } else if (norm_mode == MIRAI_NORM_EPS) {
      if (k > 1) {
        den = wsum + 1e-20f;
        divide = true;
      }
      scale = route_scale;
    } else if (norm_mode == MIRAI_NORM_L1) {
      float asum = 0.f;  // F.normalize(p=1, eps=1e-12): w / max(sum |w|, eps)
      for (int j = 0; j < k; ++j) asum += fabsf(wsel[j]);
      den = fmaxf(asum, 1e-12f);
      divide = true;
      scale = route_scale;
    } else {
      scale = route_scale;  // MIRAI_NORM_NONE: the gathered scores times route_scale
    }
    for (int j = 0; j < k; ++j) {
      float w = divide ? wsel[j] / den : wsel[j];
      if (norm_mode != MIRAI_NORM_CLAMP) w = w * scale;
      out_idx[t * k + j] = isel[j];
      out_w[t * k + j] = w;
    }
  }
}

// ============================================================================
// a2: dispatch plan.  Three passes over S = T*k flat routes, chunked by
// kPlanChunk.  (1) per-chunk expert histogram; (2) per expert, exclusive scan
// over chunks plus the segment starts; (3) per chunk, stable rank of every
// route among the routes of its expert (earlier chunks, earlier warps of this
// chunk, lower lanes of this warp) -> sorted position.  No atomics decide an
// order, so the result is deterministic and equals a stable argsort.
// ============================================================================
constexpr int kPlanThreads = 256;
constexpr int kPlanRounds = 8;
constexpr int kPlanChunk = kPlanThreads * kPlanRounds;  // 2048 routes per chunk
// Up to 4096 groups (MAGI-2 flattens heads x experts: 12 x 256 = 3072).  The
// per-chunk histograms live in dynamic shared memory sized by E.
constexpr int kPlanMaxExperts = 4096;
constexpr int kPlanWarps = 8;  // kPlanThreads / 32
inline size_t plan_hist_smem(int E) { return (size_t)E * sizeof(int); }
inline size_t plan_scatter_smem(int E) { return (size_t)(1 + kPlanWarps) * E * sizeof(int); }

// Range check shared by every dispatch-plan entry point, made before any size
// is computed from the arguments: nullptr when they are usable, else why not.
// T*k must fit the plan's int32 row offsets, so T is bounded by INT32_MAX / k
// before the product is formed (no int64 overflow for any T).
inline const char* plan_sizes_problem(int64_t num_tokens, int32_t top_k, int32_t num_experts) {
  if (top_k <= 0) return "top_k must be positive";
  if (num_experts <= 0 || num_experts > kPlanMaxExperts) return "expert count outside [1, 4096]";
  if (num_tokens < 0) return "negative token count";
  if (num_tokens > (int64_t)INT32_MAX / top_k) return "T*k exceeds the int32 range of the plan";
  return nullptr;
}

__global__ void __launch_bounds__(kPlanThreads) plan_histogram_kernel(const int64_t* __restrict__ idx,
                                                                      int64_t S, int E,
                                                                      int* __restrict__ chunk_counts) {
  extern __shared__ int hist[];  // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kPlanChunk;
  for (int r = 0; r < kPlanRounds; ++r) {
    const int64_t p = base + r * kPlanThreads + threadIdx.x;
    if (p < S) {
      const int64_t e = idx[p];
      if (e < 0 || e >= E) device_fail(MIRAI_ERR_DEVICE_BOUNDS, 100);
      else atomicAdd(&hist[e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_counts[(int64_t)blockIdx.x * E + e] = hist[e];
}

// (2a) one warp per expert: exclusive scan of its per-chunk counts, in place.
__global__ void __launch_bounds__(256) plan_chunk_scan_kernel(int* __restrict__ chunk_counts, int num_chunks, int E,
                                                              int64_t* __restrict__ counts) {
  const int lane = threadIdx.x & 31;
  const int e = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (e >= E) return;
  int carry = 0;
  for (int c0 = 0; c0 < num_chunks; c0 += 32) {
    const int c = c0 + lane;
    const int v = c < num_chunks ? chunk_counts[(int64_t)c * E + e] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (c < num_chunks) chunk_counts[(int64_t)c * E + e] = carry + incl - v;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) counts[e] = carry;
}

// (2b) one block: exclusive scan of the expert totals -> starts, offsets.
// Thread i owns experts [i*PER, (i+1)*PER) (PER = ceil(E / 1024) <= 4).
__global__ void __launch_bounds__(1024) plan_expert_scan_kernel(const int64_t* __restrict__ counts, int E,
                                                                int64_t* __restrict__ starts,
                                                                int32_t* __restrict__ offsets) {
  __shared__ int64_t warp_sums[32];
  const int per = (E + 1023) / 1024;
  const int e0 = threadIdx.x * per;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t v = 0;
  for (int i = 0; i < per; ++i)
    if (e0 + i < E) v += counts[e0 + i];
  int64_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int64_t ws = (lane < (int)(blockDim.x >> 5)) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t n = __shfl_up_sync(0xffffffffu, ws, o);
      if (lane >= o) ws += n;
    }
    warp_sums[lane] = ws;
  }
  __syncthreads();
  int64_t run = (warp > 0 ? warp_sums[warp - 1] : 0) + incl - v;
  for (int i = 0; i < per; ++i) {
    const int e = e0 + i;
    if (e >= E) break;
    starts[e] = run;
    run += counts[e];
    offsets[e] = (int32_t)run;
  }
}

__global__ void __launch_bounds__(kPlanThreads) plan_scatter_kernel(
    const int64_t* __restrict__ idx, int64_t S, int E, int k, const int* __restrict__ chunk_base,
    const int64_t* __restrict__ starts,
    int64_t* __restrict__ sort_positions, int64_t* __restrict__ sorted_tok, int64_t* __restrict__ inverse) {
  constexpr int kWarps = kPlanWarps;
  static_assert(kWarps * 32 == kPlanThreads, "one histogram row per warp");
  extern __shared__ int plan_smem[];  // running [E], then kWarps rows of [E]
  int* running = plan_smem;
  auto warp_hist = [&](int w, int e) -> int& { return plan_smem[(1 + w) * E + e]; };
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    running[e] = (int)starts[e] + chunk_base[(int64_t)blockIdx.x * E + e];
  const int64_t base = (int64_t)blockIdx.x * kPlanChunk;
  for (int r = 0; r < kPlanRounds; ++r) {
    for (int i = threadIdx.x; i < kWarps * E; i += blockDim.x) plan_smem[E + i] = 0;
    __syncthreads();
    const int64_t p = base + r * kPlanThreads + threadIdx.x;
    const bool valid = p < S;
    int e = valid ? (int)idx[p] : -1;
    if (e < 0 || e >= E) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
    const int leader = __ffs(peers) - 1;
    if (e >= 0 && lane == leader) warp_hist(warp, e) = __popc(peers);
    __syncthreads();
    if (e >= 0) {
      int pos = running[e] + rank_in_warp;
      for (int w = 0; w < warp; ++w) pos += warp_hist(w, e);
      sort_positions[pos] = p;
      sorted_tok[pos] = p / k;
      inverse[p] = pos;
    }
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
      int add = 0;
      for (int w = 0; w < kWarps; ++w) add += warp_hist(w, ee);
      running[ee] += add;
    }
    __syncthreads();
  }
}

// ============================================================================
// a3: permute rows (bf16), one warp per routed row, 16-byte vectors.
// ============================================================================
__global__ void __launch_bounds__(256) permute_rows_kernel(const uint4* __restrict__ tokens,
                                                           const int64_t* __restrict__ src_rows, int64_t S,
                                                           int vec_per_row, int64_t T,
                                                           uint4* __restrict__ routed) {
  const int lane = threadIdx.x & 31;
  const int64_t s = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (s >= S) return;
  const int64_t src = src_rows[s];
  if (src < 0 || src >= T) {
    if (lane == 0) device_fail(MIRAI_ERR_DEVICE_BOUNDS, 300);
    return;
  }
  const uint4* in = tokens + src * vec_per_row;
  uint4* out = routed + s * vec_per_row;
  for (int v = lane; v < vec_per_row; v += 32) out[v] = __ldg(in + v);
}

// ============================================================================
// a8: combine.  One warp per token; fp32 sum over the token's k routes in
// ascending sorted position, then a single rounding to the output type.
// ============================================================================
constexpr int kMaxTopK = 16;

__device__ __forceinline__ float bf16r_(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(256) combine_kernel(const uint4* __restrict__ y, const int64_t* __restrict__ inv,
                                                      const float* __restrict__ w, int64_t T, int k, int H,
                                                      int64_t S, void* __restrict__ out, int out_dtype) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (t >= T) return;
  int64_t pos[kMaxTopK];
  float wt[kMaxTopK];
  for (int j = 0; j < k; ++j) {
    pos[j] = inv[t * k + j];
    wt[j] = w ? w[t * k + j] : 1.f;
    if (pos[j] < 0 || pos[j] >= S) {
      if (lane == 0) device_fail(MIRAI_ERR_DEVICE_BOUNDS, 800);
      return;
    }
  }
  // insertion sort of (pos, weight) by position; k <= 16
  for (int a = 1; a < k; ++a) {
    const int64_t p = pos[a];
    const float ww = wt[a];
    int b = a - 1;
    while (b >= 0 && pos[b] > p) {
      pos[b + 1] = pos[b];
      wt[b + 1] = wt[b];
      --b;
    }
    pos[b + 1] = p;
    wt[b + 1] = ww;
  }
  const int vec_per_row = H / 8;
  for (int v = lane; v < vec_per_row; v += 32) {
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    for (int j = 0; j < k; ++j) {
      const uint4 u = __ldg(y + pos[j] * vec_per_row + v);
      const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
      if (out_dtype == MIRAI_COMBINE_BF16_ACCUM) {
        // bf16 tensors throughout: bf16(y * bf16(w)) added into a bf16 running sum
        const float wb = bf16r_(wt[j]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] = bf16r_(acc[2 * q] + bf16r_(bf16_lo(wd[q]) * wb));
          acc[2 * q + 1] = bf16r_(acc[2 * q + 1] + bf16r_(bf16_hi(wd[q]) * wb));
        }
        continue;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] = __fadd_rn(acc[2 * q], __fmul_rn(bf16_lo(wd[q]), wt[j]));
        acc[2 * q + 1] = __fadd_rn(acc[2 * q + 1], __fmul_rn(bf16_hi(wd[q]), wt[j]));
      }
    }
    if (out_dtype != MIRAI_DTYPE_F32) {
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(out)[t * vec_per_row + v] = o;
    } else {
      float4* o = reinterpret_cast<float4*>(out) + (t * vec_per_row + v) * 2;
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

// ============================================================================
// a8 backward: one warp per token.  grad_y rows are written in place of the
// token's routes; the score gradient is an fp32 dot product per route.
// ============================================================================
__global__ void __launch_bounds__(256) combine_backward_kernel(const uint4* __restrict__ g, const uint4* __restrict__ y,
                                                               const int64_t* __restrict__ inv,
                                                               const float* __restrict__ w, int64_t T, int k, int H,
                                                               int64_t S, uint4* __restrict__ gy,
                                                               float* __restrict__ gw) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int vec_per_row = H / 8;
  for (int j = 0; j < k; ++j) {
    const int64_t pos = inv[t * k + j];
    if (pos < 0 || pos >= S) {
      if (lane == 0) device_fail(MIRAI_ERR_DEVICE_BOUNDS, 810);
      return;
    }
    const float wt = w[t * k + j];
    float dot = 0.f;
    for (int v = lane; v < vec_per_row; v += 32) {
      const uint4 gu = __ldg(g + t * vec_per_row + v);
      const uint4 yu = __ldg(y + pos * vec_per_row + v);
      const uint32_t gw4[4] = {gu.x, gu.y, gu.z, gu.w};
      const uint32_t yw4[4] = {yu.x, yu.y, yu.z, yu.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float g0 = bf16_lo(gw4[q]), g1 = bf16_hi(gw4[q]);
        dot = fmaf(g0, bf16_lo(yw4[q]), dot);
        dot = fmaf(g1, bf16_hi(yw4[q]), dot);
        o[q] = pack_bf16x2(g0 * wt, g1 * wt);
      }
      gy[pos * vec_per_row + v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    if (lane == 0) gw[t * k + j] = dot;
  }
}

}  // namespace mirai

using namespace mirai;

static inline bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

extern "C" {

static int route_topk_impl(const char* name, const float* logits, int64_t num_tokens, int32_t num_experts,
                           int32_t top_k, int32_t score_func, const float* bias, int64_t bias_period,
                           int32_t norm_mode, float route_scale, int64_t* top_indices, float* top_weights,
                           mirai_stream_t stream) {
  if (num_tokens < 0 || num_experts <= 0 || num_experts > 1024 || top_k <= 0 || top_k > num_experts ||
      top_k > 16)
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: need 0 < k <= min(E, 16), E <= 1024 (E=%d, k=%d)", name,
                     num_experts, top_k);
  if (score_func != MIRAI_SCORE_SOFTMAX && score_func != MIRAI_SCORE_SIGMOID)
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: unknown score_func %d", name, score_func);
  if (norm_mode < MIRAI_NORM_NONE || norm_mode > MIRAI_NORM_L1)
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: unknown norm_mode %d", name, norm_mode);
  if (bias && bias_period <= 0) return set_error(MIRAI_ERR_INVALID_ARG, "%s: bias period must be positive", name);
  if (num_tokens == 0) return MIRAI_OK;
  if (!logits || !top_indices || !top_weights) return set_error(MIRAI_ERR_INVALID_ARG, "%s: null pointer", name);
  const int blocks = (int)((num_tokens + 7) / 8);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int per_lane = (num_experts + 31) / 32;
  const int64_t period = bias ? bias_period : 1;
#define MIRAI_ROUTE_LAUNCH(P)                                                                                  \
  route_topk_kernel<P><<<blocks, 256, 0, s>>>(logits, num_tokens, num_experts, top_k, score_func, bias, period, \
                                              norm_mode, route_scale, top_indices, top_weights)
  if (per_lane <= 1) MIRAI_ROUTE_LAUNCH(1);
  else if (per_lane <= 2) MIRAI_ROUTE_LAUNCH(2);
  else if (per_lane <= 4) MIRAI_ROUTE_LAUNCH(4);
  else if (per_lane <= 8) MIRAI_ROUTE_LAUNCH(8);
  else if (per_lane <= 16) MIRAI_ROUTE_LAUNCH(16);
  else MIRAI_ROUTE_LAUNCH(32);
#undef MIRAI_ROUTE_LAUNCH
  return check_launch(name);
}

int mirai_route_topk(const float* logits, int64_t num_tokens, int32_t num_experts, int32_t top_k,
                     int32_t score_func, const float* choice_bias, int32_t norm_mode, float route_scale,
                     int64_t* top_indices, float* top_weights, mirai_stream_t stream) {
  return route_topk_impl("route_topk", logits, num_tokens, num_experts, top_k, score_func, choice_bias,
                         num_tokens > 0 ? num_tokens : 1, norm_mode, route_scale, top_indices, top_weights, stream);
}

int mirai_route_topk_rows(const float* logits, int64_t num_tokens, int32_t num_experts, int32_t top_k,
                          int32_t score_func, const float* bias_rows, int64_t bias_period, int32_t norm_mode,
                          float route_scale, int64_t* top_indices, float* top_weights, mirai_stream_t stream) {
  return route_topk_impl("route_topk_rows", logits, num_tokens, num_experts, top_k, score_func, bias_rows,
                         bias_period, norm_mode, route_scale, top_indices, top_weights, stream);
}

size_t mirai_dispatch_plan_workspace_bytes(int64_t num_tokens, int32_t top_k, int32_t num_experts) {
  if (num_tokens <= 0 || mirai::plan_sizes_problem(num_tokens, top_k, num_experts) != nullptr) return 0;
  const int64_t S = num_tokens * top_k;
  const int64_t chunks = (S + kPlanChunk - 1) / kPlanChunk;
  return (size_t)(chunks * num_experts * sizeof(int));
}

int mirai_dispatch_plan(const int64_t* top_indices, int64_t num_tokens, int32_t top_k, int32_t num_experts,
                        int64_t* counts, int64_t* starts, int32_t* offsets, int64_t* sort_positions,
                        int64_t* sorted_token_indices, int64_t* inverse_order, void* workspace,
                        size_t workspace_bytes, mirai_stream_t stream) {
  if (const char* why = mirai::plan_sizes_problem(num_tokens, top_k, num_experts))
    return set_error(MIRAI_ERR_INVALID_ARG, "dispatch_plan: %s (T=%lld, k=%d, E=%d)", why, (long long)num_tokens,
                     top_k, num_experts);
  const int64_t S = num_tokens * top_k;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (!counts || !starts || !offsets) return set_error(MIRAI_ERR_INVALID_ARG, "dispatch_plan: null pointer");
  if (S == 0) {
    cudaMemsetAsync(counts, 0, sizeof(int64_t) * num_experts, s);
    cudaMemsetAsync(starts, 0, sizeof(int64_t) * num_experts, s);
    cudaMemsetAsync(offsets, 0, sizeof(int32_t) * num_experts, s);
    return check_launch("dispatch_plan(empty)", 0);  // memsets only
  }
  if (!top_indices || !sort_positions || !sorted_token_indices || !inverse_order)
    return set_error(MIRAI_ERR_INVALID_ARG, "dispatch_plan: null pointer");
  const size_t need = mirai_dispatch_plan_workspace_bytes(num_tokens, top_k, num_experts);
  if (!workspace || workspace_bytes < need)
    return set_error(MIRAI_ERR_WORKSPACE, "dispatch_plan: workspace of %zu bytes needed, %zu given", need,
                     workspace_bytes);
  const int chunks = (int)((S + kPlanChunk - 1) / kPlanChunk);
  int* cc = static_cast<int*>(workspace);
  static bool smem_attr = false;  // the scatter's histograms exceed 48 KB above 1365 experts
  if (!smem_attr) {
    cudaError_t e = cudaFuncSetAttribute(plan_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)plan_scatter_smem(kPlanMaxExperts));
    if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "dispatch_plan: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    smem_attr = true;
  }
  plan_histogram_kernel<<<chunks, kPlanThreads, plan_hist_smem(num_experts), s>>>(top_indices, S, num_experts, cc);
  plan_chunk_scan_kernel<<<(num_experts + 7) / 8, 256, 0, s>>>(cc, chunks, num_experts, counts);
  plan_expert_scan_kernel<<<1, 1024, 0, s>>>(counts, num_experts, starts, offsets);
  plan_scatter_kernel<<<chunks, kPlanThreads, plan_scatter_smem(num_experts), s>>>(
      top_indices, S, num_experts, top_k, cc, starts, sort_positions, sorted_token_indices, inverse_order);
  return check_launch("dispatch_plan", 4);
}

int mirai_permute_rows_bf16(const void* tokens, int64_t num_tokens, const int64_t* sorted_token_indices,
                            int64_t num_rows, int32_t hidden, void* routed, mirai_stream_t stream) {
  if (num_rows < 0 || hidden <= 0 || hidden % 8 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "permute_rows: hidden must be a positive multiple of 8");
  if (num_rows == 0) return MIRAI_OK;
  if (!tokens || !sorted_token_indices || !routed || misaligned16(tokens) || misaligned16(routed))
    return set_error(MIRAI_ERR_INVALID_ARG, "permute_rows: null or misaligned pointer");
  const int blocks = (int)((num_rows + 7) / 8);
  permute_rows_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(tokens), sorted_token_indices, num_rows, hidden / 8, num_tokens,
      static_cast<uint4*>(routed));
  return check_launch("permute_rows");
}

int mirai_moe_combine(const void* y_sorted, const int64_t* inverse_order, const float* top_weights,
                      int64_t num_tokens, int32_t top_k, int32_t hidden, void* out, int32_t out_dtype,
                      mirai_stream_t stream) {
  if (num_tokens < 0 || top_k <= 0 || top_k > kMaxTopK || hidden <= 0 || hidden % 8 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "combine: need 0 < k <= %d and hidden %% 8 == 0", kMaxTopK);
  if (out_dtype != MIRAI_DTYPE_BF16 && out_dtype != MIRAI_DTYPE_F32 && out_dtype != MIRAI_COMBINE_BF16_ACCUM)
    return set_error(MIRAI_ERR_INVALID_ARG, "combine: unknown out_dtype %d", out_dtype);
  if (num_tokens == 0) return MIRAI_OK;
  if (!y_sorted || !inverse_order || !out || misaligned16(y_sorted) || misaligned16(out))
    return set_error(MIRAI_ERR_INVALID_ARG, "combine: null or misaligned pointer");
  const int blocks = (int)((num_tokens + 7) / 8);
  combine_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(y_sorted), inverse_order, top_weights, num_tokens, top_k, hidden,
      num_tokens * top_k, out, out_dtype);
  return check_launch("combine");
}

int mirai_moe_combine_backward(const void* grad_out, const void* y_sorted, const int64_t* inverse_order,
                               const float* top_weights, int64_t num_tokens, int32_t top_k, int32_t hidden,
                               void* grad_y_sorted, float* grad_weights, mirai_stream_t stream) {
  if (num_tokens < 0 || top_k <= 0 || top_k > kMaxTopK || hidden <= 0 || hidden % 8 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "combine_backward: need 0 < k <= %d and hidden %% 8 == 0", kMaxTopK);
  if (num_tokens == 0) return MIRAI_OK;
  if (!grad_out || !y_sorted || !inverse_order || !top_weights || !grad_y_sorted || !grad_weights ||
      misaligned16(grad_out) || misaligned16(y_sorted) || misaligned16(grad_y_sorted))
    return set_error(MIRAI_ERR_INVALID_ARG, "combine_backward: null or misaligned pointer");
  const int blocks = (int)((num_tokens + 7) / 8);
  combine_backward_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(grad_out), static_cast<const uint4*>(y_sorted), inverse_order, top_weights,
      num_tokens, top_k, hidden, num_tokens * top_k, static_cast<uint4*>(grad_y_sorted), grad_weights);
  return check_launch("combine_backward");
}

}  // extern "C"
