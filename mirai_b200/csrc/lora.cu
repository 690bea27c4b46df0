// a10: the low-rank projections of a LoRA adapter on the expert down
// projection (ActiveExpertLoRA.batched_subset_forward,
// active_expert_lora.py:434-478).  For every routed row s of expert e:
//   out[s, j] = bf16( scale * sum_k x[s, k] * P_e[j, k] )   j < rank,
//   out[s, j] = 0                                            rank <= j < 64,
// written as a [S, 64] bf16 operand that the grouped GEMMs consume as one
// extra 64-wide k-block (so the rank-r product is fused into the down GEMM and
// into the down dX GEMM).  P_e is addressed by strides, so the same kernel
// serves lora_a [E, r, I] (forward) and lora_b [E, H, r] read transposed (dX).
//
// Rows are tiled 64 per block within expert segments; the block stages P_e in
// shared memory (fp32) and each warp reduces 8 rows with 16-byte loads.
#include "common.cuh"

namespace mirai {
namespace lr {

constexpr int kRows = 64;      // rows per block
constexpr int kThreads = 256;  // 8 warps x 8 rows
constexpr int kMaxRank = 32;
constexpr int kMaxExperts = 1024;

template <int R>
__global__ void __launch_bounds__(kThreads) lora_project_kernel(
    const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ offsets, int E, int64_t S, int K,
    const __nv_bfloat16* __restrict__ P, int64_t sE, int64_t sJ, int64_t sK, int rank, float scale,
    __nv_bfloat16* __restrict__ out) {
  extern __shared__ float sp[];  // [R][K]
  __shared__ int tile_prefix[kMaxExperts + 1];
  __shared__ int row_start[kMaxExperts + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      int cnt = 0;
      if (e < E) {
        const int64_t end = offsets[e], beg = e > 0 ? offsets[e - 1] : 0;
        cnt = end > beg ? (int)((end - beg + kRows - 1) / kRows) : 0;
        row_start[e] = (int)beg;
      }
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (e < E) tile_prefix[e] = carry + incl - cnt;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      tile_prefix[E] = carry;
      row_start[E] = (int)(E > 0 ? offsets[E - 1] : 0);
    }
  }
  __syncthreads();
  const int t = blockIdx.x;
  if (t >= tile_prefix[E]) return;
  int lo = 0, hi = E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (tile_prefix[mid] <= t) lo = mid;
    else hi = mid;
  }
  const int e = lo;
  const int m = t - tile_prefix[e];
  const int64_t seg = (int64_t)row_start[e + 1] - row_start[e];
  // stage P_e as fp32 [R][K]; rows rank..R-1 are zero
  for (int i = threadIdx.x; i < R * K; i += kThreads) {
    const int j = i / K, k = i - j * K;
    sp[i] = j < rank ? __bfloat162float(P[e * sE + j * sJ + k * sK]) : 0.f;
  }
  __syncthreads();
  for (int rr = 0; rr < kRows / 8; ++rr) {
    const int local = m * kRows + warp * (kRows / 8) + rr;
    if (local >= seg) break;
    const int64_t s = (int64_t)row_start[e] + local;
    const uint4* xr = reinterpret_cast<const uint4*>(x + s * K);
    float acc[R];
#pragma unroll
    for (int j = 0; j < R; ++j) acc[j] = 0.f;
    for (int v = lane; v < K / 8; v += 32) {
      const uint4 u = __ldg(xr + v);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      float xv[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        xv[2 * q] = bf16_lo(w[q]);
        xv[2 * q + 1] = bf16_hi(w[q]);
      }
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const float4 p0 = *reinterpret_cast<const float4*>(sp + j * K + v * 8);
        const float4 p1 = *reinterpret_cast<const float4*>(sp + j * K + v * 8 + 4);
        acc[j] = fmaf(xv[0], p0.x, acc[j]);
        acc[j] = fmaf(xv[1], p0.y, acc[j]);
        acc[j] = fmaf(xv[2], p0.z, acc[j]);
        acc[j] = fmaf(xv[3], p0.w, acc[j]);
        acc[j] = fmaf(xv[4], p1.x, acc[j]);
        acc[j] = fmaf(xv[5], p1.y, acc[j]);
        acc[j] = fmaf(xv[6], p1.z, acc[j]);
        acc[j] = fmaf(xv[7], p1.w, acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < R; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    // lanes 0..31 write the 64-wide row as bf16 pairs
    __nv_bfloat16* orow = out + s * 64;
    float v0 = 0.f, v1 = 0.f;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      if (2 * lane == j) v0 = acc[j];
      if (2 * lane + 1 == j) v1 = acc[j];
    }
    reinterpret_cast<uint32_t*>(orow)[lane] = pack_bf16x2(v0 * scale, v1 * scale);
  }
}

// Adapter-factor gradient over one expert's rows:
//   grad[e][j][k] = sum_{s in segment e} g[s, j] * x[s, k]      (fp32, rows in order)
// One block per (expert, 256 columns of K); each thread owns one column and R
// accumulators; g rows are staged through shared memory 64 at a time.
template <int R>
__global__ void __launch_bounds__(256) lora_grad_kernel(const __nv_bfloat16* __restrict__ x,
                                                        const __nv_bfloat16* __restrict__ g,
                                                        const int32_t* __restrict__ offsets, int E, int K,
                                                        int rank, float* __restrict__ grad, int64_t sE,
                                                        int64_t sJ, int64_t sK) {
  __shared__ float gs[64][R];
  const int e = blockIdx.y;
  const int col = blockIdx.x * 256 + threadIdx.x;
  const int64_t beg = e > 0 ? offsets[e - 1] : 0;
  const int64_t end = offsets[e];
  float acc[R];
#pragma unroll
  for (int j = 0; j < R; ++j) acc[j] = 0.f;
  for (int64_t s0 = beg; s0 < end; s0 += 64) {
    const int n = (int)((end - s0) < 64 ? (end - s0) : 64);
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * R; i += 256) {
      const int rr = i / R, j = i % R;
      gs[rr][j] = (rr < n && j < rank) ? __bfloat162float(g[(s0 + rr) * 64 + j]) : 0.f;
    }
    __syncthreads();
    if (col < K) {
      for (int rr = 0; rr < n; ++rr) {
        const float xv = __bfloat162float(x[(s0 + rr) * K + col]);
#pragma unroll
        for (int j = 0; j < R; ++j) acc[j] = fmaf(gs[rr][j], xv, acc[j]);
      }
    }
  }
  if (col < K) {
    for (int j = 0; j < rank && j < R; ++j) grad[e * sE + j * sJ + (int64_t)col * sK] = acc[j];
  }
}

}  // namespace lr
}  // namespace mirai

using namespace mirai;

extern "C" {

int mirai_moe_lora_project(const void* x, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                           int32_t k_dim, const void* proj, int64_t stride_e, int64_t stride_r, int64_t stride_k,
                           int32_t rank, float scale, void* out, mirai_stream_t stream) {
  if (num_experts <= 0 || num_experts > lr::kMaxExperts || num_rows < 0 || k_dim <= 0 || k_dim % 8 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "lora_project: bad sizes (E=%d, K=%d)", num_experts, k_dim);
  if (rank <= 0 || rank > lr::kMaxRank)
    return set_error(MIRAI_ERR_UNSUPPORTED, "lora_project: rank %d outside 1..%d", rank, lr::kMaxRank);
  if (num_rows == 0) return MIRAI_OK;
  if (!x || !offsets || !proj || !out || (reinterpret_cast<uintptr_t>(x) & 15u))
    return set_error(MIRAI_ERR_INVALID_ARG, "lora_project: null or misaligned pointer");
  const int R = rank <= 8 ? 8 : (rank <= 16 ? 16 : 32);
  const size_t smem = (size_t)R * k_dim * sizeof(float);
  if (smem > 200 * 1024)
    return set_error(MIRAI_ERR_UNSUPPORTED, "lora_project: rank x K = %d x %d too large", R, k_dim);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the kernel writes all 64 columns (zeros past the rank) of every row it covers
  const int64_t max_tiles = (num_rows + lr::kRows - 1) / lr::kRows + num_experts;
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  const __nv_bfloat16* pb = static_cast<const __nv_bfloat16*>(proj);
  __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(out);
#define MIRAI_LORA_LAUNCH(RR)                                                                                     \
  do {                                                                                                            \
    auto kern = lr::lora_project_kernel<RR>;                                                                      \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                          \
    kern<<<(unsigned)max_tiles, lr::kThreads, smem, s>>>(xb, offsets, num_experts, num_rows, k_dim, pb, stride_e, \
                                                         stride_r, stride_k, rank, scale, ob);                   \
  } while (0)
  if (R == 8) MIRAI_LORA_LAUNCH(8);
  else if (R == 16) MIRAI_LORA_LAUNCH(16);
  else MIRAI_LORA_LAUNCH(32);
#undef MIRAI_LORA_LAUNCH
  return check_launch("lora_project");
}

int mirai_moe_lora_grad(const void* x, const void* g_rank, const int32_t* offsets, int32_t num_experts,
                        int64_t num_rows, int32_t k_dim, int32_t rank, float* grad, int64_t stride_e,
                        int64_t stride_r, int64_t stride_k, mirai_stream_t stream) {
  if (num_experts <= 0 || num_experts > lr::kMaxExperts || num_rows < 0 || k_dim <= 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "lora_grad: bad sizes (E=%d, K=%d)", num_experts, k_dim);
  if (rank <= 0 || rank > lr::kMaxRank)
    return set_error(MIRAI_ERR_UNSUPPORTED, "lora_grad: rank %d outside 1..%d", rank, lr::kMaxRank);
  if (!x || !g_rank || !offsets || !grad) return set_error(MIRAI_ERR_INVALID_ARG, "lora_grad: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((k_dim + 255) / 256), (unsigned)num_experts);
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  const __nv_bfloat16* gb = static_cast<const __nv_bfloat16*>(g_rank);
  if (rank <= 8)
    lr::lora_grad_kernel<8><<<grid, 256, 0, s>>>(xb, gb, offsets, num_experts, k_dim, rank, grad, stride_e,
                                                 stride_r, stride_k);
  else if (rank <= 16)
    lr::lora_grad_kernel<16><<<grid, 256, 0, s>>>(xb, gb, offsets, num_experts, k_dim, rank, grad, stride_e,
                                                  stride_r, stride_k);
  else
    lr::lora_grad_kernel<32><<<grid, 256, 0, s>>>(xb, gb, offsets, num_experts, k_dim, rank, grad, stride_e,
                                                  stride_r, stride_k);
  return check_launch("lora_grad");
}

}  // extern "C"
