// a10: the low-rank side of a LoRA adapter on the expert down projection
// (ActiveExpertLoRA.batched_subset_forward, active_expert_lora.py:434-478),
// on the tensor cores.  Both kernels stream one large bf16 activation
// ([S, K], read once from HBM) against a small 64-wide rank-block operand, so
// they are HBM-bound; tcgen05 keeps the arithmetic off the critical path.
//
// lora_project: for every routed row s of expert e
//   out[s, j] = bf16( scale * sum_k x[s, k] * F_e[j, k] ),   j < 64,
// with F the adapter factor zero-padded to 64 ranks, given either as rows
// ([E*64, K], row e*64+j: lora_a padded, K-major operand) or as columns
// ([E*K, 64], row e*K+k: lora_b padded, MN-major operand).  The [S, 64]
// result is the extra k-block the fused down / down-dX GEMMs consume.
// One CTA per 128-row tile of an expert segment: D[128 x 64] in TMEM,
// A = x tile (TMA, SW128 K-major), B = factor tile (TMA, SW128).
//
// lora_grad: grad[e][j][k] = sum over segment e of g[s, j] * x[s, k], fp32.
// Computed transposed, D[k][j] (M = 128 columns of x, N = 64 ranks), reducing
// over the segment's rows 64 at a time: A = x^T (MN-major, two 64-column TMA
// boxes), B = g (MN-major).  One CTA per (expert, 128 columns); rows past the
// segment's end in its last block are zeroed in shared memory before the MMA
// so the next expert's rows never enter the sum.  Blocks are summed in row
// order by one accumulator, so the result is deterministic.
//
// Both take the rows as `nsrc` x E segments (source-major: segment s*E + e
// holds source s's rows of expert e, the layout an expert owner receives in
// the expert-parallel exchange; nsrc = 1 is one segment per expert).  A
// gradient CTA walks its expert's segments in source order.
#include "common.cuh"

namespace mirai {
namespace lr {

constexpr int kMaxRank = 32;
constexpr int kMaxExperts = 1024;     // segments (sources x experts) of one launch
constexpr int kMaxSources = 64;
constexpr int kThreads = 128;         // 4 warps: TMA producer, MMA issuer, all four drain TMEM
constexpr int kStages = 4;
constexpr int kABytes = 128 * 64 * 2; // 16 KB: 128 rows x 64 k (project) / 2 x [64 rows x 64 cols] (grad)
constexpr int kBBytes = 64 * 64 * 2;  // 8 KB: one 64 x 64 rank-block tile
constexpr int kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 64;
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + 1024;  // + alignment slack

enum FactorLayout { kFactorRows = 0, kFactorCols = 1 };

struct Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t done;
  uint32_t tmem;
  int tile_e, tile_row0, tile_rows;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void init_barriers(Barriers& b) {
  for (int s = 0; s < kStages; ++s) {
    mbar_init(&b.full[s], 1);
    mbar_init(&b.empty[s], 1);
  }
  mbar_init(&b.done, 1);
  fence_mbar_init();
}

// Waits (bounded) for TMA copies a producer may still have in flight after a
// failed wait elsewhere, so no copy lands after the CTA has exited.
__device__ __forceinline__ void drain_fulls(Barriers& b, int issued) {
  for (int i = issued - kStages > 0 ? issued - kStages : 0; i < issued; ++i)
    mbar_wait(&b.full[i % kStages], (i / kStages) & 1, 290);
}

// grad entries (e, j < rank, k in column block cb) = 0
__device__ __forceinline__ void zero_grad_tile(int e, int cb, int K, int rank, float* grad, int64_t sE, int64_t sJ,
                                               int64_t sK) {
  for (int i = threadIdx.x; i < 128 * rank; i += kThreads) {
    const int k = cb * 128 + (i & 127), j = i >> 7;
    if (k < K) grad[e * sE + j * sJ + (int64_t)k * sK] = 0.f;
  }
}

__global__ void __launch_bounds__(kThreads) lora_grad_zero_kernel(int K, int rank, float* __restrict__ grad,
                                                                  int64_t sE, int64_t sJ, int64_t sK) {
  const int ncb = (K + 127) / 128;
  zero_grad_tile(blockIdx.x / ncb, blockIdx.x % ncb, K, rank, grad, sE, sJ, sK);
}

template <int LAYOUT>
__global__ void __launch_bounds__(kThreads) lora_project_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                const __grid_constant__ CUtensorMap tmap_f,
                                                                const int32_t* __restrict__ offsets, int E, int nsrc,
                                                                int S, int K, int rank, float scale,
                                                                __nv_bfloat16* __restrict__ out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = align1024(smem_raw);
  __shared__ Barriers bar;
  __shared__ int tile_prefix[kMaxExperts + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = nsrc * E;  // segments
  if (warp == 0) {
    // tiles of 128 rows per segment, in segment order
    int carry = 0;
    for (int e0 = 0; e0 < G; e0 += 32) {
      const int e = e0 + lane;
      int cnt = 0;
      if (e < G) {
        const int end = offsets[e], beg = e > 0 ? offsets[e - 1] : 0;
        cnt = end > beg ? (end - beg + 127) / 128 : 0;
      }
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (e < G) tile_prefix[e] = carry + incl - cnt;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    __syncwarp();
    if (lane == 0) {
      const int t = blockIdx.x;
      bar.tile_e = -1;
      if (t < carry) {
        int lo = 0, hi = G;
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (tile_prefix[mid] <= t) lo = mid;
          else hi = mid;
        }
        // skip segments with no tiles that share the prefix value
        while (lo + 1 < G && tile_prefix[lo + 1] <= t) ++lo;
        const int beg = lo > 0 ? offsets[lo - 1] : 0, end = offsets[lo];
        const int m = t - tile_prefix[lo];
        bar.tile_e = lo % E;  // the segment's expert
        bar.tile_row0 = beg + m * 128;
        bar.tile_rows = min(128, end - (beg + m * 128));
      }
    }
  }
  __syncthreads();
  const int e = bar.tile_e;
  if (e < 0) return;
  const int row0 = bar.tile_row0, rows = bar.tile_rows;
  const int nk = (K + 63) / 64;
  if (warp == 1) {
    if (lane == 0) init_barriers(bar);
    __syncwarp();
    tmem_alloc(&bar.tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_f);
    int kb = 0;
    for (; kb < nk; ++kb) {
      const int st = kb % kStages;
      if (kb >= kStages && !mbar_wait(&bar.empty[st], ((kb / kStages) - 1) & 1, 280)) break;
      uint8_t* a = tiles + st * kStageBytes;
      mbar_arrive_expect_tx(&bar.full[st], kStageBytes);
      tma_load_2d(a, &tmap_x, kb * 64, row0, &bar.full[st]);
      if (LAYOUT == kFactorRows) tma_load_2d(a + kABytes, &tmap_f, kb * 64, e * 64, &bar.full[st]);
      else tma_load_2d(a + kABytes, &tmap_f, 0, e * K + kb * 64, &bar.full[st]);
    }
    if (kb < nk) drain_fulls(bar, kb);
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = make_idesc_bf16(128, 64, false, LAYOUT == kFactorCols);
    int kb = 0;
    for (; kb < nk; ++kb) {
      const int st = kb % kStages;
      if (!mbar_wait(&bar.full[st], (kb / kStages) & 1, 281)) break;
      tc_fence_after();
      const uint32_t a = smem_u32(tiles + st * kStageBytes);
      const uint32_t b = a + kABytes;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t ad = make_sdesc_sw128(a + 32 * k, 0, 1024);
        const uint64_t bd = LAYOUT == kFactorRows ? make_sdesc_sw128(b + 32 * k, 0, 1024)
                                                  : make_sdesc_sw128(b + 2048 * k, 8192, 1024);
        umma_bf16(tmem, ad, bd, idesc, (kb | k) != 0);
      }
      umma_commit(&bar.empty[st]);
    }
    // after a failed wait `done` never completes and the drain below gives up
    if (kb == nk) umma_commit(&bar.done);
  }
  __syncwarp();
  // drain: warp w owns TMEM lanes 32w..32w+31 = rows of the tile
  const bool ok = mbar_wait(&bar.done, 0, 282);
  tc_fence_after();
  uint32_t acc[32];
  tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * warp) << 16), acc);
  tmem_ld_wait();
  const int local = 32 * warp + lane;
  if (ok && local < rows && row0 + local < S) {
    uint4* orow = reinterpret_cast<uint4*>(out + (int64_t)(row0 + local) * 64);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int j = 8 * q + 2 * h;
        const float lo = j < rank ? __uint_as_float(acc[j]) * scale : 0.f;
        const float hi = j + 1 < rank ? __uint_as_float(acc[j + 1]) * scale : 0.f;
        w[h] = pack_bf16x2(lo, hi);
      }
      orow[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int q = 4; q < 8; ++q) orow[q] = z;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

__global__ void __launch_bounds__(kThreads) lora_grad_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                             const __grid_constant__ CUtensorMap tmap_g,
                                                             const int32_t* __restrict__ offsets, int E, int nsrc,
                                                             int K, int rank, float* __restrict__ grad, int64_t sE,
                                                             int64_t sJ, int64_t sK) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = align1024(smem_raw);
  __shared__ Barriers bar;
  __shared__ int seg_beg[kMaxSources], seg_end[kMaxSources];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncb = (K + 127) / 128;
  const int e = blockIdx.x / ncb, cb = blockIdx.x % ncb;
  // this expert's segments (one per source), in source order
  for (int s = threadIdx.x; s < nsrc; s += blockDim.x) {
    const int j = s * E + e;
    seg_beg[s] = j > 0 ? offsets[j - 1] : 0;
    seg_end[s] = offsets[j];
  }
  __syncthreads();
  int nb = 0;
  for (int s = 0; s < nsrc; ++s) nb += seg_end[s] > seg_beg[s] ? (seg_end[s] - seg_beg[s] + 63) / 64 : 0;
  if (nb == 0) {
    zero_grad_tile(e, cb, K, rank, grad, sE, sJ, sK);
    return;
  }
  if (warp == 1) {
    if (lane == 0) init_barriers(bar);
    __syncwarp();
    tmem_alloc(&bar.tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_g);
    int b = 0, seg = 0, s0 = seg_beg[0];
    for (; b < nb; ++b) {
      while (s0 >= seg_end[seg] && seg + 1 < nsrc) s0 = seg_beg[++seg];  // next non-empty segment
      const int st = b % kStages;
      if (b >= kStages && !mbar_wait(&bar.empty[st], ((b / kStages) - 1) & 1, 283)) break;
      uint8_t* a = tiles + st * kStageBytes;
      mbar_arrive_expect_tx(&bar.full[st], kStageBytes);
      tma_load_2d(a, &tmap_x, cb * 128, s0, &bar.full[st]);
      tma_load_2d(a + kABytes / 2, &tmap_x, cb * 128 + 64, s0, &bar.full[st]);
      tma_load_2d(a + kABytes, &tmap_g, 0, s0, &bar.full[st]);
      s0 += 64;
    }
    if (b < nb) drain_fulls(bar, b);
  } else if (warp == 1) {
    constexpr uint32_t idesc = make_idesc_bf16(128, 64, true, true);
    int b = 0, seg = 0, s0 = seg_beg[0];
    for (; b < nb; ++b) {
      while (s0 >= seg_end[seg] && seg + 1 < nsrc) s0 = seg_beg[++seg];
      const int st = b % kStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&bar.full[st], (b / kStages) & 1, 284))) break;
      uint8_t* a = tiles + st * kStageBytes;
      const int n = max(0, min(64, seg_end[seg] - s0));
      s0 += 64;
      if (n < 64) {
        // rows n..63 of this block belong to the next segment (or lie past the
        // end): zero them in all three 64-row boxes (row r = bytes r*128..+128)
        const uint4 z = make_uint4(0, 0, 0, 0);
        for (int i = n * 8 + lane; i < 64 * 8; i += 32) {
          reinterpret_cast<uint4*>(a)[i] = z;
          reinterpret_cast<uint4*>(a + kABytes / 2)[i] = z;
          reinterpret_cast<uint4*>(a + kABytes)[i] = z;
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (lane == 0) {
        tc_fence_after();
        const uint32_t sa = smem_u32(a);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t ad = make_sdesc_sw128(sa + 2048 * k, 8192, 1024);
          const uint64_t bd = make_sdesc_sw128(sa + kABytes + 2048 * k, 8192, 1024);
          umma_bf16(tmem, ad, bd, idesc, (b | k) != 0);
        }
        umma_commit(&bar.empty[st]);
      }
      __syncwarp();
    }
    if (lane == 0 && b == nb) umma_commit(&bar.done);
  }
  __syncwarp();
  const bool ok = mbar_wait(&bar.done, 0, 285);
  tc_fence_after();
  uint32_t acc[32];
  tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * warp) << 16), acc);
  tmem_ld_wait();
  const int k = cb * 128 + 32 * warp + lane;
  if (ok && k < K) {
    float* gk = grad + e * sE + (int64_t)k * sK;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < rank) gk[j * sJ] = __uint_as_float(acc[j]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace lr
}  // namespace mirai

using namespace mirai;

extern "C" {

int mirai_moe_lora_project_src(const void* x, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                               int64_t num_rows, int32_t k_dim, const void* factor, int32_t factor_layout,
                               int32_t rank, float scale, void* out, mirai_stream_t stream) {
  if (num_experts <= 0 || num_sources <= 0 || num_sources > lr::kMaxSources ||
      (int64_t)num_sources * num_experts > lr::kMaxExperts || num_rows < 0 || k_dim <= 0 || k_dim % 8 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG,
                     "lora_project: bad sizes (sources=%d, E=%d, K=%d; at most %d segments, K a multiple of 8)",
                     num_sources, num_experts, k_dim, lr::kMaxExperts);
  if (rank <= 0 || rank > lr::kMaxRank)
    return set_error(MIRAI_ERR_UNSUPPORTED, "lora_project: rank %d outside 1..%d", rank, lr::kMaxRank);
  if (factor_layout != lr::kFactorRows && factor_layout != lr::kFactorCols)
    return set_error(MIRAI_ERR_INVALID_ARG, "lora_project: unknown factor layout %d", factor_layout);
  if (num_rows >= ((int64_t)1 << 31))
    return set_error(MIRAI_ERR_INVALID_ARG, "lora_project: row count exceeds int32 range");
  if (num_rows == 0) return MIRAI_OK;
  if (!x || !offsets || !factor || !out || (reinterpret_cast<uintptr_t>(out) & 15u))
    return set_error(MIRAI_ERR_INVALID_ARG, "lora_project: null or misaligned pointer");
  CUtensorMap tx, tf;
  int rc = make_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, (uint64_t)k_dim, (uint64_t)num_rows,
                        (uint64_t)k_dim * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (factor_layout == lr::kFactorRows)
    rc = make_tmap_2d(&tf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, factor, (uint64_t)k_dim,
                      (uint64_t)num_experts * 64, (uint64_t)k_dim * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    rc = make_tmap_2d(&tf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, factor, 64, (uint64_t)num_experts * k_dim, 128,
                      64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t max_tiles = (num_rows + 127) / 128 + (int64_t)num_sources * num_experts;
  auto kern = factor_layout == lr::kFactorRows ? lr::lora_project_kernel<lr::kFactorRows>
                                               : lr::lora_project_kernel<lr::kFactorCols>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lr::kSmemBytes);
  if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "lora_project: %s", cudaGetErrorString(e));
  kern<<<(unsigned)max_tiles, lr::kThreads, lr::kSmemBytes, s>>>(tx, tf, offsets, num_experts, num_sources,
                                                                 (int)num_rows, k_dim, rank, scale,
                                                                 static_cast<__nv_bfloat16*>(out));
  return check_launch("lora_project");
}

int mirai_moe_lora_project(const void* x, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                           int32_t k_dim, const void* factor, int32_t factor_layout, int32_t rank, float scale,
                           void* out, mirai_stream_t stream) {
  return mirai_moe_lora_project_src(x, offsets, 1, num_experts, num_rows, k_dim, factor, factor_layout, rank, scale,
                                    out, stream);
}

int mirai_moe_lora_grad_src(const void* x, const void* g_rank, const int32_t* offsets, int32_t num_sources,
                            int32_t num_experts, int64_t num_rows, int32_t k_dim, int32_t rank, float* grad,
                            int64_t stride_e, int64_t stride_r, int64_t stride_k, mirai_stream_t stream) {
  if (num_experts <= 0 || num_sources <= 0 || num_sources > lr::kMaxSources ||
      (int64_t)num_sources * num_experts > lr::kMaxExperts || num_rows < 0 || k_dim <= 0 || k_dim % 8 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG,
                     "lora_grad: bad sizes (sources=%d, E=%d, K=%d; at most %d segments, K a multiple of 8)",
                     num_sources, num_experts, k_dim, lr::kMaxExperts);
  if (rank <= 0 || rank > lr::kMaxRank)
    return set_error(MIRAI_ERR_UNSUPPORTED, "lora_grad: rank %d outside 1..%d", rank, lr::kMaxRank);
  if (num_rows >= ((int64_t)1 << 31))
    return set_error(MIRAI_ERR_INVALID_ARG, "lora_grad: row count exceeds int32 range");
  if (!offsets || !grad) return set_error(MIRAI_ERR_INVALID_ARG, "lora_grad: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int ncb = (k_dim + 127) / 128;
  if (num_rows == 0) {
    // no rows at all: every gradient entry is zero
    lr::lora_grad_zero_kernel<<<(unsigned)(ncb * num_experts), lr::kThreads, 0, s>>>(k_dim, rank, grad, stride_e,
                                                                                    stride_r, stride_k);
    return check_launch("lora_grad(empty)");
  }
  if (!x || !g_rank || (reinterpret_cast<uintptr_t>(grad) & 3u))
    return set_error(MIRAI_ERR_INVALID_ARG, "lora_grad: null or misaligned pointer");
  CUtensorMap tx, tg;
  int rc = make_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, (uint64_t)k_dim, (uint64_t)num_rows,
                        (uint64_t)k_dim * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tg, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g_rank, 64, (uint64_t)num_rows, 128, 64, 64,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaError_t e =
      cudaFuncSetAttribute(lr::lora_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lr::kSmemBytes);
  if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "lora_grad: %s", cudaGetErrorString(e));
  lr::lora_grad_kernel<<<(unsigned)(ncb * num_experts), lr::kThreads, lr::kSmemBytes, s>>>(
      tx, tg, offsets, num_experts, num_sources, k_dim, rank, grad, stride_e, stride_r, stride_k);
  return check_launch("lora_grad");
}

int mirai_moe_lora_grad(const void* x, const void* g_rank, const int32_t* offsets, int32_t num_experts,
                        int64_t num_rows, int32_t k_dim, int32_t rank, float* grad, int64_t stride_e,
                        int64_t stride_r, int64_t stride_k, mirai_stream_t stream) {
  return mirai_moe_lora_grad_src(x, g_rank, offsets, 1, num_experts, num_rows, k_dim, rank, grad, stride_e,
                                 stride_r, stride_k, stream);
}

}  // extern "C"
