// a6 / a7: persistent grouped GEMMs over expert-contiguous row segments on
// sm_100a tensor cores (tcgen05.mma, fp32 accumulators in TMEM).
//
// One CTA per SM, warp-specialised:
//   warp 0      TMA producer  (A = routed activations, B = expert weight tile)
//   warp 1      UMMA issuer   (one thread) and TMEM owner
//   warps 2..5  epilogue      (TMEM -> registers -> SwiGLU / bf16 -> global)
// A STAGES-deep shared-memory ring carries the operand tiles; two TMEM
// accumulators (2 x 256 fp32 columns) let the epilogue of tile i overlap the
// main loop of tile i+1.  Tiles are (expert, 128-row block, 256-column block),
// enumerated expert-major with the column block fastest so that CTAs running
// together share one expert's weights in L2.
//
// Operand layouts (all K-major, 128-byte swizzle, 8-row x 128-byte atoms):
//   A tile  [128 rows][64 k]  = 16 KB
//   B tile  [256 rows][64 k]  = 32 KB  (gate/up: 128 rows of W1 then 128 of W3)
#include "common.cuh"
#include "tmap.h"

namespace mirai {
namespace gg {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int UMMA_K = 16;
constexpr int STAGES = 4;
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr uint32_t B_BYTES = BN * BK * 2;
constexpr int kEpiWarps = 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr int kMaxExperts = 1024;

enum Mode { GATEUP = 0, DOWN = 1 };

struct Params {
  const int32_t* offsets;  // [E] inclusive row cumsum
  int E;
  int64_t S;               // total routed rows
  int K;                   // reduction length
  int N;                   // rows of one expert's B matrix (I for gate/up, H for down)
  int n_tiles;             // column tiles per row block
  __nv_bfloat16* out;      // h [S, I] (gate/up) or y [S, H] (down)
  int64_t ldo;             // elements
  __nv_bfloat16* gate_up;  // optional [S, 2I]
};

struct Smem {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort_flag;
  int row_start[kMaxExperts + 1];
  int tile_prefix[kMaxExperts + 1];
};

constexpr size_t kSmemBytes = 1024 /*align slack*/ + STAGES * (A_BYTES + B_BYTES) + sizeof(Smem);

__device__ __forceinline__ void decode_tile(int t, const Smem& sm, int E, int n_tiles, int& e, int& m, int& n) {
  const int mt = t / n_tiles;
  n = t - mt * n_tiles;
  int lo = 0, hi = E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (sm.tile_prefix[mid] <= mt) lo = mid;
    else hi = mid;
  }
  e = lo;
  m = mt - sm.tile_prefix[e];
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b0,
                             const __grid_constant__ CUtensorMap tmap_b1, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * A_BYTES;
  Smem& sm = *reinterpret_cast<Smem*>(sB + STAGES * B_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;

  // ---- segment table: row_start[e] and exclusive prefix of 128-row blocks
  if (warp == 0) {
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      int cnt = 0;
      if (e < E) {
        const int64_t end = p.offsets[e];
        const int64_t beg = e > 0 ? p.offsets[e - 1] : 0;
        const int64_t endc = end < p.S ? end : p.S;
        cnt = endc > beg ? (int)((endc - beg + BM - 1) / BM) : 0;
        if (end < beg || end > p.S) device_fail(MIRAI_ERR_DEVICE_BOUNDS, 600 + MODE);
        sm.row_start[e] = (int)beg;
      }
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (e < E) sm.tile_prefix[e] = carry + incl - cnt;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      sm.tile_prefix[E] = carry;
      sm.row_start[E] = (int)(E > 0 ? p.offsets[E - 1] : 0);
    }
  }
  if (warp == 1) {
    if (lane == 0) {
      for (int s = 0; s < STAGES; ++s) {
        mbar_init(&sm.full[s], 1);
        mbar_init(&sm.empty[s], 1);
      }
      for (int a = 0; a < 2; ++a) {
        mbar_init(&sm.tfull[a], 1);
        mbar_init(&sm.tempty[a], kEpiWarps);
      }
      sm.abort_flag = 0;
      fence_mbar_init();
    }
    __syncwarp();
    tmem_alloc(&sm.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b0);
    if (MODE == GATEUP) prefetch_tmap(&tmap_b1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem_base = sm.tmem_base;
  const int total_tiles = sm.tile_prefix[E] * p.n_tiles;
  const int num_kb = p.K / BK;
  volatile int* abort_flag = &sm.abort_flag;

  if (warp == 0) {
    // ======================= TMA producer =======================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        int e, m, n;
        decode_tile(t, sm, E, p.n_tiles, e, m, n);
        const int row0 = sm.row_start[e] + m * BM;
        const int brow = e * p.N + n * (MODE == GATEUP ? BN / 2 : BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&sm.empty[stage], phase ^ 1, 10)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&sm.full[stage], A_BYTES + B_BYTES);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          tma_load_2d(a_dst, &tmap_a, kb * BK, row0, &sm.full[stage]);
          if (MODE == GATEUP) {
            tma_load_2d(b_dst, &tmap_b0, kb * BK, brow, &sm.full[stage]);
            tma_load_2d(b_dst + B_BYTES / 2, &tmap_b1, kb * BK, brow, &sm.full[stage]);
          } else {
            tma_load_2d(b_dst, &tmap_b0, kb * BK, brow, &sm.full[stage]);
            tma_load_2d(b_dst + B_BYTES / 2, &tmap_b0, kb * BK, brow + BN / 2, &sm.full[stage]);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ======================= UMMA issuer =======================
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&sm.tempty[acc], acc_phase ^ 1, 20)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&sm.full[stage], phase, 21)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t ad = make_sdesc_sw128(a_addr + k * UMMA_K * 2, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(b_addr + k * UMMA_K * 2, 16, 1024);
            umma_bf16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&sm.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        umma_commit(&sm.tfull[acc]);
      }
    }
  } else {
    // ======================= epilogue =======================
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int it = 0;
    for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&sm.tfull[acc], acc_phase, 30)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int e, m, n;
      decode_tile(t, sm, E, p.n_tiles, e, m, n);
      const int r = q * 32 + lane;
      const int64_t seg_rows = (int64_t)sm.row_start[e + 1] - sm.row_start[e];
      const bool valid = (int64_t)m * BM + r < seg_rows;
      const int64_t grow = (int64_t)sm.row_start[e] + (int64_t)m * BM + r;
      const uint32_t tb = tmem_base + acc * BN + ((uint32_t)(q * 32) << 16);
      if (MODE == GATEUP) {
        const int col0 = n * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < (BN / 2) / 32; ++c) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tb + c * 32, g);
          tmem_ld_32x32b_x32(tb + BN / 2 + c * 32, u);
          tmem_ld_wait();
          if (valid) {
            uint32_t hp[16], gp[16], up[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // Round where the reference's bf16 tensors round: gate, up,
              // silu(gate), and the product (experts.py:301-317).
              const float g0 = bf16r(__uint_as_float(g[2 * j])), g1 = bf16r(__uint_as_float(g[2 * j + 1]));
              const float u0 = bf16r(__uint_as_float(u[2 * j])), u1 = bf16r(__uint_as_float(u[2 * j + 1]));
              const float a0 = bf16r(g0 / (1.f + expf(-g0)));
              const float a1 = bf16r(g1 / (1.f + expf(-g1)));
              hp[j] = pack_bf16x2(a0 * u0, a1 * u1);
              gp[j] = pack_bf16x2(g0, g1);
              up[j] = pack_bf16x2(u0, u1);
            }
            uint4* dst = reinterpret_cast<uint4*>(p.out + grow * p.ldo + col0 + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = make_uint4(hp[4 * v], hp[4 * v + 1], hp[4 * v + 2], hp[4 * v + 3]);
            if (p.gate_up != nullptr) {
              const int64_t ld2 = 2 * p.ldo;
              uint4* gd = reinterpret_cast<uint4*>(p.gate_up + grow * ld2 + col0 + c * 32);
              uint4* ud = reinterpret_cast<uint4*>(p.gate_up + grow * ld2 + p.ldo + col0 + c * 32);
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                gd[v] = make_uint4(gp[4 * v], gp[4 * v + 1], gp[4 * v + 2], gp[4 * v + 3]);
                ud[v] = make_uint4(up[4 * v], up[4 * v + 1], up[4 * v + 2], up[4 * v + 3]);
              }
            }
          }
        }
      } else {
        const int col0 = n * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v32[32];
          tmem_ld_32x32b_x32(tb + c * 32, v32);
          tmem_ld_wait();
          if (valid) {
            uint32_t yp[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) yp[j] = pack_bf16x2(__uint_as_float(v32[2 * j]), __uint_as_float(v32[2 * j + 1]));
            uint4* dst = reinterpret_cast<uint4*>(p.out + grow * p.ldo + col0 + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = make_uint4(yp[4 * v], yp[4 * v + 1], yp[4 * v + 2], yp[4 * v + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int MODE>
int launch_bf16(const void* a, const void* b0, const void* b1, const int32_t* offsets, int E, int64_t S, int K,
                int N, void* out, void* gate_up, cudaStream_t stream) {
  CUtensorMap ta, tb0, tb1;
  int rc = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, (uint64_t)K, (uint64_t)S, (uint64_t)K * 2, BK,
                        BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tb0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b0, (uint64_t)K, (uint64_t)E * N, (uint64_t)K * 2,
                    BK, BN / 2, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (MODE == GATEUP) {
    rc = make_tmap_2d(&tb1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b1, (uint64_t)K, (uint64_t)E * N, (uint64_t)K * 2,
                      BK, BN / 2, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    tb1 = tb0;
  }
  Params p;
  p.offsets = offsets;
  p.E = E;
  p.S = S;
  p.K = K;
  p.N = N;
  p.n_tiles = MODE == GATEUP ? N / (BN / 2) : N / BN;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = N;
  p.gate_up = static_cast<__nv_bfloat16*>(gate_up);
  auto kern = grouped_gemm_bf16_kernel<MODE>;
  static bool attr_set[2] = {false, false};
  if (!attr_set[MODE]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_set[MODE] = true;
  }
  const int64_t max_tiles = ((S + BM - 1) / BM + E) * (int64_t)p.n_tiles;
  const int grid = (int)(max_tiles < sm_count() ? max_tiles : sm_count());
  kern<<<grid, kThreads, kSmemBytes, stream>>>(ta, tb0, tb1, p);
  return check_launch(MODE == GATEUP ? "gateup_swiglu_bf16" : "down_bf16");
}

}  // namespace gg
}  // namespace mirai

using namespace mirai;

static inline bool mis16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

extern "C" {

int mirai_moe_gateup_swiglu_bf16(const void* x_sorted, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                 int32_t hidden, int32_t inter, const void* w1, const void* w3, void* h,
                                 void* gate_up, mirai_stream_t stream) {
  if (num_experts <= 0 || num_experts > gg::kMaxExperts || num_rows < 0 || hidden <= 0 || inter <= 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "gateup_swiglu_bf16: bad sizes (E=%d, S=%lld, H=%d, I=%d)", num_experts,
                     (long long)num_rows, hidden, inter);
  if (hidden % gg::BK != 0 || inter % (gg::BN / 2) != 0)
    return set_error(MIRAI_ERR_UNSUPPORTED, "gateup_swiglu_bf16: needs hidden %% 64 == 0 and inter %% 128 == 0 "
                     "(H=%d, I=%d)", hidden, inter);
  if (num_rows == 0) return MIRAI_OK;
  if (num_rows >= (int64_t)1 << 31) return set_error(MIRAI_ERR_UNSUPPORTED, "gateup_swiglu_bf16: S >= 2^31");
  if (!x_sorted || !offsets || !w1 || !w3 || !h || mis16(h) || (gate_up && mis16(gate_up)))
    return set_error(MIRAI_ERR_INVALID_ARG, "gateup_swiglu_bf16: null or misaligned pointer");
  return gg::launch_bf16<gg::GATEUP>(x_sorted, w1, w3, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                                     reinterpret_cast<cudaStream_t>(stream));
}

int mirai_moe_down_bf16(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows, int32_t inter,
                        int32_t hidden, const void* w2, void* y, mirai_stream_t stream) {
  if (num_experts <= 0 || num_experts > gg::kMaxExperts || num_rows < 0 || hidden <= 0 || inter <= 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "down_bf16: bad sizes (E=%d, S=%lld, I=%d, H=%d)", num_experts,
                     (long long)num_rows, inter, hidden);
  if (inter % gg::BK != 0 || hidden % gg::BN != 0)
    return set_error(MIRAI_ERR_UNSUPPORTED, "down_bf16: needs inter %% 64 == 0 and hidden %% 256 == 0 (I=%d, H=%d)",
                     inter, hidden);
  if (num_rows == 0) return MIRAI_OK;
  if (num_rows >= (int64_t)1 << 31) return set_error(MIRAI_ERR_UNSUPPORTED, "down_bf16: S >= 2^31");
  if (!h || !offsets || !w2 || !y || mis16(y))
    return set_error(MIRAI_ERR_INVALID_ARG, "down_bf16: null or misaligned pointer");
  return gg::launch_bf16<gg::DOWN>(h, w2, nullptr, offsets, num_experts, num_rows, inter, hidden, y, nullptr,
                                   reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
