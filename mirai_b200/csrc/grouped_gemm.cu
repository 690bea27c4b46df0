// a6 / a7: persistent grouped GEMMs over expert-contiguous row segments on
// sm_100a tensor cores (tcgen05.mma, fp32 accumulators in TMEM), with the
// frozen expert weights read as bf16, NF4 or INT8.
//
// One CTA per SM, warp-specialised:
//   warp 0       TMA producer: A (routed activations) and, for bf16 weights,
//                B; for NF4 / INT8 weights the raw codes of B
//   warp 1       UMMA issuer (one elected thread) and TMEM owner
//   warps 2..5   epilogue: TMEM -> registers -> SwiGLU / bf16 -> global
//   warps 6..9   (NF4 / INT8 only) dequantisers: raw codes in shared memory ->
//                exact bf16 weights written in the UMMA operand layout
// An A/B ring of STAGES shared-memory slots carries the operand tiles; two
// TMEM accumulators (2 x 256 fp32 columns) let the epilogue of tile i overlap
// the main loop of tile i+1.  Tiles are (expert, 128-row block, column
// block), enumerated expert-major with the column block fastest so that CTAs
// running together share one expert's weights in L2.
//
// Operand layouts (K-major, 128-byte swizzle, 8-row x 128-byte atoms):
//   A tile  [128 rows][64 k]  = 16 KB
//   B tile  [256 rows][64 k]  = 32 KB  (gate/up: 128 rows of W1 then 128 of W3;
//                                        down: 256 rows of W2)
// Dequantisation is bit-exact with the reference's dequantise-then-matmul:
//   NF4  w = bf16( code[nibble] * (ncode[q] * nabsmax + offset) )  (quant.py:413-431)
//   INT8 w = bf16( q * scale[row] )                                 (quant.py:238-260, g = 0)
#include "common.cuh"
#include "tmap.h"

namespace mirai {
namespace gg {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int UMMA_K = 16;
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr uint32_t B_BYTES = BN * BK * 2;
constexpr int kEpiWarps = 4;
constexpr int kDeqWarps = 4;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr int kMaxExperts = 1024;
constexpr int kMaxKBlocks = 64;  // K <= 4096 for the quantised formats

enum Mode { GATEUP = 0, DOWN = 1 };
enum WFmt { W_BF16 = 0, W_NF4 = 1, W_INT8 = 2 };

template <int WF> struct Cfg;
template <> struct Cfg<W_BF16> {
  static constexpr int STAGES = 4;
  static constexpr uint32_t RAW_BYTES = 0;
  static constexpr int THREADS = 64 + 32 * kEpiWarps;
};
template <> struct Cfg<W_NF4> {
  static constexpr int STAGES = 3;
  static constexpr uint32_t RAW_BYTES = BN * BK / 2;  // 8 KB of packed nibbles
  static constexpr int THREADS = 64 + 32 * (kEpiWarps + kDeqWarps);
};
template <> struct Cfg<W_INT8> {
  static constexpr int STAGES = 3;
  static constexpr uint32_t RAW_BYTES = BN * BK;  // 16 KB of int8
  static constexpr int THREADS = 64 + 32 * (kEpiWarps + kDeqWarps);
};

// One B half (128 weight rows) of a quantised key.
struct QHalf {
  const uint8_t* absmax;       // NF4: [E, out*in/64] codes
  const float* nested_absmax;  // NF4: [E, n_nested]
  const float* offset;         // NF4: [E]
  const float* code;           // NF4: [16]
  const float* nested_code;    // NF4: [256]
  const float* scale;          // INT8: [E, out]
  int n_nested;                // per expert
};

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
  QHalf q[2];              // quantised B halves (gate/up: W1, W3; down: W2, W2)
  int nbs_shift;           // log2(nested_blocksize)
};

template <int WF>
struct Smem {
  uint64_t full[Cfg<WF>::STAGES];
  uint64_t empty[Cfg<WF>::STAGES];
  uint64_t raw_full[Cfg<WF>::STAGES];
  uint64_t raw_empty[Cfg<WF>::STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort_flag;
  int row_start[kMaxExperts + 1];
  int tile_prefix[kMaxExperts + 1];
};

// Extra shared memory of the dequantisers: per-tile absmax codes, the
// byte -> (code[hi], code[lo]) table and the nested code map per B half.
struct DeqSmem {
  uint8_t absq[2][128 * kMaxKBlocks];
  float2 lut[2][256];
  float ncode[2][256];
};

template <int WF>
constexpr size_t smem_bytes() {
  return 1024 + Cfg<WF>::STAGES * (A_BYTES + B_BYTES + Cfg<WF>::RAW_BYTES) + sizeof(Smem<WF>) +
         (WF == W_BF16 ? 0 : sizeof(DeqSmem));
}

template <int WF>
__device__ __forceinline__ void decode_tile(int t, const Smem<WF>& sm, int E, int n_tiles, int& e, int& m,
                                            int& n) {
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

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Weight row (within the [E * N] row space) of B half h for tile (e, n).
template <int MODE>
__device__ __forceinline__ int b_row(const Params& p, int e, int n, int h) {
  return MODE == GATEUP ? e * p.N + n * (BN / 2) : e * p.N + n * BN + h * (BN / 2);
}

template <int MODE, int WF>
__global__ void __launch_bounds__(Cfg<WF>::THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b0,
                        const __grid_constant__ CUtensorMap tmap_b1, const Params p) {
  constexpr int STAGES = Cfg<WF>::STAGES;
  constexpr uint32_t RAW_BYTES = Cfg<WF>::RAW_BYTES;
  constexpr bool QUANT = WF != W_BF16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sRaw = sB + STAGES * B_BYTES;
  Smem<WF>& sm = *reinterpret_cast<Smem<WF>*>(sRaw + STAGES * RAW_BYTES);
  DeqSmem* dq = reinterpret_cast<DeqSmem*>(reinterpret_cast<uint8_t*>(&sm) + sizeof(Smem<WF>));

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
        mbar_init(&sm.full[s], QUANT ? 1 + kDeqWarps : 1);
        mbar_init(&sm.empty[s], 1);
        mbar_init(&sm.raw_full[s], 1);
        mbar_init(&sm.raw_empty[s], kDeqWarps);
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
    prefetch_tmap(&tmap_b1);
  }
  if (QUANT && warp >= 2 + kEpiWarps) {
    const int d = threadIdx.x - 32 * (2 + kEpiWarps);
    if (WF == W_NF4) {
      for (int h = 0; h < 2; ++h) {
        for (int i = d; i < 256; i += 32 * kDeqWarps) {
          dq->lut[h][i] = make_float2(__ldg(p.q[h].code + (i >> 4)), __ldg(p.q[h].code + (i & 15)));
          dq->ncode[h][i] = __ldg(p.q[h].nested_code + i);
        }
      }
    }
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
        decode_tile<WF>(t, sm, E, p.n_tiles, e, m, n);
        const int row0 = sm.row_start[e] + m * BM;
        const int br0 = b_row<MODE>(p, e, n, 0);
        const int br1 = b_row<MODE>(p, e, n, 1);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&sm.empty[stage], phase ^ 1, 10)) {
            *abort_flag = 1;
            break;
          }
          if (!QUANT) {
            mbar_arrive_expect_tx(&sm.full[stage], A_BYTES + B_BYTES);
            uint8_t* b_dst = sB + stage * B_BYTES;
            tma_load_2d(b_dst, &tmap_b0, kb * BK, br0, &sm.full[stage]);
            tma_load_2d(b_dst + B_BYTES / 2, MODE == GATEUP ? &tmap_b1 : &tmap_b0, kb * BK, br1, &sm.full[stage]);
          } else {
            mbar_arrive_expect_tx(&sm.full[stage], A_BYTES);
          }
          tma_load_2d(sA + stage * A_BYTES, &tmap_a, kb * BK, row0, &sm.full[stage]);
          if (QUANT) {
            if (!mbar_wait(&sm.raw_empty[stage], phase ^ 1, 11)) {
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&sm.raw_full[stage], RAW_BYTES);
            uint8_t* r_dst = sRaw + stage * RAW_BYTES;
            constexpr int kbx = WF == W_NF4 ? BK / 2 : BK;  // raw bytes of one row per k-block
            tma_load_2d(r_dst, &tmap_b0, kb * kbx, br0, &sm.raw_full[stage]);
            tma_load_2d(r_dst + RAW_BYTES / 2, MODE == GATEUP ? &tmap_b1 : &tmap_b0, kb * kbx, br1,
                        &sm.raw_full[stage]);
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
  } else if (warp < 2 + kEpiWarps) {
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
      decode_tile<WF>(t, sm, E, p.n_tiles, e, m, n);
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
  } else if (QUANT) {
    // ======================= dequantisers =======================
    // Thread d owns B row d of each half (rows d and 128 + d of the tile).
    const int d = threadIdx.x - 32 * (2 + kEpiWarps);
    const int nkb = num_kb;
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
      int e, m, n;
      decode_tile<WF>(t, sm, E, p.n_tiles, e, m, n);
      int wrow[2];  // row inside the expert's [out, in] matrix
      float s_off[2] = {0.f, 0.f};
      float row_scale[2] = {0.f, 0.f};
      const float* nab[2] = {nullptr, nullptr};
      for (int h = 0; h < 2; ++h) wrow[h] = b_row<MODE>(p, e, n, h) - e * p.N + d;
      if (WF == W_NF4) {
        // stage this tile's absmax codes: 128 rows x nkb bytes per half, contiguous
        named_bar_sync(1, 32 * kDeqWarps);
        for (int h = 0; h < 2; ++h) {
          const uint4* src = reinterpret_cast<const uint4*>(p.q[h].absmax + (size_t)b_row<MODE>(p, e, n, h) * nkb);
          uint4* dst = reinterpret_cast<uint4*>(dq->absq[h]);
          for (int i = d; i < 8 * nkb; i += 32 * kDeqWarps) dst[i] = __ldg(src + i);
          s_off[h] = __ldg(p.q[h].offset + e);
          nab[h] = p.q[h].nested_absmax + (size_t)e * p.q[h].n_nested;
        }
        named_bar_sync(1, 32 * kDeqWarps);
      } else {
        for (int h = 0; h < 2; ++h) row_scale[h] = __ldg(p.q[h].scale + (size_t)e * p.N + wrow[h]);
      }
      for (int kb = 0; kb < nkb; ++kb) {
        bool ok = mbar_wait(&sm.raw_full[stage], phase, 40);
        ok = ok && mbar_wait(&sm.empty[stage], phase ^ 1, 41);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        const uint8_t* raw = sRaw + stage * RAW_BYTES;
        const uint32_t bst = smem_u32(sB + stage * B_BYTES);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t row_addr = bst + (uint32_t)(h * 128 + d) * 128u;
          const int sw = d & 7;
          if (WF == W_NF4) {
            const uint32_t qcode = dq->absq[h][d * nkb + kb];
            const int nidx = (wrow[h] * nkb + kb) >> p.nbs_shift;
            const float scale = __fadd_rn(__fmul_rn(dq->ncode[h][qcode], __ldg(nab[h] + nidx)), s_off[h]);
            const uint4* rp = reinterpret_cast<const uint4*>(raw + h * (RAW_BYTES / 2) + d * 32);
            const uint4 r0 = rp[0], r1 = rp[1];
            const uint32_t words[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
            const float2* lut = dq->lut[h];
#pragma unroll
            for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = elements 8c .. 8c+7 = raw bytes 4c .. 4c+3
              uint32_t o[4];
#pragma unroll
              for (int b = 0; b < 4; ++b) {
                const float2 f = lut[(words[c] >> (8 * b)) & 0xFFu];
                o[b] = pack_bf16x2(__fmul_rn(f.x, scale), __fmul_rn(f.y, scale));
              }
              st_shared_v4(row_addr + (uint32_t)((c ^ sw) << 4), o[0], o[1], o[2], o[3]);
            }
          } else {
            const float scale = row_scale[h];
            const uint4* rp = reinterpret_cast<const uint4*>(raw + h * (RAW_BYTES / 2) + d * 64);
#pragma unroll
            for (int v = 0; v < 4; ++v) {  // 16 int8 -> two 16-byte bf16 chunks
              const uint4 r = rp[v];
              const uint32_t words[4] = {r.x, r.y, r.z, r.w};
              uint32_t o[8];
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                const uint32_t biased = words[w] ^ 0x80808080u;  // q + 128 as unsigned bytes
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                  // 0x4B0000uu is the float 2^23 + uu: subtracting 2^23 + 128 recovers q exactly
                  const float q0 = __uint_as_float(__byte_perm(biased, 0x4B000000u, 0x7540u + 2 * b)) - 8388736.f;
                  const float q1 = __uint_as_float(__byte_perm(biased, 0x4B000000u, 0x7541u + 2 * b)) - 8388736.f;
                  o[2 * w + b] = pack_bf16x2(__fmul_rn(q0, scale), __fmul_rn(q1, scale));
                }
              }
              st_shared_v4(row_addr + (uint32_t)(((2 * v) ^ sw) << 4), o[0], o[1], o[2], o[3]);
              st_shared_v4(row_addr + (uint32_t)(((2 * v + 1) ^ sw) << 4), o[4], o[5], o[6], o[7]);
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.raw_empty[stage]);
          mbar_arrive(&sm.full[stage]);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int MODE, int WF>
int launch(const CUtensorMap& ta, const CUtensorMap& tb0, const CUtensorMap& tb1, const Params& p,
           cudaStream_t stream) {
  auto kern = grouped_gemm_kernel<MODE, WF>;
  constexpr size_t smem = smem_bytes<WF>();
  static_assert(smem <= 232448, "shared memory budget exceeded");
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  const int64_t max_tiles = ((p.S + BM - 1) / BM + p.E) * (int64_t)p.n_tiles;
  const int grid = (int)(max_tiles < sm_count() ? max_tiles : sm_count());
  kern<<<grid, Cfg<WF>::THREADS, smem, stream>>>(ta, tb0, tb1, p);
  return check_launch(MODE == GATEUP ? "gateup_swiglu" : "down");
}

static inline bool mis16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0; }

// Shared host-side checks and the A-operand tensor map.
template <int MODE>
int prepare(const char* name, const void* a, const int32_t* offsets, int E, int64_t S, int K, int N, void* out,
            void* gate_up, Params& p, CUtensorMap& ta) {
  if (E <= 0 || E > kMaxExperts || S < 0 || K <= 0 || N <= 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: bad sizes (E=%d, S=%lld, K=%d, N=%d)", name, E, (long long)S, K, N);
  const int ntile = MODE == GATEUP ? BN / 2 : BN;
  if (K % BK != 0 || N % ntile != 0)
    return set_error(MIRAI_ERR_UNSUPPORTED, "%s: needs K %% %d == 0 and N %% %d == 0 (K=%d, N=%d)", name, BK, ntile,
                     K, N);
  if (S >= (int64_t)1 << 31) return set_error(MIRAI_ERR_UNSUPPORTED, "%s: more than 2^31 routed rows", name);
  if (!a || !offsets || !out || mis16(out) || (gate_up && mis16(gate_up)))
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: null or misaligned pointer", name);
  p.offsets = offsets;
  p.E = E;
  p.S = S;
  p.K = K;
  p.N = N;
  p.n_tiles = N / ntile;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = N;
  p.gate_up = static_cast<__nv_bfloat16*>(gate_up);
  p.nbs_shift = 8;
  p.q[0] = QHalf{};
  p.q[1] = QHalf{};
  return make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, (uint64_t)K, (uint64_t)S, (uint64_t)K * 2, BK, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

int bf16_weight_map(CUtensorMap& m, const void* w, int E, int N, int K) {
  if (!w) return set_error(MIRAI_ERR_INVALID_ARG, "null weight pointer");
  return make_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, (uint64_t)K, (uint64_t)E * N, (uint64_t)K * 2, BK,
                      BN / 2, CU_TENSOR_MAP_SWIZZLE_128B);
}

int nf4_half(CUtensorMap& m, QHalf& q, int& nbs_shift, const mirai_nf4_weight* w, int E, int N, int K) {
  if (!w || !w->packed || !w->absmax || !w->nested_absmax || !w->offset || !w->code || !w->nested_code)
    return set_error(MIRAI_ERR_INVALID_ARG, "nf4 weight: null buffer");
  if (w->blocksize != BK)
    return set_error(MIRAI_ERR_UNSUPPORTED, "nf4 weight: blocksize %d (the fused kernel decodes blocksize 64)",
                     w->blocksize);
  if (w->nested_blocksize <= 0 || (w->nested_blocksize & (w->nested_blocksize - 1)) != 0)
    return set_error(MIRAI_ERR_UNSUPPORTED, "nf4 weight: nested blocksize %d is not a power of two",
                     w->nested_blocksize);
  if (K / BK > kMaxKBlocks)
    return set_error(MIRAI_ERR_UNSUPPORTED, "nf4 weight: in_features %d exceeds %d", K, BK * kMaxKBlocks);
  if (mis16(w->absmax)) return set_error(MIRAI_ERR_INVALID_ARG, "nf4 weight: absmax codes not 16-byte aligned");
  nbs_shift = __builtin_ctz((unsigned)w->nested_blocksize);
  const int64_t blocks_per_expert = (int64_t)N * K / BK;
  q.absmax = w->absmax;
  q.nested_absmax = w->nested_absmax;
  q.offset = w->offset;
  q.code = w->code;
  q.nested_code = w->nested_code;
  q.scale = nullptr;
  q.n_nested = (int)((blocks_per_expert + w->nested_blocksize - 1) / w->nested_blocksize);
  // packed nibbles as a [E*N rows, K/2 bytes] byte tensor; one box = 128 rows x 32 bytes
  return make_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w->packed, (uint64_t)K / 2, (uint64_t)E * N,
                      (uint64_t)K / 2, BK / 2, BN / 2, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int int8_half(CUtensorMap& m, QHalf& q, const mirai_int8_weight* w, int E, int N, int K) {
  if (!w || !w->q || !w->scale) return set_error(MIRAI_ERR_INVALID_ARG, "int8 weight: null buffer");
  q = QHalf{};
  q.scale = w->scale;
  return make_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w->q, (uint64_t)K, (uint64_t)E * N, (uint64_t)K, BK,
                      BN / 2, CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace gg
}  // namespace mirai

using namespace mirai;
using namespace mirai::gg;

extern "C" {

int mirai_moe_gateup_swiglu_bf16(const void* x_sorted, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                 int32_t hidden, int32_t inter, const void* w1, const void* w3, void* h,
                                 void* gate_up, mirai_stream_t stream) {
  Params p;
  CUtensorMap ta, t0, t1;
  if (num_rows == 0 && num_experts > 0) return MIRAI_OK;
  int rc = prepare<GATEUP>("gateup_swiglu_bf16", x_sorted, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                           p, ta);
  if (!rc) rc = bf16_weight_map(t0, w1, num_experts, inter, hidden);
  if (!rc) rc = bf16_weight_map(t1, w3, num_experts, inter, hidden);
  if (rc) return rc;
  return launch<GATEUP, W_BF16>(ta, t0, t1, p, reinterpret_cast<cudaStream_t>(stream));
}

int mirai_moe_gateup_swiglu_nf4(const void* x_sorted, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                int32_t hidden, int32_t inter, const mirai_nf4_weight* w1, const mirai_nf4_weight* w3,
                                void* h, void* gate_up, mirai_stream_t stream) {
  Params p;
  CUtensorMap ta, t0, t1;
  if (num_rows == 0 && num_experts > 0) return MIRAI_OK;
  int rc = prepare<GATEUP>("gateup_swiglu_nf4", x_sorted, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                           p, ta);
  int s0 = 8, s1 = 8;
  if (!rc) rc = nf4_half(t0, p.q[0], s0, w1, num_experts, inter, hidden);
  if (!rc) rc = nf4_half(t1, p.q[1], s1, w3, num_experts, inter, hidden);
  if (!rc && s0 != s1) rc = set_error(MIRAI_ERR_UNSUPPORTED, "gateup_swiglu_nf4: w1/w3 nested blocksizes differ");
  if (rc) return rc;
  p.nbs_shift = s0;
  return launch<GATEUP, W_NF4>(ta, t0, t1, p, reinterpret_cast<cudaStream_t>(stream));
}

int mirai_moe_gateup_swiglu_int8(const void* x_sorted, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                 int32_t hidden, int32_t inter, const mirai_int8_weight* w1,
                                 const mirai_int8_weight* w3, void* h, void* gate_up, mirai_stream_t stream) {
  Params p;
  CUtensorMap ta, t0, t1;
  if (num_rows == 0 && num_experts > 0) return MIRAI_OK;
  int rc = prepare<GATEUP>("gateup_swiglu_int8", x_sorted, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                           p, ta);
  if (!rc) rc = int8_half(t0, p.q[0], w1, num_experts, inter, hidden);
  if (!rc) rc = int8_half(t1, p.q[1], w3, num_experts, inter, hidden);
  if (rc) return rc;
  return launch<GATEUP, W_INT8>(ta, t0, t1, p, reinterpret_cast<cudaStream_t>(stream));
}

int mirai_moe_down_bf16(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows, int32_t inter,
                        int32_t hidden, const void* w2, void* y, mirai_stream_t stream) {
  Params p;
  CUtensorMap ta, t0;
  if (num_rows == 0 && num_experts > 0) return MIRAI_OK;
  int rc = prepare<DOWN>("down_bf16", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, p, ta);
  if (!rc) rc = bf16_weight_map(t0, w2, num_experts, hidden, inter);
  if (rc) return rc;
  return launch<DOWN, W_BF16>(ta, t0, t0, p, reinterpret_cast<cudaStream_t>(stream));
}

int mirai_moe_down_nf4(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows, int32_t inter,
                       int32_t hidden, const mirai_nf4_weight* w2, void* y, mirai_stream_t stream) {
  Params p;
  CUtensorMap ta, t0;
  if (num_rows == 0 && num_experts > 0) return MIRAI_OK;
  int rc = prepare<DOWN>("down_nf4", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, p, ta);
  int s = 8;
  if (!rc) rc = nf4_half(t0, p.q[0], s, w2, num_experts, hidden, inter);
  if (rc) return rc;
  p.q[1] = p.q[0];
  p.nbs_shift = s;
  return launch<DOWN, W_NF4>(ta, t0, t0, p, reinterpret_cast<cudaStream_t>(stream));
}

int mirai_moe_down_int8(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows, int32_t inter,
                        int32_t hidden, const mirai_int8_weight* w2, void* y, mirai_stream_t stream) {
  Params p;
  CUtensorMap ta, t0;
  if (num_rows == 0 && num_experts > 0) return MIRAI_OK;
  int rc = prepare<DOWN>("down_int8", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, p, ta);
  if (!rc) rc = int8_half(t0, p.q[0], w2, num_experts, hidden, inter);
  if (rc) return rc;
  p.q[1] = p.q[0];
  return launch<DOWN, W_INT8>(ta, t0, t0, p, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
