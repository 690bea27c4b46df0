// a6 / a7 / a9: persistent grouped GEMMs over expert-contiguous row segments
// on sm_100a tensor cores (tcgen05.mma, fp32 accumulators in TMEM), with the
// frozen expert weights read as bf16, NF4 or INT8.
//
// Modes (one kernel template):
//   GATEUP    h = silu(x W1^T) * (x W3^T)            B = W1/W3 rows  (K-major)
//   DOWN      y = h W2^T                              B = W2 rows     (K-major)
//   DXDOWN    dgu = swiglu_bwd(dy W2, gate, up)       B = W2 columns  (MN-major)
//   DXGATEUP  dx = dgate W1 + dup W3                  B = W1;W3       (MN-major)
//
// Warp roles in every CTA:
//   TMA producer    A tiles; B tiles (bf16); the LoRA rank block
//   UMMA issuer     one thread; owns the TMEM accumulators
//   raw producer    (NF4 / INT8) packed codes into their own ring, and for NF4
//                   pairs each tile's absmax codes by one bulk copy
//   epilogue        TMEM -> registers -> SwiGLU (+bwd) / bf16 -> global
//   dequantisers    (NF4 / INT8) raw codes -> exact bf16 weights in the UMMA
//                   operand layout
// NF4 / INT8 on CTA pairs run 16 dequantiser warps beside 4 epilogue warps
// (768 threads) with registers rebalanced per warpgroup by setmaxnreg; the
// single-CTA variants run 8 (or none) with one register budget.
// Two TMEM accumulators (2 x 256 fp32 columns) overlap the epilogue of tile i
// with the main loop of tile i+1.  Tiles are (expert, row block, column
// block), expert-major with the column block fastest so that the CTAs running
// together share one expert's weights in L2.
//
// PAIR = true runs each tile on a CTA pair (cluster of 2, tcgen05 cta_group::2):
// the A rows of every 256-row sub-tile are split between the two SMs (128
// each) and the B operand is split along N, so each SM stages, and for
// NF4/INT8 decodes, only half of B.  The even CTA issues the M=256 UMMAs;
// completion is multicast to both CTAs.  No TMA multicast is used.
// Every format uses one 256-row sub-tile x 256 columns per tile (RT = 1,
// TN = 256).  The geometry also admits RT = 2 sub-tiles of 128 columns that
// share one decoded B block (half the decode work per FLOP); on B200 that shape
// measured slower for NF4 and bf16 alike (0.80 vs 0.73 ms, 0.75 vs 0.59 ms for
// the c2 gate/up GEMM), because N = 128 UMMAs re-read A from shared memory twice
// as often and shared-memory bandwidth, not decode, becomes the limit.
// PAIR = false is the single-SM 128-row x 256-column variant.
//
// Operand layouts (128-byte swizzle), per CTA:
//   A  RT x [128 rows][64 k] K-major = RT x 16 KB
//   B  K-major:  [B_ROWS rows][64 k]           (8-row x 128 B atoms, SBO 1 KB)
//      MN-major: [B_ROWS/64 x 64 n][64 k rows] (atoms 8 k-rows x 64 n; LBO 8 KB
//                                               between 64-n blocks, SBO 1 KB)
// Dequantisation is bit-exact with the reference's dequantise-then-matmul:
//   NF4  w = bf16( code[nibble] * (ncode[q] * nabsmax + offset) )  (quant.py:413-431)
//   INT8 w = bf16( q * scale[row] )                                 (quant.py:238-260, g = 0)
#include "common.cuh"
#include "tmap.h"

namespace mirai {
namespace gg {

constexpr int BM = 128;  // rows of A per CTA and sub-tile
constexpr int BN = 256;  // accumulator columns per tile (RT x TN)
constexpr int BK = 64;
constexpr int UMMA_K = 16;
constexpr uint32_t A_BYTES = BM * BK * 2;
// epilogue warps: 8 when the SM has no dequantisers (two per TMEM lane
// quarter, splitting the columns), 4 otherwise
constexpr int epi_warps(int wf) { return wf == 0 ? 8 : 4; }
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr int kMaxExperts = 1024;
constexpr int kMaxK = 4096;        // reduction length supported by the quantised formats
constexpr int kMaxNested = 512;    // nested absmax entries per expert and key

enum Mode { GATEUP = 0, DOWN = 1, DXDOWN = 2, DXGATEUP = 3 };
enum WFmt { W_BF16 = 0, W_NF4 = 1, W_INT8 = 2 };

// How a mode's two weight keys (if any) share a B tile: side by side along N
// (gate/up: the gate columns, then the up columns of the same channels) or
// one after the other along K (gate/up dX: K = [gate | up]).  Whether B is
// read K-major or MN-major is a separate template flag of the kernel: the
// reference's compressed experts store W as [E, out, in], so their forward
// reads B K-major and their dX MN-major; MAGI-2's experts store W as
// [E, in, out] (grouped_moe.py:109-154), the other way round.
template <int MODE> struct MCfg {
  static constexpr bool NSPLIT = MODE == GATEUP;
  static constexpr bool KSPLIT = MODE == DXGATEUP;
  static constexpr bool TWO_KEYS = NSPLIT || KSPLIT;
  // B layout of the reference's compressed-expert layout ([E, out, in]) in this mode
  static constexpr bool MN_NATIVE = MODE == DXDOWN || MODE == DXGATEUP;
};

// Gate/up activation applied by the GATEUP epilogue (and differentiated by the
// DXDOWN epilogue): SwiGLU h = silu(g) * u (experts.py:301-317), or MAGI-2's
// swiglu7 h = g' sigmoid(1.702 g') (u' + 1) with g' = min(g, 7) and
// u' = clamp(u, -7, 7) (grouped_moe.py:287-335).
enum Act { ACT_SWIGLU = 0, ACT_SWIGLU7 = 1 };

// Per (format, pairing) geometry.
template <int WF, bool PAIR> struct Cfg {
  static constexpr bool QUANT = WF != W_BF16;
  static constexpr int RT = 1;                                           // row sub-tiles per tile
  static constexpr int TN = BN / RT;                                     // output columns per tile
  static constexpr int SUB_M = PAIR ? 2 * BM : BM;                       // rows per sub-tile (UMMA M)
  static constexpr int TILE_M = RT * SUB_M;                              // rows per tile
  static constexpr uint32_t A_STAGE = RT * A_BYTES;                      // A per CTA per stage
  static constexpr int B_ROWS = PAIR ? TN / 2 : TN;                      // B rows / n-columns per CTA
  static constexpr uint32_t B_BYTES = B_ROWS * BK * 2;                   // bf16 B per CTA per stage
  static constexpr int ROW_BYTES = WF == W_NF4 ? BK / 2 : (WF == W_INT8 ? BK : 0);  // raw bytes / 64 elements
  static constexpr uint32_t RAW_BYTES = B_ROWS * ROW_BYTES;
  // WIDE (NF4 / INT8 on CTA pairs): 16 dequantiser warps, with the registers split per
  // warpgroup (setmaxnreg) so that they fit beside the epilogue.  Warps:
  //   WIDE:  0 TMA producer, 1 MMA, 2 raw-code producer, 3 spare | 4..7 epilogue | 8..23 dequant
  //   else:  0 TMA producer, 1 MMA, 2.. epilogue, then dequant (8 warps), then raw-code producer
  static constexpr bool WIDE = QUANT && PAIR;
  static constexpr int DEQ_WARPS = WIDE ? 16 : (QUANT ? 8 : 0);
  static constexpr int DEQ_THREADS = 32 * DEQ_WARPS;
  // Dequantisers: one thread per B row and k-block; KG groups of B_ROWS
  // threads take the k-blocks in turn (group g: k-blocks g, g+KG, ...).
  static constexpr int KG = QUANT ? DEQ_THREADS / B_ROWS : 1;
  static constexpr int GROUP_WARPS = QUANT ? B_ROWS / 32 : 0;            // dequant warps per group
  // (bf16 pairs: 5 operand stages, leaving room for the staged epilogue's boxes)
  static constexpr int STAGES = WF == W_BF16 ? (PAIR ? 5 : 4) : (PAIR ? 4 : 3);
  // raw-code ring: its own producer warp runs ahead of the operand ring
  static constexpr int RAW_STAGES = WF == W_BF16 ? 1 : (PAIR ? (WF == W_NF4 ? 8 : 4) : (WF == W_NF4 ? 4 : 2));
  static constexpr int EPI_WARPS = epi_warps(WF);
  static constexpr int EPI_FIRST = WIDE ? 4 : 2;
  static constexpr int DEQ_FIRST = WIDE ? 8 : 2 + EPI_WARPS;
  static constexpr int RAW_WARP = WIDE ? 2 : DEQ_FIRST + DEQ_WARPS;
  static constexpr int THREADS = WIDE ? 32 * (DEQ_FIRST + DEQ_WARPS)
                                      : 64 + 32 * EPI_WARPS + (WF == W_BF16 ? 0 : DEQ_THREADS + 32);
  // WIDE register split: launched at 80 registers per thread (65536 / 768,
  // rounded down to a multiple of 8), then producer warpgroup -> 48,
  // epilogue -> 144, dequantisers -> 72: 128*48 + 128*144 + 512*72 = 61440 =
  // 768 * 80, the launch allocation (setmaxnreg.inc draws only on registers
  // the block was launched with; the host checks the compiled count).
  static constexpr int LAUNCH_REGS = 80;
  static constexpr int REG_WG0 = 48, REG_EPI = 144, REG_DEQ = 72;
  static_assert(!WIDE || 128 * REG_WG0 + 128 * REG_EPI + DEQ_THREADS * REG_DEQ <= THREADS * LAUNCH_REGS,
                "the register split must fit in the launch allocation");
  static_assert(!QUANT || (DEQ_THREADS % B_ROWS == 0 && STAGES % KG == 0 && RAW_STAGES % KG == 0),
                "each dequantiser group must own whole stages");
};

// One quantised key (W1, W3 or W2).
struct QKey {
  const uint8_t* absmax;       // NF4: [E, out*in/64] codes
  const float* nested_absmax;  // NF4: [E, n_nested]
  const float* offset;         // NF4: [E]
  const float* code;           // NF4: [16]
  const float* nested_code;    // NF4: [256]
  const float* scale;          // INT8: [E, out]
  int n_nested;                // NF4: per expert
};

struct Params {
  const int32_t* offsets;  // [E] inclusive row cumsum
  int E;
  int64_t S;               // total routed rows
  int K;                   // reduction length
  int N;                   // output columns per row (I, H, I, H by mode)
  int n_tiles;             // column tiles per row block
  int krows;               // MN modes: K rows of one expert in one key (H for W2, I for W1/W3)
  int kb_half;             // DXGATEUP: k-blocks taken from W1 before W3
  int out_rows;            // K-major modes: rows of one expert's B matrix per key
  __nv_bfloat16* out;      // h [S,I] | y [S,H] | dgu [S,2I] | dx [S,H]
  int64_t ldo;             // elements
  __nv_bfloat16* gate_up;  // GATEUP: optional saved [S,2I] output; DXDOWN: saved input
  QKey q[2];               // quantised keys (index 1 used by GATEUP / DXGATEUP)
  int nbs_shift;           // log2(nested_blocksize)
  int has_ext;             // 1: one extra bf16 k-block (the LoRA rank block) from tmap_xa / tmap_xb
  int nsrc;                // row sources: segment s*(E/nsrc) + w holds source s's rows for weight expert w
  int act;                 // Act of the gate/up epilogue (GATEUP) and of its backward (DXDOWN)
  int prev_end;            // 1: segment 0 starts at offsets[-1] (a later chunk of > kMaxExperts groups)
};

// Control block in shared memory.  16-byte aligned size: the dequantiser
// scratch that follows it is written with 16-byte vector stores.
template <int WF, bool PAIR>
struct alignas(16) Smem {
  uint64_t full[Cfg<WF, PAIR>::STAGES];
  uint64_t empty[Cfg<WF, PAIR>::STAGES];
  uint64_t raw_full[Cfg<WF, PAIR>::RAW_STAGES];
  uint64_t raw_empty[Cfg<WF, PAIR>::RAW_STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t absq_full[2];   // NF4 pair K-major: the tile's absmax codes, prefetched
  uint64_t absq_empty[2];
  uint32_t tmem_base;
  int abort_flag;
  int row_start[kMaxExperts + 1];  // per segment, in tile order
  int seg_rows[kMaxExperts + 1];
  int tile_prefix[kMaxExperts + 1];
};

// Dequantiser scratch: per-tile absmax codes (or INT8 row scales), the
// expert's nested absmax, and the code tables, per key.
struct alignas(16) DeqSmem {
  uint8_t absq[16384];
  float nested[2][kMaxNested];
  float ncode[2][256];
  float code[2][16];
};

// Staged epilogue (CTA pairs): each epilogue warp writes 32 rows x 32 bf16
// columns of an output into one of STG_BUFS shared-memory boxes (64-byte TMA
// swizzle) and a TMA store writes the box to global memory, instead of every
// lane storing its own row (32 cache lines per warp store, whose wavefronts
// share the shared-memory port with the operand traffic).
constexpr int STG_BUFS = 3;
constexpr uint32_t STG_BOX = 32 * 64;  // bytes: 32 rows x 32 bf16
// (CTA pairs only: the single-CTA variants, kept for A/B measurement, have no room left)
template <int WF, bool PAIR> __host__ __device__ constexpr bool staged_epilogue() { return PAIR; }

template <int WF, bool PAIR>
constexpr size_t smem_bytes() {
  using C = Cfg<WF, PAIR>;
  static_assert(sizeof(Smem<WF, PAIR>) % 16 == 0 && (C::RAW_STAGES * C::RAW_BYTES) % 16 == 0,
                "the dequantiser scratch must start 16-byte aligned");
  return 1024 + C::STAGES * (C::A_STAGE + C::B_BYTES) + (WF == W_BF16 ? 0 : C::RAW_STAGES * C::RAW_BYTES) +
         sizeof(Smem<WF, PAIR>) +
         (WF == W_BF16 ? 0 : sizeof(DeqSmem)) +
         (staged_epilogue<WF, PAIR>() ? 1024 + (size_t)C::EPI_WARPS * STG_BUFS * STG_BOX : 0);
}

// Tile t -> segment j (in tile order), weight expert e, row block m, column
// block n.  Segments are visited weight-expert-major (all sources of expert 0,
// then of expert 1, ...) so that concurrent tiles share one expert's weights.
template <int WF, bool PAIR>
__device__ __forceinline__ void decode_tile(int t, const Smem<WF, PAIR>& sm, int units, int n_tiles, int& j,
                                            int& e, int& m, int& n) {
  // units: segments (one source: segment = expert), or experts (several sources)
  const int mt = t / n_tiles;
  n = t - mt * n_tiles;
  int lo = 0, hi = units;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (sm.tile_prefix[mid] <= mt) lo = mid;
    else hi = mid;
  }
  j = lo;
  e = lo;
  m = mt - sm.tile_prefix[lo];
}

// Several sources: an expert's rows are its nsrc segments e*nsrc + s (tile
// order), cut into BM-row blocks segment by segment; tile m of the expert takes
// blocks m*BPT .. m*BPT + BPT-1 (BPT = CTAs per tile), so a CTA pair can hold
// blocks of two sources and no tile is cut at a source boundary beyond a
// block.  Block q: first memory row and rows (0 past the expert's last block).
template <int WF, bool PAIR>
__device__ __forceinline__ void source_block(const Smem<WF, PAIR>& sm, int e, int nsrc, int q, int& row, int& rows) {
  for (int s = 0; s < nsrc; ++s) {
    const int len = sm.seg_rows[e * nsrc + s];
    const int nb = (len + BM - 1) / BM;
    if (q < nb) {
      row = sm.row_start[e * nsrc + s] + q * BM;
      rows = min(BM, len - q * BM);
      return;
    }
    q -= nb;
  }
  row = 0;
  rows = 0;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// MAGI-2's swiglu7 on bf16 gate / up values, in fp32 (grouped_moe.py:287-306):
// g' = min(g, 7), u' = clamp(u, -7, 7), h = g' sigmoid(1.702 g') (u' + 1).
__device__ __forceinline__ float swiglu7(float g, float u) {
  const float gc = fminf(g, 7.f), uc = fminf(fmaxf(u, -7.f), 7.f);
  const float sg = __fdividef(1.f, 1.f + __expf(-1.702f * gc));
  return gc * sg * (uc + 1.f);
}

// Its backward (grouped_moe.py:309-335): given dh, the gradients of the
// unclamped gate and up; the clamps pass no gradient outside their ranges.
__device__ __forceinline__ void swiglu7_backward(float dh, float g, float u, float& dg, float& du) {
  const float gc = fminf(g, 7.f), uc = fminf(fmaxf(u, -7.f), 7.f);
  const float sg = __fdividef(1.f, 1.f + __expf(-1.702f * gc));
  const float dgate = g <= 7.f ? sg + 1.702f * gc * sg * (1.f - sg) : 0.f;
  dg = dh * dgate * (uc + 1.f);
  du = (u >= -7.f && u <= 7.f) ? dh * (gc * sg) : 0.f;
}

// Per-warpgroup register budget (all four warps of the group execute it).
template <int N> __device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N> __device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
  return d;
}

// ---------------------------------------------------------------------------
// NF4 decode without memory lookups.  For one 64-element block the 16
// possible outputs bf16(code[j] * scale) are formed once; their low and high
// bytes are split into lo[4] / hi[4] (4 entries per register) so that PRMT
// can select one entry per output byte from a 4-bit index.
struct Nf4Tab {
  uint32_t lo[4], hi[4];
};

__device__ __forceinline__ void nf4_table(const float* code, float scale, Nf4Tab& t) {
  uint32_t q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = pack_bf16x2(__fmul_rn(code[2 * i], scale), __fmul_rn(code[2 * i + 1], scale));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    t.lo[j] = prmt(q[2 * j], q[2 * j + 1], 0x6420);
    t.hi[j] = prmt(q[2 * j], q[2 * j + 1], 0x7531);
  }
}

// One packed word = 8 elements, the first element in the high nibble of
// byte 0.  Produces 4 registers of bf16 pairs in element order.
__device__ __forceinline__ void nf4_word(uint32_t w, const Nf4Tab& t, uint32_t (&o)[4]) {
  const uint32_t sel = w & 0x77777777u;  // entry within the 8-entry half
  const uint32_t selh = sel >> 16;
  const uint32_t wsh = w << 4;
  // byte masks: 0xFF where the nibble's bit 3 is set (entries 8..15), from the
  // sign-replicating PRMT mode on the byte whose msb is that bit
  const uint32_t m0 = prmt(w, wsh, 0x9D8C);
  const uint32_t m1 = prmt(w, wsh, 0xBFAE);
  const uint32_t lo0 = (prmt(t.lo[0], t.lo[1], sel) & ~m0) | (prmt(t.lo[2], t.lo[3], sel) & m0);
  const uint32_t hi0 = (prmt(t.hi[0], t.hi[1], sel) & ~m0) | (prmt(t.hi[2], t.hi[3], sel) & m0);
  const uint32_t lo1 = (prmt(t.lo[0], t.lo[1], selh) & ~m1) | (prmt(t.lo[2], t.lo[3], selh) & m1);
  const uint32_t hi1 = (prmt(t.hi[0], t.hi[1], selh) & ~m1) | (prmt(t.hi[2], t.hi[3], selh) & m1);
  // selector nibbles address [second, first, fourth, third] element of each byte pair
  o[0] = prmt(lo0, hi0, 0x4051);
  o[1] = prmt(lo0, hi0, 0x6273);
  o[2] = prmt(lo1, hi1, 0x4051);
  o[3] = prmt(lo1, hi1, 0x6273);
}

// 16 int8 (one uint4) -> 16 bf16(q * scale) as 8 registers.
__device__ __forceinline__ void int8_x16(const uint4 r, float scale, uint32_t (&o)[8]) {
  const uint32_t words[4] = {r.x, r.y, r.z, r.w};
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
}

// K-major modes: first weight row (within the [E * out_rows] row space) of the
// B block `h` (TN/2 rows) of tile (e, n): h = 0/1 are the two halves of the
// TN-column tile (gate/up: W1 and W3 rows n*TN/2..; down: W2 rows n*TN + h*TN/2..).
template <int MODE, int TN>
__device__ __forceinline__ int kmajor_row(const Params& p, int e, int n, int h) {
  return MODE == GATEUP ? e * p.out_rows + n * (TN / 2) : e * p.out_rows + n * TN + h * (TN / 2);
}

template <int MODE, int WF, bool PAIR, bool BMN>
__global__ void __launch_bounds__(Cfg<WF, PAIR>::THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b0,
                        const __grid_constant__ CUtensorMap tmap_b1, const __grid_constant__ CUtensorMap tmap_xa,
                        const __grid_constant__ CUtensorMap tmap_xb, const __grid_constant__ CUtensorMap tmap_o0,
                        const __grid_constant__ CUtensorMap tmap_o1, const __grid_constant__ CUtensorMap tmap_o2,
                        const Params p) {
  using C = Cfg<WF, PAIR>;
  constexpr int STAGES = C::STAGES;
  constexpr uint32_t B_BYTES = C::B_BYTES;
  constexpr uint32_t RAW_BYTES = C::RAW_BYTES;
  constexpr int TILE_M = C::TILE_M;
  constexpr int RT = C::RT;
  constexpr int TN = C::TN;
  constexpr int SUB_M = C::SUB_M;
  constexpr uint32_t A_STAGE = C::A_STAGE;
  constexpr bool QUANT = WF != W_BF16;
  constexpr bool MN = BMN;
  using MC = MCfg<MODE>;
  // B layouts other than the compressed-expert one run on CTA pairs only
  static_assert(PAIR || MN == MC::MN_NATIVE, "the transposed weight layout runs on CTA pairs");
  // NF4 on CTA pairs: each tile's absmax codes reach one of two buffers a
  // tile ahead of use, so the dequantisers never stop to stage them.  K-major,
  // they are one contiguous run of B_ROWS x K/64 bytes, bulk-copied by the
  // raw-code producer; MN-major, K rows of B_ROWS/64 bytes strided by the
  // weight row, gathered by the spare warp of warpgroup 0.
  constexpr bool PREFETCH = WF == W_NF4 && PAIR;
  constexpr int ABUF = 8192;  // bytes per prefetch buffer: B_ROWS x K/64 or K x B_ROWS/64, K <= 4096
  static_assert(!PREFETCH || (C::WIDE && C::RAW_WARP == 2), "the absmax gatherer is warp 3 of the wide layout");
  static_assert(!PREFETCH || MN || C::B_ROWS * (kMaxK / BK) <= ABUF, "a K-major tile's codes fit one buffer");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = sA + STAGES * A_STAGE;
  uint8_t* sRaw = sB + STAGES * B_BYTES;
  constexpr int RAW_STAGES = C::RAW_STAGES;
  Smem<WF, PAIR>& sm = *reinterpret_cast<Smem<WF, PAIR>*>(sRaw + (QUANT ? RAW_STAGES * RAW_BYTES : 0));
  DeqSmem* dq = reinterpret_cast<DeqSmem*>(reinterpret_cast<uint8_t*>(&sm) + sizeof(Smem<WF, PAIR>));
  constexpr bool STAGED = staged_epilogue<WF, PAIR>();
  // staging boxes of the epilogue warps (1024-byte aligned: the swizzle pattern repeats every 512 bytes)
  uint8_t* sStage = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(dq) + (QUANT ? sizeof(DeqSmem) : 0) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // position in the CTA pair
  // this CTA's key of an N-split tile, and the key / k-block-in-key of a k-block
  auto key_of = [&](int kb) -> int {
    return MC::KSPLIT ? (kb >= p.kb_half ? 1 : 0) : ((MC::NSPLIT && PAIR) ? (int)rank : 0);
  };
  auto kk_of = [&](int kb, int key) -> int { return (MC::KSPLIT && key) ? kb - p.kb_half : kb; };
  // MN-major: first column (in the key's matrix) of 64-column block nb of this CTA's B
  auto mn_col = [&](int n, int nb) -> int {
    return MC::NSPLIT ? n * (C::TN / 2) + nb * 64 : n * C::TN + (int)rank * C::B_ROWS + nb * 64;
  };
  const bool leader = rank == 0;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // tile-scheduling unit
  const int num_units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  // shared::cluster address of a barrier of this CTA as seen from the pair's leader
  auto leader_addr = [&](uint64_t* bar) -> uint32_t {
    return PAIR ? mapa_shared(smem_u32(bar), 0) : smem_u32(bar);
  };
  // the leader's `full` barriers as seen from this CTA (stage s at + 8 s)
  const uint32_t full_leader0 = leader_addr(&sm.full[0]);

  // ---- segment table, in tile order j: row_start / seg_rows and the exclusive
  // prefix of TILE_M-row blocks.  Tile-order segment j is memory segment
  // g = (j % nsrc) * (E / nsrc) + j / nsrc (offsets are inclusive ends in memory order).
  if (warp == 0) {
    const int nsrc = p.nsrc, wexp = E / nsrc;
    int carry = 0;
    for (int j0 = 0; j0 < E; j0 += 32) {
      const int j = j0 + lane;
      int cnt = 0;
      if (j < E) {
        const int g = (j % nsrc) * wexp + j / nsrc;
        const int64_t end = p.offsets[g];
        const int64_t beg = (g > 0 || p.prev_end) ? p.offsets[g - 1] : 0;
        const int64_t endc = end < p.S ? end : p.S;
        cnt = endc > beg ? (int)((endc - beg + TILE_M - 1) / TILE_M) : 0;
        if (end < beg || end > p.S) device_fail(MIRAI_ERR_DEVICE_BOUNDS, 600 + MODE);
        sm.row_start[j] = (int)beg;
        sm.seg_rows[j] = endc > beg ? (int)(endc - beg) : 0;
      }
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (j < E) sm.tile_prefix[j] = carry + incl - cnt;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) sm.tile_prefix[E] = carry;
    if (nsrc > 1) {
      // several sources: tiles per expert = its BM-row blocks over all its
      // segments, CTAs-per-tile at a time; the prefix is over experts instead
      constexpr int BPT = PAIR ? 2 : 1;
      __syncwarp();  // the segment table above is complete
      carry = 0;
      for (int e0 = 0; e0 < wexp; e0 += 32) {
        const int e = e0 + lane;
        int blocks = 0;
        if (e < wexp)
          for (int s = 0; s < nsrc; ++s) blocks += (sm.seg_rows[e * nsrc + s] + BM - 1) / BM;
        const int cnt = (blocks + BPT - 1) / BPT;
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        if (e < wexp) sm.tile_prefix[e] = carry + incl - cnt;
        carry += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) sm.tile_prefix[wexp] = carry;
    }
  }
  if (warp == 1) {
    if (lane == 0) {
      const int pair_mult = PAIR ? 2 : 1;
      for (int s = 0; s < STAGES; ++s) {
        // full: the leader's producer arrive (with the bytes of both CTAs) plus
        // every dequantiser warp of the pair
        mbar_init(&sm.full[s], 1 + (QUANT ? C::GROUP_WARPS * pair_mult : 0));
        mbar_init(&sm.empty[s], 1);
      }
      for (int s = 0; s < RAW_STAGES; ++s) {
        mbar_init(&sm.raw_full[s], 1);
        mbar_init(&sm.raw_empty[s], C::GROUP_WARPS);
      }
      for (int a = 0; a < 2; ++a) {
        mbar_init(&sm.absq_full[a], 32);  // every lane of the gathering warp
        mbar_init(&sm.absq_empty[a], C::DEQ_WARPS);
        mbar_init(&sm.tfull[a], 1);
        mbar_init(&sm.tempty[a], C::EPI_WARPS * pair_mult);
      }
      sm.abort_flag = 0;
      fence_mbar_init();
    }
    __syncwarp();
    if (PAIR) {
      tmem_alloc_pair(&sm.tmem_base, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&sm.tmem_base, TMEM_COLS);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b0);
    prefetch_tmap(&tmap_b1);
  }
  if (WF == W_NF4 && warp >= C::DEQ_FIRST && warp < C::DEQ_FIRST + C::DEQ_WARPS) {
    const int d = threadIdx.x - 32 * C::DEQ_FIRST;
    for (int h = 0; h < 2; ++h) {
      for (int i = d; i < 256; i += C::DEQ_THREADS) dq->ncode[h][i] = __ldg(p.q[h].nested_code + i);
      if (d < 16) dq->code[h][d] = __ldg(p.q[h].code + d);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA signal
  tc_fence_after();

  const uint32_t tmem_base = sm.tmem_base;
  const int units = p.nsrc > 1 ? E / p.nsrc : E;  // tile-order units: segments, or experts
  const int total_tiles = sm.tile_prefix[units] * p.n_tiles;
  constexpr int BPT = PAIR ? 2 : 1;               // BM-row blocks per tile
  static_assert(RT == 1, "source blocks assume one row sub-tile per tile");
  const int num_kb = p.K / BK;
  // the rank block of a fused LoRA adapter is one more k-block: A from tmap_xa
  // ([S, 64] bf16), B from tmap_xb (bf16, the layout of this mode's B)
  const int total_kb = num_kb + p.has_ext;
  volatile int* abort_flag = &sm.abort_flag;

  // Role bodies; dispatched below.
  auto role_producer = [&]() {
    // ======================= TMA producer =======================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = unit; t < total_tiles && !*abort_flag; t += num_units) {
        int j, e, m, n;
        decode_tile<WF, PAIR>(t, sm, units, p.n_tiles, j, e, m, n);
        int row0 = sm.row_start[j] + m * TILE_M + (int)rank * BM;
        if (p.nsrc > 1) {  // this CTA's block (a past-the-end block loads rows 0..: never stored)
          int rows;
          source_block(sm, e, p.nsrc, m * BPT + (int)rank, row0, rows);
        }
        // sub-tiles holding rows of this segment (the first always does)
        const int seg_rows = p.nsrc > 1 ? TILE_M : sm.seg_rows[j];
        const int n_live = (RT == 2 && m * TILE_M + SUB_M >= seg_rows) ? 1 : RT;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&sm.empty[stage], phase ^ 1, 10)) {
            *abort_flag = 1;
            break;
          }
          const uint32_t full_addr = full_leader0 + 8u * stage;
          const bool ext = kb == num_kb;  // the fused rank block
          // B source for this k-block: its key, the k-block inside the key
          const int key = key_of(kb), kk = kk_of(kb, key);
          const CUtensorMap* mb = key ? &tmap_b1 : &tmap_b0;
          const int krow = MN ? e * p.krows + kk * BK : 0;
          const int pair_mult = PAIR ? 2 : 1;
          if (leader) {
            const uint32_t bytes = pair_mult * (n_live * A_BYTES + ((QUANT && !ext) ? 0u : B_BYTES));
            // the leader's own barrier: a CTA-local arrive carries the bytes of both CTAs
            mbar_arrive_expect_tx(&sm.full[stage], bytes);
          }
          auto load = [&](void* dst, const CUtensorMap* map, int x, int y) {
            if (PAIR) tma_load_2d_pair(dst, map, x, y, full_addr);
            else tma_load_2d(dst, map, x, y, &sm.full[stage]);
          };
          if (ext) {
            uint8_t* b_dst = sB + stage * B_BYTES;
            if (MN) {
#pragma unroll
              for (int nb = 0; nb < C::B_ROWS / 64; ++nb)
                load(b_dst + nb * 8192, &tmap_xb, n * TN + (int)rank * C::B_ROWS + nb * 64, e * BK);
            } else if (PAIR) {
              load(b_dst, &tmap_xb, 0, kmajor_row<MODE, TN>(p, e, n, (int)rank));
            } else {
              load(b_dst, &tmap_xb, 0, kmajor_row<MODE, TN>(p, e, n, 0));
              load(b_dst + B_BYTES / 2, &tmap_xb, 0, kmajor_row<MODE, TN>(p, e, n, 1));
            }
          } else if (!QUANT) {
            uint8_t* b_dst = sB + stage * B_BYTES;
            if (MN) {
              // this CTA's 64-column blocks of the key's [K, N] matrix
#pragma unroll
              for (int nb = 0; nb < C::B_ROWS / 64; ++nb) load(b_dst + nb * 8192, mb, mn_col(n, nb), krow);
            } else if (PAIR) {
              // B_ROWS rows per CTA: gate/up -> rank 0 W1, rank 1 W3; others -> rows block `rank`
              load(b_dst, mb, kk * BK, kmajor_row<MODE, TN>(p, e, n, (int)rank));
            } else {
              load(b_dst, MODE == GATEUP ? &tmap_b0 : mb, kk * BK, kmajor_row<MODE, TN>(p, e, n, 0));
              load(b_dst + B_BYTES / 2, MODE == GATEUP ? &tmap_b1 : mb, kk * BK, kmajor_row<MODE, TN>(p, e, n, 1));
            }
          }
          for (int sub = 0; sub < n_live; ++sub) {
            uint8_t* a_dst = sA + stage * A_STAGE + sub * A_BYTES;
            if (ext) load(a_dst, &tmap_xa, 0, row0 + sub * SUB_M);
            else load(a_dst, &tmap_a, kb * BK, row0 + sub * SUB_M);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // tail: wait for the final MMA completion of every stage so that no
      // commit from the pair's leader targets this CTA after it exits
      for (int i = 0; i < STAGES; ++i) {
        if (!mbar_wait(&sm.empty[stage], phase ^ 1, 12)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  };
  auto role_mma = [&]() {
    // ======================= UMMA issuer (the leader of a pair) =======================
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_bf16(SUB_M, TN, false, MN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = unit; t < total_tiles && !*abort_flag; t += num_units, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&sm.tempty[acc], acc_phase ^ 1, 20)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        int j, e, m, n;
        decode_tile<WF, PAIR>(t, sm, units, p.n_tiles, j, e, m, n);
        const int seg_rows = p.nsrc > 1 ? TILE_M : sm.seg_rows[j];
        const int n_live = (RT == 2 && m * TILE_M + SUB_M >= seg_rows) ? 1 : RT;
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&sm.full[stage], phase, 21)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
          for (int sub = 0; sub < n_live; ++sub) {
            const uint32_t a_addr = smem_u32(sA + stage * A_STAGE + sub * A_BYTES);
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k) {
              const uint64_t ad = make_sdesc_sw128(a_addr + k * UMMA_K * 2, 16, 1024);
              const uint64_t bd = MN ? make_sdesc_sw128(b_addr + k * UMMA_K * 128, 8192, 1024)
                                     : make_sdesc_sw128(b_addr + k * UMMA_K * 2, 16, 1024);
              if (PAIR) umma_bf16_pair(d_tmem + sub * TN, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
              else umma_bf16(d_tmem + sub * TN, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            }
          }
          if (PAIR) umma_commit_pair(&sm.empty[stage], 0x3);
          else umma_commit(&sm.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        if (PAIR) umma_commit_pair(&sm.tfull[acc], 0x3);
        else umma_commit(&sm.tfull[acc]);
      }
    }
  };
  auto role_epilogue = [&]() {
    // ======================= epilogue =======================
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    // warps sharing a lane quarter split the 32-column chunks between them
    constexpr int NSPLIT = C::EPI_WARPS / 4;
    const int part = (warp - C::EPI_FIRST) / 4;
    const uint32_t tempty_leader0 = leader_addr(&sm.tempty[0]), tempty_leader1 = leader_addr(&sm.tempty[1]);
    int stg = 0;  // the next staging box of this warp
    // Write one 32 x 32 bf16 block (this lane's row: 16 packed words) through a
    // staging box to `map` at (col, row0): the whole warp, rows row0..row0+31 all valid.
    auto stage_store = [&](const CUtensorMap* map, int col, int64_t row0, const uint32_t (&w)[16]) {
      uint8_t* box = sStage + ((warp - C::EPI_FIRST) * STG_BUFS + stg) * STG_BOX;
      if (lane == 0) bulk_wait_group_read<STG_BUFS - 1>();  // the box's previous store has read it
      __syncwarp();
      const uint32_t rowaddr = smem_u32(box) + (uint32_t)lane * 64u;
      const uint32_t sw = (uint32_t)(lane >> 1) & 3u;  // 64-byte swizzle: 16-byte chunk ^= row bits 1..2
#pragma unroll
      for (int v = 0; v < 4; ++v)
        st_shared_v4(rowaddr + (((uint32_t)v ^ sw) << 4), w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(map, box, col, (int)row0);
        bulk_commit_group();
      }
      stg = stg + 1 == STG_BUFS ? 0 : stg + 1;
    };
    int it = 0;
    for (int t = unit; t < total_tiles && !*abort_flag; t += num_units, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      int j, e, m, n;
      decode_tile<WF, PAIR>(t, sm, units, p.n_tiles, j, e, m, n);
      int blk_row = 0, blk_rows = 0;  // several sources: this CTA's block
      if (p.nsrc > 1) source_block(sm, e, p.nsrc, m * BPT + (int)rank, blk_row, blk_rows);
      const int64_t seg_rows = sm.seg_rows[j];
      if (MODE == DXDOWN && p.gate_up != nullptr) {
        // The SwiGLU backward reads this tile's saved gate and up columns: start
        // bringing this thread's row of both into L2 while the accumulator fills.
        const int col0 = n * TN;
        const int cols = min(TN, p.N - col0);
        for (int sub = 0; sub < RT && cols > 0; ++sub) {
          const int lr = q * 32 + lane;
          const int r = sub * SUB_M + (int)rank * BM + lr;
          const bool live = p.nsrc > 1 ? lr < blk_rows : (int64_t)m * TILE_M + r < seg_rows;
          if (!live || part != 0) continue;
          const int64_t grow = p.nsrc > 1 ? (int64_t)blk_row + lr : (int64_t)sm.row_start[j] + (int64_t)m * TILE_M + r;
          const __nv_bfloat16* base = p.gate_up + grow * 2 * (int64_t)p.N + col0;
          prefetch_l2_bulk(base, (uint32_t)cols * 2u);
          prefetch_l2_bulk(base + p.N, (uint32_t)cols * 2u);
        }
      }
      if (!mbar_wait(&sm.tfull[acc], acc_phase, 30)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      for (int sub = 0; sub < RT; ++sub) {
      // no rows in this sub-tile (warp-uniform; several sources: blocks say)
      if (p.nsrc == 1 && (int64_t)m * TILE_M + sub * SUB_M >= seg_rows) break;
      const int r = sub * SUB_M + (int)rank * BM + q * 32 + lane;  // row inside the tile
      const int lr = q * 32 + lane;                                 // row inside this CTA's block
      const bool valid = p.nsrc > 1 ? lr < blk_rows : (int64_t)m * TILE_M + r < seg_rows;
      const int64_t grow = p.nsrc > 1 ? (int64_t)blk_row + lr : (int64_t)sm.row_start[j] + (int64_t)m * TILE_M + r;
      const uint32_t tb = tmem_base + acc * BN + sub * TN + ((uint32_t)(q * 32) << 16);
      // all 32 rows of this warp belong to the segment: stores go through TMA boxes
      const bool boxed = STAGED && __all_sync(0xffffffffu, valid);
      const int64_t row0 = __shfl_sync(0xffffffffu, grow, 0);
      if (MODE == GATEUP) {
        const int col0 = n * (TN / 2);
        constexpr int NCH = TN / 64;  // 32-column chunks of gate (and of up)
#pragma unroll 1
        for (int c = part * (NCH / NSPLIT); c < (part + 1) * (NCH / NSPLIT); ++c) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tb + c * 32, g);
          tmem_ld_32x32b_x32(tb + TN / 2 + c * 32, u);
          tmem_ld_wait();
          if (valid && col0 + c * 32 < p.N) {  // the last tile of an I % 128 == 64 layer is half empty
            uint32_t hp[16], gp[16], up[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // Round where the reference's bf16 tensors round: gate and up (the
              // GEMM outputs), then SwiGLU's silu(gate) and product (experts.py:301-317)
              // or swiglu7 in fp32 on the bf16 gate/up (grouped_moe.py:287-306).
              // (column pairs as bf16x2: the product of two bf16 values is exact in fp32, so
              // mul.rn.bf16x2 rounds it as an fp32 multiply and a bf16 rounding would)
              gp[j] = pack_bf16x2(__uint_as_float(g[2 * j]), __uint_as_float(g[2 * j + 1]));
              up[j] = pack_bf16x2(__uint_as_float(u[2 * j]), __uint_as_float(u[2 * j + 1]));
              const float g0 = bf16_lo(gp[j]), g1 = bf16_hi(gp[j]);
              if (p.act == ACT_SWIGLU7) {
                hp[j] = pack_bf16x2(swiglu7(g0, bf16_lo(up[j])), swiglu7(g1, bf16_hi(up[j])));
              } else {
                const float a0 = __fdividef(g0, 1.f + __expf(-g0));
                const float a1 = __fdividef(g1, 1.f + __expf(-g1));
                hp[j] = bf16x2_mul(pack_bf16x2(a0, a1), up[j]);
              }
            }
            if (boxed) {
              stage_store(&tmap_o0, col0 + c * 32, row0, hp);
              if (p.gate_up != nullptr) {
                stage_store(&tmap_o1, col0 + c * 32, row0, gp);
                stage_store(&tmap_o2, col0 + c * 32, row0, up);
              }
              continue;
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
      } else if (MODE == DXDOWN && p.gate_up != nullptr) {
        // dgu = SwiGLU backward of the saved (gate, up) given dh = dy W2
        // (without saved gate/up: dh itself, [S, I], by the plain epilogue below)
        // (autograd of experts.py:301-317 in bf16: mul, silu backward)
        const int64_t ld2 = 2 * (int64_t)p.N;
        constexpr int NCH = TN / 32;
        const int c_first = part * (NCH / NSPLIT), c_end = (part + 1) * (NCH / NSPLIT);
        // the saved gate/up of the next chunk are loaded while this chunk computes
        uint4 gnext[4], unext[4];
        auto load_gu = [&](int c) {
          const int col = n * TN + c * 32;
          if (valid && col < p.N) {
            const uint4* gs = reinterpret_cast<const uint4*>(p.gate_up + grow * ld2 + col);
            const uint4* us = reinterpret_cast<const uint4*>(p.gate_up + grow * ld2 + p.N + col);
#pragma unroll
            for (int v = 0; v < 4; ++v) gnext[v] = gs[v], unext[v] = us[v];
          }
        };
        load_gu(c_first);
#pragma unroll 1
        for (int c = c_first; c < c_end; ++c) {
          const int col = n * TN + c * 32;
          uint32_t gw[16], uw[16];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            gw[4 * v] = gnext[v].x, gw[4 * v + 1] = gnext[v].y, gw[4 * v + 2] = gnext[v].z, gw[4 * v + 3] = gnext[v].w;
            uw[4 * v] = unext[v].x, uw[4 * v + 1] = unext[v].y, uw[4 * v + 2] = unext[v].z, uw[4 * v + 3] = unext[v].w;
          }
          if (c + 1 < c_end) load_gu(c + 1);
          uint32_t v32[32];
          tmem_ld_32x32b_x32(tb + c * 32, v32);
          tmem_ld_wait();
          if (valid && col < p.N) {
            uint32_t dg[16], du[16];
            // (the register budget of the NF4 / INT8 epilogue warps keeps them on the per-element form)
            if (WF != W_BF16 || p.act == ACT_SWIGLU7) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                float dgo[2], duo[2];
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                  const float dh = bf16r(__uint_as_float(v32[2 * j + hh]));
                  const float gv = hh ? bf16_hi(gw[j]) : bf16_lo(gw[j]);
                  const float uv = hh ? bf16_hi(uw[j]) : bf16_lo(uw[j]);
                  if (p.act == ACT_SWIGLU7) {
                    swiglu7_backward(dh, gv, uv, dgo[hh], duo[hh]);
                    continue;
                  }
                  const float sg = __fdividef(1.f, 1.f + __expf(-gv));
                  const float act = bf16r(gv * sg);
                  const float dact = bf16r(dh * uv);
                  duo[hh] = dh * act;
                  dgo[hh] = dact * sg * (1.f + gv * (1.f - sg));
                }
                dg[j] = pack_bf16x2(dgo[0], dgo[1]);
                du[j] = pack_bf16x2(duo[0], duo[1]);
              }
            } else {
              // Column pairs as bf16x2: dh, silu(g) and the products dh*up, dh*act are the
              // reference's bf16 tensors; a product of two bf16 values is exact in fp32, so the
              // packed multiply rounds it exactly as an fp32 multiply and a bf16 rounding would.
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const uint32_t dh2 = pack_bf16x2(__uint_as_float(v32[2 * j]), __uint_as_float(v32[2 * j + 1]));
                const float g0 = bf16_lo(gw[j]), g1 = bf16_hi(gw[j]);
                const float s0 = __fdividef(1.f, 1.f + __expf(-g0));
                const float s1 = __fdividef(1.f, 1.f + __expf(-g1));
                const uint32_t dact2 = bf16x2_mul(dh2, uw[j]);
                du[j] = bf16x2_mul(dh2, pack_bf16x2(g0 * s0, g1 * s1));
                const float d0 = bf16_lo(dact2), d1 = bf16_hi(dact2);
                dg[j] = pack_bf16x2(d0 * s0 * (1.f + g0 * (1.f - s0)), d1 * s1 * (1.f + g1 * (1.f - s1)));
              }
            }
            if (boxed) {
              stage_store(&tmap_o0, col, row0, dg);  // the gate half of dgu
              stage_store(&tmap_o1, col, row0, du);  // the up half
              continue;
            }
            uint4* gd = reinterpret_cast<uint4*>(p.out + grow * ld2 + col);
            uint4* ud = reinterpret_cast<uint4*>(p.out + grow * ld2 + p.N + col);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              gd[v] = make_uint4(dg[4 * v], dg[4 * v + 1], dg[4 * v + 2], dg[4 * v + 3]);
              ud[v] = make_uint4(du[4 * v], du[4 * v + 1], du[4 * v + 2], du[4 * v + 3]);
            }
          }
        }
      } else {
        const int col0 = n * TN;
        constexpr int NCH = TN / 32;
#pragma unroll 1
        for (int c = part * (NCH / NSPLIT); c < (part + 1) * (NCH / NSPLIT); ++c) {
          uint32_t v32[32];
          tmem_ld_32x32b_x32(tb + c * 32, v32);
          tmem_ld_wait();
          if (valid && col0 + c * 32 < p.N) {
            uint32_t yp[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) yp[j] = pack_bf16x2(__uint_as_float(v32[2 * j]), __uint_as_float(v32[2 * j + 1]));
            if (boxed) {
              stage_store(&tmap_o0, col0 + c * 32, row0, yp);
              continue;
            }
            uint4* dst = reinterpret_cast<uint4*>(p.out + grow * p.ldo + col0 + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = make_uint4(yp[4 * v], yp[4 * v + 1], yp[4 * v + 2], yp[4 * v + 3]);
          }
        }
      }
      }  // sub-tiles
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
        else mbar_arrive(&sm.tempty[acc]);
      }
    }
    // this warp's TMA stores have written global memory (and read their boxes) before the CTA exits
    if (STAGED && lane == 0) bulk_wait_group_all();
    __syncwarp();
  };
  auto role_raw = [&]() {
    // ======================= raw-code producer (NF4 / INT8) =======================
    // Streams this CTA's share of the packed codes of every k-block into the
    // raw ring, up to RAW_STAGES ahead of the dequantisers.
    if (lane == 0) {
      int rstage = 0;
      uint32_t rphase = 0;
      constexpr int RB = C::ROW_BYTES;
      for (int t = unit; t < total_tiles && !*abort_flag; t += num_units) {
        int j, e, m, n;
        decode_tile<WF, PAIR>(t, sm, units, p.n_tiles, j, e, m, n);
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&sm.raw_empty[rstage], rphase ^ 1, 11)) {
            *abort_flag = 1;
            break;
          }
          const bool ext = kb == num_kb;  // the rank block has no raw codes: an empty stage
          mbar_arrive_expect_tx(&sm.raw_full[rstage], ext ? 0u : RAW_BYTES);
          if (!ext) {
            const int key = key_of(kb), kk = kk_of(kb, key);
            const CUtensorMap* mb = key ? &tmap_b1 : &tmap_b0;
            const int krow = MN ? e * p.krows + kk * BK : 0;
            uint8_t* r_dst = sRaw + rstage * RAW_BYTES;
            if (MN) {
#pragma unroll
              for (int nb = 0; nb < C::B_ROWS / 64; ++nb)
                tma_load_2d(r_dst + nb * 64 * RB, mb, mn_col(n, nb) * RB / 64, krow, &sm.raw_full[rstage]);
            } else if (PAIR) {
              tma_load_2d(r_dst, mb, kk * RB, kmajor_row<MODE, TN>(p, e, n, (int)rank), &sm.raw_full[rstage]);
            } else {
              tma_load_2d(r_dst, MODE == GATEUP ? &tmap_b0 : mb, kk * RB, kmajor_row<MODE, TN>(p, e, n, 0),
                          &sm.raw_full[rstage]);
              tma_load_2d(r_dst + RAW_BYTES / 2, MODE == GATEUP ? &tmap_b1 : mb, kk * RB,
                          kmajor_row<MODE, TN>(p, e, n, 1), &sm.raw_full[rstage]);
            }
          }
          if (++rstage == RAW_STAGES) {
            rstage = 0;
            rphase ^= 1;
          }
        }
      }
    }
  };
  auto role_absq = [&]() {
    // ======================= absmax gatherer (NF4 pairs) =======================
    // Fills one of two buffers with a tile's absmax codes a tile ahead of the
    // dequantisers (which release them), laid out so that the 32 lanes of a
    // dequantiser warp, reading the codes of 32 consecutive B rows for one
    // k-block, read 32 consecutive bytes (one shared-memory wavefront):
    //   K-major: buffer[kb * B_ROWS + r] = code of (this CTA's weight row r, k-block kb);
    //   MN-major: buffer[kk * NB + j] = code of (k-row kk, this CTA's column block j).
    constexpr int NB = C::B_ROWS / 64;
    const int nblk_row = p.N / 64;  // NF4 blocks per weight row (MN-major)
    int tl = 0;
    for (int t = unit; t < total_tiles && !*abort_flag; t += num_units, ++tl) {
      int j, e, m, n;
      decode_tile<WF, PAIR>(t, sm, units, p.n_tiles, j, e, m, n);
      const int buf = tl & 1;
      if (tl >= 2 && !mbar_wait(&sm.absq_empty[buf], ((tl >> 1) - 1) & 1, 14)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* dst = dq->absq + buf * ABUF;
      if (!MN) {
        // this CTA's weight rows of the tile: `rows` x num_kb codes, contiguous in
        // global memory (row-major, 16-byte aligned: rows is a multiple of 64)
        const int first = kmajor_row<MODE, TN>(p, e, n, (int)rank) - e * p.out_rows;
        const int rows = min(C::B_ROWS, p.out_rows - first);
        // k-blocks per weight row of one key: a K-split tile takes the first kb_half
        // k-blocks from key 0 and the rest from key 1
        const int nkbk = MC::KSPLIT ? p.kb_half : num_kb;
        for (int kq = 0; kq < (MC::KSPLIT ? 2 : 1); ++kq) {
          const int key = MC::KSPLIT ? kq : (MC::NSPLIT ? (int)rank : 0);
          const uint4* src = reinterpret_cast<const uint4*>(
              p.q[key].absmax + (size_t)kmajor_row<MODE, TN>(p, e, n, (int)rank) * nkbk);
          const int chunks = rows > 0 ? rows * nkbk / 16 : 0;
#pragma unroll 1
          for (int c = lane; c < chunks; c += 32) {
            const uint4 v = __ldg(src + c);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            int r = (16 * c) / nkbk, kb = 16 * c - r * nkbk;
#pragma unroll
            for (int b = 0; b < 16; ++b) {
              dst[(kq * nkbk + kb) * C::B_ROWS + r] = (uint8_t)(w[b >> 2] >> (8 * (b & 3)));
              if (++kb == nkbk) kb = 0, ++r;
            }
          }
        }
        mbar_arrive(&sm.absq_full[buf]);  // release: this lane's stores are visible to the waiters
        continue;
      }
      const int nb0 = mn_col(n, 0) / 64;  // first column block of this CTA in the key's rows (even)
      static_assert(!(PREFETCH && MN) || NB == 2, "one 16-bit load covers this CTA's two column blocks");
      if (NB == 2 && (nblk_row & 1) == 0 && nb0 + 1 < nblk_row) {
        // both codes of a k-row in one aligned 16-bit load, four k-rows in flight per lane
#pragma unroll 4
        for (int kk = lane; kk < p.K; kk += 32) {
          const int key = MC::KSPLIT ? (kk >= p.krows ? 1 : 0) : (MC::NSPLIT ? (int)rank : 0);
          const int wr = (MC::KSPLIT && key) ? kk - p.krows : kk;
          const uint8_t* src = p.q[key].absmax + ((size_t)e * p.krows + wr) * nblk_row + nb0;
          reinterpret_cast<uint16_t*>(dst)[kk] = __ldg(reinterpret_cast<const uint16_t*>(src));
        }
      } else {
#pragma unroll 1
        for (int kk = lane; kk < p.K; kk += 32) {
          const int key = MC::KSPLIT ? (kk >= p.krows ? 1 : 0) : (MC::NSPLIT ? (int)rank : 0);
          const int wr = (MC::KSPLIT && key) ? kk - p.krows : kk;
          const uint8_t* src = p.q[key].absmax + ((size_t)e * p.krows + wr) * nblk_row;
#pragma unroll
          for (int jj = 0; jj < NB; ++jj)
            dst[kk * NB + jj] = nb0 + jj < nblk_row ? __ldg(src + nb0 + jj) : (uint8_t)0;
        }
      }
      mbar_arrive(&sm.absq_full[buf]);  // release: this lane's stores are visible to the waiters
    }
  };
  auto role_dequant = [&]() {
    // ======================= dequantisers =======================
    // One thread per B row (K-major: a weight row; MN-major: one k-row of a
    // 64-column block) and k-block: each thread decodes a whole 64-element
    // block, i.e. one NF4 absmax block.  The KG groups of B_ROWS threads take
    // the k-blocks of this CTA's sequence in turn (group g: g, g+KG, ...), so
    // a group has KG main-loop steps to deliver each of its blocks.
    constexpr int RB = C::ROW_BYTES;
    constexpr int KG = C::KG;
    const int d = threadIdx.x - 32 * C::DEQ_FIRST;
    const int grp = d / C::B_ROWS;
    const int row = d % C::B_ROWS;      // B row inside the stage
    const int nkb = num_kb;
    // K-major: TN/2-row block and row in it; MN-major: 64-column block and k-row
    const int kblk = MN ? 0 : (PAIR ? (int)rank : row / (TN / 2));
    const int kr = MN ? row & 63 : row % (TN / 2);
    const int nbq = MN ? row >> 6 : 0;  // local 64-column block (MN)
    const int nbase = MN ? (int)rank * C::B_ROWS / 64 : 0;  // first 64-column block of this CTA in the tile
    const int nblk_row = p.N / 64;      // MN: NF4 blocks per weight row
    const int sw = row & 7;             // 128-byte swizzle phase of this operand row
    float code[16];
    int cur_key = -1;
    int gk = 0;  // position in this CTA's k-block sequence over all its tiles
    bool failed = false;
    int tl = 0;  // tiles of this CTA so far
    // per-tile staging through shared memory (NF4 unless prefetched; INT8 MN-major)
    constexpr bool STAGE = (WF == W_NF4 && !PREFETCH) || (WF == W_INT8 && MN);
    for (int t = unit; t < total_tiles && !failed && !*abort_flag; t += num_units, ++tl) {
      int j, e, m, n;
      decode_tile<WF, PAIR>(t, sm, units, p.n_tiles, j, e, m, n);
      // key of this thread's rows (K-major, N-split keys); K-split keys follow the k-block
      const int row_key = (!MN && MC::NSPLIT) ? kblk : 0;
      const int wrow_base = MN ? 0 : kmajor_row<MODE, TN>(p, e, n, kblk) - e * p.out_rows;  // first weight row
      const int abuf = tl & 1;
      if (PREFETCH && !mbar_wait(&sm.absq_full[abuf], (tl >> 1) & 1, 42)) {
        failed = true;
        *abort_flag = 1;
        break;
      }
      // ---- stage this tile's scale inputs in shared memory
      if (STAGE) named_bar_sync(1, C::DEQ_THREADS);
      if (WF == W_NF4 && !PREFETCH) {
        if (!MN) {
          const int nblk = PAIR ? 1 : 2;
          for (int h = 0; h < nblk; ++h) {
            const int blk = PAIR ? (int)rank : h;
            // rows of this half inside the expert's matrix (a multiple of 64: N % 64 == 0)
            const int first = kmajor_row<MODE, TN>(p, e, n, blk) - e * p.out_rows;
            const int rows = min(TN / 2, p.out_rows - first);
            if (rows <= 0) continue;  // past the last row
            const int key = MC::NSPLIT ? blk : 0;
            const uint4* src = reinterpret_cast<const uint4*>(
                p.q[key].absmax + (size_t)kmajor_row<MODE, TN>(p, e, n, blk) * nkb);
            uint4* dst = reinterpret_cast<uint4*>(dq->absq + h * (TN / 2) * nkb);
            for (int i = d; i < rows * nkb / 16; i += C::DEQ_THREADS) dst[i] = __ldg(src + i);
          }
        } else {
          // absq[kk * NB + j] = code of (k-row kk, this CTA's column block j)
          constexpr int NB = C::B_ROWS / 64;
          for (int i = d; i < p.K * NB; i += C::DEQ_THREADS) {
            const int kk = i / NB, j = i % NB;
            const int key = (MC::KSPLIT && kk >= p.krows) ? 1 : 0;
            const int wr = kk - key * p.krows;
            const int nbg = n * (TN / 64) + nbase + j;
            dq->absq[i] = nbg < nblk_row
                              ? __ldg(p.q[key].absmax + ((size_t)e * p.krows + wr) * nblk_row + nbg) : (uint8_t)0;
          }
        }
        for (int h = 0; h < (MC::TWO_KEYS ? 2 : 1); ++h)
          for (int i = d; i < p.q[h].n_nested; i += C::DEQ_THREADS)
            dq->nested[h][i] = __ldg(p.q[h].nested_absmax + (size_t)e * p.q[h].n_nested + i);
      } else if (WF == W_INT8 && MN) {
        // INT8 MN-major: the scale belongs to the k-row (output channel of W)
        float* srow = reinterpret_cast<float*>(dq->absq);
        for (int kk = d; kk < p.K; kk += C::DEQ_THREADS) {
          const int key = (MC::KSPLIT && kk >= p.krows) ? 1 : 0;
          srow[kk] = __ldg(p.q[key].scale + (size_t)e * p.krows + (kk - key * p.krows));
        }
      }
      if (STAGE) named_bar_sync(1, C::DEQ_THREADS);
      // K-major: is this thread's weight row inside the expert's matrix?  (The
      // last tile of a down projection whose N is not a multiple of TN is half empty.)
      const bool row_live = MN || (wrow_base + kr < p.out_rows);
      float row_scale = 0.f;
      if (WF == W_INT8 && !MN && row_live)
        row_scale = __ldg(p.q[row_key].scale + (size_t)e * p.out_rows + wrow_base + kr);
      float off[2] = {0.f, 0.f};
      if (WF == W_NF4) {
        off[0] = __ldg(p.q[0].offset + e);
        off[1] = MC::TWO_KEYS ? __ldg(p.q[1].offset + e) : off[0];
      }
      const int absq_row = PAIR ? 0 : kblk;  // absq block of this thread (K-major)
      // this group's k-blocks of the tile: positions gk0 + kb with (gk0 + kb) % KG == grp
      const int gk0 = gk;
      gk += total_kb;
      for (int kb = ((grp - gk0) % KG + KG) % KG; kb < total_kb; kb += KG) {
        const int g = gk0 + kb;
        const int st = g % STAGES, rst = g % RAW_STAGES;
        const uint32_t ph = (uint32_t)(g / STAGES) & 1u, rph = (uint32_t)(g / RAW_STAGES) & 1u;
        bool ok = mbar_wait(&sm.raw_full[rst], rph, 40);
        ok = ok && mbar_wait(&sm.empty[st], ph ^ 1, 41);
        if (!ok) {
          failed = true;
          *abort_flag = 1;
          break;
        }
        if (kb != nkb) {  // the rank block arrives by TMA: nothing to decode
          const uint8_t* raw = sRaw + rst * RAW_BYTES + row * RB;
          const uint32_t row_addr = smem_u32(sB + st * B_BYTES) + (uint32_t)row * 128u;
          // the k-block's key: K-split by k-block, N-split by this CTA (pairs) or by row half
          const int key = MC::KSPLIT ? (kb >= p.kb_half ? 1 : 0) : (MN ? key_of(kb) : row_key);
          const int kk0 = kk_of(kb, key);  // k-block inside the key's matrix
          if (WF == W_NF4) {
            // the row's 32 code bytes as two 16-byte loads; rows 4..7 of every 8 take the halves
            // in the other order, so that each 8-lane phase of a load covers all 32 banks
            const uint4* raw4 = reinterpret_cast<const uint4*>(raw);
            const bool swap = (row & 4) != 0;
            const uint4 ra = raw4[swap ? 1 : 0], rb = raw4[swap ? 0 : 1];
            const uint4 r0 = swap ? rb : ra, r1 = swap ? ra : rb;
            const uint32_t words[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
            if (key != cur_key) {
#pragma unroll
              for (int j = 0; j < 16; ++j) code[j] = dq->code[key][j];
              cur_key = key;
            }
            int blk;
            uint32_t qcode;
            bool live = row_live;
            if (!MN) {
              blk = (wrow_base + kr) * (MC::KSPLIT ? p.kb_half : nkb) + kk0;
              qcode = PREFETCH ? dq->absq[abuf * ABUF + kb * C::B_ROWS + kr]
                               : dq->absq[absq_row * (TN / 2) * nkb + kr * nkb + kb];
            } else {
              const int kk = kb * BK + kr;                           // k-row across both keys
              const int wr = (MC::KSPLIT && key) ? kk - p.krows : kk;  // k-row inside the key's matrix
              const int nbg = mn_col(n, 0) / 64 + nbq;
              live = nbg < nblk_row;
              blk = wr * nblk_row + nbg;
              qcode = dq->absq[(PREFETCH ? abuf * ABUF : 0) + kk * (C::B_ROWS / 64) + nbq];
            }
            // rows past the weight matrix (a partial last tile) read no scale: their block index
            // lies beyond the expert's nested absmax
            const float nabs = !live ? 0.f
                               : PREFETCH ? __ldg(p.q[key].nested_absmax + (size_t)e * p.q[key].n_nested +
                                                  (blk >> p.nbs_shift))
                                          : dq->nested[key][blk >> p.nbs_shift];
            const float scale = live ? __fadd_rn(__fmul_rn(dq->ncode[key][qcode], nabs), off[key]) : 0.f;
            Nf4Tab tab;
            nf4_table(code, scale, tab);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint32_t o[4];
              nf4_word(words[c], tab, o);
              st_shared_v4(row_addr + (uint32_t)((c ^ sw) << 4), o[0], o[1], o[2], o[3]);
            }
          } else {
            const float iscale = MN ? reinterpret_cast<const float*>(dq->absq)[kb * BK + kr] : row_scale;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t o[8];
              int8_x16(reinterpret_cast<const uint4*>(raw)[v], iscale, o);
              st_shared_v4(row_addr + (uint32_t)(((2 * v) ^ sw) << 4), o[0], o[1], o[2], o[3]);
              st_shared_v4(row_addr + (uint32_t)(((2 * v + 1) ^ sw) << 4), o[4], o[5], o[6], o[7]);
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.raw_empty[rst]);
          if (PAIR) mbar_arrive_cluster(full_leader0 + 8u * st);
          else mbar_arrive(&sm.full[st]);
        }
      }
      if (PREFETCH && !failed) {  // this warp is done with the tile's absmax buffer
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.absq_empty[abuf]);
      }
    }
  };

  if (C::WIDE) {
    // One register budget per warpgroup, set once at the top of its branch so
    // that it covers all the code the group runs.
    if (warp < 4) {
      setmaxnreg_dec<C::REG_WG0>();
      if (warp == 0) role_producer();
      else if (warp == 1) role_mma();
      else if (warp == C::RAW_WARP) role_raw();
      else if (PREFETCH && warp == 3) role_absq();
    } else if (warp < 8) {
      setmaxnreg_inc<C::REG_EPI>();
      role_epilogue();
    } else {
      setmaxnreg_dec<C::REG_DEQ>();
      role_dequant();
    }
  } else {
    if (warp == 0) role_producer();
    else if (warp == 1) role_mma();
    else if (warp >= C::EPI_FIRST && warp < C::EPI_FIRST + C::EPI_WARPS) role_epilogue();
    else if (QUANT && warp == C::RAW_WARP) role_raw();
    else if (QUANT && warp >= C::DEQ_FIRST) role_dequant();
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// CTA pairs are used unless MIRAI_B200_CTA_PAIR=0 (kept for A/B measurement).
static bool use_pairs() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("MIRAI_B200_CTA_PAIR");
    v = (s && s[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <int MODE, int WF, bool PAIR, bool BMN>
int launch_impl(const CUtensorMap& ta, const CUtensorMap& tb0, const CUtensorMap& tb1, const CUtensorMap& txa,
                const CUtensorMap& txb, const CUtensorMap* to, const Params& p,
                cudaStream_t stream) {
  using C = Cfg<WF, PAIR>;
  auto kern = grouped_gemm_kernel<MODE, WF, PAIR, BMN>;
  constexpr size_t smem = smem_bytes<WF, PAIR>();
  static_assert(smem <= 232448, "shared memory budget exceeded");
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    if (C::WIDE) {
      // the per-warpgroup register split needs the launch allocation it was sized for
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, kern);
      if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
      if (fa.numRegs < C::LAUNCH_REGS)
        return set_error(MIRAI_ERR_UNSUPPORTED, "grouped GEMM compiled with %d registers per thread; the register "
                         "split needs %d", fa.numRegs, C::LAUNCH_REGS);
    }
    attr_set = true;
  }
  Params q = p;
  q.n_tiles = MODE == GATEUP ? (q.N + C::TN / 2 - 1) / (C::TN / 2) : (q.N + C::TN - 1) / C::TN;
  const int64_t max_tiles = ((q.S + C::TILE_M - 1) / C::TILE_M + q.E) * (int64_t)q.n_tiles;
  static const char* names[4] = {"gateup_swiglu", "down", "down_dx", "gateup_dx"};
  const int limit = gemm_sm_limit();
  const int sms = (limit > 0 && limit < sm_count()) ? limit : sm_count();
  if (!PAIR) {
    const int grid = (int)(max_tiles < sms ? max_tiles : sms);
    kern<<<grid, C::THREADS, smem, stream>>>(ta, tb0, tb1, txa, txb, to[0], to[1], to[2], q);
    return check_launch(names[MODE]);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(C::THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // The kernel is persistent: launch no more pairs than can be resident at
  // once (cluster placement can leave some SMs unpaired), else the surplus
  // pairs run as a second wave.
  static int resident_pairs = 0;
  if (resident_pairs <= 0) {
    cfg.gridDim = dim3((unsigned)(sms & ~1), 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sms / 2;
    }
    resident_pairs = n;
    if (getenv("MIRAI_B200_DEBUG")) fprintf(stderr, "[mirai_b200] %s: %d resident CTA pairs\n", names[MODE], n);
  }
  int64_t units = max_tiles < resident_pairs ? max_tiles : resident_pairs;
  if (units > sms / 2) units = sms / 2;  // the SM limit, in pairs
  cfg.gridDim = dim3((unsigned)(2 * units), 1, 1);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb0, tb1, txa, txb, to[0], to[1], to[2], q);
  if (e != cudaSuccess) return set_error(MIRAI_ERR_CUDA, "%s: launch failed: %s", names[MODE], cudaGetErrorString(e));
  return check_launch(names[MODE]);
}

// BMN: B read MN-major.  The compressed-expert layout ([E, out, in]) has its
// native B layout per mode (every format, single CTAs or pairs); the MAGI-2
// layout ([E, in, out]) reads the other way round, for bf16 and NF4, on pairs.
template <int MODE, int WF, bool BMN>
int launch(const CUtensorMap& ta, const CUtensorMap& tb0, const CUtensorMap& tb1, const CUtensorMap& txa,
           const CUtensorMap& txb, const CUtensorMap* to, const Params& p,
           cudaStream_t stream) {
  if constexpr (BMN == MCfg<MODE>::MN_NATIVE) {
    return use_pairs() ? launch_impl<MODE, WF, true, BMN>(ta, tb0, tb1, txa, txb, to, p, stream)
                       : launch_impl<MODE, WF, false, BMN>(ta, tb0, tb1, txa, txb, to, p, stream);
  } else if constexpr (WF == W_INT8) {
    return set_error(MIRAI_ERR_UNSUPPORTED, "INT8 experts are read in the [E, out, in] layout only");
  } else {
    if (!use_pairs())
      return set_error(MIRAI_ERR_UNSUPPORTED, "the [E, in, out] weight layout runs on CTA pairs "
                       "(MIRAI_B200_CTA_PAIR=0 is set)");
    return launch_impl<MODE, WF, true, BMN>(ta, tb0, tb1, txa, txb, to, p, stream);
  }
}

static inline bool mis16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0; }

// Shared host-side checks, the A-operand tensor map and the mode geometry.
template <int MODE>
int prepare(const char* name, const void* a, const int32_t* offsets, int E, int64_t S, int K, int N, void* out,
            void* gate_up, Params& p, CUtensorMap& ta, bool dh_only, bool bmn) {
  if (E <= 0 || E > kMaxExperts || S < 0 || K <= 0 || N <= 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: bad sizes (E=%d, S=%lld, K=%d, N=%d)", name, E, (long long)S, K, N);
  // column granularity: every mode masks a partial last tile (gate/up: 128 W1
  // rows beside 128 W3 rows; the others: 256 columns) in 32-column chunks and,
  // for NF4/INT8, by weight row, so N % 64 is enough
  const int ntile = 64;
  if (K % BK != 0 || N % ntile != 0 || (MCfg<MODE>::KSPLIT && (K / 2) % BK != 0))
    return set_error(MIRAI_ERR_UNSUPPORTED, "%s: needs K %% %d == 0 and N %% %d == 0 (K=%d, N=%d)", name, BK, ntile,
                     K, N);
  if (S >= (int64_t)1 << 31) return set_error(MIRAI_ERR_UNSUPPORTED, "%s: more than 2^31 routed rows", name);
  if (!a || !offsets || !out || mis16(out) || (gate_up && mis16(gate_up)))
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: null or misaligned pointer", name);
  if (MODE == DXDOWN && !gate_up && !dh_only)
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: saved gate/up is required", name);
  if (dh_only) gate_up = nullptr;
  p = Params{};
  p.offsets = offsets;
  p.E = E;
  p.S = S;
  p.K = K;
  p.N = N;
  p.n_tiles = 0;  // set per tile geometry at launch
  p.krows = bmn ? (MCfg<MODE>::KSPLIT ? K / 2 : K) : 0;
  p.kb_half = MCfg<MODE>::KSPLIT ? (K / 2) / BK : 0;
  p.out_rows = N;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = N;
  p.gate_up = static_cast<__nv_bfloat16*>(gate_up);
  p.nbs_shift = 8;
  p.nsrc = 1;
  return make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, (uint64_t)K, (uint64_t)S, (uint64_t)K * 2, BK, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

// bf16 weight map.  K-major: [E*rows, cols] with boxes of 64 cols x box_rows rows.
// MN-major: the same matrix read as [E*rows (k), cols (n)] with 64 x 64 boxes.
int bf16_weight_map(CUtensorMap& m, const void* w, int E, int rows, int cols, bool mn, int box_rows) {
  if (!w) return set_error(MIRAI_ERR_INVALID_ARG, "null weight pointer");
  return make_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, (uint64_t)cols, (uint64_t)E * rows,
                      (uint64_t)cols * 2, 64, mn ? 64 : box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

int nf4_key(CUtensorMap& m, QKey& q, int& nbs_shift, const mirai_nf4_weight* w, int E, int rows, int cols, bool mn,
            int box_rows) {
  if (!w || !w->packed || !w->absmax || !w->nested_absmax || !w->offset || !w->code || !w->nested_code)
    return set_error(MIRAI_ERR_INVALID_ARG, "nf4 weight: null buffer");
  if (w->blocksize != 64)
    return set_error(MIRAI_ERR_UNSUPPORTED, "nf4 weight: blocksize %d (the fused kernel decodes blocksize 64)",
                     w->blocksize);
  if (w->nested_blocksize < 64 || (w->nested_blocksize & (w->nested_blocksize - 1)) != 0)
    return set_error(MIRAI_ERR_UNSUPPORTED, "nf4 weight: nested blocksize %d is not a power of two >= 64",
                     w->nested_blocksize);
  if (cols % 64 != 0) return set_error(MIRAI_ERR_UNSUPPORTED, "nf4 weight: in_features %d %% 64 != 0", cols);
  if (mis16(w->absmax)) return set_error(MIRAI_ERR_INVALID_ARG, "nf4 weight: absmax codes not 16-byte aligned");
  nbs_shift = __builtin_ctz((unsigned)w->nested_blocksize);
  const int64_t blocks_per_expert = (int64_t)rows * cols / 64;
  q.absmax = w->absmax;
  q.nested_absmax = w->nested_absmax;
  q.offset = w->offset;
  q.code = w->code;
  q.nested_code = w->nested_code;
  q.scale = nullptr;
  q.n_nested = (int)((blocks_per_expert + w->nested_blocksize - 1) / w->nested_blocksize);
  if (q.n_nested > kMaxNested)
    return set_error(MIRAI_ERR_UNSUPPORTED, "nf4 weight: %d nested absmax blocks per expert (max %d)", q.n_nested,
                     kMaxNested);
  // packed nibbles as a [E*rows, cols/2] byte tensor; boxes of one 64-element
  // block per row: box_rows rows (K-major) or 64 rows (MN-major)
  return make_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w->packed, (uint64_t)cols / 2, (uint64_t)E * rows,
                      (uint64_t)cols / 2, 32, mn ? 64 : box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int int8_key(CUtensorMap& m, QKey& q, const mirai_int8_weight* w, int E, int rows, int cols, bool mn, int box_rows) {
  if (!w || !w->q || !w->scale) return set_error(MIRAI_ERR_INVALID_ARG, "int8 weight: null buffer");
  q = QKey{};
  q.scale = w->scale;
  return make_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w->q, (uint64_t)cols, (uint64_t)E * rows, (uint64_t)cols,
                      64, mn ? 64 : box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Bind one weight key in any format.  rows x cols is one expert's matrix.
struct WeightArg {
  int fmt;
  const void* bf16;
  const mirai_nf4_weight* nf4;
  const mirai_int8_weight* int8;
};

int bind_key(const WeightArg& w, CUtensorMap& m, QKey& q, int& shift, int E, int rows, int cols, bool mn,
             int box_rows) {
  if (w.fmt == W_BF16) return bf16_weight_map(m, w.bf16, E, rows, cols, mn, box_rows);
  if (w.fmt == W_NF4) return nf4_key(m, q, shift, w.nf4, E, rows, cols, mn, box_rows);
  return int8_key(m, q, w.int8, E, rows, cols, mn, box_rows);
}

// Rows of one K-major B box (TN/2: the half of a tile's columns one CTA of a
// pair holds, or one of the two boxes of a single-CTA tile).
static int kmajor_box_rows(int fmt) {
  static_assert(Cfg<W_BF16, true>::TN == Cfg<W_NF4, true>::TN && Cfg<W_NF4, true>::TN == Cfg<W_NF4, false>::TN,
                "one column-tile width for every format");
  (void)fmt;
  return Cfg<W_BF16, true>::TN / 2;
}

// The optional rank block of a fused LoRA adapter: ext_a [S, 64] bf16 (one
// k-block of A) and ext_b, bf16 in the layout of this mode's B:
// down forward [E*H rows, 64] (K-major); down dX [E*64 rows, I] (MN-major).
struct RankBlock {
  const void* a;
  const void* b;
};

// One launch over at most kMaxExperts groups (see run).
template <int MODE>
int run_groups(const char* name, const void* a, const int32_t* offsets, int E, int64_t S, int K, int N, void* out,
               void* gate_up, const WeightArg& w0, const WeightArg& w1, int rows, int cols, mirai_stream_t stream,
               const RankBlock* ext, int nsrc, bool dh_only, bool mn, int act, bool prev_end) {
  Params p;
  CUtensorMap ta, t0, t1, txa, txb;
  const int box_rows = kmajor_box_rows(w0.fmt);
  int rc = prepare<MODE>(name, a, offsets, nsrc * E, S, K, N, out, gate_up, p, ta, dh_only, mn);
  p.nsrc = nsrc;
  p.act = act;
  p.prev_end = prev_end ? 1 : 0;
  if (!rc && ext) {
    if (!ext->a || !ext->b) rc = set_error(MIRAI_ERR_INVALID_ARG, "%s: null rank-block operand", name);
    if (!rc)
      rc = make_tmap_2d(&txa, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ext->a, 64, (uint64_t)S, 128, BK, BM,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc) {
      if (mn)  // [E*64 rank rows (k), N cols]
        rc = make_tmap_2d(&txb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ext->b, (uint64_t)N, (uint64_t)E * BK,
                          (uint64_t)N * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
      else  // [E*N rows, 64 rank cols (k)]
        rc = make_tmap_2d(&txb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ext->b, 64, (uint64_t)E * N, 128, BK,
                          box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    p.has_ext = 1;
  }
  if (!rc && w0.fmt != W_BF16 && K > kMaxK)
    rc = set_error(MIRAI_ERR_UNSUPPORTED, "%s: reduction length %d exceeds %d", name, K, kMaxK);
  int s0 = 8, s1 = 8;
  if (!rc) rc = bind_key(w0, t0, p.q[0], s0, E, rows, cols, mn, box_rows);
  if (!rc && MCfg<MODE>::TWO_KEYS) rc = bind_key(w1, t1, p.q[1], s1, E, rows, cols, mn, box_rows);
  if (!rc && MCfg<MODE>::TWO_KEYS && s0 != s1)
    rc = set_error(MIRAI_ERR_UNSUPPORTED, "%s: the two keys use different nested blocksizes", name);
  if (rc) return rc;
  if (!MCfg<MODE>::TWO_KEYS) {
    t1 = t0;
    p.q[1] = p.q[0];
  }
  p.nbs_shift = s0;
  if (!ext) {
    txa = ta;
    txb = t0;
  }
  // output maps of the staged epilogue (32 x 32 bf16 boxes, 64-byte swizzle); a map that
  // a mode does not store through is a copy of another (never used)
  CUtensorMap to[3];
  {
    const bool dgu = MODE == DXDOWN && p.gate_up != nullptr;  // [S, 2N]: gate half, then up half
    const uint64_t ld = dgu ? 2 * (uint64_t)N : (uint64_t)N;
    char* o = static_cast<char*>(out);
    rc = make_tmap_2d(&to[0], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, o, (uint64_t)N, (uint64_t)S, ld * 2, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_64B);
    if (!rc)
      rc = dgu ? make_tmap_2d(&to[1], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, o + (size_t)N * 2, (uint64_t)N,
                              (uint64_t)S, ld * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)
         : (MODE == GATEUP && gate_up)
             ? make_tmap_2d(&to[1], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, gate_up, (uint64_t)N, (uint64_t)S,
                            4 * (uint64_t)N, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)
             : (to[1] = to[0], MIRAI_OK);
    if (!rc)
      rc = (MODE == GATEUP && gate_up)
               ? make_tmap_2d(&to[2], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, static_cast<char*>(gate_up) + (size_t)N * 2,
                              (uint64_t)N, (uint64_t)S, 4 * (uint64_t)N, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)
               : (to[2] = to[0], MIRAI_OK);
    if (rc) return rc;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  constexpr bool NAT = MCfg<MODE>::MN_NATIVE;
  switch (w0.fmt) {
    case W_BF16:
      return mn == NAT ? launch<MODE, W_BF16, NAT>(ta, t0, t1, txa, txb, to, p, st)
                       : launch<MODE, W_BF16, !NAT>(ta, t0, t1, txa, txb, to, p, st);
    case W_NF4:
      return mn == NAT ? launch<MODE, W_NF4, NAT>(ta, t0, t1, txa, txb, to, p, st)
                       : launch<MODE, W_NF4, !NAT>(ta, t0, t1, txa, txb, to, p, st);
    default:
      return mn == NAT ? launch<MODE, W_INT8, NAT>(ta, t0, t1, txa, txb, to, p, st)
                       : launch<MODE, W_INT8, !NAT>(ta, t0, t1, txa, txb, to, p, st);
  }
}

// One expert's share of each weight buffer, to start a chunk of groups at
// group g0 (bf16 / NF4 / INT8 buffers are [E, rows, cols] in their encodings).
struct KeyShift {
  mirai_nf4_weight nf4;
  mirai_int8_weight int8;
};
static WeightArg shift_weight(const WeightArg& w, int64_t g0, int rows, int cols, KeyShift& hold) {
  const int64_t n = (int64_t)rows * cols;
  WeightArg r = w;
  if (w.fmt == W_BF16) {
    r.bf16 = static_cast<const uint8_t*>(w.bf16) + g0 * n * 2;
  } else if (w.fmt == W_NF4) {
    hold.nf4 = *w.nf4;
    const int64_t blocks = n / 64;
    const int64_t nested = (blocks + w.nf4->nested_blocksize - 1) / w.nf4->nested_blocksize;
    hold.nf4.packed += g0 * n / 2;
    hold.nf4.absmax += g0 * blocks;
    hold.nf4.nested_absmax += g0 * nested;
    hold.nf4.offset += g0;
    r.nf4 = &hold.nf4;
  } else {
    hold.int8 = *w.int8;
    hold.int8.q += g0 * n;
    hold.int8.scale += g0 * rows;
    r.int8 = &hold.int8;
  }
  return r;
}

// E weight experts; nsrc > 1: `offsets` has nsrc * E segments, source-major
// (segment s*E + e = rows of source s for expert e).  bmn: read B MN-major
// (the native layout of the mode's compressed-expert weights, or the MAGI-2
// [E, in, out] layout read the other way); act: the gate/up activation.
// More than kMaxExperts groups (one source) run as consecutive launches over
// chunks of kMaxExperts groups, each starting at the previous chunk's end.
template <int MODE>
int run(const char* name, const void* a, const int32_t* offsets, int E, int64_t S, int K, int N, void* out,
        void* gate_up, const WeightArg& w0, const WeightArg& w1, int rows, int cols, mirai_stream_t stream,
        const RankBlock* ext = nullptr, int nsrc = 1, bool dh_only = false, int bmn = -1, int act = ACT_SWIGLU) {
  if (nsrc <= 0 || E <= 0 || (nsrc > 1 && (int64_t)nsrc * E > kMaxExperts))
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: %d sources x %d experts outside 1..%d segments", name, nsrc, E,
                     kMaxExperts);
  const bool mn = bmn < 0 ? MCfg<MODE>::MN_NATIVE : bmn != 0;
  if (S == 0) return MIRAI_OK;
  if (E > kMaxExperts) {
    if (ext) return set_error(MIRAI_ERR_UNSUPPORTED, "%s: a rank block with more than %d groups", name, kMaxExperts);
    for (int g0 = 0; g0 < E; g0 += kMaxExperts) {
      const int Ec = E - g0 < kMaxExperts ? E - g0 : kMaxExperts;
      KeyShift h0, h1;
      const WeightArg c0 = shift_weight(w0, g0, rows, cols, h0);
      const WeightArg c1 = MCfg<MODE>::TWO_KEYS ? shift_weight(w1, g0, rows, cols, h1) : c0;
      const int rc = run_groups<MODE>(name, a, offsets + g0, Ec, S, K, N, out, gate_up, c0, c1, rows, cols,
                                      stream, nullptr, 1, dh_only, mn, act, g0 > 0);
      if (rc) return rc;
    }
    return MIRAI_OK;
  }
  return run_groups<MODE>(name, a, offsets, E, S, K, N, out, gate_up, w0, w1, rows, cols, stream, ext, nsrc, dh_only,
                          mn, act, false);
}

inline WeightArg wb(const void* w) { return WeightArg{W_BF16, w, nullptr, nullptr}; }
inline WeightArg wn(const mirai_nf4_weight* w) { return WeightArg{W_NF4, nullptr, w, nullptr}; }
inline WeightArg wi(const mirai_int8_weight* w) { return WeightArg{W_INT8, nullptr, nullptr, w}; }

}  // namespace gg
}  // namespace mirai

using namespace mirai::gg;

// ---- any weight layout and activation (MAGI-2 multi-head grouped experts and
// the compressed-expert layout alike), any number of groups.
//   layout MIRAI_LAYOUT_OUT_IN: w1/w3 [G, I, H], w2 [G, H, I] (compressed experts)
//          MIRAI_LAYOUT_IN_OUT: w1/w3 [G, H, I], w2 [G, I, H] (MAGI-2 W_gate/W_up/W_down)
static int layout_ok(const char* name, int32_t layout, int32_t act) {
  if (layout != MIRAI_LAYOUT_OUT_IN && layout != MIRAI_LAYOUT_IN_OUT)
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: unknown weight layout %d", name, layout);
  if (act != MIRAI_ACT_SWIGLU && act != MIRAI_ACT_SWIGLU7)
    return set_error(MIRAI_ERR_INVALID_ARG, "%s: unknown activation %d", name, act);
  return MIRAI_OK;
}

template <int MODE>
static int run_ex(const char* name, const void* a, const int32_t* offsets, int32_t groups, int64_t S, int K, int N,
                  void* out, void* gate_up, const WeightArg& w0, const WeightArg& w1, int32_t layout, int32_t act,
                  mirai_stream_t stream) {
  if (int rc = layout_ok(name, layout, act)) return rc;
  const bool in_out = layout == MIRAI_LAYOUT_IN_OUT;
  // one key's [rows, cols] per group: OUT_IN stores [out, in], IN_OUT [in, out]
  int rows, cols;
  switch (MODE) {
    case GATEUP: rows = in_out ? K : N, cols = in_out ? N : K; break;           // K = H, N = I
    case DOWN: rows = in_out ? K : N, cols = in_out ? N : K; break;             // K = I, N = H
    case DXDOWN: rows = in_out ? N : K, cols = in_out ? K : N; break;           // K = H, N = I
    default: rows = in_out ? N : K / 2, cols = in_out ? K / 2 : N; break;      // K = 2I, N = H
  }
  const bool mn = in_out != MCfg<MODE>::MN_NATIVE;
  return run<MODE>(name, a, offsets, groups, S, K, N, out, gate_up, w0, w1, rows, cols, stream, nullptr, 1,
                   MODE == DXDOWN && gate_up == nullptr, mn ? 1 : 0, act);
}

extern "C" {

// ---- forward: gate/up + SwiGLU.  B = W1/W3 [E, I, H]: rows I, cols H.
int mirai_moe_gateup_swiglu_bf16(const void* x_sorted, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                 int32_t hidden, int32_t inter, const void* w1, const void* w3, void* h,
                                 void* gate_up, mirai_stream_t stream) {
  return run<GATEUP>("gateup_swiglu_bf16", x_sorted, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                     wb(w1), wb(w3), inter, hidden, stream);
}
int mirai_moe_gateup_swiglu_nf4(const void* x_sorted, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                int32_t hidden, int32_t inter, const mirai_nf4_weight* w1, const mirai_nf4_weight* w3,
                                void* h, void* gate_up, mirai_stream_t stream) {
  return run<GATEUP>("gateup_swiglu_nf4", x_sorted, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                     wn(w1), wn(w3), inter, hidden, stream);
}
int mirai_moe_gateup_swiglu_int8(const void* x_sorted, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                 int32_t hidden, int32_t inter, const mirai_int8_weight* w1,
                                 const mirai_int8_weight* w3, void* h, void* gate_up, mirai_stream_t stream) {
  return run<GATEUP>("gateup_swiglu_int8", x_sorted, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                     wi(w1), wi(w3), inter, hidden, stream);
}

// ---- forward over source-major segments (expert-parallel receive buffers).
int mirai_moe_gateup_swiglu_src_bf16(const void* x_sorted, const int32_t* offsets, int32_t num_sources,
                                     int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter,
                                     const void* w1, const void* w3, void* h, void* gate_up, mirai_stream_t stream) {
  return run<GATEUP>("gateup_swiglu_src_bf16", x_sorted, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                     wb(w1), wb(w3), inter, hidden, stream, nullptr, num_sources);
}
int mirai_moe_gateup_swiglu_src_nf4(const void* x_sorted, const int32_t* offsets, int32_t num_sources,
                                    int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter,
                                    const mirai_nf4_weight* w1, const mirai_nf4_weight* w3, void* h, void* gate_up,
                                    mirai_stream_t stream) {
  return run<GATEUP>("gateup_swiglu_src_nf4", x_sorted, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                     wn(w1), wn(w3), inter, hidden, stream, nullptr, num_sources);
}
int mirai_moe_gateup_swiglu_src_int8(const void* x_sorted, const int32_t* offsets, int32_t num_sources,
                                     int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter,
                                     const mirai_int8_weight* w1, const mirai_int8_weight* w3, void* h,
                                     void* gate_up, mirai_stream_t stream) {
  return run<GATEUP>("gateup_swiglu_src_int8", x_sorted, offsets, num_experts, num_rows, hidden, inter, h, gate_up,
                     wi(w1), wi(w3), inter, hidden, stream, nullptr, num_sources);
}
int mirai_moe_down_src_bf16(const void* h, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                            int64_t num_rows, int32_t inter, int32_t hidden, const void* w2, void* y,
                            mirai_stream_t stream) {
  return run<DOWN>("down_src_bf16", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, wb(w2), wb(w2),
                   hidden, inter, stream, nullptr, num_sources);
}
int mirai_moe_down_src_nf4(const void* h, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                           int64_t num_rows, int32_t inter, int32_t hidden, const mirai_nf4_weight* w2, void* y,
                           mirai_stream_t stream) {
  return run<DOWN>("down_src_nf4", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, wn(w2), wn(w2),
                   hidden, inter, stream, nullptr, num_sources);
}
int mirai_moe_down_src_int8(const void* h, const int32_t* offsets, int32_t num_sources, int32_t num_experts,
                            int64_t num_rows, int32_t inter, int32_t hidden, const mirai_int8_weight* w2, void* y,
                            mirai_stream_t stream) {
  return run<DOWN>("down_src_int8", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, wi(w2), wi(w2),
                   hidden, inter, stream, nullptr, num_sources);
}

// ---- forward: down.  B = W2 [E, H, I]: rows H, cols I.
int mirai_moe_down_bf16(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows, int32_t inter,
                        int32_t hidden, const void* w2, void* y, mirai_stream_t stream) {
  return run<DOWN>("down_bf16", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, wb(w2), wb(w2), hidden,
                   inter, stream);
}
int mirai_moe_down_nf4(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows, int32_t inter,
                       int32_t hidden, const mirai_nf4_weight* w2, void* y, mirai_stream_t stream) {
  return run<DOWN>("down_nf4", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, wn(w2), wn(w2), hidden,
                   inter, stream);
}
int mirai_moe_down_int8(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows, int32_t inter,
                        int32_t hidden, const mirai_int8_weight* w2, void* y, mirai_stream_t stream) {
  return run<DOWN>("down_int8", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, wi(w2), wi(w2), hidden,
                   inter, stream);
}

// ---- dX: down.  dh = dy W2 (K = H, N = I), SwiGLU backward fused.  B = W2 read MN-major.
int mirai_moe_down_dx_bf16(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                           int32_t hidden, int32_t inter, const void* w2, const void* gate_up, void* grad_gate_up,
                           mirai_stream_t stream) {
  return run<DXDOWN>("down_dx_bf16", grad_y, offsets, num_experts, num_rows, hidden, inter, grad_gate_up,
                     const_cast<void*>(gate_up), wb(w2), wb(w2), hidden, inter, stream);
}
int mirai_moe_down_dx_nf4(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                          int32_t hidden, int32_t inter, const mirai_nf4_weight* w2, const void* gate_up,
                          void* grad_gate_up, mirai_stream_t stream) {
  return run<DXDOWN>("down_dx_nf4", grad_y, offsets, num_experts, num_rows, hidden, inter, grad_gate_up,
                     const_cast<void*>(gate_up), wn(w2), wn(w2), hidden, inter, stream);
}
int mirai_moe_down_dx_int8(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                           int32_t hidden, int32_t inter, const mirai_int8_weight* w2, const void* gate_up,
                           void* grad_gate_up, mirai_stream_t stream) {
  return run<DXDOWN>("down_dx_int8", grad_y, offsets, num_experts, num_rows, hidden, inter, grad_gate_up,
                     const_cast<void*>(gate_up), wi(w2), wi(w2), hidden, inter, stream);
}

// ---- dX over source-major segments (the expert-parallel backward on an expert
// owner; num_sources = 1 equals the entry points above).  down_dx_src with
// gate_up == NULL writes dh = dy W2 [S, I] without the SwiGLU backward.
#define MIRAI_DX_SRC(SUF, WT, WRAP)                                                                            \
  int mirai_moe_down_dx_src_##SUF(const void* grad_y, const int32_t* offsets, int32_t num_sources,          \
                                  int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter, WT w2, \
                                  const void* gate_up, void* grad_gate_up, mirai_stream_t stream) {           \
    return run<DXDOWN>("down_dx_src_" #SUF, grad_y, offsets, num_experts, num_rows, hidden, inter,            \
                       grad_gate_up, const_cast<void*>(gate_up), WRAP(w2), WRAP(w2), hidden, inter, stream,   \
                       nullptr, num_sources, gate_up == nullptr);                                              \
  }                                                                                                            \
  int mirai_moe_gateup_dx_src_##SUF(const void* grad_gate_up, const int32_t* offsets, int32_t num_sources,  \
                                    int32_t num_experts, int64_t num_rows, int32_t inter, int32_t hidden,    \
                                    WT w1, WT w3, void* dx_sorted, mirai_stream_t stream) {                    \
    return run<DXGATEUP>("gateup_dx_src_" #SUF, grad_gate_up, offsets, num_experts, num_rows, 2 * inter,     \
                         hidden, dx_sorted, nullptr, WRAP(w1), WRAP(w3), inter, hidden, stream, nullptr,     \
                         num_sources);                                                                         \
  }
MIRAI_DX_SRC(bf16, const void*, wb)
MIRAI_DX_SRC(nf4, const mirai_nf4_weight*, wn)
MIRAI_DX_SRC(int8, const mirai_int8_weight*, wi)
#undef MIRAI_DX_SRC

// ---- LoRA on the down projection, fused as one extra k-block (a10).
int mirai_moe_down_lora_bf16(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                             int32_t inter, int32_t hidden, const void* w2, const void* rank_a, const void* rank_b,
                             void* y, mirai_stream_t stream) {
  const RankBlock rb{rank_a, rank_b};
  return run<DOWN>("down_lora_bf16", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, wb(w2), wb(w2),
                   hidden, inter, stream, &rb);
}
int mirai_moe_down_lora_nf4(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                            int32_t inter, int32_t hidden, const mirai_nf4_weight* w2, const void* rank_a,
                            const void* rank_b, void* y, mirai_stream_t stream) {
  const RankBlock rb{rank_a, rank_b};
  return run<DOWN>("down_lora_nf4", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, wn(w2), wn(w2),
                   hidden, inter, stream, &rb);
}
int mirai_moe_down_lora_int8(const void* h, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                             int32_t inter, int32_t hidden, const mirai_int8_weight* w2, const void* rank_a,
                             const void* rank_b, void* y, mirai_stream_t stream) {
  const RankBlock rb{rank_a, rank_b};
  return run<DOWN>("down_lora_int8", h, offsets, num_experts, num_rows, inter, hidden, y, nullptr, wi(w2), wi(w2),
                   hidden, inter, stream, &rb);
}
int mirai_moe_down_dx_lora_bf16(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                int32_t hidden, int32_t inter, const void* w2, const void* gate_up,
                                const void* rank_a, const void* rank_b, void* grad_gate_up, mirai_stream_t stream) {
  const RankBlock rb{rank_a, rank_b};
  return run<DXDOWN>("down_dx_lora_bf16", grad_y, offsets, num_experts, num_rows, hidden, inter, grad_gate_up,
                     const_cast<void*>(gate_up), wb(w2), wb(w2), hidden, inter, stream, &rb);
}
int mirai_moe_down_dx_lora_nf4(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                               int32_t hidden, int32_t inter, const mirai_nf4_weight* w2, const void* gate_up,
                               const void* rank_a, const void* rank_b, void* grad_gate_up, mirai_stream_t stream) {
  const RankBlock rb{rank_a, rank_b};
  return run<DXDOWN>("down_dx_lora_nf4", grad_y, offsets, num_experts, num_rows, hidden, inter, grad_gate_up,
                     const_cast<void*>(gate_up), wn(w2), wn(w2), hidden, inter, stream, &rb);
}
int mirai_moe_down_dx_lora_int8(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                int32_t hidden, int32_t inter, const mirai_int8_weight* w2, const void* gate_up,
                                const void* rank_a, const void* rank_b, void* grad_gate_up, mirai_stream_t stream) {
  const RankBlock rb{rank_a, rank_b};
  return run<DXDOWN>("down_dx_lora_int8", grad_y, offsets, num_experts, num_rows, hidden, inter, grad_gate_up,
                     const_cast<void*>(gate_up), wi(w2), wi(w2), hidden, inter, stream, &rb);
}

// ---- LoRA rank block over source-major segments (the expert-parallel train step
// on an expert owner; num_sources = 1 equals the entry points above).
#define MIRAI_LORA_SRC(SUF, WT, WRAP)                                                                          \
  int mirai_moe_down_lora_src_##SUF(const void* h, const int32_t* offsets, int32_t num_sources,             \
                                    int32_t num_experts, int64_t num_rows, int32_t inter, int32_t hidden,    \
                                    WT w2, const void* rank_a, const void* rank_b, void* y,                 \
                                    mirai_stream_t stream) {                                                 \
    const RankBlock rb{rank_a, rank_b};                                                                      \
    return run<DOWN>("down_lora_src_" #SUF, h, offsets, num_experts, num_rows, inter, hidden, y, nullptr,    \
                     WRAP(w2), WRAP(w2), hidden, inter, stream, &rb, num_sources);                           \
  }                                                                                                          \
  int mirai_moe_down_dx_lora_src_##SUF(const void* grad_y, const int32_t* offsets, int32_t num_sources,     \
                                       int32_t num_experts, int64_t num_rows, int32_t hidden, int32_t inter, \
                                       WT w2, const void* gate_up, const void* rank_a, const void* rank_b,   \
                                       void* grad_gate_up, mirai_stream_t stream) {                          \
    const RankBlock rb{rank_a, rank_b};                                                                      \
    return run<DXDOWN>("down_dx_lora_src_" #SUF, grad_y, offsets, num_experts, num_rows, hidden, inter,      \
                       grad_gate_up, const_cast<void*>(gate_up), WRAP(w2), WRAP(w2), hidden, inter, stream,  \
                       &rb, num_sources, gate_up == nullptr);                                                \
  }
MIRAI_LORA_SRC(bf16, const void*, wb)
MIRAI_LORA_SRC(nf4, const mirai_nf4_weight*, wn)
MIRAI_LORA_SRC(int8, const mirai_int8_weight*, wi)
#undef MIRAI_LORA_SRC

// ---- dX: down without the SwiGLU backward: dh = dy W2 [S, I] (+ the rank block).  The rotated
// INT8 format rotates dh before the SwiGLU backward (mirai_swiglu_backward_rotated).
int mirai_moe_down_dh_int8(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                           int32_t hidden, int32_t inter, const mirai_int8_weight* w2, void* dh,
                           mirai_stream_t stream) {
  return run<DXDOWN>("down_dh_int8", grad_y, offsets, num_experts, num_rows, hidden, inter, dh, nullptr, wi(w2),
                     wi(w2), hidden, inter, stream, nullptr, 1, true);
}
int mirai_moe_down_dh_lora_int8(const void* grad_y, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                                int32_t hidden, int32_t inter, const mirai_int8_weight* w2, const void* rank_a,
                                const void* rank_b, void* dh, mirai_stream_t stream) {
  const RankBlock rb{rank_a, rank_b};
  return run<DXDOWN>("down_dh_lora_int8", grad_y, offsets, num_experts, num_rows, hidden, inter, dh, nullptr,
                     wi(w2), wi(w2), hidden, inter, stream, &rb, 1, true);
}

// ---- dX: gate/up.  dx = [dgate | dup] [W1 ; W3] (K = 2I, N = H).  B = W1/W3 read MN-major.
int mirai_moe_gateup_dx_bf16(const void* grad_gate_up, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                             int32_t inter, int32_t hidden, const void* w1, const void* w3, void* dx_sorted,
                             mirai_stream_t stream) {
  return run<DXGATEUP>("gateup_dx_bf16", grad_gate_up, offsets, num_experts, num_rows, 2 * inter, hidden, dx_sorted,
                       nullptr, wb(w1), wb(w3), inter, hidden, stream);
}
int mirai_moe_gateup_dx_nf4(const void* grad_gate_up, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                            int32_t inter, int32_t hidden, const mirai_nf4_weight* w1, const mirai_nf4_weight* w3,
                            void* dx_sorted, mirai_stream_t stream) {
  return run<DXGATEUP>("gateup_dx_nf4", grad_gate_up, offsets, num_experts, num_rows, 2 * inter, hidden, dx_sorted,
                       nullptr, wn(w1), wn(w3), inter, hidden, stream);
}
int mirai_moe_gateup_dx_int8(const void* grad_gate_up, const int32_t* offsets, int32_t num_experts, int64_t num_rows,
                             int32_t inter, int32_t hidden, const mirai_int8_weight* w1, const mirai_int8_weight* w3,
                             void* dx_sorted, mirai_stream_t stream) {
  return run<DXGATEUP>("gateup_dx_int8", grad_gate_up, offsets, num_experts, num_rows, 2 * inter, hidden, dx_sorted,
                       nullptr, wi(w1), wi(w3), inter, hidden, stream);
}

#define MIRAI_EX_ENTRIES(SUF, WT, WRAP)                                                                          \
  int mirai_moe_gateup_ex_##SUF(const void* x_sorted, const int32_t* offsets, int32_t num_groups,              \
                                int64_t num_rows, int32_t hidden, int32_t inter, WT w1, WT w3, int32_t layout, \
                                int32_t activation, void* h, void* gate_up, mirai_stream_t stream) {          \
    return run_ex<GATEUP>("gateup_ex_" #SUF, x_sorted, offsets, num_groups, num_rows, hidden, inter, h,         \
                          gate_up, WRAP(w1), WRAP(w3), layout, activation, stream);                             \
  }                                                                                                              \
  int mirai_moe_down_ex_##SUF(const void* h, const int32_t* offsets, int32_t num_groups, int64_t num_rows,     \
                              int32_t inter, int32_t hidden, WT w2, int32_t layout, void* y,                    \
                              mirai_stream_t stream) {                                                           \
    return run_ex<DOWN>("down_ex_" #SUF, h, offsets, num_groups, num_rows, inter, hidden, y, nullptr, WRAP(w2), \
                        WRAP(w2), layout, MIRAI_ACT_SWIGLU, stream);                                             \
  }                                                                                                              \
  int mirai_moe_down_dx_ex_##SUF(const void* grad_y, const int32_t* offsets, int32_t num_groups,               \
                                 int64_t num_rows, int32_t hidden, int32_t inter, WT w2, int32_t layout,       \
                                 int32_t activation, const void* gate_up, void* grad_gate_up,                  \
                                 mirai_stream_t stream) {                                                        \
    if (!gate_up) return set_error(MIRAI_ERR_INVALID_ARG, "down_dx_ex_" #SUF ": saved gate/up is required");   \
    return run_ex<DXDOWN>("down_dx_ex_" #SUF, grad_y, offsets, num_groups, num_rows, hidden, inter,            \
                          grad_gate_up, const_cast<void*>(gate_up), WRAP(w2), WRAP(w2), layout, activation,     \
                          stream);                                                                               \
  }                                                                                                              \
  int mirai_moe_gateup_dx_ex_##SUF(const void* grad_gate_up, const int32_t* offsets, int32_t num_groups,       \
                                   int64_t num_rows, int32_t inter, int32_t hidden, WT w1, WT w3,              \
                                   int32_t layout, void* dx_sorted, mirai_stream_t stream) {                   \
    return run_ex<DXGATEUP>("gateup_dx_ex_" #SUF, grad_gate_up, offsets, num_groups, num_rows, 2 * inter,      \
                            hidden, dx_sorted, nullptr, WRAP(w1), WRAP(w3), layout, MIRAI_ACT_SWIGLU, stream); \
  }
MIRAI_EX_ENTRIES(bf16, const void*, wb)
MIRAI_EX_ENTRIES(nf4, const mirai_nf4_weight*, wn)
#undef MIRAI_EX_ENTRIES

}  // extern "C"
