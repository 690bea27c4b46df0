// a5: the block-Hadamard rotation of the reference's INT8 format, applied to
// activations so that the INT8 grouped GEMMs read the stored codes as they are.
//
// The reference quantises W rotated (quant.py:189-235: q*s = W H, per group of
// g input features) and de-rotates the weight before its bf16 matmul
// (quant.py:238-260).  H = h4 (x) ... (x) h4 / sqrt(g), g = 4^m, with
// h4[i][j] = -1 where i + j == 3 and +1 elsewhere (quant.py:103-122), is
// symmetric and orthogonal, so (rotated_int8.py:7-21)
//     y  = x W^T      = (x H) (q s)^T        forward: rotate the GEMM input
//     dx = dy W       = (dy (q s)) H         backward: rotate the GEMM output
// mirai_rotate_rows applies "row times H" to every g-wide group of a row-major
// matrix; mirai_swiglu_backward_rotated rotates the down projection's input
// gradient and applies the SwiGLU backward in the same pass.
//
// Fast transform: along one base-4 digit of the index, (v h4)_j = S - 2 v_{3-j}
// with S = v0 + v1 + v2 + v3; the m digits are transformed in turn, in fp32,
// and the result is scaled by 2^-m (exact).  Each CTA holds a 4096-element
// tile (whole groups, g | 4096); a thread keeps 16 elements in registers and
// transforms two digits at a time, exchanging through shared memory between
// digit pairs.  HBM-bound: one read and one write per element.
#include "common.cuh"

namespace mirai {
namespace rot {

constexpr int kTile = 4096;
constexpr int kThreads = 256;  // 16 elements per thread
// padded shared-memory index: +4 words every 32 (conflict-free 16-byte rows of
// 16 contiguous elements) and +16 every 256 (conflict-free 16-strided reads)
__device__ __forceinline__ int pad(int i) { return i + (i >> 5) * 4 + (i >> 8) * 16; }
constexpr int kSmemWords = kTile + (kTile / 32) * 4 + (kTile / 256) * 16;

// transform digit 0 of v[base + {0, s, 2s, 3s}]
template <int S>
__device__ __forceinline__ void h4(float (&v)[16], int b) {
  const float a0 = v[b], a1 = v[b + S], a2 = v[b + 2 * S], a3 = v[b + 3 * S];
  const float sum = (a0 + a1) + (a2 + a3);
  v[b] = fmaf(-2.f, a3, sum);
  v[b + S] = fmaf(-2.f, a2, sum);
  v[b + 2 * S] = fmaf(-2.f, a1, sum);
  v[b + 3 * S] = fmaf(-2.f, a0, sum);
}

// the 16 values are [digit1][digit0]; transform digit 0 and, if `two`, digit 1
__device__ __forceinline__ void h16(float (&v)[16], bool two) {
#pragma unroll
  for (int b = 0; b < 16; b += 4) h4<1>(v, b);
  if (two) {
#pragma unroll
    for (int b = 0; b < 4; ++b) h4<4>(v, b);
  }
}

__device__ __forceinline__ void load16(const void* src, int dtype, int64_t e0, float (&v)[16]) {
  if (dtype == MIRAI_DTYPE_BF16) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(src) + e0);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint4 r = __ldg(p + q);
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * q + 2 * j] = bf16_lo(w[j]);
        v[8 * q + 2 * j + 1] = bf16_hi(w[j]);
      }
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(src) + e0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 r = __ldg(p + q);
      v[4 * q] = r.x, v[4 * q + 1] = r.y, v[4 * q + 2] = r.z, v[4 * q + 3] = r.w;
    }
  }
}

__device__ __forceinline__ void store16(void* dst, int dtype, int64_t e0, const float (&v)[16]) {
  if (dtype == MIRAI_DTYPE_BF16) {
    uint4* p = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(dst) + e0);
#pragma unroll
    for (int q = 0; q < 2; ++q)
      p[q] = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                        pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
  } else {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(dst) + e0);
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }
}

// SwiGLU backward of one row segment given dh (the autograd of
// silu(gate) * up in bf16, as the fused down-dX epilogue computes it).
struct SwigluBwd {
  const __nv_bfloat16* gate_up;  // [rows, 2I]
  __nv_bfloat16* out;            // [rows, 2I]
  int inter;
  __device__ __forceinline__ void operator()(int64_t e0, float (&dh)[16]) const {
    const int64_t row = e0 / inter;
    const int col = (int)(e0 - row * inter);
    const uint4* gs = reinterpret_cast<const uint4*>(gate_up + row * 2 * inter + col);
    const uint4* us = reinterpret_cast<const uint4*>(gate_up + row * 2 * inter + inter + col);
    uint32_t gw[8], uw[8], dg[8], du[8];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint4 a = __ldg(gs + q), b = __ldg(us + q);
      gw[4 * q] = a.x, gw[4 * q + 1] = a.y, gw[4 * q + 2] = a.z, gw[4 * q + 3] = a.w;
      uw[4 * q] = b.x, uw[4 * q + 1] = b.y, uw[4 * q + 2] = b.z, uw[4 * q + 3] = b.w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float dgo[2], duo[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float d = __bfloat162float(__float2bfloat16_rn(dh[2 * j + hh]));
        const float gv = hh ? bf16_hi(gw[j]) : bf16_lo(gw[j]);
        const float uv = hh ? bf16_hi(uw[j]) : bf16_lo(uw[j]);
        const float sg = __fdividef(1.f, 1.f + __expf(-gv));
        const float act = __bfloat162float(__float2bfloat16_rn(gv * sg));
        const float dact = __bfloat162float(__float2bfloat16_rn(d * uv));
        duo[hh] = d * act;
        dgo[hh] = dact * sg * (1.f + gv * (1.f - sg));
      }
      dg[j] = pack_bf16x2(dgo[0], dgo[1]);
      du[j] = pack_bf16x2(duo[0], duo[1]);
    }
    uint4* gd = reinterpret_cast<uint4*>(out + row * 2 * inter + col);
    uint4* ud = reinterpret_cast<uint4*>(out + row * 2 * inter + inter + col);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      gd[q] = make_uint4(dg[4 * q], dg[4 * q + 1], dg[4 * q + 2], dg[4 * q + 3]);
      ud[q] = make_uint4(du[4 * q], du[4 * q + 1], du[4 * q + 2], du[4 * q + 3]);
    }
  }
};

struct PlainStore {
  void* out;
  int dtype;
  __device__ __forceinline__ void operator()(int64_t e0, float (&v)[16]) const { store16(out, dtype, e0, v); }
};

// digits: m = log4(group).  total: elements (a multiple of 16 and of group).
template <class Epilogue>
__global__ void __launch_bounds__(kThreads) rotate_kernel(const void* in, int in_dtype, int64_t total,
                                                          int digits, Epilogue epi) {
  __shared__ __align__(16) float sm[kSmemWords];
  const int t = threadIdx.x;
  const float scale = __uint_as_float((uint32_t)(127 - digits) << 23);  // 2^-m
  const int64_t tiles = (total + kTile - 1) / kTile;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t base = tile * kTile;
    const int64_t e0 = base + 16 * t;
    const bool live = e0 < total;  // total % 16 == 0: a thread's 16 elements are all in or all out
    float v[16];
    if (live) load16(in, in_dtype, e0, v);
    else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.f;
    }
    h16(v, digits >= 2);  // digits 0 and 1: the thread's 16 contiguous elements
    int done = digits < 2 ? digits : 2;
    int s = 16;  // stride of the next digit pair
    bool strided = false;
    while (done < digits) {
      // write back in the current layout, then gather 16 elements at stride s:
      // element hi * 16s + mid * s + lo, thread t = hi * s + lo
      __syncthreads();  // the previous pass's reads of sm are complete
      if (!strided) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<float4*>(&sm[pad(16 * t + 4 * q)]) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2],
                                                                             v[4 * q + 3]);
      } else {
        const int ps = s / 16, hi = t / ps, lo = t - hi * ps;
#pragma unroll
        for (int mid = 0; mid < 16; ++mid) sm[pad(hi * 16 * ps + mid * ps + lo)] = v[mid];
      }
      __syncthreads();
      const int hi = t / s, lo = t - hi * s;
#pragma unroll
      for (int mid = 0; mid < 16; ++mid) v[mid] = sm[pad(hi * 16 * s + mid * s + lo)];
      h16(v, digits - done >= 2);
      done += digits - done >= 2 ? 2 : 1;
      strided = true;
      s *= 16;
    }
    if (strided) {  // back to 16 contiguous elements per thread
      const int ps = s / 16, hi = t / ps, lo = t - hi * ps;
      __syncthreads();
#pragma unroll
      for (int mid = 0; mid < 16; ++mid) sm[pad(hi * 16 * ps + mid * ps + lo)] = v[mid];
      __syncthreads();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 r = *reinterpret_cast<const float4*>(&sm[pad(16 * t + 4 * q)]);
        v[4 * q] = r.x, v[4 * q + 1] = r.y, v[4 * q + 2] = r.z, v[4 * q + 3] = r.w;
      }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] *= scale;
    if (live) epi(e0, v);
  }
}

inline int digits_of(int group) {
  int m = 0;
  for (int g = group; g > 1; g >>= 2) ++m;
  return m;
}

inline bool valid_group(int group) {
  return group >= 4 && group <= kTile && (group & (group - 1)) == 0 && (__builtin_ctz((unsigned)group) % 2) == 0;
}

inline int grid_for(int64_t total) {
  const int64_t tiles = (total + kTile - 1) / kTile;
  const int64_t cap = (int64_t)sm_count() * 8;
  return (int)(tiles < cap ? tiles : cap);
}

}  // namespace rot
}  // namespace mirai

using namespace mirai;

extern "C" {

int mirai_rotate_rows(const void* in, int32_t in_dtype, int64_t rows, int32_t cols, int32_t group, void* out,
                      int32_t out_dtype, mirai_stream_t stream) {
  if (!rot::valid_group(group))
    return set_error(MIRAI_ERR_INVALID_ARG, "rotate_rows: group %d is not a power of 4 in [4, %d]", group, rot::kTile);
  if (rows < 0 || cols <= 0 || cols % group != 0 || cols % 16 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "rotate_rows: cols %d must be a multiple of the group %d and of 16", cols,
                     group);
  const bool dt_ok = [](int d) { return d == MIRAI_DTYPE_BF16 || d == MIRAI_DTYPE_F32; }(in_dtype) &&
                     (out_dtype == MIRAI_DTYPE_BF16 || out_dtype == MIRAI_DTYPE_F32);
  if (!dt_ok) return set_error(MIRAI_ERR_INVALID_ARG, "rotate_rows: dtypes %d -> %d", in_dtype, out_dtype);
  if (rows == 0) return MIRAI_OK;
  if (!in || !out || (reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return set_error(MIRAI_ERR_INVALID_ARG, "rotate_rows: null or misaligned pointer");
  const int64_t total = rows * (int64_t)cols;
  rot::rotate_kernel<rot::PlainStore><<<rot::grid_for(total), rot::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      in, in_dtype, total, rot::digits_of(group), rot::PlainStore{out, out_dtype});
  return check_launch("rotate_rows");
}

int mirai_swiglu_backward_rotated(const void* dh, const void* gate_up, int64_t rows, int32_t inter, int32_t group,
                                  void* grad_gate_up, mirai_stream_t stream) {
  if (!rot::valid_group(group))
    return set_error(MIRAI_ERR_INVALID_ARG, "swiglu_backward_rotated: group %d is not a power of 4 in [4, %d]", group,
                     rot::kTile);
  if (rows < 0 || inter <= 0 || inter % group != 0 || inter % 16 != 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "swiglu_backward_rotated: inter %d must be a multiple of %d and 16", inter,
                     group);
  if (rows == 0) return MIRAI_OK;
  if (!dh || !gate_up || !grad_gate_up || (reinterpret_cast<uintptr_t>(dh) & 15) ||
      (reinterpret_cast<uintptr_t>(gate_up) & 15) || (reinterpret_cast<uintptr_t>(grad_gate_up) & 15))
    return set_error(MIRAI_ERR_INVALID_ARG, "swiglu_backward_rotated: null or misaligned pointer");
  const int64_t total = rows * (int64_t)inter;
  const rot::SwigluBwd epi{static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(grad_gate_up),
                           inter};
  rot::rotate_kernel<rot::SwigluBwd><<<rot::grid_for(total), rot::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      dh, MIRAI_DTYPE_BF16, total, rot::digits_of(group), epi);
  return check_launch("swiglu_backward_rotated");
}

}  // extern "C"
