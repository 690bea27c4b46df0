// Weight ingest on the GPU: NF4 (blocksize 64, double-quantised absmax) and
// per-output-channel INT8, producing the buffers the reference stores
// (experts.py:998-1031 for NF4, quant.py:189-235 with group_size 0 for INT8).
//
// NF4 follows the published construction the reference delegates to
// bitsandbytes (quant.py:315-358): absmax over 64 consecutive elements of the
// row-major expert matrix, x * (1 / absmax) mapped to the nearest NF4 value
// (a value above a midpoint takes the upper code), two codes per byte with
// the first element in the high nibble; then the fp32 absmax vector minus its
// mean is quantised blockwise (256) to the nearest entry of the 8-bit
// dynamic-tree map (ties to the lower entry).
#include "common.cuh"

namespace mirai {
namespace qz {

// One warp per 64-element block: lane l holds elements 2l, 2l+1.
__global__ void __launch_bounds__(256) nf4_blocks_kernel(const __nv_bfloat16* __restrict__ w, int64_t nblocks,
                                                         const float* __restrict__ code,
                                                         uint8_t* __restrict__ packed, float* __restrict__ absmax) {
  __shared__ float mids[15];
  if (threadIdx.x < 15)
    mids[threadIdx.x] = (float)(((double)code[threadIdx.x] + (double)code[threadIdx.x + 1]) / 2.0);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t b = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (b >= nblocks) return;
  const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(w + b * 64)[lane];
  const float x0 = __bfloat162float(v.x), x1 = __bfloat162float(v.y);
  float m = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float inv = m == 0.f ? 0.f : __fdiv_rn(1.f, m);
  const float n0 = __fmul_rn(x0, inv), n1 = __fmul_rn(x1, inv);
  int q0 = 0, q1 = 0;
#pragma unroll
  for (int i = 0; i < 15; ++i) {
    q0 += n0 > mids[i];
    q1 += n1 > mids[i];
  }
  packed[b * 32 + lane] = (uint8_t)((q0 << 4) | q1);
  if (lane == 0) absmax[b] = m;
}

// One CTA per expert: offset = mean(absmax) (fp64 sum), then blockwise 8-bit
// quantisation of (absmax - offset) against the sorted dynamic map.
__global__ void __launch_bounds__(1024) nf4_nested_kernel(const float* __restrict__ absmax, int64_t blocks_per_expert,
                                                          int nested_bs, int n_nested,
                                                          const float* __restrict__ ncode,
                                                          uint8_t* __restrict__ absmax_q,
                                                          float* __restrict__ nested_absmax,
                                                          float* __restrict__ offset) {
  __shared__ float table[256];
  __shared__ double partial[32];
  __shared__ float s_off;
  const int e = blockIdx.x;
  const float* a = absmax + (int64_t)e * blocks_per_expert;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) table[i] = ncode[i];
  double sum = 0.0;
  for (int64_t i = threadIdx.x; i < blocks_per_expert; i += blockDim.x) sum += (double)a[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x < 32) {
    double s = threadIdx.x < (blockDim.x >> 5) ? partial[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) {
      s_off = (float)(s / (double)blocks_per_expert);
      offset[e] = s_off;
    }
  }
  __syncthreads();
  const float off = s_off;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int nb = threadIdx.x >> 5; nb < n_nested; nb += warps) {
    const int64_t base = (int64_t)nb * nested_bs;
    float m = 0.f;
    for (int j = lane; j < nested_bs; j += 32) {
      const int64_t i = base + j;
      if (i < blocks_per_expert) m = fmaxf(m, fabsf(__fsub_rn(a[i], off)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float inv = m == 0.f ? 0.f : __fdiv_rn(1.f, m);
    for (int j = lane; j < nested_bs; j += 32) {
      const int64_t i = base + j;
      if (i >= blocks_per_expert) break;
      const float x = __fmul_rn(__fsub_rn(a[i], off), inv);
      int lo = 0, hi = 256;  // first index with table[idx] >= x
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (table[mid] < x) lo = mid + 1;
        else hi = mid;
      }
      int h = lo < 1 ? 1 : (lo > 255 ? 255 : lo);
      const int l = h - 1;
      const float dl = fabsf(__fsub_rn(x, table[l]));
      const float dh = fabsf(__fsub_rn(table[h], x));
      absmax_q[(int64_t)e * blocks_per_expert + i] = (uint8_t)(dh < dl ? h : l);
    }
    if (lane == 0) nested_absmax[(int64_t)e * n_nested + nb] = m;
  }
}

// NF4 -> bf16 [E, out, in] (nf4_dequantize_stack, quant.py:380-434): a
// thread decodes 4 code bytes (8 elements) per step, kDequantItems steps a
// block-width apart, so that a warp reads 128 contiguous bytes and writes 512
// per step (HBM-bound: 2.25 bytes moved per element);
// w = bf16(code[nibble] * (ncode[q] * nested_absmax + offset)), the same
// rounding as the grouped GEMMs' in-loop decode.
constexpr int kDequantItems = 8;  // 8-element chunks per thread

__global__ void __launch_bounds__(256) nf4_dequant_kernel(const uint32_t* __restrict__ packed,
                                                          const uint8_t* __restrict__ absmax,
                                                          const float* __restrict__ nested_absmax,
                                                          const float* __restrict__ offset,
                                                          const float* __restrict__ code,
                                                          const float* __restrict__ ncode, int per_expert,
                                                          int nested_bs, int n_nested, uint4* __restrict__ out) {
  __shared__ float s_code[16], s_ncode[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) s_ncode[i] = ncode[i];
  if (threadIdx.x < 16) s_code[threadIdx.x] = code[threadIdx.x];
  __syncthreads();
  // grid: x = blocks of kDequantItems x 256 chunks of one expert, y = expert (no 64-bit
  // division per thread); each thread issues all its loads before decoding
  const int e = blockIdx.y;
  const int cpe = per_expert / 8;  // 8-element chunks per expert
  const int base = blockIdx.x * (blockDim.x * kDequantItems) + threadIdx.x;
  const float off = __ldg(offset + e);
  const uint32_t* pk = packed + (int64_t)e * cpe;
  const uint8_t* am = absmax + (int64_t)e * (per_expert / 64);
  const float* na = nested_absmax + (int64_t)e * n_nested;
  const bool pow2 = (nested_bs & (nested_bs - 1)) == 0;
  const int nshift = 31 - __clz(nested_bs);
  uint32_t w[kDequantItems];
  uint8_t q[kDequantItems];
  float nabs[kDequantItems];
#pragma unroll
  for (int i = 0; i < kDequantItems; ++i) {
    const int cl = base + i * blockDim.x;
    if (cl < cpe) {
      const int blk = cl >> 3;  // absmax block inside the expert
      w[i] = __ldg(pk + cl);
      q[i] = __ldg(am + blk);
      nabs[i] = __ldg(na + (pow2 ? blk >> nshift : blk / nested_bs));
    }
  }
  uint4* dst = out + (int64_t)e * cpe;
#pragma unroll
  for (int i = 0; i < kDequantItems; ++i) {
    const int cl = base + i * blockDim.x;
    if (cl >= cpe) break;
    const float scale = __fadd_rn(__fmul_rn(s_ncode[q[i]], nabs[i]), off);
    uint32_t o[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t byte = (w[i] >> (8 * b)) & 0xFFu;  // first element in the high nibble
      o[b] = pack_bf16x2(__fmul_rn(s_code[byte >> 4], scale), __fmul_rn(s_code[byte & 15u], scale));
    }
    dst[cl] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// INT8 per row: scale = max(amax / 127, 1e-30); q = clamp(rint(x / scale), +-127).
template <typename T>
__global__ void __launch_bounds__(256) int8_rows_kernel(const T* __restrict__ w, int64_t rows, int64_t in,
                                                        int8_t* __restrict__ q, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const T* row = w + r * in;
  float m = 0.f;
  for (int64_t i = lane; i < in; i += 32) m = fmaxf(m, fabsf((float)row[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float s = fmaxf(__fdiv_rn(m, 127.f), 1e-30f);
  for (int64_t i = lane; i < in; i += 32) {
    const float v = rintf(__fdiv_rn((float)row[i], s));
    q[r * in + i] = (int8_t)fminf(fmaxf(v, -127.f), 127.f);
  }
  if (lane == 0) scale[r] = s;
}

}  // namespace qz
}  // namespace mirai

using namespace mirai;

extern "C" {

size_t mirai_nf4_quantize_workspace_bytes(int32_t num_experts, int64_t out_features, int64_t in_features) {
  if (num_experts <= 0 || out_features <= 0 || in_features <= 0) return 0;
  return (size_t)num_experts * (size_t)(out_features * in_features / 64) * sizeof(float);
}

int mirai_nf4_quantize(const void* weight_bf16, int32_t num_experts, int64_t out_features, int64_t in_features,
                       const float* code, const float* nested_code, int32_t blocksize, int32_t nested_blocksize,
                       uint8_t* packed, uint8_t* absmax, float* nested_absmax, float* offset, void* workspace,
                       size_t workspace_bytes, mirai_stream_t stream) {
  if (num_experts <= 0 || out_features <= 0 || in_features <= 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "nf4_quantize: bad sizes");
  if (blocksize != 64 || nested_blocksize <= 0)
    return set_error(MIRAI_ERR_UNSUPPORTED, "nf4_quantize: blocksize must be 64 (got %d)", blocksize);
  const int64_t per = out_features * in_features;
  if (per % 64 != 0) return set_error(MIRAI_ERR_UNSUPPORTED, "nf4_quantize: out*in must be a multiple of 64");
  if (!weight_bf16 || !code || !nested_code || !packed || !absmax || !nested_absmax || !offset)
    return set_error(MIRAI_ERR_INVALID_ARG, "nf4_quantize: null pointer");
  const size_t need = mirai_nf4_quantize_workspace_bytes(num_experts, out_features, in_features);
  if (!workspace || workspace_bytes < need)
    return set_error(MIRAI_ERR_WORKSPACE, "nf4_quantize: workspace of %zu bytes needed", need);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t bpe = per / 64;
  const int64_t nblocks = bpe * num_experts;
  float* am = static_cast<float*>(workspace);
  qz::nf4_blocks_kernel<<<(unsigned)((nblocks + 7) / 8), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(weight_bf16), nblocks, code, packed, am);
  const int n_nested = (int)((bpe + nested_blocksize - 1) / nested_blocksize);
  qz::nf4_nested_kernel<<<num_experts, 1024, 0, s>>>(am, bpe, nested_blocksize, n_nested, nested_code, absmax,
                                                      nested_absmax, offset);
  return check_launch("nf4_quantize", 2);
}

int mirai_nf4_dequantize(const uint8_t* packed, const uint8_t* absmax, const float* nested_absmax,
                         const float* offset, const float* code, const float* nested_code, int32_t num_experts,
                         int64_t out_features, int64_t in_features, int32_t blocksize, int32_t nested_blocksize,
                         void* out_bf16, mirai_stream_t stream) {
  if (num_experts <= 0 || out_features <= 0 || in_features <= 0)
    return set_error(MIRAI_ERR_INVALID_ARG, "nf4_dequantize: bad sizes");
  if (blocksize != 64 || nested_blocksize <= 0)
    return set_error(MIRAI_ERR_UNSUPPORTED, "nf4_dequantize: blocksize must be 64 (got %d)", blocksize);
  const int64_t per = out_features * in_features;
  if (per % 64 != 0) return set_error(MIRAI_ERR_UNSUPPORTED, "nf4_dequantize: out*in must be a multiple of 64");
  if (per >= ((int64_t)1 << 31) || num_experts > 65535)
    return set_error(MIRAI_ERR_UNSUPPORTED, "nf4_dequantize: at most 2^31 elements per expert and 65535 experts");
  if (!packed || !absmax || !nested_absmax || !offset || !code || !nested_code || !out_bf16 ||
      (reinterpret_cast<uintptr_t>(packed) & 15u) || (reinterpret_cast<uintptr_t>(out_bf16) & 15u))
    return set_error(MIRAI_ERR_INVALID_ARG, "nf4_dequantize: null or misaligned pointer");
  const int n_nested = (int)((per / 64 + nested_blocksize - 1) / nested_blocksize);
  const dim3 grid((unsigned)((per / 8 + 256 * qz::kDequantItems - 1) / (256 * qz::kDequantItems)),
                  (unsigned)num_experts);
  qz::nf4_dequant_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(packed), absmax, nested_absmax, offset, code, nested_code, (int)per,
      nested_blocksize, n_nested, static_cast<uint4*>(out_bf16));
  return check_launch("nf4_dequantize");
}

int mirai_int8_quantize_rows(const void* weight, int32_t weight_dtype, int64_t rows, int64_t in_features, int8_t* q,
                             float* scale, mirai_stream_t stream) {
  if (rows < 0 || in_features <= 0) return set_error(MIRAI_ERR_INVALID_ARG, "int8_quantize_rows: bad sizes");
  if (rows == 0) return MIRAI_OK;
  if (!weight || !q || !scale) return set_error(MIRAI_ERR_INVALID_ARG, "int8_quantize_rows: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((rows + 7) / 8);
  if (weight_dtype == MIRAI_DTYPE_F32)
    qz::int8_rows_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(weight), rows, in_features, q, scale);
  else if (weight_dtype == MIRAI_DTYPE_BF16)
    qz::int8_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(weight), rows,
                                                             in_features, q, scale);
  else
    return set_error(MIRAI_ERR_INVALID_ARG, "int8_quantize_rows: unknown weight dtype %d", weight_dtype);
  return check_launch("int8_quantize_rows");
}

}  // extern "C"
