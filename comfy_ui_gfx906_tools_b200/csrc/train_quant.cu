// Block-16 int4 quantizers of the reference's int4 training backward, in the
// layout gemm_int4(qblock = 16) reads: packed int8 [rows, K/2] (element e of
// each 32-element chunk in word e/8, nibble e%8, so a chunk's two 16-element
// blocks are words 0-1 and 2-3) and fp32 scales [rows, K/16].
//
// Reference: int4_train_quant.hip (nodes/ComfyUI-Gfx906Int4/csrc), quant16
// (:35-55), quant_rows_b16 (:59-85), quant_cols_b16 (:87-123), behind
// quantize_int4_rows / quantize_int4_cols (binding.cpp:317-356). Numerics
// kept identical: scale = max(amax, 1e-8) * (1/7) in fp32, t = v / scale
// (IEEE division), round to nearest even or, stochastically, floor(t + u)
// with u = 24 bits of a counter-based hash of (seed, element index), codes
// clamped to [-8, 7]; the optional transform of a 16-row column group is
// v <- (H16 / 4) diag(signs) v as four butterfly stages of exact pair
// sums / differences (the same pairs in the same stage order as the
// reference, so the fp32 results agree bit for bit).
//
// The hash is lowbias32 (Chris Wellons' integer hash, "hash prospector"):
// x ^= x >> 16; x *= 0x7feb352d; x ^= x >> 15; x *= 0x846ca68b; x ^= x >> 16.
//
// B200 layout of the work (memory-bound kernels):
//   rows  one thread per 16-element block: two 16-byte loads, one 8-byte
//         packed store and one scale store, consecutive threads consecutive
//         blocks of a row (coalesced both ways).
//   cols  one thread per (column, pair of 16-row groups): 32 coalesced
//         2-byte loads down the column (consecutive threads take consecutive
//         columns) and one 16-byte packed + one 8-byte scale store per
//         thread, a whole 32-row chunk of the transposed output.
#include "common.cuh"
#include "kernels.h"

namespace gfx {
namespace trainq {

__device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// uniform in [0, 1) with 24 random bits, per (seed, 64-bit element index)
__device__ __forceinline__ float hash_uniform(uint32_t seed, unsigned long long element) {
  const uint32_t h = lowbias32(seed ^ lowbias32((uint32_t)element ^ lowbias32((uint32_t)(element >> 32))));
  return (float)(h >> 8) * (1.0f / 16777216.0f);
}

// 16 values -> 16 nibbles (two words) and the block scale
template <bool kSR>
__device__ __forceinline__ float quant_block16(const float (&v)[16], uint32_t seed, unsigned long long first,
                                               uint32_t& lo, uint32_t& hi) {
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[e]));
  const float s = fmaxf(amax, 1e-8f) * (1.0f / 7.0f);
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const float t = __fdiv_rn(v[e], s);
    const float r = kSR ? floorf(__fadd_rn(t, hash_uniform(seed, first + e))) : rintf(t);
    const int code = (int)fminf(fmaxf(r, -8.0f), 7.0f);
    w[e >> 3] |= ((uint32_t)code & 0xFu) << (4 * (e & 7));
  }
  lo = w[0];
  hi = w[1];
  return s;
}

template <bool kSR>
__global__ void __launch_bounds__(256) quant_rows16_kernel(const __half* __restrict__ x, long long row_stride, int R,
                                                           int C, uint32_t seed, uint2* __restrict__ packed,
                                                           float* __restrict__ scale) {
  const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // 16-element block
  const int per_row = C / 16;
  if (b >= (long long)R * per_row) return;
  const int r = (int)(b / per_row), j = (int)(b % per_row);
  const uint4* src = reinterpret_cast<const uint4*>(x + r * row_stride + j * 16);
  const uint4 a = src[0], c = src[1];
  const uint32_t raw[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
  float v[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&raw[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
  uint32_t lo, hi;
  scale[b] = quant_block16<kSR>(v, seed, (unsigned long long)r * C + (unsigned long long)j * 16, lo, hi);
  packed[b] = make_uint2(lo, hi);
}

// (H16 / 4) diag(signs) v: four stages of pair sums and differences
__device__ __forceinline__ void hadamard16(float (&v)[16], const float (&sg)[16]) {
#pragma unroll
  for (int t = 0; t < 16; ++t) v[t] = __fmul_rn(v[t], sg[t]);
#pragma unroll
  for (int h = 1; h < 16; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if ((i & h) == 0) {
        const float a = v[i], b = v[i + h];
        v[i] = __fadd_rn(a, b);
        v[i + h] = __fsub_rn(a, b);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < 16; ++t) v[t] = __fmul_rn(v[t], 0.25f);
}

template <bool kRHT, bool kSR>
__global__ void __launch_bounds__(256) quant_cols16_kernel(const __half* __restrict__ x, long long row_stride, int R,
                                                           int C, const float* __restrict__ signs, uint32_t seed,
                                                           uint4* __restrict__ packed, float2* __restrict__ scale) {
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int chunks = R / 32;  // pairs of 16-row groups
  if (id >= (long long)C * chunks) return;
  const int c = (int)(id % C), g2 = (int)(id / C);
  float sg[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) sg[t] = kRHT ? signs[t] : 1.0f;
  uint32_t w[4];
  float s[2];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row0 = g2 * 32 + half * 16;
    float v[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) v[t] = __half2float(x[(long long)(row0 + t) * row_stride + c]);
    if constexpr (kRHT) hadamard16(v, sg);
    s[half] = quant_block16<kSR>(v, seed, (unsigned long long)c * R + row0, w[2 * half], w[2 * half + 1]);
  }
  packed[(long long)c * chunks + g2] = make_uint4(w[0], w[1], w[2], w[3]);
  scale[(long long)c * chunks + g2] = make_float2(s[0], s[1]);
}

}  // namespace trainq

int launch_quantize_int4_rows(const void* x, long long row_stride, int R, int C, int sr, uint32_t seed, void* packed,
                              float* scale, cudaStream_t st) {
  const long long n = (long long)R * (C / 16);
  if (n == 0) return GFX_OK;
  const unsigned grid = (unsigned)((n + 255) / 256);
  if (sr)
    trainq::quant_rows16_kernel<true><<<grid, 256, 0, st>>>((const __half*)x, row_stride, R, C, seed,
                                                             (uint2*)packed, scale);
  else
    trainq::quant_rows16_kernel<false><<<grid, 256, 0, st>>>((const __half*)x, row_stride, R, C, seed,
                                                              (uint2*)packed, scale);
  return check_launch("quant_rows16_kernel");
}

int launch_quantize_int4_cols(const void* x, long long row_stride, int R, int C, const float* signs, int sr,
                              uint32_t seed, void* packed, float* scale, cudaStream_t st) {
  const long long n = (long long)C * (R / 32);
  if (n == 0) return GFX_OK;
  const unsigned grid = (unsigned)((n + 255) / 256);
  const __half* xh = (const __half*)x;
  uint4* p = (uint4*)packed;
  float2* s = (float2*)scale;
  if (signs && sr)
    trainq::quant_cols16_kernel<true, true><<<grid, 256, 0, st>>>(xh, row_stride, R, C, signs, seed, p, s);
  else if (signs)
    trainq::quant_cols16_kernel<true, false><<<grid, 256, 0, st>>>(xh, row_stride, R, C, signs, seed, p, s);
  else if (sr)
    trainq::quant_cols16_kernel<false, true><<<grid, 256, 0, st>>>(xh, row_stride, R, C, signs, seed, p, s);
  else
    trainq::quant_cols16_kernel<false, false><<<grid, 256, 0, st>>>(xh, row_stride, R, C, signs, seed, p, s);
  return check_launch("quant_cols16_kernel");
}

}  // namespace gfx
