// Weight-format kernels: dequantize, ggml Q4_0 repack, block-32 int4 / int8
// quantizers, fp32 -> fp16 scale conversion.
//
// These are memory-bound byte/integer kernels: one thread per 32-element block
// (or per 8-element nibble word), coalesced 16-byte accesses where the format
// allows, grid sized in whole multiples of the SM count by the hardware
// scheduler (plain 1-D grids; each thread does a constant amount of work).
//
// Bit-exactness contract (checked against the CPU oracle in tests):
//  * int4_dequant: code * scale is one IEEE fp32 multiply; bf16/f16 outputs
//    round that product to nearest-even once (int4_train_test.py:46-52,
//    nodes.py:51-52).
//  * quantize_pack_int4: ops.quantize_pack_int4 (ops.py:108-126): amax over
//    the block, clamp_min(1e-8), scale = amax / 7 (div_mode 0, IEEE division:
//    torch on CPU) or amax * (1/7) (div_mode 1: torch on CUDA, and the
//    reference's HIP quantizer int4_gemm_scaled.hip:210-211), codes =
//    clamp(rint(v / scale), -8, 7) with an IEEE division and round-half-even.
//  * quantize_int8: int8_gemm.hip:217-246 (amax * (1/127), rint, +-127).
//  * repack_q4_0: ops.repack_q4_0_native (ops.py:129-164), lossless.
#include "common.cuh"
#include "kernels.h"

namespace gfx {

// ---------------------------------------------------------------------------
// dequant: one thread per 32-bit nibble word (8 elements)
// ---------------------------------------------------------------------------
template <bool kF16Scale, typename OutT>
__global__ void int4_dequant_kernel(const uint32_t* __restrict__ wq, const void* __restrict__ ws,
                                    OutT* __restrict__ out, int64_t words, int words_per_group_log2) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= words) return;
  const uint32_t w = wq[i];
  const int64_t grp = i >> words_per_group_log2;  // 4 words per 32-group, 2 per 16-group; rows are whole groups
  const float s = kF16Scale ? __half2float(reinterpret_cast<const __half*>(ws)[grp])
                            : reinterpret_cast<const float*>(ws)[grp];
  OutT v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int code = (int)((w >> (4 * e)) & 0xF) - (int)(((w >> (4 * e)) & 0x8) << 1);  // sign-extend nibble
    v[e] = from_f32<OutT>(__fmul_rn((float)code, s));
  }
  OutT* dst = out + i * 8;
  if constexpr (sizeof(OutT) == 4) {
    reinterpret_cast<float4*>(dst)[0] = make_float4(to_f32(v[0]), to_f32(v[1]), to_f32(v[2]), to_f32(v[3]));
    reinterpret_cast<float4*>(dst)[1] = make_float4(to_f32(v[4]), to_f32(v[5]), to_f32(v[6]), to_f32(v[7]));
  } else {
    uint4 packed;
    uint16_t* h = reinterpret_cast<uint16_t*>(&packed);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = *reinterpret_cast<uint16_t*>(&v[e]);
    *reinterpret_cast<uint4*>(dst) = packed;
  }
}

int launch_int4_dequant(const void* wq, const void* ws, int scale_dtype, void* out, int out_dtype, int N, int K,
                        cudaStream_t stream, int qblock) {
  const int64_t words = (int64_t)N * K / 8;
  if (words == 0) return GFX_OK;
  const int threads = 256;
  const unsigned blocks = (unsigned)((words + threads - 1) / threads);
  const bool f16s = scale_dtype == GFX_SCALE_F16;
#define DQ(F16S, T) \
  int4_dequant_kernel<F16S, T><<<blocks, threads, 0, stream>>>((const uint32_t*)wq, ws, (T*)out, words, \
                                                                 qblock == 16 ? 1 : 2)
  if (out_dtype == GFX_DTYPE_F32) { if (f16s) DQ(true, float); else DQ(false, float); }
  else if (out_dtype == GFX_DTYPE_F16) { if (f16s) DQ(true, __half); else DQ(false, __half); }
  else { if (f16s) DQ(true, __nv_bfloat16); else DQ(false, __nv_bfloat16); }
#undef DQ
  return check_launch("int4_dequant_kernel");
}

// ---------------------------------------------------------------------------
// Q4_0 repack: one thread per 18-byte ggml block
// ---------------------------------------------------------------------------
__global__ void repack_q4_0_kernel(const uint8_t* __restrict__ raw, uint4* __restrict__ packed,
                                   float* __restrict__ scale, __half* __restrict__ scale_f16, int64_t blocks) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= blocks) return;
  const uint8_t* src = raw + b * 18;
  const uint16_t dbits = (uint16_t)src[0] | ((uint16_t)src[1] << 8);
  uint8_t qs[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) qs[i] = src[2 + i];
  // element e: offset-8 nibble u_e (split-half: e < 16 low nibble of byte e,
  // else high nibble of byte e-16); native nibble = (u_e - 8) & 0xF = u_e ^ 8.
  uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const uint32_t u = e < 16 ? (qs[e] & 0xF) : (qs[e - 16] >> 4);
    words[e >> 3] |= ((u ^ 8u) & 0xFu) << (4 * (e & 7));
  }
  packed[b] = make_uint4(words[0], words[1], words[2], words[3]);
  __half_raw hr;
  hr.x = dbits;
  const __half d = __half(hr);
  if (scale) scale[b] = __half2float(d);
  if (scale_f16) scale_f16[b] = d;
}

int launch_repack_q4_0(const void* raw, void* packed, float* scale, void* scale_f16, int N, int K,
                       cudaStream_t stream) {
  const int64_t blocks = (int64_t)N * (K / 32);
  if (blocks == 0) return GFX_OK;
  const int threads = 256;
  repack_q4_0_kernel<<<(unsigned)((blocks + threads - 1) / threads), threads, 0, stream>>>(
      (const uint8_t*)raw, (uint4*)packed, scale, (__half*)scale_f16, blocks);
  return check_launch("repack_q4_0_kernel");
}

// ---------------------------------------------------------------------------
// Q8_0 repack: one thread per 34-byte ggml block (fp16 d + 32 int8 codes)
// ---------------------------------------------------------------------------
// value = q * d: the int8 codes are already the W8A16 weight, d becomes its
// fp32 group scale. Lossless; blocks start on even addresses (34-byte stride),
// so the codes are read as 16 halfwords and written as two 16-byte stores.
__global__ void repack_q8_0_kernel(const uint16_t* __restrict__ raw, uint4* __restrict__ q,
                                   float* __restrict__ scale, int64_t blocks) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= blocks) return;
  const uint16_t* src = raw + b * 17;
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = (uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16);
  q[2 * b] = make_uint4(w[0], w[1], w[2], w[3]);
  q[2 * b + 1] = make_uint4(w[4], w[5], w[6], w[7]);
  __half_raw hr;
  hr.x = src[0];
  scale[b] = __half2float(__half(hr));
}

int launch_repack_q8_0(const void* raw, void* q, float* scale, int N, int K, cudaStream_t stream) {
  const int64_t blocks = (int64_t)N * (K / 32);
  if (blocks == 0) return GFX_OK;
  const int threads = 256;
  repack_q8_0_kernel<<<(unsigned)((blocks + threads - 1) / threads), threads, 0, stream>>>(
      (const uint16_t*)raw, (uint4*)q, scale, blocks);
  return check_launch("repack_q8_0_kernel");
}

// ---------------------------------------------------------------------------
// block-32 quantizers: one thread per block
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load_block32(const T* src, float (&v)[32]) {
#pragma unroll
  for (int e = 0; e < 32; ++e) v[e] = to_f32(src[e]);
}

template <typename T>
__global__ void quantize_pack_int4_kernel(const T* __restrict__ x, uint4* __restrict__ packed,
                                          float* __restrict__ scale, int64_t blocks, int div_mode) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= blocks) return;
  float v[32];
  load_block32(x + b * 32, v);
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(v[e]));
  amax = fmaxf(amax, 1e-8f);
  const float s = div_mode == 0 ? __fdiv_rn(amax, 7.0f) : __fmul_rn(amax, 1.0f / 7.0f);
  uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const float q = fminf(fmaxf(rintf(__fdiv_rn(v[e], s)), -8.0f), 7.0f);
    words[e >> 3] |= ((uint32_t)(int)q & 0xFu) << (4 * (e & 7));
  }
  packed[b] = make_uint4(words[0], words[1], words[2], words[3]);
  scale[b] = s;
}

template <typename T>
__global__ void quantize_int8_kernel(const T* __restrict__ x, uint4* __restrict__ q, float* __restrict__ scale,
                                     int64_t blocks) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= blocks) return;
  float v[32];
  load_block32(x + b * 32, v);
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(v[e]));
  const float s = __fmul_rn(fmaxf(amax, 1e-8f), 1.0f / 127.0f);
  uint32_t words[8];
#pragma unroll
  for (int wd = 0; wd < 8; ++wd) {
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float qv = fminf(fmaxf(rintf(__fdiv_rn(v[4 * wd + e], s)), -127.0f), 127.0f);
      word |= ((uint32_t)(int)qv & 0xFFu) << (8 * e);
    }
    words[wd] = word;
  }
  q[2 * b] = make_uint4(words[0], words[1], words[2], words[3]);
  q[2 * b + 1] = make_uint4(words[4], words[5], words[6], words[7]);
  scale[b] = s;
}

int launch_quantize_pack_int4(const void* x, int x_dtype, void* packed, float* scale, int64_t rows, int K,
                              int div_mode, cudaStream_t stream) {
  const int64_t blocks = rows * (K / 32);
  if (blocks == 0) return GFX_OK;
  const int threads = 128;
  const unsigned grid = (unsigned)((blocks + threads - 1) / threads);
  if (x_dtype == GFX_DTYPE_F32)
    quantize_pack_int4_kernel<float><<<grid, threads, 0, stream>>>((const float*)x, (uint4*)packed, scale, blocks,
                                                                   div_mode);
  else if (x_dtype == GFX_DTYPE_F16)
    quantize_pack_int4_kernel<__half><<<grid, threads, 0, stream>>>((const __half*)x, (uint4*)packed, scale, blocks,
                                                                    div_mode);
  else
    quantize_pack_int4_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>((const __nv_bfloat16*)x,
                                                                           (uint4*)packed, scale, blocks, div_mode);
  return check_launch("quantize_pack_int4_kernel");
}

int launch_quantize_int8(const void* x, int x_dtype, void* q, float* scale, int64_t rows, int K,
                         cudaStream_t stream) {
  const int64_t blocks = rows * (K / 32);
  if (blocks == 0) return GFX_OK;
  const int threads = 128;
  const unsigned grid = (unsigned)((blocks + threads - 1) / threads);
  if (x_dtype == GFX_DTYPE_F32)
    quantize_int8_kernel<float><<<grid, threads, 0, stream>>>((const float*)x, (uint4*)q, scale, blocks);
  else if (x_dtype == GFX_DTYPE_F16)
    quantize_int8_kernel<__half><<<grid, threads, 0, stream>>>((const __half*)x, (uint4*)q, scale, blocks);
  else
    quantize_int8_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>((const __nv_bfloat16*)x, (uint4*)q, scale,
                                                                      blocks);
  return check_launch("quantize_int8_kernel");
}

// ---------------------------------------------------------------------------
// fp32 -> fp16 scales with an exactness count
// ---------------------------------------------------------------------------
__global__ void scales_to_f16_kernel(const float* __restrict__ s, __half* __restrict__ s16, int64_t n,
                                     int* __restrict__ inexact) {
  int bad = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = s[i];
    const __half h = __float2half_rn(v);
    s16[i] = h;
    bad += (__half2float(h) != v) ? 1 : 0;
  }
  bad = __reduce_add_sync(0xffffffffu, bad);
  if ((threadIdx.x & 31) == 0 && bad) atomicAdd(inexact, bad);
}

int launch_scales_to_f16(const float* s, void* s16, int64_t n, int* inexact, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(inexact, 0, sizeof(int), stream);
  if (e != cudaSuccess) return set_error(GFX_ERR_CUDA, "scales_to_f16: memset failed: %s", cudaGetErrorString(e));
  if (n == 0) return GFX_OK;
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  if (blocks > 4096) blocks = 4096;
  scales_to_f16_kernel<<<(unsigned)blocks, threads, 0, stream>>>(s, (__half*)s16, n, inexact);
  return check_launch("scales_to_f16_kernel");
}

// ---------------------------------------------------------------------------
// block-diagonal randomized Hadamard rotation of activations
// ---------------------------------------------------------------------------
// out[r, g*G + i] = sum_j H_G[i, j] * sign[j] * x[r, g*G + j] / sqrt(G): the
// reference's `flat @ R^T` with R = H_G / sqrt(G) * diag(sign)
// (ops.py:68-105), evaluated as a fast Walsh-Hadamard transform instead of a
// G x G matmul: one warp per (row, group), E = G/32 consecutive elements per
// lane; butterflies of stride < E stay in registers, wider ones exchange
// through warp shuffles. fp32 arithmetic; the summation order differs from a
// matmul, so results agree with it to fp32 rounding, not bit for bit.
template <int E, typename InT, typename OutT>
__global__ void hadamard_rotate_kernel(const InT* __restrict__ x, const float* __restrict__ sign,
                                       OutT* __restrict__ out, int64_t items, int K) {
  constexpr int G = 32 * E;
  const int64_t item = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (item >= items) return;  // whole warps leave together (items are per warp)
  const int64_t groups_per_row = K / G;
  const int64_t row = item / groups_per_row, g = item % groups_per_row;
  const int64_t base = row * K + g * G + lane * E;
  float v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = to_f32(x[base + e]) * sign[lane * E + e];
  // strides inside a lane's E elements
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if ((e & h) == 0) {
        const float a = v[e], b = v[e + h];
        v[e] = a + b;
        v[e + h] = a - b;
      }
    }
  }
  // strides across lanes: element index bit h*E <-> lane bit h
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
    const bool upper = (lane & h) != 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, v[e], h);
      v[e] = upper ? other - v[e] : v[e] + other;
    }
  }
  const float norm = rsqrtf((float)G);
#pragma unroll
  for (int e = 0; e < E; ++e) out[base + e] = from_f32<OutT>(v[e] * norm);
}

template <int E, typename InT>
static int launch_hadamard_in(const void* x, const float* sign, void* out, int out_dtype, int64_t items, int K,
                              cudaStream_t st) {
  const int threads = 256;
  const int64_t blocks = (items * 32 + threads - 1) / threads;
  if (out_dtype == GFX_DTYPE_F32)
    hadamard_rotate_kernel<E, InT, float><<<blocks, threads, 0, st>>>((const InT*)x, sign, (float*)out, items, K);
  else if (out_dtype == GFX_DTYPE_F16)
    hadamard_rotate_kernel<E, InT, __half><<<blocks, threads, 0, st>>>((const InT*)x, sign, (__half*)out, items, K);
  else
    hadamard_rotate_kernel<E, InT, __nv_bfloat16>
        <<<blocks, threads, 0, st>>>((const InT*)x, sign, (__nv_bfloat16*)out, items, K);
  return check_launch("hadamard_rotate_kernel");
}

template <int E>
static int launch_hadamard_e(const void* x, int x_dtype, const float* sign, void* out, int out_dtype, int64_t items,
                             int K, cudaStream_t st) {
  if (x_dtype == GFX_DTYPE_F32) return launch_hadamard_in<E, float>(x, sign, out, out_dtype, items, K, st);
  if (x_dtype == GFX_DTYPE_F16) return launch_hadamard_in<E, __half>(x, sign, out, out_dtype, items, K, st);
  return launch_hadamard_in<E, __nv_bfloat16>(x, sign, out, out_dtype, items, K, st);
}

int launch_hadamard_rotate(const void* x, int x_dtype, const float* sign, void* out, int out_dtype, int64_t rows,
                           int K, int group, cudaStream_t stream) {
  const int64_t items = rows * (K / group);
  if (items == 0) return GFX_OK;
  if (group == 32) return launch_hadamard_e<1>(x, x_dtype, sign, out, out_dtype, items, K, stream);
  if (group == 64) return launch_hadamard_e<2>(x, x_dtype, sign, out, out_dtype, items, K, stream);
  return launch_hadamard_e<4>(x, x_dtype, sign, out, out_dtype, items, K, stream);
}

}  // namespace gfx
