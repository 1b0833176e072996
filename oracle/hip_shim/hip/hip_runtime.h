/* Stand-in for the HIP runtime header, so that the reference's own HIP
 * kernel sources (nodes/ComfyUI-Gfx906Int4/csrc/int4_gemm_scaled.hip,
 * int8_gemm.hip, int4_train_quant.hip) compile unmodified with nvcc as CUDA for the B200, as a
 * test oracle. It maps the few HIP names those files use onto CUDA and
 * restates the two gfx906 dot-product builtins they call from the ISA's
 * definition. TEST INFRASTRUCTURE ONLY: nothing of the product links it. */
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

typedef cudaStream_t hipStream_t;

/* The gfx906 occupancy hint has no CUDA meaning. */
#define amdgpu_waves_per_eu(n) unused

/* v_dot8_i32_i4: eight signed 4-bit products of the nibbles of a and b (nibble
 * i = bits 4i..4i+3, two's complement) summed onto c; clamp = false wraps. */
__device__ __forceinline__ int gfx906_ref_sdot8(int a, int b, int c, bool) {
  int s = c;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int x = (int)((unsigned)a << (28 - 4 * i)) >> 28;
    const int y = (int)((unsigned)b << (28 - 4 * i)) >> 28;
    s += x * y;
  }
  return s;
}

/* v_dot4_i32_i8: four signed 8-bit products of the bytes of a and b onto c
 * (the same operation as CUDA's __dp4a on signed operands). */
__device__ __forceinline__ int gfx906_ref_sdot4(int a, int b, int c, bool) { return __dp4a(a, b, c); }

#define __builtin_amdgcn_sdot8(a, b, c, clamp) gfx906_ref_sdot8((a), (b), (c), (clamp))
#define __builtin_amdgcn_sdot4(a, b, c, clamp) gfx906_ref_sdot4((a), (b), (c), (clamp))

/* clang's __builtin_bit_cast on CUDA's __half2, which nvcc rejects as not
 * trivially copyable: the same bit copy through memcpy. */
#include <cstring>
template <typename To, typename From>
__host__ __device__ __forceinline__ To gfx906_ref_bit_cast(const From& f) {
  static_assert(sizeof(To) == sizeof(From), "bit cast between types of different sizes");
  To t;
  memcpy(&t, &f, sizeof(To));
  return t;
}
#define __builtin_bit_cast(T, v) gfx906_ref_bit_cast<T>(v)
