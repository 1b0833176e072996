// C entry points onto the reference's own gfx906 kernels, compiled from their
// sources (int4_gemm_scaled.hip, int8_gemm.hip, int4_train_quant.hip) for sm_100a through the HIP
// stand-in headers in oracle/hip_shim/. TEST INFRASTRUCTURE ONLY: the GPU
// parity tests run these next to this repository's kernels and the numpy
// oracle to pin the reference's integer semantics (block-scaled int4 / int8
// GEMMs, the int4 / int8 quantizers), which its Python cannot express.
// Built by oracle/build_ref.py into oracle/_ref/libgfx906_ref.so.
#include <cstdint>

#include <cuda_runtime.h>

// The reference's dispatchers, as declared by its binding
// (nodes/ComfyUI-Gfx906Int4/csrc/binding.cpp:8-19).
void quantize_int4_dispatch(int dtype, const void* x, void* packed, float* scale, long total_blocks,
                            cudaStream_t stream);
void gemm_dispatch(int dtype, int qblock, const void* A, const float* As, const void* B, const float* Bs,
                   const void* bias, void* C, int M, int N, int n_blocks, int splits, float* workspace,
                   cudaStream_t stream);
void quantize_int8_dispatch(int dtype, const void* x, void* q, float* scale, long total_blocks, cudaStream_t stream);
void gemm_int8_dispatch(int dtype, int config, const void* A, const float* As, const void* B, const float* Bs,
                        const void* bias, void* C, int M, int N, int n_blocks, const int* geom, cudaStream_t stream);
// (nodes/ComfyUI-Gfx906Int4/csrc/train_kernels.hpp:10-13, int4_train_quant.hip:125-151)
void quant_rows_b16_dispatch(const void* x, long long row_stride, int R, int C, bool sr, uint32_t seed, void* packed,
                             float* scale, cudaStream_t stream);
void quant_cols_b16_dispatch(const void* x, long long row_stride, int R, int C, const float* signs, bool sr,
                             uint32_t seed, void* packed, float* scale, cudaStream_t stream);

extern "C" {

// Each returns the CUDA error code of the launch (0 = success).
int ref_quantize_int4(int dtype, const void* x, void* packed, float* scale, long total_blocks, void* stream) {
  quantize_int4_dispatch(dtype, x, packed, scale, total_blocks, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}

// n_blocks = K / 32 (16-byte loads per row); workspace: fp32 [splits, M, N] when splits > 1.
int ref_gemm_int4(int dtype, int qblock, const void* A, const float* As, const void* B, const float* Bs,
                  const void* bias, void* C, int M, int N, int n_blocks, int splits, float* workspace, void* stream) {
  gemm_dispatch(dtype, qblock, A, As, B, Bs, bias, C, M, N, n_blocks, splits, workspace, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}

int ref_quantize_int8(int dtype, const void* x, void* q, float* scale, long total_blocks, void* stream) {
  quantize_int8_dispatch(dtype, x, q, scale, total_blocks, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}

int ref_gemm_int8(int dtype, int config, const void* A, const float* As, const void* B, const float* Bs,
                  const void* bias, void* C, int M, int N, int n_blocks, void* stream) {
  gemm_int8_dispatch(dtype, config, A, As, B, Bs, bias, C, M, N, n_blocks, nullptr, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}

int ref_quant_rows_b16(const void* x, long long row_stride, int R, int C, int sr, unsigned seed, void* packed,
                       float* scale, void* stream) {
  quant_rows_b16_dispatch(x, row_stride, R, C, sr != 0, seed, packed, scale, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}

int ref_quant_cols_b16(const void* x, long long row_stride, int R, int C, const float* signs, int sr, unsigned seed,
                       void* packed, float* scale, void* stream) {
  quant_cols_b16_dispatch(x, row_stride, R, C, signs, sr != 0, seed, packed, scale, (cudaStream_t)stream);
  return (int)cudaGetLastError();
}

}  // extern "C"
