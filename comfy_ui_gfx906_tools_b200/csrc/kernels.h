// Internal launcher declarations shared by the C-ABI layer (capi.cu) and the
// kernel translation units. Not part of the public ABI (include/gfx906_b200.h).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gfx {

constexpr int kMaxSplits = 16;
// Split-K arrival counters occupy this many bytes at the start of the
// workspace (65536 tiles); the fp32 partials follow.
constexpr size_t kSplitKCounterBytes = 256 * 1024;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Where the small-M kernel stores y: `count` copies (one per target buffer, for
// example every rank's copy of a symmetric-memory buffer reached over NVLink),
// each [M, ldy] with this launch's N columns starting at column col0. A single
// local target with fence_sys 0 runs the plain kernel (y = ptr[0], [M, N]);
// anything else runs the all-gather variant, whose threads end with a
// system-scope fence so that a following cross-GPU barrier publishes the peer
// stores.
constexpr int kMaxOutTargets = 8;
struct OutTargets {
  void* ptr[kMaxOutTargets];
  int count;
  int ldy;
  int col0;
  int fence_sys;
};

// W4A16, small M (split-K / stream-K, mma.sync register dequant) -- w4a16_smallm.cu
int launch_w4a16_smallm(const void* x, const void* wq, const void* ws, int scale_dtype, const void* bias, void* y,
                        int out_dtype, int M, int N, int K, int splits, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream, int sms);
int launch_w4a16_smallm_targets(const void* x, const void* wq, const void* ws, int scale_dtype, const void* bias,
                                const OutTargets& out, int out_dtype, int M, int N, int K, int splits,
                                void* workspace, size_t workspace_bytes, cudaStream_t stream, int sms);
int launch_peer_barrier(int* const* flags, int n_ranks, int rank, cudaStream_t stream);

size_t smallm_workspace_bytes(int M, int N, int K, int splits, int sms);
int smallm_auto_splits(int M, int N, int K, int sms);
int smallm_device_status(int clear);

// W4A16 / W8A16, large M (tcgen05 + TMEM, persistent) -- w4a16_tc.cu
// qblock 32 (fp32 or fp16 scales [N, K/32]) or 16 (fp32 scales [N, K/16]; any M)
int launch_w4a16_tc(const void* x, const void* wq, const void* ws, int scale_dtype, const void* bias, void* y,
                    int out_dtype, int M, int N, int K, cudaStream_t stream, int sms, int qblock = 32);
// The same GEMM storing y into tg.count buffers (tg.ptr[q][m * tg.ldy + n], fp32 or fp16 32-groups, one CTA
// per tile) and fencing at system scope: the token-row split's GEMM and all-gather in one kernel.
int launch_w4a16_tc_targets(const void* x, const void* wq, const void* ws, int scale_dtype, const void* bias,
                            const OutTargets& tg, int out_dtype, int M, int N, int K, cudaStream_t stream, int sms);
bool w4a16_tc_supported(int M, int N, int K, int scale_dtype);
int tc_device_status(int clear);
int selftest_device_status(int clear);
int launch_w8a16_tc(const void* x, const void* wq, const void* ws, int per_channel, const void* bias, void* y,
                    int out_dtype, int M, int N, int K, cudaStream_t stream, int sms);

// integer-exact W4A4 (the reference's int4 x int4 block GEMM, bit for bit) -- w4a4_exact.cu
// a_q4 [M, K/2] / b_q4 [N, K/2] packed int4, fp32 scales [M|N, K/qblock]; workspace of
// w4a4_exact_workspace(M, N, K, qblock) bytes, 16-byte aligned. splits 0 = the reference's plan.
size_t w4a4_exact_workspace(int M, int N, int K, int qblock);
int w4a4_exact_splits(int M, int N, int K, int splits, int sms);
int launch_w4a4_exact(const void* a_q4, const float* a_scale, const void* b_q4, const float* b_scale, int qblock,
                      const void* bias, void* y, int out_dtype, int M, int N, int K, int splits, void* workspace,
                      cudaStream_t stream, int sms);
int w4a4x_device_status(int clear);

// block-16 int4 training quantizers -- train_quant.cu
// x fp16 [R, C] (rows row_stride elements apart). rows: C % 32 == 0 -> packed [R, C/2], scale [R, C/16].
// cols: R % 32 == 0 -> packed [C, R/2], scale [C, R/16] (transposed; signs: 16 floats or null).
int launch_quantize_int4_rows(const void* x, long long row_stride, int R, int C, int sr, uint32_t seed, void* packed,
                              float* scale, cudaStream_t stream);
int launch_quantize_int4_cols(const void* x, long long row_stride, int R, int C, const float* signs, int sr,
                              uint32_t seed, void* packed, float* scale, cudaStream_t stream);

// fused quantized attention, head dim 128 -- attention.cu
// qk_mode 0 fp16 / 1 int8 / 2 int4, pv_mode 0 fp16 / 1 u8; layouts as the C ABI's attention().
constexpr int kAttentionMaxTiles = 1024;  // key tiles a keep mask may cover (65536 keys)
int attention_rows_per_block(int qk_mode);
// tcgen05 kernel -- attention_tc.cu (launch_attention routes to it when selected)
bool attention_tc_selected(int qk_mode, bool keep);
int launch_attention_tc(int qk_mode, int pv_mode, const void* q, const float* q_scale, const void* k,
                        const float* k_scale, const void* vt, const float* v_scale, const uint8_t* keep, void* out,
                        int B, int H, int KVH, int Lq, int Lk, float skip_below, cudaStream_t stream);
int attn_tc_device_status(int clear);
int launch_attention(int qk_mode, int pv_mode, const void* q, const float* q_scale, const void* k,
                     const float* k_scale, const void* vt, const float* v_scale, const uint8_t* keep, void* out,
                     int B, int H, int KVH, int Lq, int Lk, float skip_below, cudaStream_t stream);

// loaders / helpers -- pack.cu
int launch_int4_dequant(const void* wq, const void* ws, int scale_dtype, void* out, int out_dtype, int N, int K,
                        cudaStream_t stream, int qblock = 32);
int launch_repack_q4_0(const void* raw, void* packed, float* scale, void* scale_f16, int N, int K,
                       cudaStream_t stream);
int launch_quantize_pack_int4(const void* x, int x_dtype, void* packed, float* scale, int64_t rows, int K,
                              int div_mode, cudaStream_t stream);
int launch_quantize_int8(const void* x, int x_dtype, void* q, float* scale, int64_t rows, int K,
                         cudaStream_t stream);
int launch_scales_to_f16(const float* s, void* s16, int64_t n, int* inexact, cudaStream_t stream);
int launch_repack_q8_0(const void* raw, void* q, float* scale, int N, int K, cudaStream_t stream);
int launch_hadamard_rotate(const void* x, int x_dtype, const float* sign, void* out, int out_dtype, int64_t rows,
                           int K, int group, cudaStream_t stream);

}  // namespace gfx
