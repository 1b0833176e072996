/*
 * gfx906_b200.h -- C ABI of the B200 (sm_100a) int4 / int8 weight-only linear
 * library: the drop-in boundary under the reference's Python operator layer.
 *
 * Reference: luna-niemitalo/comfy_ui_gfx906_tools, nodes/ComfyUI-Gfx906Int4.
 * Each entry point names the reference interface it replaces (path:line).
 *
 * Conventions
 *  - All pointers are device pointers unless stated; the caller owns every
 *    buffer (inputs, outputs, workspaces). The library never allocates or
 *    frees caller memory.
 *  - Work is enqueued on `stream` (a cudaStream_t) of the current device; the
 *    caller makes the device that owns the buffers current first (the
 *    reference binds a CUDAGuard for the same reason, binding.cpp:56-59).
 *  - Return 0 on success, otherwise a GFX_ERR_* code; gfx_last_error() then
 *    holds a message (thread-local) with expected vs actual values. Nothing
 *    aborts the process.
 *  - dtype codes follow the reference binding (binding.cpp:45-50):
 *    0 = float32, 1 = float16, 2 = bfloat16.
 *  - Packed int4 weight layout (ops.py:108-126, int4_gemm_scaled.hip:6-10):
 *    int8 [N, K/2], two's-complement nibbles, element e of each 32-chunk is
 *    nibble e%8 of little-endian 32-bit word e/8; scales [N, K/32].
 */
#ifndef GFX906_B200_H
#define GFX906_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* gfx_stream_t; /* == cudaStream_t */

#define GFX_OK 0
#define GFX_ERR_INVALID 1     /* bad argument (shape, dtype, null pointer)          */
#define GFX_ERR_UNSUPPORTED 2 /* valid for the reference, not supported here (yet)  */
#define GFX_ERR_WORKSPACE 3   /* workspace missing or smaller than required         */
#define GFX_ERR_CUDA 4        /* CUDA runtime / launch error                        */
#define GFX_ERR_DEVICE 5      /* a bounded device-side wait gave up (see status)    */

#define GFX_DTYPE_F32 0
#define GFX_DTYPE_F16 1
#define GFX_DTYPE_BF16 2

#define GFX_SCALE_F32 0 /* scales float32 [N, K/32] (the reference's format)      */
#define GFX_SCALE_F16 1 /* scales float16 [N, K/32] (only when exactly fp16)      */

/* Message for the last failing call on this host thread ("" if none). */
const char* gfx_last_error(void);

/* Library version: major * 10000 + minor * 100 + patch. */
int gfx_version(void);

/* Device-side status word of the current device: 0 = healthy, else the code
 * of the first bounded wait that gave up. Synchronises the device. clear != 0
 * resets the word to 0. */
int gfx_device_status(int clear);

/* Output-channel split of one W4A16 GEMM with the all-gather fused into its
 * epilogue (no reference counterpart: the reference splits tokens or the batch
 * across two GPUs, row_split.py:122-241; this is the B200 form of an
 * output-channel split for M <= 64). This rank computes y[:, rank*N_local :
 * (rank+1)*N_local] from its shard w_q4 [N_local, K/2] / w_scale and bias
 * [N_local] (or NULL), and stores it into EVERY rank's y buffer
 * (y_ranks[q]: rank q's [M, n_ranks*N_local] buffer, mapped on this device,
 * e.g. symmetric memory reached over NVLink) with plain stores and a
 * system-scope fence. Follow it with gfx_peer_barrier before reading y; a
 * buffer must not be rewritten while a peer may still read it (alternate two
 * buffers). 1 <= n_ranks <= 8, M <= 64; other arguments as w4a16_gemm. */
int w4a16_gemm_allgather(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype,
                         const void* bias, void* const* y_ranks, int n_ranks, int rank, int out_dtype, int M,
                         int N_local, int K, int splits, void* workspace, size_t workspace_bytes,
                         gfx_stream_t stream);

/* Token-row split of one W4A16 GEMM with the all-gather fused into its
 * epilogue (no reference counterpart: the reference splits a DiT's image rows
 * across two GPUs and exchanges K/V, row_split.py:122-241; this is the B200
 * form of the token-row split of one linear, the survey's first multi-GPU
 * case). This rank computes rows [row0, row0 + M) of y from its activations
 * x [M, K] and stores them into EVERY rank's y buffer (y_ranks[q]: rank q's
 * [M_total, N] buffer, mapped on this device, e.g. symmetric memory reached
 * over NVLink) with plain stores and a system-scope fence; M > 64 runs the
 * tcgen05 kernel (fp32 or fp16 32-group scales), M <= 64 the small-M kernel.
 * Follow it with gfx_peer_barrier before reading y. Other arguments as
 * w4a16_gemm. */
int w4a16_gemm_rows_allgather(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype,
                              const void* bias, void* const* y_ranks, int n_ranks, int row0, int out_dtype, int M,
                              int N, int K, int splits, void* workspace, size_t workspace_bytes, gfx_stream_t stream);

/* Cross-GPU barrier over NVLink-mapped flags (no reference counterpart):
 * flags_ranks[q] is rank q's int[n_ranks + 1] (zero before the first call).
 * The epoch lives on the device: slot n_ranks of this rank's own array counts
 * the barriers it passed, so the call takes no per-call argument and can be
 * captured in a CUDA graph. With e = that count + 1, this rank stores e into
 * flags_ranks[q][rank] for every q (release, system scope), waits until
 * flags_ranks[rank][q] >= e for every q (acquire, system scope) and stores e
 * back into its counter. A wait that exceeds 2 s records status 7
 * (gfx_device_status) and returns. */
int gfx_peer_barrier(int* const* flags_ranks, int n_ranks, int rank, gfx_stream_t stream);

/* Failure-detection check (no reference counterpart; used by the tests): one
 * CTA waits on an mbarrier nothing arrives on, gives up after timeout_us
 * (0 < timeout_us <= 1e6) and records status code 6 in the device status
 * word, exactly as a stuck GEMM pipeline would; the context stays usable.
 * Returns 0 once launched; read the outcome with gfx_device_status. */
int gfx_selftest_wait_timeout(int timeout_us, void* stream);

/*
 * W4A16 GEMM:  y[M, N] = x[M, K] @ dequant(w_q4, w_scale)^T (+ bias)
 *
 * Replaces the int4 GEMM under Gfx906Int4Ops.Linear.forward -> int4_linear
 * (ops.py:167-183 -> binding.cpp:73-112 gemm_int4 -> int4_gemm_scaled.hip
 * int4_gemm_kernel), keeping the weight buffers, layout and scale format; the
 * activation stays bf16 (weight-only), the accumulation is fp32.
 *   x        bf16 [M, K] row-major (x_dtype must be GFX_DTYPE_BF16)
 *   w_q4     int8 [N, K/2] packed as above;  K % 32 == 0
 *   w_scale  [N, K/32], GFX_SCALE_F32 or GFX_SCALE_F16
 *   bias     [N] in out_dtype, or NULL (binding.cpp:97: bias dtype == out dtype)
 *   y        [M, N] in out_dtype
 *   splits   split-K count, 0 = automatic (gemm_int4's `splits`, binding.cpp:101-105)
 *   workspace / workspace_bytes: scratch for split-K partials, at least
 *            w4a16_workspace_bytes(M, N, K, splits); must hold zeros before
 *            its first use; every call leaves its counters at zero again.
 * M == 0 is a no-op (binding.cpp:93).
 */
int w4a16_gemm(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype,
               const void* bias, void* y, int out_dtype, int M, int N, int K, int splits, void* workspace,
               size_t workspace_bytes, gfx_stream_t stream);

/*
 * W4A16 GEMM with a choice of scale block (gemm_int4's `qblock`,
 * binding.cpp:73-112 / int4_gemm_scaled.hip:153-160, SUB = 2 for qblock 16).
 * qblock 32: exactly w4a16_gemm. qblock 16: w_scale is float32 [N, K/16] (one
 * scale per 16 elements, the reference's training format, train_linear.py:
 * 45-67), any M, no workspace; each weight becomes bf16(code * scale) of its
 * own 16-group. Other arguments as w4a16_gemm.
 */
int w4a16_gemm_qblock(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype, int qblock,
                      const void* bias, void* y, int out_dtype, int M, int N, int K, int splits, void* workspace,
                      size_t workspace_bytes, gfx_stream_t stream);

/*
 * Integer-exact W4A4 GEMM: replaces gemm_int4 (binding.cpp:73-112) with the
 * reference's numerics bit for bit -- int4_gemm_kernel's per-block chain
 * acc = fmaf((float)dot, a_scale * b_scale, acc) over 32-element blocks (two
 * 16-element halves, low then high, for qblock 16; int4_gemm_scaled.hip:
 * 147-160), each split-K slice's chain from 0 and the slices summed in order
 * (splitk_reduce_kernel, :182-191), then + bias, one conversion to out_dtype.
 * a_q4 [M, K/2] / b_q4 [N, K/2]: packed int4 (quantize_int4 / quantize_pack_int4
 * layout), 16-byte aligned; a_scale [M, K/qblock] / b_scale [N, K/qblock]
 * float32 (b_scale 16-byte aligned); bias [N] in out_dtype or NULL; y [M, N]
 * out_dtype.
 * splits: 0 = the reference's auto_splits (binding.cpp:36-43) evaluated with
 * this device's SM count, or 1..8. The split count changes the rounding, as in
 * the reference; w4a4_gemm_exact_splits reports the count a call would use.
 * workspace: >= w4a4_gemm_exact_workspace_bytes(M, N, K, qblock) bytes,
 * 16-byte aligned (e5m2 copies of A, transposed A scales and, when K/qblock
 * is not a multiple of 4, a padded copy of B_scale; rewritten every call).
 * Errors as gemm_int4's TORCH_CHECKs (K % 32, qblock, splits, dtypes).
 */
size_t w4a4_gemm_exact_workspace_bytes(int M, int N, int K, int qblock);
int w4a4_gemm_exact_splits(int M, int N, int K, int splits);
int w4a4_gemm_exact(const void* a_q4, const float* a_scale, const void* b_q4, const float* b_scale, int qblock,
                    const void* bias, void* y, int out_dtype, int M, int N, int K, int splits, void* workspace,
                    size_t workspace_bytes, gfx_stream_t stream);

/*
 * Block-16 int4 quantizers of the int4 training backward (quantize_int4_rows /
 * quantize_int4_cols, binding.cpp:317-356; int4_train_quant.hip:35-123), in
 * the layout w4a4_gemm_exact(qblock = 16) reads. x: fp16 [R, C], rows
 * row_stride elements apart (a multiple of 8, 16-byte aligned rows).
 * scale = max(amax, 1e-8) * (1/7), code = clamp(round(v / scale), -8, 7) with
 * round to nearest even (sr = 0) or floor(v / scale + u) (sr != 0), u a
 * counter-based hash of (seed, element index) in [0, 1) with 24 bits.
 * rows: blocks of 16 along each row, C % 32 == 0 -> packed int8 [R, C/2],
 *       scale float32 [R, C/16].
 * cols: blocks of 16 along each column, transposed: R % 32 == 0 -> packed
 *       int8 [C, R/2], scale float32 [C, R/16]; with signs (16 floats, else
 *       NULL) each 16-row group is first rotated by (H16 / 4) diag(signs).
 */
int quantize_int4_rows(const void* x, int64_t row_stride, int R, int C, int sr, uint32_t seed, void* packed,
                       float* scale, gfx_stream_t stream);
int quantize_int4_cols(const void* x, int64_t row_stride, int R, int C, const float* signs, int sr, uint32_t seed,
                       void* packed, float* scale, gfx_stream_t stream);

/*
 * Fused quantized attention, head dim 128 (attention(), binding.cpp:114-170;
 * attention_kernel, attention.hip:83-357). Inputs as the reference's prepare
 * step writes them (attention.py:50-81): scores in log2 units (softmax scale
 * * log2(e) folded into Q, or into q_scale for the int modes).
 *   qk_mode 0 fp16: Q [B, H, Lq, 128] / K [B, KVH, Lk, 128] fp16, no scales.
 *   qk_mode 1 int8: Q, K int8 per token, q_scale [B, H, Lq], k_scale [B, KVH, Lk].
 *   qk_mode 2 int4: Q, K packed int4 [.., 64 bytes] (element 2i in the low
 *                   nibble of byte i), scales as int8.
 *   pv_mode 0 fp16: Vt [B, KVH, ceil(Lk/64), 128, 64] fp16 (64-key tiles,
 *                   channel-major), no v_scale.
 *   pv_mode 1 u8:   Vt as above in uint8 (value + 128), v_scale
 *                   [B, KVH, ceil(Lk/64), 128] fp32.
 * keep: NULL or uint8 [B, H, ceil(Lq / attention_block_rows(qk_mode)),
 * ceil(Lk/64)], nonzero = visit that key tile (at most attention_max_tiles()
 * tiles; every query block must keep one). skip_below: a key tile whose
 * largest attention weight is below this fraction of the running row maximum
 * for all 16 rows of a warp skips its P.V (0 = never). H % KVH == 0 (GQA:
 * head h reads KV head h / (H / KVH)). out: fp16 [B, Lq, H * 128].
 * Q, K, Vt 16-byte aligned.
 */
int attention(int qk_mode, int pv_mode, const void* q, const float* q_scale, const void* k, const float* k_scale,
              const void* vt, const float* v_scale, const uint8_t* keep, void* out, int B, int H, int KVH, int Lq,
              int Lk, float skip_below, gfx_stream_t stream);
/* Query rows per block of the keep mask (64 for fp16 Q.K, 128 for the int
 * modes; attention_block_rows, binding.cpp:17), or -1 for a bad mode. */
int attention_block_rows(int qk_mode);
/* Key tiles a keep mask may cover (attention_max_tiles, binding.cpp:21). */
int attention_max_tiles(void);

/*
 * W4A16 GEMM that allocates nothing (no counterpart in the reference).
 * For callers that cannot allocate device memory -- a plugin host that passes
 * only its input/output device pointers and owns the memory budget, or code
 * that must not issue a synchronising cudaMalloc -- yet need the small-M path,
 * whose w4a16_gemm call requires a caller-provided scratch workspace.
 * Same arguments and result as w4a16_gemm without the workspace; M <= 64 only
 * (M > 64: call w4a16_gemm with a NULL workspace, that kernel needs no
 * scratch). The scratch is a fixed 8 MiB array in the library's device memory,
 * held by every GPU that loads the library until the process exits; shapes
 * needing more are rejected with GFX_ERR_UNSUPPORTED. The first call on a
 * device looks the array up and clears it (make it before any stream capture).
 * All calls share the array: calls that overlap on the GPU race, so serialise
 * them.
 */
int w4a16_gemm_noalloc(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype,
                       const void* bias, void* y, int out_dtype, int M, int N, int K, int splits,
                       gfx_stream_t stream);

/* Scratch bytes w4a16_gemm needs for (M, N, K, splits) on the current device. */
size_t w4a16_workspace_bytes(int M, int N, int K, int splits);

/* Split-K count w4a16_gemm picks when splits == 0 (gemm_int4_auto_splits,
 * binding.cpp:358-361 / auto_splits binding.cpp:36-43). */
int w4a16_auto_splits(int M, int N, int K);

/*
 * W8A16 GEMM:  y = x @ dequant_int8(w_q8, w_scale)^T (+ bias)
 * The int8 sibling of w4a16_gemm (gemm_int8, binding.cpp:190-217; weights
 * from quantize_int8, binding.cpp:174-186), on the tcgen05 kernel for every M.
 *   w_q8     int8 [N, K];  K % 32 == 0
 *   w_scale  float32 [N, K/32] (block scales, the reference layout) when
 *            scale_per_channel == 0: each weight becomes bf16(q * scale);
 *            float16 [N] per-output-channel scale when scale_per_channel == 1:
 *            the exact codes are multiplied and the fp32 result is scaled.
 *   workspace is not used (pass NULL, 0).
 */
int w8a16_gemm(const void* x, int x_dtype, const void* w_q8, const void* w_scale, int scale_per_channel,
               const void* bias, void* y, int out_dtype, int M, int N, int K, int splits, void* workspace,
               size_t workspace_bytes, gfx_stream_t stream);

size_t w8a16_workspace_bytes(int M, int N, int K, int splits);

/*
 * Block-32 int4 quantize + pack (ops.quantize_pack_int4, ops.py:108-126; the
 * activation quantizer quantize_int4, binding.cpp:53-68 /
 * int4_gemm_scaled.hip:197-220, is div_mode 1).
 *   x       [rows, K] in x_dtype; K % 32 == 0
 *   packed  int8 [rows, K/2];  scale float32 [rows, K/32]
 *   div_mode 0: scale = amax / 7 as an IEEE division (torch on CPU);
 *            1: scale = amax * (1/7) (torch on CUDA, and the HIP kernel).
 */
int quantize_pack_int4(const void* x, int x_dtype, void* packed, float* scale, int64_t rows, int K, int div_mode,
                       gfx_stream_t stream);

/* Block-32 int8 quantize (quantize_int8, binding.cpp:174-186 /
 * int8_gemm.hip:217-246): q int8 [rows, K], scale float32 [rows, K/32]. */
int quantize_int8(const void* x, int x_dtype, void* q, float* scale, int64_t rows, int K, gfx_stream_t stream);

/* Lossless ggml Q4_0 -> native repack (ops.repack_q4_0_native, ops.py:129-164).
 *   raw     N*(K/32)*18 bytes of Q4_0 blocks (2-byte fp16 d + 16 nibble bytes)
 *   packed  int8 [N, K/2];  scale float32 [N, K/32];  scale_f16 float16 [N, K/32]
 *           (either scale pointer may be NULL). */
int repack_q4_0(const void* raw, void* packed, float* scale, void* scale_f16, int N, int K, gfx_stream_t stream);

/* Lossless ggml Q8_0 -> int8 weight repack (no reference kernel: the
 * reference dequantizes Q8_0 GGUF tensors and re-quantizes them to int4,
 * nodes.py:294-301; its GGUF report names a lossless Q8_0 repack onto the int8
 * path as the follow-up). raw: N*(K/32) blocks of 34 bytes (fp16 d, 32 int8
 * codes), 2-byte aligned; q int8 [N, K] (16-byte aligned) and scale float32
 * [N, K/32] = d: exactly the block-scale int8 format w8a16_gemm reads. */
int repack_q8_0(const void* raw, void* q, float* scale, int N, int K, gfx_stream_t stream);

/* Dequantize packed int4 weights: out[N, K] = code * scale, computed as one
 * fp32 multiply and, for out_dtype bf16/f16, rounded to nearest-even once
 * (int4_train_test.py:46-52; nodes.py:51-52). The bf16 output is the exact
 * operand the W4A16 tensor-core kernel multiplies with. */
int int4_dequant(const void* w_q4, const void* w_scale, int scale_dtype, void* out, int out_dtype, int N, int K,
                 gfx_stream_t stream);

/* int4_dequant with a choice of scale block: qblock 32 (scales [N, K/32]) or
 * 16 (scales [N, K/16], the reference's qblock=16 format,
 * int4_gemm_scaled.hip:153-160); same arithmetic. */
int int4_dequant_qblock(const void* w_q4, const void* w_scale, int scale_dtype, int qblock, void* out, int out_dtype,
                        int N, int K, gfx_stream_t stream);

/* Convert float32 scales to float16 and count the ones that did not survive
 * the round trip exactly (*inexact, a device int, is overwritten). */
int scales_to_f16(const float* scale, void* scale_f16, int64_t n, int* inexact, gfx_stream_t stream);

/* Block-diagonal randomized Hadamard rotation of activations (the forward
 * half of rotation_group != 0 in int4_linear, ops.py:85-105,176-179):
 *   out[r, g*group + i] = sum_j H[i, j] * sign[j] * x[r, g*group + j] / sqrt(group)
 * with H the Sylvester Hadamard matrix of order group (32, 64 or 128) and
 * sign[group] the float +-1 vector of get_group_rotation. x, out [rows, K]
 * (K % group == 0), dtype codes 0/1/2; out may not alias x. Computed as a
 * fast Walsh-Hadamard transform in fp32, equal to the reference's fp32
 * matmul up to fp32 rounding. */
int hadamard_rotate(const void* x, int x_dtype, const float* sign, void* out, int out_dtype, int64_t rows, int K,
                    int group, gfx_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GFX906_B200_H */
