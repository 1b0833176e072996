// W4A16 small-M GEMM (M <= 64 per token block): the HBM-bound weight stream.
//
// y[M, N] = x[M, K] @ (code[N, K] * scale[N, K/32])^T (+ bias), x bf16.
//
// Reference counterpart: int4_gemm_kernel + splitk_reduce_kernel
// (nodes/ComfyUI-Gfx906Int4/csrc/int4_gemm_scaled.hip:53-191) as called from
// gemm_int4 (binding.cpp:73-112) with split-K for narrow problems
// (auto_splits, binding.cpp:36-43). The weight layout and scale format are the
// reference's; the design is B200-first:
//
//  * one producer warp streams 128-byte (K = 256) nibble rows of a 64/128-row
//    weight slab with TMA (SWIZZLE_128B) into an S-stage shared-memory ring,
//    and the slab's group scales with cp.async (completion on the same
//    mbarrier), so a CTA keeps tens of KB of weights in flight;
//  * consumer warps read one 32-bit nibble word per row with ldmatrix (the
//    swizzle makes it conflict-free), turn nibbles into EXACT bf16 integer
//    codes with one LOP3 + one bf16x2 subtract per pair (magic-number
//    0x4300|u = 128+u), and run mma.sync m16n8k16 with the weights as the
//    16-row A operand and the tokens as the 8-column B operand (swap-AB);
//  * every MMA covers exactly one 32-element scale group, so the group's fp32
//    partial is scaled in registers (acc += partial * scale). Codes and x are
//    exact in bf16 and the tensor core accumulates in fp32, so the result is
//    the fp32 dequant-then-matmul up to fp32 rounding (the operand never
//    rounds to bf16);
//  * K is split across CTAs when the N tiles alone cannot fill the GPU; each
//    split writes fp32 partials to the workspace and the last CTA of a tile
//    (arrival counter, no spinning) sums them in split order -- deterministic
//    -- adds the bias, converts and stores, and re-arms the counter to zero.
//
// The K order inside one 16-wide MMA step is permuted (both operands the
// same way) so that each thread's four weights per register pair come out of
// one nibble word with no byte shuffles: k-slot (2t, 2t+1) of step s holds
// elements (8t + 2s, 8t + 2s + 4) and slot (2t + 8, 2t + 9) holds
// (8t + 2s + 1, 8t + 2s + 5) of the 32-group.
#include "common.cuh"
#include "kernels.h"

namespace gfx {

namespace splitk {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStageK = 256;               // K elements per pipeline stage
constexpr int kStageBytesPerRow = kStageK / 2;  // 128 nibble bytes = one SW128 row
constexpr int kGroupsPerStage = kStageK / 32;
constexpr int kStages = 6;

template <int MT, bool kF16Scale>
struct Layout {
  static constexpr int kRows = kConsumerWarps * MT * 16;        // weight rows per CTA
  static constexpr int kNibBytes = kRows * kStageBytesPerRow;    // per stage
  // scales: one padded row per weight row (pitch avoids bank conflicts)
  static constexpr int kScaleWordsPerRow = kF16Scale ? 4 : 8;    // 32-bit words of real data
  static constexpr int kScalePitch = kScaleWordsPerRow + 1;      // words
  static constexpr int kScaleBytes = kRows * kScalePitch * 4;
  static constexpr int kScaleBytesAligned = (kScaleBytes + 1023) / 1024 * 1024;
  static constexpr int kStageBytes = kNibBytes + kScaleBytesAligned;
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kStages * kStageBytes + 2 * kStages * 8 + 16;
};

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// Two nibbles (at bit 4i and 4i+16 of w after the shift) -> bf16x2 exact codes.
__device__ __forceinline__ uint32_t nib_pair_to_bf16x2(uint32_t w_shifted) {
  // (w & 0x000F000F) ^ 0x43084308 == 0x4300 | (nib ^ 8) in each half: 128 + u,
  // u = nib ^ 8 = code + 8 for a two's-complement nibble.
  const uint32_t magic = and_xor(w_shifted, 0x000F000Fu, 0x43084308u);
  __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&magic);
  const __nv_bfloat162 off = __floats2bfloat162_rn(136.0f, 136.0f);
  __nv_bfloat162 c = __hsub2(v, off);  // (128 + u) - 136 = code, exact
  return *reinterpret_cast<uint32_t*>(&c);
}

template <int MT, int NT, bool kF16Scale, typename OutT>
__global__ void __launch_bounds__(kThreads) w4a16_splitk_kernel(
    const __grid_constant__ CUtensorMap nib_map, const __nv_bfloat16* __restrict__ x, const void* __restrict__ wscale,
    const OutT* __restrict__ bias, OutT* __restrict__ y, float* __restrict__ partials, int* __restrict__ counters,
    int M, int N, int K, int splits) {
  using L = Layout<MT, kF16Scale>;
  constexpr int kTok = 8 * NT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * L::kStageBytes);
  uint64_t* empty = full + kStages;
  int* s_flag = reinterpret_cast<int*>(empty + kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * L::kRows;  // first weight row of this CTA
  const int split = blockIdx.y;
  const int tok0 = blockIdx.z * kTok;
  const int groups = K >> 5;
  const int k_stages = (K + kStageK - 1) / kStageK;
  const int st_begin = (int)(((long long)k_stages * split) / splits);
  const int st_end = (int)(((long long)k_stages * (split + 1)) / splits);
  const int n_iters = st_end - st_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1 + 32);              // producer lane 0 (expect_tx) + 32 cp.async arrivals
      mbar_init(&empty[s], kConsumerWarps);     // one arrival per consumer warp
    }
    fence_barrier_init();
  }
  __syncthreads();

  float acc[MT][NT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;

  bool ok = true;
  if (warp == kConsumerWarps) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) tma_prefetch_desc(&nib_map);
    for (int it = 0; it < n_iters; ++it) {
      const int stage = it % kStages;
      const uint32_t phase = (it / kStages) & 1;
      if (!mbar_wait(&empty[stage], phase ^ 1, kDevErrEmptyBarrierTimeout)) { ok = false; break; }
      uint8_t* st = smem + stage * L::kStageBytes;
      const int ks = st_begin + it;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[stage], L::kNibBytes);
        tma_load_2d(st, &nib_map, &full[stage], ks * kStageBytesPerRow, row0);
      }
      uint32_t* sc = reinterpret_cast<uint32_t*>(st + L::kNibBytes);
      constexpr int kWords = L::kRows * L::kScaleWordsPerRow;
      for (int i = lane; i < kWords; i += 32) {
        const int r = i / L::kScaleWordsPerRow;
        const int wd = i % L::kScaleWordsPerRow;
        const int n = row0 + r;
        const int g = ks * kGroupsPerStage + wd * (kF16Scale ? 2 : 1);
        const bool valid = (n < N) && (g < groups);
        const uint8_t* src = reinterpret_cast<const uint8_t*>(wscale);
        if (valid) src += ((size_t)n * groups + g) * (kF16Scale ? 2 : 4);
        cp_async_4(&sc[r * L::kScalePitch + wd], src, valid ? 4u : 0u);
      }
      cp_async_mbar_arrive_noinc(&full[stage]);
    }
  } else {
    // ------------------------------ consumers -----------------------------
    const int g_ = lane >> 2;  // row within an 8-row half / token within an n-tile
    const int t_ = lane & 3;   // thread-in-quad: nibble word / k quad
    // ldmatrix row address components (matrix i = lane/8, row j = lane%8)
    const int lm_i = lane >> 3, lm_j = lane & 7;
    for (int it = 0; it < n_iters; ++it) {
      const int stage = it % kStages;
      const uint32_t phase = (it / kStages) & 1;
      if (!mbar_wait(&full[stage], phase, kDevErrFullBarrierTimeout)) { ok = false; break; }
      const uint8_t* st = smem + stage * L::kStageBytes;
      const uint32_t nib_base = smem_u32(st);
      const uint32_t* sc = reinterpret_cast<const uint32_t*>(st + L::kNibBytes);
      const int kbase = (st_begin + it) * kStageK;
#pragma unroll
      for (int gp = 0; gp < kGroupsPerStage; gp += 2) {
        // B fragments (x) for groups gp and gp+1: 8 consecutive k per thread.
        uint32_t xf[2][NT][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int k = kbase + (gp + h) * 32 + 8 * t_;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int tok = tok0 + nt * 8 + g_;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (tok < M && k < K) v = ldg_nc_v4(x + (size_t)tok * K + k);
            xf[h][nt][0] = v.x; xf[h][nt][1] = v.y; xf[h][nt][2] = v.z; xf[h][nt][3] = v.w;
          }
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int rbase = warp * MT * 16 + mt * 16;
          const int lrow = rbase + lm_j + (lm_i & 1) * 8;
          const int lgrp = gp + (lm_i >> 1);
          uint32_t w[4];  // (row g, grp gp), (row g+8, gp), (row g, gp+1), (row g+8, gp+1)
          ldmatrix_x4(nib_base + lrow * kStageBytesPerRow + ((lgrp ^ (lrow & 7)) << 4), w[0], w[1], w[2], w[3]);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t wr = w[2 * h], wr8 = w[2 * h + 1];
            float s_r, s_r8;
            const int r_lo = rbase + g_, r_hi = rbase + g_ + 8;
            if (kF16Scale) {
              const __half* sch = reinterpret_cast<const __half*>(sc);
              s_r = __half2float(sch[r_lo * L::kScalePitch * 2 + gp + h]);
              s_r8 = __half2float(sch[r_hi * L::kScalePitch * 2 + gp + h]);
            } else {
              const float* scf = reinterpret_cast<const float*>(sc);
              s_r = scf[r_lo * L::kScalePitch + gp + h];
              s_r8 = scf[r_hi * L::kScalePitch + gp + h];
            }
            // step 0: slots (2t,2t+1) <- (n0,n4), (2t+8,2t+9) <- (n1,n5)
            // step 1: slots (2t,2t+1) <- (n2,n6), (2t+8,2t+9) <- (n3,n7)
            const uint32_t a00 = nib_pair_to_bf16x2(wr), a01 = nib_pair_to_bf16x2(wr8);
            const uint32_t a02 = nib_pair_to_bf16x2(wr >> 4), a03 = nib_pair_to_bf16x2(wr8 >> 4);
            const uint32_t a10 = nib_pair_to_bf16x2(wr >> 8), a11 = nib_pair_to_bf16x2(wr8 >> 8);
            const uint32_t a12 = nib_pair_to_bf16x2(wr >> 12), a13 = nib_pair_to_bf16x2(wr8 >> 12);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint32_t* xv = xf[h][nt];
              const float zero[4] = {0.f, 0.f, 0.f, 0.f};
              float p[4];
              mma_bf16_16816(p, a00, a01, a02, a03, prmt(xv[0], xv[2], 0x5410), prmt(xv[0], xv[2], 0x7632), zero);
              mma_bf16_16816(p, a10, a11, a12, a13, prmt(xv[1], xv[3], 0x5410), prmt(xv[1], xv[3], 0x7632), p);
              acc[mt][nt][0] = fmaf(p[0], s_r, acc[mt][nt][0]);
              acc[mt][nt][1] = fmaf(p[1], s_r, acc[mt][nt][1]);
              acc[mt][nt][2] = fmaf(p[2], s_r8, acc[mt][nt][2]);
              acc[mt][nt][3] = fmaf(p[3], s_r8, acc[mt][nt][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }
  }
  // A bounded wait that gave up makes the whole CTA leave (the status word
  // says which wait); every thread reaches this barrier either way.
  if (!__syncthreads_and(ok)) return;

  // --------------------------------- epilogue ---------------------------------
  if (splits == 1) {
    if (warp < kConsumerWarps) {
      const int g_ = lane >> 2, t_ = lane & 3;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int n = row0 + warp * MT * 16 + mt * 16 + g_ + half * 8;
          if (n >= N) continue;
          const float b = bias ? to_f32(bias[n]) : 0.0f;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int tok = tok0 + nt * 8 + 2 * t_ + c;
              if (tok < M) y[(size_t)tok * N + n] = from_f32<OutT>(acc[mt][nt][half * 2 + c] + b);
            }
          }
        }
      }
    }
    return;
  }

  const int m_pad = gridDim.z * kTok;
  if (warp < kConsumerWarps) {
    const int g_ = lane >> 2, t_ = lane & 3;
    float* part = partials + (size_t)split * m_pad * N;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int n = row0 + warp * MT * 16 + mt * 16 + g_ + half * 8;
        if (n >= N) continue;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int tok = tok0 + nt * 8 + 2 * t_ + c;
            part[(size_t)tok * N + n] = acc[mt][nt][half * 2 + c];
          }
        }
      }
    }
  }
  __threadfence();
  __syncthreads();
  int* counter = counters + blockIdx.z * gridDim.x + blockIdx.x;
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(counter, 1);
    *s_flag = (prev == splits - 1);
  }
  __syncthreads();
  if (!*s_flag) return;
  __threadfence();
  // last CTA of this tile: fixed-order reduction over splits
  const int rows = min(L::kRows, N - row0);
  for (int i = threadIdx.x; i < kTok * L::kRows; i += kThreads) {
    const int tl = i / L::kRows, r = i % L::kRows;
    const int tok = tok0 + tl;
    if (r >= rows || tok >= M) continue;
    const int n = row0 + r;
    float v = 0.0f;
    for (int s = 0; s < splits; ++s) v += __ldcg(partials + ((size_t)s * m_pad + tok) * N + n);
    if (bias) v += to_f32(bias[n]);
    y[(size_t)tok * N + n] = from_f32<OutT>(v);
  }
  if (threadIdx.x == 0) *counter = 0;  // re-arm for the next call
}

}  // namespace splitk

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
GFX_DEFINE_STATUS_READER(splitk_device_status)

struct SplitKPlan {
  int mt, nt, rows, tok, row_blocks, tok_blocks, splits;
};

static SplitKPlan splitk_plan(int M, int N, int K, int splits_req, int sms) {
  SplitKPlan p{};
  if (M <= 8) { p.mt = 2; p.nt = 1; }
  else if (M <= 16) { p.mt = 2; p.nt = 2; }
  else if (M <= 32) { p.mt = 2; p.nt = 4; }
  else { p.mt = 1; p.nt = 8; }
  p.rows = splitk::kConsumerWarps * p.mt * 16;
  p.tok = 8 * p.nt;
  p.row_blocks = (N + p.rows - 1) / p.rows;
  p.tok_blocks = (M + p.tok - 1) / p.tok;
  const int k_stages = (K + splitk::kStageK - 1) / splitk::kStageK;
  int s = splits_req;
  if (s <= 0) {
    // Enough CTAs for two resident per SM; each split keeps >= 1 stage.
    const int tiles = p.row_blocks * p.tok_blocks;
    const int target = 2 * sms;
    s = (target + tiles - 1) / tiles;
  }
  p.splits = s < 1 ? 1 : (s > k_stages ? k_stages : s);
  if (p.splits > kMaxSplits) p.splits = kMaxSplits;
  return p;
}

size_t splitk_workspace_bytes(int M, int N, int K, int splits_req, int sms) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  SplitKPlan p = splitk_plan(M, N, K, splits_req, sms);
  if (p.splits <= 1) return 0;
  const size_t part = (size_t)p.splits * p.tok_blocks * p.tok * N * sizeof(float);
  return kSplitKCounterBytes + align_up(part, 256);
}

int splitk_auto_splits(int M, int N, int K, int sms) { return splitk_plan(M, N, K, 0, sms).splits; }

template <int MT, int NT, bool F16S, typename OutT>
static int launch_splitk_t(const SplitKPlan& p, const CUtensorMap& map, const void* x, const void* ws,
                           const void* bias, void* y, float* part, int* cnt, int M, int N, int K, cudaStream_t st) {
  using L = splitk::Layout<MT, F16S>;
  auto kern = splitk::w4a16_splitk_kernel<MT, NT, F16S, OutT>;
  static bool attr_set[64] = {false};  // per device
  int dev = current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    attr_set[dev] = true;
  }
  dim3 grid(p.row_blocks, p.splits, p.tok_blocks);
  kern<<<grid, splitk::kThreads, L::kSmemBytes, st>>>(map, (const __nv_bfloat16*)x, ws, (const OutT*)bias, (OutT*)y,
                                                     part, cnt, M, N, K, p.splits);
  return check_launch("w4a16_splitk_kernel");
}

template <int MT, int NT, bool F16S>
static int launch_splitk_out(int out_dtype, const SplitKPlan& p, const CUtensorMap& map, const void* x,
                             const void* ws, const void* bias, void* y, float* part, int* cnt, int M, int N, int K,
                             cudaStream_t st) {
  if (out_dtype == GFX_DTYPE_F32)
    return launch_splitk_t<MT, NT, F16S, float>(p, map, x, ws, bias, y, part, cnt, M, N, K, st);
  if (out_dtype == GFX_DTYPE_F16)
    return launch_splitk_t<MT, NT, F16S, __half>(p, map, x, ws, bias, y, part, cnt, M, N, K, st);
  return launch_splitk_t<MT, NT, F16S, __nv_bfloat16>(p, map, x, ws, bias, y, part, cnt, M, N, K, st);
}

template <bool F16S>
static int launch_splitk_shape(int out_dtype, const SplitKPlan& p, const CUtensorMap& map, const void* x,
                               const void* ws, const void* bias, void* y, float* part, int* cnt, int M, int N, int K,
                               cudaStream_t st) {
  if (p.nt == 1) return launch_splitk_out<2, 1, F16S>(out_dtype, p, map, x, ws, bias, y, part, cnt, M, N, K, st);
  if (p.nt == 2) return launch_splitk_out<2, 2, F16S>(out_dtype, p, map, x, ws, bias, y, part, cnt, M, N, K, st);
  if (p.nt == 4) return launch_splitk_out<2, 4, F16S>(out_dtype, p, map, x, ws, bias, y, part, cnt, M, N, K, st);
  return launch_splitk_out<1, 8, F16S>(out_dtype, p, map, x, ws, bias, y, part, cnt, M, N, K, st);
}

int launch_w4a16_splitk(const void* x, const void* wq, const void* ws, int scale_dtype, const void* bias, void* y,
                        int out_dtype, int M, int N, int K, int splits_req, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream, int sms) {
  SplitKPlan p = splitk_plan(M, N, K, splits_req, sms);
  float* part = nullptr;
  int* cnt = nullptr;
  if (p.splits > 1) {
    const size_t need = splitk_workspace_bytes(M, N, K, splits_req, sms);
    if (workspace == nullptr || workspace_bytes < need)
      return set_error(GFX_ERR_WORKSPACE, "w4a16_gemm: split-K workspace of %zu bytes required, got %zu (ptr %p)",
                       need, workspace_bytes, workspace);
    if ((size_t)p.tok_blocks * p.row_blocks * sizeof(int) > kSplitKCounterBytes)
      return set_error(GFX_ERR_UNSUPPORTED, "w4a16_gemm: %d x %d split-K tiles exceed the %zu-byte counter region",
                       p.tok_blocks, p.row_blocks, kSplitKCounterBytes);
    // Counters live at a fixed offset (the first kSplitKCounterBytes) so that
    // calls of any shape sharing one workspace always find them re-armed to
    // zero; the fp32 partials follow and need no initial value.
    cnt = reinterpret_cast<int*>(workspace);
    part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + kSplitKCounterBytes);
  }
  CUtensorMap map;
  int rc = make_tmap_2d(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                        splitk::kStageBytesPerRow, (uint32_t)p.rows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (scale_dtype == GFX_SCALE_F16)
    return launch_splitk_shape<true>(out_dtype, p, map, x, ws, bias, y, part, cnt, M, N, K, stream);
  return launch_splitk_shape<false>(out_dtype, p, map, x, ws, bias, y, part, cnt, M, N, K, stream);
}

}  // namespace gfx
