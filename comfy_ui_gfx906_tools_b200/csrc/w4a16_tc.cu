// Weight-only GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), large M.
//
// int4: y[M, N] = x[M, K] @ bf16(code[N, K] * scale[N, K/32])^T (+ bias)
// int8: y[M, N] = x @ bf16(q[N, K] * scale[N, K/32])^T, or, with one scale per
//       output channel, (x @ q^T) * scale[N] (+ bias)
//
// Reference counterparts: int4_gemm_kernel (nodes/ComfyUI-Gfx906Int4/csrc/
// int4_gemm_scaled.hip:53-180) behind gemm_int4 (binding.cpp:73-112), and
// int8_gemm_kernel (csrc/int8_gemm.hip:66-213) behind gemm_int8
// (binding.cpp:190-217). Same weight buffers; int4 weights are dequantized to
// the bf16 values the reference's W4A16 emulation multiplies with
// (nodes.py:43-52), bit for bit, and multiplied on the tensor cores with fp32
// accumulation.
//
// Design (one persistent CTA per SM, 14 warps, swap-AB):
//   D[n, m] (TMEM, 128 lanes = weight rows, 256 fp32 columns = tokens)
//     = W_tile[128 x K] (A, dequantized bf16 in SMEM, K-major SWIZZLE_128B)
//     * X_tile[256 x K]^T (B, bf16 in SMEM via TMA, K-major SWIZZLE_128B)
//   Putting the 128-row weight tile on the MMA's M side lets one dequantized
//   weight element feed 256 tokens, which halves the dequant work per FLOP
//   compared with a 128-token tile.
//   warp 4      TMA producer: x tile (TMA, 32 KB), packed weight tile (TMA:
//               int4 4 KB SWIZZLE_32B, int8 8 KB SWIZZLE_64B) per 64-wide K
//               stage, and the group scales of 4 stages at a time (one TMA
//               box of 8 groups x 128 rows into one of two chunk buffers;
//               per-stage cp.async when the scale rows are not 16-byte
//               aligned). Gathering a row's 4 scale bytes per stage with
//               cp.async measured as half of all shared-memory wavefronts,
//               most of them bank conflicts.
//   warps 6-13  dequant: each thread turns 32 weights of one row into bf16 in
//               the UMMA canonical SW128 layout, then a proxy fence and an
//               mbarrier arrival hand the stage to the MMA.
//   warp 5      TMEM allocation + one elected thread issuing tcgen05.mma
//               (M=128, N=256, K=16; 4 per stage) and tcgen05.commit.
//   warps 0-3   epilogue: tcgen05.ld of the accumulator (warp w owns TMEM
//               lanes 32w..32w+31), (* channel scale) + bias, convert, store.
//               The accumulator is double-buffered (2 x 256 columns = all
//               512), so the epilogue of tile i overlaps the main loop of
//               tile i+1.
// CTA-pair variant (C = 2, opt-in): a cluster of two CTAs on one TPC
// computes a 256-row x 256-token tile with tcgen05.mma.cta_group::2 (M=256):
// each CTA dequantizes its own 128 weight rows and TMA-loads HALF of the
// x tile (128 tokens); the MMA, issued by CTA 0, reads A and B from both
// CTAs' shared memory and writes each CTA's 128 x 256 accumulator into its own
// TMEM. Per SM this halves the x bytes per stage (16 KB instead of 32 KB), so
// six stages fit instead of four. CTA 1's dequant and epilogue warps arrive on
// CTA 0's barriers (mbarrier.arrive on a shared::cluster address); CTA 0's MMA thread
// signals both CTAs' barriers with one tcgen05.commit per CTA.
// Exact int4 dequant: with fp16-valued scales the product code*scale is exact
// in fp32 and one rounding to bf16 equals the reference's two roundings; it is
// computed as fma.rn.bf16x2(code, s_hi, code * s_lo) with s = s_hi + s_lo split
// into two bf16 parts (code * s_lo is exact in bf16), 2.5 ops per element.
// General fp32 scales use an fp32 multiply then one cvt.rn to bf16; with
// 16-element groups (the reference's qblock=16) each half of a 32-element
// item takes its own scale. int8 codes are exact in bf16; a per-channel scale
// is applied to the fp32 accumulator.
// Every mbarrier wait is bounded (common.cuh).
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace gfx {

GFX_DEFINE_STATUS_READER(tc_device_status)

namespace tc {

constexpr int kTileN = 128;       // weight rows per tile (MMA M)
constexpr int kTileM = 256;       // tokens per tile (MMA N)
constexpr int kStageK = 64;       // K per pipeline stage (one 128-byte swizzle row of bf16)
constexpr int kUmmaK = 16;
#ifndef GFX_TC_DEQ_WARPS
#define GFX_TC_DEQ_WARPS 8
#endif
constexpr int kEpiWarps = 4, kProducerWarp = 4, kMmaWarp = 5, kDequantWarp0 = 6, kDequantWarps = GFX_TC_DEQ_WARPS;
constexpr int kThreads = (kDequantWarp0 + kDequantWarps) * 32;
static_assert(kDequantWarps == 8 || kDequantWarps == 16, "dequant warps: 8 or 16");
#ifndef GFX_TC_DEQ_GROUPS
#define GFX_TC_DEQ_GROUPS 2
#endif
// Dequant warp groups working on different stages at once (1, 2, 4 or 8).
constexpr int kDeqGroups = GFX_TC_DEQ_GROUPS;
static_assert(kDeqGroups == 1 || kDeqGroups == 2 || kDeqGroups == 4 || kDeqGroups == 8, "bad dequant grouping");
constexpr int kAccCols = kTileM;  // fp32 columns per accumulator
constexpr int kTmemCols = 2 * kAccCols;
constexpr int kWBytes = kTileN * kStageK * 2;  // 16 KB
constexpr int kBarrierBytes = 320;
constexpr int kSmemLimit = 232448;  // 227 KB per CTA

// Weight formats.
enum Fmt : int {
  kInt4GroupF32 = 0,  // int4 nibbles, fp32 scale per 32-group (the reference's format)
  kInt4GroupF16 = 1,  // int4 nibbles, fp16-valued scale per 32-group (exact fp16 copy)
  kInt8GroupF32 = 2,  // int8, fp32 scale per 32-group (the reference's quantize_int8 format)
  kInt8ChanF16 = 3,   // int8, fp16 scale per output channel
  kInt4Group16F32 = 4,  // int4 nibbles, fp32 scale per 16-group (the reference's qblock=16 format)
};

template <int F, int C>
struct Traits {
  static constexpr int kXRows = kTileM / C;                    // tokens this CTA loads per stage
  static constexpr int kXBytes = kXRows * kStageK * 2;         // 32 KB, or 16 KB per CTA of a pair
  static constexpr bool kInt8 = F == kInt8GroupF32 || F == kInt8ChanF16;
  static constexpr bool kG16 = F == kInt4Group16F32;  // four 16-groups per 64-wide K stage
  static constexpr bool kChannel = F == kInt8ChanF16;
  static constexpr bool kF16Group = F == kInt4GroupF16;
  static constexpr int kQRowBytes = kInt8 ? kStageK : kStageK / 2;  // packed bytes per row per stage
  static constexpr int kQBytes = kTileN * kQRowBytes;
  static constexpr int kGroupsPerStage = kChannel ? 0 : (kG16 ? 4 : 2);
  static constexpr int kScaleElem = kF16Group ? 2 : 4;
  // per-stage scale area of the cp.async path, [row][group]
  static constexpr int kScaleBytes = kChannel ? 0 : (kTileN * kGroupsPerStage * kScaleElem + 1023) / 1024 * 1024;
  // TMA path: one 2-D box of 8 groups x 128 rows ("a chunk", [row][8 groups],
  // 16 B of fp16 or 32 B of fp32 per row) covers the scales of kChunkStages
  // consecutive stages; two chunk buffers alternate.
  static constexpr int kChunkGroups = 8;
  static constexpr int kChunkStages = kChannel ? 1 : kChunkGroups / kGroupsPerStage;
  static constexpr int kChunkRowBytes = kChunkGroups * kScaleElem;
  static constexpr int kChunkBytes = kChannel ? 0 : kTileN * kChunkRowBytes;
  static constexpr int kStageBytes = kXBytes + kWBytes + kQBytes + kScaleBytes;
  static constexpr int kFit = (kSmemLimit - 1024 - kBarrierBytes - 2 * kChunkBytes) / kStageBytes;
  static constexpr int kStages = kFit > 6 ? 6 : kFit;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 2 * kChunkBytes + kBarrierBytes;
  static_assert(kStageBytes % 1024 == 0, "stage bases must stay 1024-byte aligned");
  static_assert(kStages >= 3, "pipeline too shallow");
};

// Instruction descriptor, kind::f16: D f32, A/B bf16, both K-major,
// M = 128 per CTA (256 for a pair), N = 256.
template <int C>
constexpr uint32_t idesc_f16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTileM >> 3) << 17) |
         ((uint32_t)((kTileN * C) >> 4) << 24);
}

__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// One 32-bit nibble word (elements 8j..8j+7 of a row) -> 8 bf16 = 16 bytes.
template <bool kF16Scale>
__device__ __forceinline__ uint4 dequant_nibble_word(uint32_t w, float s, uint32_t s_hi2, uint32_t s_lo2) {
  uint32_t out[4];
  if constexpr (kF16Scale) {
    const uint32_t t2 = w >> 4;
    constexpr uint32_t kOne = 0x3F803F80u, kMinus136 = 0xC308C308u;  // bf16x2 (1, 1), (-136, -136)
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      // nibbles 2p (bits 0-3) and 2p+1 (bits 16-19), offset-8 magic 0x4300|u = 128+u
      const uint32_t t = prmt(w, t2, 0x0400u + 0x0101u * p);
      const uint32_t magic = and_xor(t, 0x000F000Fu, 0x43084308u);
      const uint32_t code = bf16x2_fma(magic, kOne, kMinus136);   // exact integer codes
      const uint32_t lo = bf16x2_mul(code, s_lo2);                  // exact (<= 7 significant bits)
      out[p] = bf16x2_fma(code, s_hi2, lo);                         // RN(code * s), one rounding
    }
  } else {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t n0 = (w >> (8 * p)) & 0xFu, n1 = (w >> (8 * p + 4)) & 0xFu;
      const float c0 = __uint_as_float(0x4B000000u | (n0 ^ 8u)) - 8388616.0f;  // exact code
      const float c1 = __uint_as_float(0x4B000000u | (n1 ^ 8u)) - 8388616.0f;
      out[p] = pack_bf16x2_rn(__fmul_rn(c0, s), __fmul_rn(c1, s));
    }
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// Four int8 weights (one word) -> two bf16x2. Scaled: RN(float(q) * s); else the exact code.
template <bool kScaled>
__device__ __forceinline__ uint2 dequant_int8_word(uint32_t w, float s) {
  const uint32_t xo = w ^ 0x80808080u;  // offset binary u = q + 128
  float f[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bytes [u_i, 0, 0, 0x4B] -> float 2^23 + u_i, minus 2^23 + 128 -> q_i exactly
    f[i] = __uint_as_float(prmt(xo, 0x4Bu, 0x4650u + i)) - 8388736.0f;
    if (kScaled) f[i] = __fmul_rn(f[i], s);
  }
  return make_uint2(pack_bf16x2_rn(f[0], f[1]), pack_bf16x2_rn(f[2], f[3]));
}

struct Smem {
  uint8_t* stage0;     // stage s starts at stage0 + s * kStageBytes
  uint8_t* chunk0;     // scale chunk b starts at chunk0 + b * kChunkBytes
  uint64_t* full;      // [kStages] packed weights (+ cp.async scales) landed; with a pair, the x slice too
  uint64_t* xfull;     // [kStages] one CTA: the x tile landed (the dequant does not wait for it)
  uint64_t* wready;    // [kStages] dequantized weights written
  uint64_t* empty;     // [kStages] MMAs done reading the stage
  uint64_t* acc_full;  // [2]
  uint64_t* acc_empty; // [2]
  uint64_t* drain;     // [1]
  uint64_t* sfull;     // [2] scale chunk landed
  uint64_t* sempty;    // [2] every dequant warp is done with the chunk
  uint32_t* tmem_base;
};

// kPeers: the epilogue stores every output element into each of tg.count
// buffers (tg.ptr[q][m * tg.ldy + n], e.g. every rank's y mapped over NVLink,
// offset to this rank's rows), then fences at system scope: the GEMM and the
// all-gather of a token-row split in one kernel.
template <int F, typename OutT, int C, bool kPeers = false>
__global__ void __launch_bounds__(kThreads, 1) wq_tc_kernel(const __grid_constant__ CUtensorMap x_map,
                                                            const __grid_constant__ CUtensorMap q_map,
                                                            const __grid_constant__ CUtensorMap s_map, int scale_tma,
                                                            const void* __restrict__ wscale,
                                                            const OutT* __restrict__ bias, OutT* __restrict__ y,
                                                            int M, int N, int K, int* status_host,
                                                            const __grid_constant__ OutTargets tg) {
  using T = Traits<F, C>;
  constexpr int kStages = T::kStages;
  constexpr int kStageBytes = T::kStageBytes;
  constexpr int kXBytes = T::kXBytes;
  constexpr int kPairRows = kTileN * C;  // weight rows per (pair) tile
  // Dequant groups must divide the stage count: a group's parity wait on
  // full[s] is exact only if the load kStages iterations earlier (the same
  // group's previous item on that stage) has already landed.
  constexpr int kG = kStages % kDeqGroups == 0 ? kDeqGroups : (kStages % 2 == 0 ? 2 : 1);
  constexpr int kCS = T::kChunkStages;
  static_assert(T::kChannel || kCS % kG == 0, "every dequant group must touch every scale chunk");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Smem sm;
  sm.stage0 = base;
  sm.chunk0 = base + kStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm.chunk0 + 2 * T::kChunkBytes);
  sm.full = bars;
  sm.wready = bars + kStages;
  sm.empty = bars + 2 * kStages;
  sm.xfull = bars + 3 * kStages;
  sm.acc_full = bars + 4 * kStages;
  sm.acc_empty = bars + 4 * kStages + 2;
  sm.drain = bars + 4 * kStages + 4;
  sm.sfull = bars + 4 * kStages + 5;
  sm.sempty = bars + 4 * kStages + 7;
  sm.tmem_base = reinterpret_cast<uint32_t*>(bars + 4 * kStages + 9);
  static_assert((4 * kStages + 9) * 8 + 4 <= kBarrierBytes, "barrier area");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cr = C == 2 ? cluster_ctarank() : 0u;  // rank within the pair
  const bool leader = cr == 0;
  const int tiles_n = (N + kPairRows - 1) / kPairRows;
  const int tiles_m = (M + kTileM - 1) / kTileM;
  const int num_tiles = tiles_n * tiles_m;
  const int first_tile = blockIdx.x / C, tile_step = gridDim.x / C;
  const int k_stages = (K + kStageK - 1) / kStageK;
  const int groups = T::kG16 ? K >> 4 : K >> 5;
  const bool stma = !T::kChannel && scale_tma != 0;  // host: aligned strides and k_stages % kCS == 0

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], (T::kChannel || stma) ? 1 : 1 + 32);
      mbar_init(&sm.xfull[s], 1);
      mbar_init(&sm.wready[s], kDequantWarps / kG * C);  // one group; a pair's arrive on CTA 0
      mbar_init(&sm.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.acc_full[a], 1);
      mbar_init(&sm.acc_empty[a], kEpiWarps * C);
      mbar_init(&sm.sfull[a], 1);
      mbar_init(&sm.sempty[a], kDequantWarps);
    }
    mbar_init(sm.drain, 1);
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc<C>(sm.tmem_base, kTmemCols);
  tc_fence_before();
  if constexpr (C == 2) {
    cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  pdl_trigger();

  bool ok = true;
  if (warp == kProducerWarp) {
    // -------------------------------- producer --------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&x_map);
      tma_prefetch_desc(&q_map);
      if (stma) tma_prefetch_desc(&s_map);
      // the first tile's first weight stages stream into L2 while the previous
      // kernel of the stream finishes
      if (first_tile < num_tiles) {
        const int n0 = (first_tile % tiles_n) * kPairRows + (int)cr * kTileN;
        const int pre = k_stages < kStages ? k_stages : kStages;
        for (int ks = 0; ks < pre; ++ks) tma_prefetch_l2_2d(&q_map, ks * T::kQRowBytes, n0);
      }
    }
    pdl_wait();
    uint32_t kit = 0;
    for (int tile = first_tile; tile < num_tiles && ok; tile += tile_step) {
      const int n0 = (tile % tiles_n) * kPairRows + (int)cr * kTileN;
      const int m0 = (tile / tiles_n) * kTileM + (int)cr * T::kXRows;
      for (int ks = 0; ks < k_stages; ++ks, ++kit) {
        const int s = kit % kStages;
        const uint32_t ph = (kit / kStages) & 1;
        if (!mbar_wait(&sm.empty[s], ph ^ 1, kDevErrEmptyBarrierTimeout)) { ok = false; break; }
        if (stma && kit % kCS == 0) {
          // the scales of stages kit .. kit + kCS - 1 (one tile: k_stages % kCS == 0)
          const uint32_t c = kit / kCS;
          const int b = c & 1;
          if (!mbar_wait(&sm.sempty[b], ((c >> 1) & 1) ^ 1, kDevErrEmptyBarrierTimeout)) { ok = false; break; }
          if (lane == 0) {
            mbar_arrive_expect_tx(&sm.sfull[b], T::kChunkBytes);
            tma_load_2d(sm.chunk0 + b * T::kChunkBytes, &s_map, &sm.sfull[b], ks * T::kGroupsPerStage, n0);
          }
        }
        uint8_t* st = sm.stage0 + s * kStageBytes;
        if (lane == 0) {
          // One CTA: the packed weights on full[s] (all the dequant waits for,
          // issued first) and the x tile on xfull[s] (only the MMA waits for
          // it). A pair keeps both on full[s]: CTA 1's dequant warps vouch for
          // its x slice when they arrive on CTA 0's wready.
          uint64_t* xbar = C == 1 ? &sm.xfull[s] : &sm.full[s];
          mbar_arrive_expect_tx(&sm.full[s], T::kQBytes + (C == 1 ? 0 : kXBytes));
          tma_load_2d(st + kXBytes + kWBytes, &q_map, &sm.full[s], ks * T::kQRowBytes, n0);
          if (C == 1) mbar_arrive_expect_tx(xbar, kXBytes);
          tma_load_2d(st, &x_map, xbar, ks * kStageK, m0);
        }
        if (!T::kChannel && !stma) {
          // cp.async fallback: this stage's scales into its [row][group] area,
          // then one no-increment arrival per lane when they have landed
          uint8_t* sc = st + kXBytes + kWBytes + T::kQBytes;
          constexpr int kGS = T::kGroupsPerStage;
          const int g0 = ks * kGS;
#pragma unroll
          for (int j = 0; j < kGS * kTileN / 32; ++j) {
            const int i = lane + 32 * j, r = i % kTileN, g = i / kTileN, n = n0 + r;
            const bool valid = n < N && (g0 + g) < groups;
            const uint8_t* src = reinterpret_cast<const uint8_t*>(wscale);
            if (valid) src += ((size_t)n * groups + g0 + g) * T::kScaleElem;
            if constexpr (T::kScaleElem == 4) {
              cp_async_4(sc + 4 * (r * kGS + g), src, valid ? 4u : 0u);
            } else if (g == 0) {
              // fp16: the two scales of a row are one aligned 4-byte word (K % 64 == 0)
              cp_async_4(sc + 4 * r, src, valid ? 4u : 0u);
            }
          }
          cp_async_mbar_arrive_noinc(&sm.full[s]);
        }
      }
    }
  } else if (warp >= kDequantWarp0) {
    // -------------------------------- dequant ---------------------------------
    // reads only shared memory the producer filled after its pdl_wait()
    // The dequant warps form kG groups; group q dequantizes the stages with
    // kit % kG == q, so kG stages are in flight at once. A stage holds 256
    // items (128 rows x two 32-element halves of the 64-wide stage). A warp
    // takes 16 rows x both halves per round: lane l -> row 16 b + (l & 7) +
    // 8 (l >> 4), half (l >> 3) & 1. Then the 8 lanes of each quarter-warp
    // store 8 different rows and the two quarters of each half-warp store
    // different halves of the same 8 rows, so every 16-byte store of a
    // half-warp lands on a distinct bank group of the 128-byte swizzle atom.
    constexpr int kGroupThreads = kDequantWarps * 32 / kG;
    constexpr int kWarpsPerGroup = kGroupThreads / 32;
    constexpr int kRounds = (kTileN / 16 + kWarpsPerGroup - 1) / kWarpsPerGroup;  // 16-row blocks per warp
    const int dt = (warp - kDequantWarp0) * 32 + lane;
    const int q = dt / kGroupThreads, wg = (dt % kGroupThreads) >> 5;
    const int r_in = (lane & 7) + 8 * (lane >> 4), g = (lane >> 3) & 1;
    // fp16 scales by TMA: each thread keeps its rows' 16-byte chunk rows (8
    // scales) in registers across its group's stages of the chunk, loaded
    // once with a conflict-free 16-byte load (a 2-byte load per stage from
    // 16-byte rows is a 2-way bank conflict between rows r and r + 8)
    uint4 scache[kRounds];
#pragma unroll
    for (int rd = 0; rd < kRounds; ++rd) scache[rd] = make_uint4(0u, 0u, 0u, 0u);
    uint32_t kit = 0;
    for (int tile = first_tile; tile < num_tiles && ok; tile += tile_step) {
      for (int ks = 0; ks < k_stages; ++ks, ++kit) {
        if ((int)(kit % kG) != q) continue;
        const int s = kit % kStages;
        const uint32_t ph = (kit / kStages) & 1;
        uint8_t* st = sm.stage0 + s * kStageBytes;
        if (!mbar_wait(&sm.full[s], ph, kDevErrFullBarrierTimeout)) { ok = false; break; }
        const uint8_t* qt = st + kXBytes + kWBytes;
        // scale of (row r, group gg of this stage): a chunk [row][8 groups] or
        // the stage's own [row][group] area
        const uint8_t* sbase;
        int srow_bytes, sgroup0;
        uint32_t c = 0;
        if (stma) {
          c = kit / kCS;
          if (!mbar_wait(&sm.sfull[c & 1], (c >> 1) & 1, kDevErrFullBarrierTimeout)) { ok = false; break; }
          sbase = sm.chunk0 + (c & 1) * T::kChunkBytes;
          srow_bytes = T::kChunkRowBytes;
          sgroup0 = (int)(kit % kCS) * T::kGroupsPerStage;
          if constexpr (T::kF16Group) {
            if ((int)(kit % kCS) < kG) {  // this group's first stage of the chunk
#pragma unroll
              for (int rd = 0; rd < kRounds; ++rd) {
                const int blk = rd * kWarpsPerGroup + wg;
                if (blk < kTileN / 16) scache[rd] = lds128(smem_u32(sbase) + (blk * 16 + r_in) * T::kChunkRowBytes);
              }
            }
          }
        } else {
          sbase = qt + T::kQBytes;
          srow_bytes = T::kGroupsPerStage * T::kScaleElem;
          sgroup0 = 0;
        }
#pragma unroll
        for (int rd = 0; rd < kRounds; ++rd) {
          const int blk = rd * kWarpsPerGroup + wg;
          if (kTileN / 16 % kWarpsPerGroup != 0 && blk >= kTileN / 16) break;
          const int r = blk * 16 + r_in;  // weight row within the tile
          const uint32_t wrow = smem_u32(st + kXBytes) + r * 128;
          const int c0 = 4 * g, sw = r & 7;
          const uint8_t* srow = sbase + r * srow_bytes;
          if constexpr (!T::kInt8) {
            // SWIZZLE_32B nibble tile: 16-byte half h of row r sits at half h ^ ((r >> 2) & 1)
            const uint4 qw = lds128(smem_u32(qt) + r * 32 + ((g ^ ((r >> 2) & 1)) << 4));
            float sf, sf1;
            uint32_t s_hi2 = 0, s_lo2 = 0;
            if constexpr (T::kG16) {
              // words 0-1 of the 32-element half are 16-group 2g, words 2-3 group 2g+1
              sf = reinterpret_cast<const float*>(srow)[sgroup0 + 2 * g];
              sf1 = reinterpret_cast<const float*>(srow)[sgroup0 + 2 * g + 1];
            } else if constexpr (T::kF16Group) {
              if (stma) {
                const uint4 cv = scache[rd];
                const int k4 = (int)(kit % kCS);
                const uint32_t w = k4 == 0 ? cv.x : (k4 == 1 ? cv.y : (k4 == 2 ? cv.z : cv.w));
                sf = __half2float(__ushort_as_half((unsigned short)(g ? (w >> 16) : (w & 0xFFFFu))));
              } else {
                sf = __half2float(reinterpret_cast<const __half*>(srow)[sgroup0 + g]);
              }
              const float hi = __uint_as_float(__float_as_uint(sf) & 0xFFFF0000u);
              const float lo = sf - hi;  // exact; at most 3 significant bits for an fp16 value
              const uint32_t hb = __float_as_uint(hi) >> 16;
              const uint32_t lb = __float_as_uint(lo) >> 16;  // exact truncation (low bits are zero)
              s_hi2 = hb | (hb << 16);
              s_lo2 = lb | (lb << 16);
            } else {
              sf = reinterpret_cast<const float*>(srow)[sgroup0 + g];
            }
            if constexpr (!T::kG16) sf1 = sf;
            constexpr bool kF16 = T::kF16Group;
            sts128(wrow + (((c0 + 0) ^ sw) << 4), dequant_nibble_word<kF16>(qw.x, sf, s_hi2, s_lo2));
            sts128(wrow + (((c0 + 1) ^ sw) << 4), dequant_nibble_word<kF16>(qw.y, sf, s_hi2, s_lo2));
            sts128(wrow + (((c0 + 2) ^ sw) << 4), dequant_nibble_word<kF16>(qw.z, sf1, s_hi2, s_lo2));
            sts128(wrow + (((c0 + 3) ^ sw) << 4), dequant_nibble_word<kF16>(qw.w, sf1, s_hi2, s_lo2));
          } else {
            // SWIZZLE_64B int8 tile (64-byte rows): chunk c of row r sits at c ^ ((r >> 1) & 3)
            const float sf = T::kChannel ? 1.0f : reinterpret_cast<const float*>(srow)[sgroup0 + g];
            const int xr = (r >> 1) & 3;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const uint4 qw = lds128(smem_u32(qt) + r * 64 + (((2 * g + j) ^ xr) << 4));
              const uint2 a = dequant_int8_word<!T::kChannel>(qw.x, sf), b = dequant_int8_word<!T::kChannel>(qw.y, sf);
              const uint2 cc = dequant_int8_word<!T::kChannel>(qw.z, sf), d = dequant_int8_word<!T::kChannel>(qw.w, sf);
              sts128(wrow + (((c0 + 2 * j) ^ sw) << 4), make_uint4(a.x, a.y, b.x, b.y));
              sts128(wrow + (((c0 + 2 * j + 1) ^ sw) << 4), make_uint4(cc.x, cc.y, d.x, d.y));
            }
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          // this CTA's x slice and dequantized rows of stage s are in place
          if constexpr (C == 1) {
            mbar_arrive(&sm.wready[s]);
          } else {
            mbar_arrive_cluster(&sm.wready[s], 0);
          }
          // this warp's last stage of the scale chunk: the producer may refill it
          if (stma && (int)(kit % kCS) >= kCS - kG) mbar_arrive(&sm.sempty[c & 1]);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------- MMA -----------------------------------
    // One thread of CTA 0 issues for the pair; CTA 1's MMA warp only waits for
    // the drain before the collective TMEM release.
    if (leader) {
      constexpr uint32_t kId = idesc_f16<C>();
      uint32_t kit = 0;
      int it = 0;
      for (int tile = first_tile; tile < num_tiles && ok; tile += tile_step, ++it) {
        const int acc = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(&sm.acc_empty[acc], aph ^ 1, kDevErrMmaBarrierTimeout)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * kAccCols;
        for (int ks = 0; ks < k_stages; ++ks, ++kit) {
          const int s = kit % kStages;
          const uint32_t ph = (kit / kStages) & 1;
          // wready[s] complete => every arriving dequant warp saw its CTA's full[s]
          if (!mbar_wait(C == 1 ? &sm.xfull[s] : &sm.full[s], ph, kDevErrFullBarrierTimeout) ||
              !mbar_wait(&sm.wready[s], ph, kDevErrFullBarrierTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t xa = smem_u32(sm.stage0 + s * kStageBytes);
            const uint32_t wa = xa + kXBytes;
            const uint64_t adesc = sw128_desc(wa), bdesc = sw128_desc(xa);
#pragma unroll
            for (int k = 0; k < kStageK / kUmmaK; ++k) {
              // advance 16 elements (32 bytes) along K inside the swizzle atom
              umma_f16<C>(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), kId, (ks | k) != 0);
            }
#pragma unroll
            for (uint32_t rk = 0; rk < (uint32_t)C; ++rk) {
              umma_commit<C>(&sm.empty[s], rk);
              if (ks == k_stages - 1) umma_commit<C>(&sm.acc_full[acc], rk);
            }
          }
          __syncwarp();
        }
      }
      // drain: every MMA this thread issued has completed before TMEM is freed
      if (lane == 0) {
#pragma unroll
        for (uint32_t rk = 0; rk < (uint32_t)C; ++rk) umma_commit<C>(sm.drain, rk);
      }
      __syncwarp();
    }
    if (!mbar_wait(sm.drain, 0, kDevErrMmaBarrierTimeout)) ok = false;
  } else {
    // -------------------------------- epilogue --------------------------------
    pdl_wait();  // y, bias and channel scales are touched only after the previous kernel
    int it = 0;
    for (int tile = first_tile; tile < num_tiles && ok; tile += tile_step, ++it) {
      const int n0 = (tile % tiles_n) * kPairRows + (int)cr * kTileN;
      const int m0 = (tile / tiles_n) * kTileM;
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (!mbar_wait(&sm.acc_full[acc], aph, kDevErrEpilogueBarrierTimeout)) { ok = false; break; }
      tc_fence_after();
      const int n = n0 + warp * 32 + lane;
      const bool n_ok = n < N;
      const float b = (bias != nullptr && n_ok) ? to_f32(bias[n]) : 0.0f;
      const float cs = (T::kChannel && n_ok) ? __half2float(reinterpret_cast<const __half*>(wscale)[n]) : 1.0f;
      const uint32_t taddr = tmem + acc * kAccCols + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < kAccCols; c += 32) {
        uint32_t v[32];
        tmem_ld32(taddr + c, v);
        const int mbase = m0 + c;
        if (n_ok) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = mbase + j;
            const float a = T::kChannel ? __fmul_rn(__uint_as_float(v[j]), cs) : __uint_as_float(v[j]);
            if (m < M) {
              const OutT v = from_f32<OutT>(a + b);
              if constexpr (kPeers) {
                for (int t = 0; t < tg.count; ++t) static_cast<OutT*>(tg.ptr[t])[(size_t)m * tg.ldy + n] = v;
              } else {
                y[(size_t)m * N + n] = v;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (C == 1) {
          mbar_arrive(&sm.acc_empty[acc]);
        } else {
          mbar_arrive_cluster(&sm.acc_empty[acc], 0);
        }
      }
    }
  }

  if constexpr (kPeers) {
    if (warp < kEpiWarps) __threadfence_system();  // the peer stores are visible before the flag barrier
  }
  if (!ok) mirror_device_error(status_host);
  tc_fence_before();
  if constexpr (C == 2) {
    cluster_sync_all();  // no CTA leaves while its peer may still touch its barriers or smem
  } else {
    __syncthreads();
  }
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc<C>(tmem, kTmemCols);
}

}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
bool w4a16_tc_supported(int M, int N, int K, int scale_dtype) {
  (void)N;
  if (M <= 64) return false;  // the small-M kernel owns the HBM-bound regime
  if (K % 32 != 0) return false;
  if (scale_dtype == GFX_SCALE_F16 && K % 64 != 0) return false;
  return true;
}

// CTA count per tile. One CTA is the default: on B200 the pair variant
// (cta_group::2) measured 2-8% slower on the Flux shapes at M = 4608 although
// it halves the activation bytes per SM, so the per-SM limit is not the x
// tile traffic. GFX906_B200_TC_CTA=2 selects the pair (tests, measurement).
static int tc_ctas(int M) {
  (void)M;
  const char* e = getenv("GFX906_B200_TC_CTA");
  if (e && e[0] == '2' && e[1] == 0) return 2;
  return 1;
}

template <int F, typename OutT, int C, bool kPeers = false>
static int launch_tc_t(const CUtensorMap& xm, const CUtensorMap& qm, const CUtensorMap& sm_map, int scale_tma,
                       const void* ws, const void* bias, void* y, int M, int N, int K, cudaStream_t st, int sms,
                       const OutTargets* tg = nullptr) {
  using T = tc::Traits<F, C>;
  auto kern = tc::wq_tc_kernel<F, OutT, C, kPeers>;
  static bool attr_set[64] = {false};
  static int max_clusters[64] = {0};
  const int dev = current_device();
  const bool cached = dev >= 0 && dev < 64 && attr_set[dev];
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.blockDim = dim3(tc::kThreads);
  cfg.dynamicSmemBytes = T::kSmemBytes;
  cfg.stream = st;
  cfg.attrs = attr;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 1;
  if (C == 2) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  int clusters = sms / C;
  if (!cached) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T::kSmemBytes);
    if (e != cudaSuccess)
      return set_error(GFX_ERR_CUDA, "wq_tc: cannot set %d bytes of shared memory: %s", T::kSmemBytes,
                       cudaGetErrorString(e));
    if (C == 2) {
      // pairs must sit on two SMs of one cluster slot; ask how many fit at once
      cfg.gridDim = dim3(2 * clusters);
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        return set_error(GFX_ERR_CUDA, "wq_tc: no co-resident CTA pair possible: %s", cudaGetErrorString(e));
      }
      if (dev >= 0 && dev < 64) max_clusters[dev] = n;
      clusters = n < clusters ? n : clusters;
    }
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  } else if (C == 2 && max_clusters[dev] > 0 && max_clusters[dev] < clusters) {
    clusters = max_clusters[dev];
  }
  const int rows = tc::kTileN * C;
  const int tiles = ((N + rows - 1) / rows) * ((M + tc::kTileM - 1) / tc::kTileM);
  const int units = tiles < clusters ? tiles : clusters;
  cfg.gridDim = dim3(C * units);
  OutTargets none{};
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, xm, qm, sm_map, scale_tma, ws, (const OutT*)bias, (OutT*)y, M, N, K,
                                     host_status_word(dev), tg ? *tg : none);
  if (e != cudaSuccess) return set_error(GFX_ERR_CUDA, "wq_tc_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("wq_tc_kernel");
}

template <int F>
static int launch_tc_out(int out_dtype, const void* x, const CUtensorMap& qm, const void* ws, const void* bias,
                         void* y, int M, int N, int K, cudaStream_t st, int sms, const OutTargets* tg = nullptr) {
  const int C = tg ? 1 : tc_ctas(M);
  CUtensorMap xm;
  // x box: 64 K-elements x (256 tokens, or the 128 of one CTA of a pair), SWIZZLE_128B
  int rc = make_tmap_2d(&xm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2,
                        tc::kStageK, tc::kTileM / C, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // Scales by TMA, one box of 8 groups x 128 rows per chunk of stages, when
  // the scale rows are 16-byte aligned and no chunk crosses a tile's K end;
  // otherwise per-stage cp.async.
  using T1 = tc::Traits<F, 1>;
  CUtensorMap sm_map;
  memset(&sm_map, 0, sizeof(sm_map));
  int scale_tma = 0;
  if constexpr (!T1::kChannel) {
    const uint64_t groups = (uint64_t)K / (T1::kG16 ? 16 : 32);
    const int k_stages = (K + tc::kStageK - 1) / tc::kStageK;
    if ((groups * T1::kScaleElem) % 16 == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0 &&
        k_stages % T1::kChunkStages == 0) {
      rc = cached_tmap_2d(&sm_map, T1::kScaleElem == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                          ws, groups, (uint64_t)N, groups * T1::kScaleElem, T1::kChunkGroups, tc::kTileN,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
      scale_tma = 1;
    }
  }
  if (tg != nullptr) {
    if constexpr (F == tc::kInt4GroupF32 || F == tc::kInt4GroupF16) {
      if (out_dtype == GFX_DTYPE_F32)
        return launch_tc_t<F, float, 1, true>(xm, qm, sm_map, scale_tma, ws, bias, y, M, N, K, st, sms, tg);
      if (out_dtype == GFX_DTYPE_F16)
        return launch_tc_t<F, __half, 1, true>(xm, qm, sm_map, scale_tma, ws, bias, y, M, N, K, st, sms, tg);
      return launch_tc_t<F, __nv_bfloat16, 1, true>(xm, qm, sm_map, scale_tma, ws, bias, y, M, N, K, st, sms, tg);
    } else {
      return set_error(GFX_ERR_UNSUPPORTED, "wq_tc: peer-store outputs take int4 weights with 32-element groups");
    }
  }
  if (C == 2) {
    if (out_dtype == GFX_DTYPE_F32)
      return launch_tc_t<F, float, 2>(xm, qm, sm_map, scale_tma, ws, bias, y, M, N, K, st, sms);
    if (out_dtype == GFX_DTYPE_F16)
      return launch_tc_t<F, __half, 2>(xm, qm, sm_map, scale_tma, ws, bias, y, M, N, K, st, sms);
    return launch_tc_t<F, __nv_bfloat16, 2>(xm, qm, sm_map, scale_tma, ws, bias, y, M, N, K, st, sms);
  }
  if (out_dtype == GFX_DTYPE_F32)
    return launch_tc_t<F, float, 1>(xm, qm, sm_map, scale_tma, ws, bias, y, M, N, K, st, sms);
  if (out_dtype == GFX_DTYPE_F16)
    return launch_tc_t<F, __half, 1>(xm, qm, sm_map, scale_tma, ws, bias, y, M, N, K, st, sms);
  return launch_tc_t<F, __nv_bfloat16, 1>(xm, qm, sm_map, scale_tma, ws, bias, y, M, N, K, st, sms);
}

int launch_w4a16_tc(const void* x, const void* wq, const void* ws, int scale_dtype, const void* bias, void* y,
                    int out_dtype, int M, int N, int K, cudaStream_t stream, int sms, int qblock) {
  CUtensorMap qm;
  int rc = cached_tmap_2d(&qm, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                    tc::kStageK / 2, tc::kTileN, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  if (qblock == 16) return launch_tc_out<tc::kInt4Group16F32>(out_dtype, x, qm, ws, bias, y, M, N, K, stream, sms);
  if (scale_dtype == GFX_SCALE_F16)
    return launch_tc_out<tc::kInt4GroupF16>(out_dtype, x, qm, ws, bias, y, M, N, K, stream, sms);
  return launch_tc_out<tc::kInt4GroupF32>(out_dtype, x, qm, ws, bias, y, M, N, K, stream, sms);
}

int launch_w4a16_tc_targets(const void* x, const void* wq, const void* ws, int scale_dtype, const void* bias,
                            const OutTargets& tg, int out_dtype, int M, int N, int K, cudaStream_t stream, int sms) {
  CUtensorMap qm;
  int rc = cached_tmap_2d(&qm, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                          tc::kStageK / 2, tc::kTileN, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  if (scale_dtype == GFX_SCALE_F16)
    return launch_tc_out<tc::kInt4GroupF16>(out_dtype, x, qm, ws, bias, tg.ptr[0], M, N, K, stream, sms, &tg);
  return launch_tc_out<tc::kInt4GroupF32>(out_dtype, x, qm, ws, bias, tg.ptr[0], M, N, K, stream, sms, &tg);
}

int launch_w8a16_tc(const void* x, const void* wq, const void* ws, int per_channel, const void* bias, void* y,
                    int out_dtype, int M, int N, int K, cudaStream_t stream, int sms) {
  CUtensorMap qm;
  int rc = cached_tmap_2d(&qm, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)K, (uint64_t)N, (uint64_t)K, tc::kStageK,
                    tc::kTileN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  if (per_channel) return launch_tc_out<tc::kInt8ChanF16>(out_dtype, x, qm, ws, bias, y, M, N, K, stream, sms);
  return launch_tc_out<tc::kInt8GroupF32>(out_dtype, x, qm, ws, bias, y, M, N, K, stream, sms);
}

}  // namespace gfx
