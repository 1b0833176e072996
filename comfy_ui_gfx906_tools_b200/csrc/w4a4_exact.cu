// Integer-exact W4A4 GEMM on the 5th-generation tensor cores: the reference's
// own production numerics, bit for bit.
//
// C[m, n] = sum over 32-element blocks b, in order, of the fp32 chain
//   acc = fmaf((float)dot_b(A[m], B[n]), A_scale[m, b] * B_scale[n, b], acc)
// with dot_b the exact integer dot product of the block's int4 codes (two
// 16-element halves with their own scales when qblock = 16), the split-K
// partition of the reference (each split's chain starts at 0, partials summed
// in split order), then + bias and one conversion to the output dtype.
// Reference: int4_gemm_kernel (nodes/ComfyUI-Gfx906Int4/csrc/
// int4_gemm_scaled.hip:53-180, the chain at :147-160), splitk_reduce_kernel
// (:182-191), gemm_launch (:229-248) and auto_splits (binding.cpp:36-43).
//
// Design: the integer block dot products run on the tensor cores as
// tcgen05.mma.kind::f8f6f4 with e5m2 operands. Every int4 code (-8..7) is
// exact in e5m2, every product is an integer of magnitude <= 64, and a
// 32-element dot is an integer of magnitude <= 2048, so the fp32 result of
// one K = 32 MMA (a fresh accumulator per block) is the exact integer dot.
// The per-block fp32 chain (one rounding per multiply and per fma, as the
// reference) runs on the CUDA cores, in packed f32x2 instructions, in
// registers that hold the accumulators across the whole K loop.
//
// One persistent CTA per SM, 20 warps:
//   warp 0      producer: TMA of the activation tile (e5m2, prepared once per
//               call by e5m2_prepass_kernel) and of the weight nibbles per
//               128-wide K stage (4-stage ring, freed by the MMAs), and of both
//               operands' scales (8-stage ring, freed by the rescale warps).
//   warp 1      TMEM allocation; one thread issues one MMA per 32-element
//               block (M = 128 weight rows, N = the tile's token columns,
//               K = 32) into one of 4 TMEM slots and commits it.
//   warps 2-3   unpack: weight nibbles -> e5m2 in the UMMA K-major
//               SWIZZLE_128B layout, proxy fence, mbarrier arrive.
//   warps 4-19  rescale: four warps per TMEM lane quarter, one column group
//               each; per block all TMEM reads, one wait, release the slot,
//               then the fp32 chain. Measured: with one 16-column read in
//               flight per warp and 8 rescale warps, the TMEM read latency
//               (not the FMA pipe) set the pace, ~1300 cycles per block.
//               At the end of a tile: + bias, convert, store.
// Every mbarrier wait is bounded (common.cuh).
#include <string.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace gfx {

GFX_DEFINE_STATUS_READER(w4a4x_device_status)

namespace w4a4x {

constexpr int kRows = 128;        // weight rows per tile (MMA M, TMEM lanes)
constexpr int kStageK = 128;      // K elements per stage: one 128-byte e5m2 row = 4 blocks
constexpr int kBlocks = 4;        // 32-element blocks per stage
constexpr int kSlots = 4;         // TMEM slots, one block's dot products each
constexpr int kStages = 4;         // activation / weight stages (freed by the MMAs)
constexpr int kSStages = 8;        // scale stages (freed by the rescale warps, which trail the MMAs)
constexpr int kProducerWarp = 0, kMmaWarp = 1, kUnpackWarp0 = 2, kUnpackWarps = 2, kRescaleWarp0 = 4,
              kRescaleWarps = 16;
constexpr int kThreads = (kRescaleWarp0 + kRescaleWarps) * 32;
constexpr int kSmemLimit = 232448;

// Token tile per template: 128 tokens for 32-element blocks, 64 when the
// rescale threads also carry the split partial sum or (qblock 16) two
// products per block (the low half's dots in columns 0..63, the high half's
// in 64..127).
template <int SUB, bool kSplit>
struct Cfg {
  static constexpr int kTok = (SUB == 2 || kSplit) ? 64 : 128;
  static constexpr int kCols = SUB == 2 ? 2 * kTok : kTok;  // MMA N = TMEM columns per slot
  static constexpr int kTPT = kTok / 4;                      // tokens per rescale thread (4 column groups)
  static constexpr int kScalesPerStage = kBlocks * SUB;
  static constexpr int kActBytes = kCols * kStageK;          // e5m2 token rows (MMA B)
  static constexpr int kWBytes = kRows * kStageK;            // e5m2 weight rows (MMA A)
  static constexpr int kQBytes = kRows * kStageK / 2;        // weight nibbles
  static constexpr int kSaBytes = kScalesPerStage * kTok * 4;  // activation scales [scale][token]
  static constexpr int kSbBytes = kRows * kScalesPerStage * 4;  // weight scales [row][scale]
  static constexpr int kStageBytes = kActBytes + kWBytes + kQBytes;
  static constexpr int kScaleBytes = (kSaBytes + kSbBytes + 1023) / 1024 * 1024;
  static constexpr int kTmemCols = kSlots * kCols;
  static constexpr int kBarrierBytes = 512;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kSStages * kScaleBytes + kBarrierBytes;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory");
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation");
};

// Instruction descriptor, kind::f8f6f4: D f32, A and B e5m2, both K-major,
// M = 128, N = kCols.
template <int kCols>
__host__ __device__ constexpr uint32_t idesc_e5m2() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kCols >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
}

// Eight two's-complement nibbles of one word (element i in bits 4i..4i+3)
// -> eight e5m2 bytes. e5m2 is the high byte of an IEEE half, and an integer
// -8..7 as a half has a zero low byte, so the conversion is exact: the
// nibbles become halves 0x6400 | (c ^ 8) = 1024 + (c ^ 8) (or that times 16
// for the odd nibble of a byte), one half-precision add or fma subtracts the
// offset exactly, and a byte permute keeps the high bytes. Byte order of the
// result: elements (0, 4, 1, 5) then (2, 6, 3, 7). The order inside a word
// does not change a block's dot product as long as both operands use it,
// which they do (the activation pre-pass and the weight unpack both call
// this function).
__device__ __forceinline__ uint2 nibbles_to_e5m2(uint32_t w) {
  constexpr uint32_t kMinus1032 = 0xE408E408u;  // half2 (-1032, -1032)
  constexpr uint32_t kSixteenth = 0x2C002C00u;  // half2 (1/16, 1/16)
  constexpr uint32_t kMinus72 = 0xD480D480u;    // half2 (-72, -72)
  const uint32_t w2 = w >> 8;
  uint32_t h0 = and_xor(w, 0x000F000Fu, 0x64086408u);   // elements 0, 4
  uint32_t h1 = and_xor(w, 0x00F000F0u, 0x64806480u);   // elements 1, 5 (times 16)
  uint32_t h2 = and_xor(w2, 0x000F000Fu, 0x64086408u);  // elements 2, 6
  uint32_t h3 = and_xor(w2, 0x00F000F0u, 0x64806480u);  // elements 3, 7 (times 16)
  asm("add.rn.f16x2 %0, %0, %1;" : "+r"(h0) : "r"(kMinus1032));
  asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(h1) : "r"(kSixteenth), "r"(kMinus72));
  asm("add.rn.f16x2 %0, %0, %1;" : "+r"(h2) : "r"(kMinus1032));
  asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(h3) : "r"(kSixteenth), "r"(kMinus72));
  return make_uint2(prmt(h0, h1, 0x7531u), prmt(h2, h3, 0x7531u));
}

// One 16-byte item (a 32-element block of one row) -> 32 e5m2 bytes.
__device__ __forceinline__ void block_to_e5m2(const uint4& q, uint4& lo, uint4& hi) {
  const uint2 a = nibbles_to_e5m2(q.x), b = nibbles_to_e5m2(q.y);
  const uint2 c = nibbles_to_e5m2(q.z), d = nibbles_to_e5m2(q.w);
  lo = make_uint4(a.x, a.y, b.x, b.y);
  hi = make_uint4(c.x, c.y, d.x, d.y);
}

// Activation pre-pass: packed int4 [M, K/2] -> e5m2 [M, K] (SUB 1), or for
// 16-element scale blocks two copies, one with each block's high half zeroed
// and one with its low half zeroed, so one K = 32 MMA yields both halves'
// dots in separate columns. One thread per 32-element block.
template <int SUB>
__global__ void __launch_bounds__(256) e5m2_prepass_kernel(const uint4* __restrict__ a_q4, uint4* __restrict__ a_lo,
                                                           uint4* __restrict__ a_hi, long blocks) {
  const long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b < blocks) {
    uint4 lo, hi;
    block_to_e5m2(a_q4[b], lo, hi);
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    if constexpr (SUB == 1) {
      a_lo[2 * b] = lo;
      a_lo[2 * b + 1] = hi;
    } else {
      a_lo[2 * b] = lo;
      a_lo[2 * b + 1] = z;
      a_hi[2 * b] = z;
      a_hi[2 * b + 1] = hi;
    }
  }
  pdl_trigger();
}

// Activation scales [M, S] -> [S, Mp] (token-contiguous, Mp = M rounded up
// to 4 so the rows of the TMA view are 16-byte aligned).
__global__ void __launch_bounds__(256) scale_transpose_kernel(const float* __restrict__ s, float* __restrict__ st,
                                                              int M, int S, int Mp) {
  __shared__ float tile[32][33];
  const int m0 = blockIdx.x * 32, j0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int m = m0 + r, j = j0 + threadIdx.x;
    tile[r][threadIdx.x] = (m < M && j < S) ? s[(size_t)m * S + j] : 0.0f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int j = j0 + r, m = m0 + threadIdx.x;
    if (j < S && m < Mp) st[(size_t)j * Mp + m] = tile[threadIdx.x][r];
  }
  pdl_trigger();
}

// Weight scales [N, S] -> [N, Sp] with Sp = S rounded up to 4 (zeros after
// column S), for K whose scale rows are not 16-byte multiples (TMA rows must be).
__global__ void __launch_bounds__(256) scale_pad_kernel(const float* __restrict__ s, float* __restrict__ sp, int N,
                                                        int S, int Sp) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < (long)N * Sp) {
    const int n = (int)(i / Sp), j = (int)(i % Sp);
    sp[i] = j < S ? s[(size_t)n * S + j] : 0.0f;
  }
  pdl_trigger();
}

// The reference's split-K reduction (splitk_reduce_kernel,
// int4_gemm_scaled.hip:182-191): v = 0; v += partial[s] in slice order; + bias.
template <typename OutT>
__global__ void __launch_bounds__(256) split_reduce_kernel(const float* __restrict__ part, int P,
                                                           const OutT* __restrict__ bias, OutT* __restrict__ y, int M,
                                                           int N) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  if (i < (long)M * N) {
    float v = 0.0f;
    for (int s = 0; s < P; ++s) v = __fadd_rn(v, part[(size_t)s * M * N + i]);
    if (bias != nullptr) v = __fadd_rn(v, to_f32(bias[i % N]));
    y[i] = from_f32<OutT>(v);
  }
}

struct Smem {
  uint8_t* stage0;     // stage s at stage0 + s * kStageBytes: [act e5m2 | W e5m2 | W nibbles]
  uint8_t* scale0;     // scale stage i at scale0 + i * kScaleBytes: [act scales [scale][token] | W scales [row][scale]]
  uint64_t* full;      // [kStages] the stage's TMA loads landed
  uint64_t* wready;    // [kStages] unpacked weights written
  uint64_t* empty;     // [kStages] MMAs done with the stage
  uint64_t* sfull;     // [kSStages] the scale stage landed
  uint64_t* sempty;    // [kSStages] every rescale warp is done with the scale stage
  uint64_t* dfull;     // [kSlots] a block's dot products are in the slot
  uint64_t* dempty;    // [kSlots] every rescale warp has read the slot
  uint64_t* drain;     // [1] every MMA issued has completed
  uint32_t* tmem_base;
};

__device__ __forceinline__ float4 lds_f32x4(uint32_t addr) {
  const uint4 v = lds128(addr);
  return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
}

// acc[i..i+3] = fma(d[i..i+3], sa[i..i+3] * sb, acc[i..i+3]): the reference's
// fmaf((float)dot, sa * sb, acc), two lanes per packed instruction (each
// element rounded exactly as the scalar operations round it).
__device__ __forceinline__ void chain4(float* acc, const uint32_t* d, float4 sa, float sb) {
  const float2 sb2 = make_float2(sb, sb);
  const float2 t01 = __fmul2_rn(make_float2(sa.x, sa.y), sb2);
  const float2 t23 = __fmul2_rn(make_float2(sa.z, sa.w), sb2);
  const float2 a01 = __ffma2_rn(make_float2(__uint_as_float(d[0]), __uint_as_float(d[1])), t01,
                                make_float2(acc[0], acc[1]));
  const float2 a23 = __ffma2_rn(make_float2(__uint_as_float(d[2]), __uint_as_float(d[3])), t23,
                                make_float2(acc[2], acc[3]));
  acc[0] = a01.x;
  acc[1] = a01.y;
  acc[2] = a23.x;
  acc[3] = a23.y;
}

// kMode 0: one chain per output. 1: the reference's split-K slices run one
// after another in the CTA (the partial sum in registers). 2: the slices run
// in parallel as separate work items, each storing its fp32 partial to
// y[slice][M][N] (no bias); split_reduce_kernel sums them in slice order.
template <typename OutT, int SUB, int kMode>
__global__ void __launch_bounds__(kThreads, 1) w4a4x_kernel(const __grid_constant__ CUtensorMap a_map,
                                                            const __grid_constant__ CUtensorMap a2_map,
                                                            const __grid_constant__ CUtensorMap q_map,
                                                            const __grid_constant__ CUtensorMap s_map,
                                                            const __grid_constant__ CUtensorMap sb_map,
                                                            const OutT* __restrict__ bias, OutT* __restrict__ y,
                                                            int M, int N, int K, int split_blocks, int n_par,
                                                            int* status_host) {
  constexpr bool kSplit = kMode == 1, kPar = kMode == 2;
  using T = Cfg<SUB, kSplit>;
  constexpr int kTok = T::kTok, kCols = T::kCols, kTPT = T::kTPT, kSPS = T::kScalesPerStage;
  constexpr int kStageBytes = T::kStageBytes, kActBytes = T::kActBytes, kWBytes = T::kWBytes,
                kQBytes = T::kQBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Smem sm;
  sm.stage0 = base;
  sm.scale0 = base + kStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm.scale0 + kSStages * T::kScaleBytes);
  sm.full = bars;
  sm.wready = bars + kStages;
  sm.empty = bars + 2 * kStages;
  sm.sfull = bars + 3 * kStages;
  sm.sempty = bars + 3 * kStages + kSStages;
  sm.dfull = bars + 3 * kStages + 2 * kSStages;
  sm.dempty = sm.dfull + kSlots;
  sm.drain = sm.dfull + 2 * kSlots;
  sm.tmem_base = reinterpret_cast<uint32_t*>(sm.drain + 1);
  static_assert((3 * kStages + 2 * kSStages + 2 * kSlots + 1) * 8 + 4 <= T::kBarrierBytes, "barrier area");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nb = K / 32;               // 32-element blocks per row
  const int tiles_m = (M + kTok - 1) / kTok;
  const int tiles_n = (N + kRows - 1) / kRows;
  const int num_tiles = tiles_m * tiles_n;
  const int num_items = num_tiles * (kPar ? n_par : 1);  // work items: (tile, slice)
  // the 32-element blocks [kb0, kb1) and stages [ks0, ks1) of a work item
  auto item_range = [&](int item, int& kb0, int& kb1, int& ks0, int& ks1) {
    kb0 = kPar ? (item % n_par) * split_blocks : 0;
    kb1 = kPar ? (kb0 + split_blocks < nb ? kb0 + split_blocks : nb) : nb;
    ks0 = kb0 / kBlocks;
    ks1 = (kb1 + kBlocks - 1) / kBlocks;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.wready[s], kUnpackWarps);
      mbar_init(&sm.empty[s], 1);
    }
    for (int i = 0; i < kSStages; ++i) {
      mbar_init(&sm.sfull[i], 1);
      mbar_init(&sm.sempty[i], kRescaleWarps);
    }
    for (int b = 0; b < kSlots; ++b) {
      mbar_init(&sm.dfull[b], 1);
      mbar_init(&sm.dempty[b], kRescaleWarps);
    }
    mbar_init(sm.drain, 1);
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tc::tmem_alloc<1>(sm.tmem_base, T::kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  pdl_trigger();

  bool ok = true;
  if (warp == kProducerWarp) {
    // -------------------------------- producer --------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&a_map);
      if (SUB == 2) tma_prefetch_desc(&a2_map);
      tma_prefetch_desc(&q_map);
      tma_prefetch_desc(&s_map);
      tma_prefetch_desc(&sb_map);
      pdl_wait();  // the activation copies come from the pre-pass kernels
      uint32_t kit = 0, aissued = 0, sissued = 0;  // stages issued: activation/weight, scales
      for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
        const int tile = kPar ? item / n_par : item;
        const int m0 = (tile % tiles_m) * kTok, n0 = (tile / tiles_m) * kRows;
        int kb0, kb1, ks0, ks1;
        item_range(item, kb0, kb1, ks0, ks1);
        for (int ks = ks0; ks < ks1; ++ks, ++kit) {
          const int s = kit % kStages;
          const uint32_t ph = (kit / kStages) & 1;
          if (!mbar_wait(&sm.empty[s], ph ^ 1, kDevErrEmptyBarrierTimeout)) { ok = false; break; }
          uint8_t* st = sm.stage0 + s * kStageBytes;
          mbar_arrive_expect_tx(&sm.full[s], kActBytes + kQBytes);
          tma_load_2d(st, &a_map, &sm.full[s], ks * kStageK, m0);
          if constexpr (SUB == 2) tma_load_2d(st + kTok * kStageK, &a2_map, &sm.full[s], ks * kStageK, m0);
          tma_load_2d(st + kActBytes + kWBytes, &q_map, &sm.full[s], ks * (kStageK / 2), n0);
          // the scales go to their own, deeper ring: only the rescale warps, which
          // trail the MMAs, hold it
          const int si = kit % kSStages;
          if (!mbar_wait(&sm.sempty[si], ((kit / kSStages) & 1) ^ 1, kDevErrEmptyBarrierTimeout)) {
            ok = false;
            aissued = kit + 1;
            break;
          }
          uint8_t* sc = sm.scale0 + si * T::kScaleBytes;
          mbar_arrive_expect_tx(&sm.sfull[si], T::kSaBytes + T::kSbBytes);
          tma_load_2d(sc, &s_map, &sm.sfull[si], m0, ks * kSPS);
          tma_load_2d(sc + T::kSaBytes, &sb_map, &sm.sfull[si], ks * kSPS, n0);
          aissued = sissued = kit + 1;
        }
      }
      if (!ok) {
        // loads still in flight land before the CTA leaves
        for (uint32_t k = aissued > (uint32_t)kStages ? aissued - kStages : 0u; k < aissued; ++k)
          (void)mbar_wait_for(&sm.full[k % kStages], (k / kStages) & 1, kDevErrFullBarrierTimeout, kWaitTimeoutNs);
        for (uint32_t k = sissued > (uint32_t)kSStages ? sissued - kSStages : 0u; k < sissued; ++k)
          (void)mbar_wait_for(&sm.sfull[k % kSStages], (k / kSStages) & 1, kDevErrFullBarrierTimeout,
                              kWaitTimeoutNs);
      }
    }
  } else if (warp >= kUnpackWarp0 && warp < kUnpackWarp0 + kUnpackWarps) {
    // --------------------------------- unpack ---------------------------------
    // Lane l takes the 32-element block l & 3 of rows 8i + (l >> 2) of the
    // warp's 64 rows: the warp reads 512 contiguous nibble bytes per step and
    // its 16-byte stores fall on 8 distinct bank groups per 8 lanes.
    const int u = warp - kUnpackWarp0;
    const int c = lane & 3;
    uint32_t kit = 0;
    for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
      int kb0, kb1, ks0, ks1;
      item_range(item, kb0, kb1, ks0, ks1);
      for (int ks = ks0; ks < ks1; ++ks, ++kit) {
        const int s = kit % kStages;
        const uint32_t ph = (kit / kStages) & 1;
        if (!mbar_wait(&sm.full[s], ph, kDevErrFullBarrierTimeout)) { ok = false; break; }
        const uint32_t wa = smem_u32(sm.stage0 + s * kStageBytes + kActBytes);
        const uint32_t qa = wa + kWBytes;
#pragma unroll
        for (int i = 0; i < kRows / kUnpackWarps / 8; ++i) {
          const int r = kRows / kUnpackWarps * u + 8 * i + (lane >> 2);
          uint4 lo, hi;
          block_to_e5m2(lds128(qa + r * (kStageK / 2) + c * 16), lo, hi);
          const uint32_t row = wa + (r >> 3) * 1024 + (r & 7) * 128;
          sts128(row + (((2 * c) ^ (r & 7)) << 4), lo);
          sts128(row + (((2 * c + 1) ^ (r & 7)) << 4), hi);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.wready[s]);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------- MMA -----------------------------------
    constexpr uint32_t kId = idesc_e5m2<kCols>();
    uint32_t kit = 0, bit = 0;
    for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
      int kb0, kb1, ks0, ks1;
      item_range(item, kb0, kb1, ks0, ks1);
      for (int ks = ks0; ks < ks1 && ok; ++ks, ++kit) {
        const int s = kit % kStages;
        const uint32_t ph = (kit / kStages) & 1;
        if (!mbar_wait(&sm.full[s], ph, kDevErrFullBarrierTimeout) ||
            !mbar_wait(&sm.wready[s], ph, kDevErrFullBarrierTimeout)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t xa = smem_u32(sm.stage0 + s * kStageBytes);
        const uint64_t adesc = tc::sw128_desc(xa + kActBytes), bdesc = tc::sw128_desc(xa);
        const int nblk = kb1 - ks * kBlocks < kBlocks ? kb1 - ks * kBlocks : kBlocks;
        for (int j = 0; j < nblk; ++j, ++bit) {
          const int slot = bit % kSlots;
          if (!mbar_wait(&sm.dempty[slot], ((bit / kSlots) & 1) ^ 1, kDevErrMmaBarrierTimeout)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          if (lane == 0) {
            // block j = bytes 32j..32j+31 of every 128-byte row: +2 in the
            // descriptors' 16-byte address units; a fresh accumulator per block
            tc::umma_f8f6f4(tmem + slot * kCols, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j), kId, 0u);
            tc::umma_commit<1>(&sm.dfull[slot]);
            if (j == nblk - 1) tc::umma_commit<1>(&sm.empty[s]);
          }
          __syncwarp();
        }
      }
    }
    if (lane == 0) tc::umma_commit<1>(sm.drain);
    __syncwarp();
    if (!mbar_wait(sm.drain, 0, kDevErrMmaBarrierTimeout)) ok = false;
  } else {
    // -------------------------------- rescale ---------------------------------
    // Each thread owns one weight row (its TMEM lane) and kTPT token columns;
    // the four warps on one SM sub-partition own the four column groups of one
    // lane quarter. Per block a warp issues all its TMEM reads, waits once,
    // releases the slot and runs the chain; the sub-partition's other warps
    // cover the read latency.
    pdl_wait();  // bias and y only after the previous kernel of the stream
    const int q = warp & 3;                                      // TMEM lanes 32q .. 32q + 31
    const int t0 = ((warp - kRescaleWarp0) >> 2) * kTPT;         // first token column of this thread
    constexpr int kNCh = kTPT / 16;                              // 16-column chunks per block half
    constexpr int kMaxChunks = kNCh * SUB;                       // SUB 2: chunk c = tokens 16 (c / 2), half c % 2
    uint32_t kit = 0, bit = 0;
    for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
      const int tile = kPar ? item / n_par : item;
      int kb0, kb1, ks0, ks1;
      item_range(item, kb0, kb1, ks0, ks1);
      const int m0 = (tile % tiles_m) * kTok, n0 = (tile / tiles_m) * kRows;
      const int n = n0 + 32 * q + lane;
      const int live_tok = M - m0 - t0;  // tokens of this thread's columns inside M (may be <= 0)
      int nlive = live_tok <= 0 ? 0 : (live_tok + 15) / 16;
      if (nlive > kNCh) nlive = kNCh;
      const int nch = nlive * SUB;  // chunks holding tokens < M
      float acc[kTPT], tot[kSplit ? kTPT : 1];
#pragma unroll
      for (int i = 0; i < kTPT; ++i) acc[i] = 0.0f;
#pragma unroll
      for (int i = 0; i < (kSplit ? kTPT : 1); ++i) tot[i] = 0.0f;
      const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
      for (int kb = kb0; kb < kb1 && ok; ++kb, ++bit) {
        const int j = kb % kBlocks;
        const int si = kit % kSStages;
        if (j == 0) {
          // a new scale stage: visible to this thread once it observed sfull itself
          if (!mbar_wait(&sm.sfull[si], (kit / kSStages) & 1, kDevErrFullBarrierTimeout)) { ok = false; break; }
        }
        const uint32_t sa_base = smem_u32(sm.scale0 + si * T::kScaleBytes);
        const int slot = bit % kSlots;
        if (!mbar_wait(&sm.dfull[slot], (bit / kSlots) & 1, kDevErrEpilogueBarrierTimeout)) { ok = false; break; }
        tc::tc_fence_after();
        uint32_t d[kMaxChunks][16];
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c) {
          const int col = SUB == 1 ? t0 + 16 * c : (c & 1) * kTok + t0 + 16 * (c >> 1);
          if (c < nch) tc::tmem_ld16_nowait(lane_base + slot * kCols + col, d[c]);
        }
        float sbv[SUB];  // this row's weight scales for the block (zero past N or K)
        {
          const uint32_t a = sa_base + T::kSaBytes + (uint32_t)(((32 * q + lane) * kSPS + SUB * j) * 4);
          sbv[0] = lds_f32(a);
          if (SUB == 2) sbv[SUB - 1] = lds_f32(a + 4);
        }
        if constexpr (kSplit) {
          if (kb > 0 && kb % split_blocks == 0) {  // a new split's chain starts at 0
#pragma unroll
            for (int i = 0; i < kTPT; ++i) {
              tot[i] = __fadd_rn(tot[i], acc[i]);
              acc[i] = 0.0f;
            }
          }
        }
        tc::tmem_wait_ld();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.dempty[slot]);
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c) {
          if (c < nch) {
            const int tc0 = SUB == 1 ? 16 * c : 16 * (c >> 1);     // first token of the chunk (thread-relative)
            const int sidx = SUB * j + (SUB == 2 ? (c & 1) : 0);  // scale index within the stage
            const float sb = sbv[SUB == 2 ? (c & 1) : 0];
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              chain4(acc + tc0 + i, d[c] + i, lds_f32x4(sa_base + (uint32_t)((sidx * kTok + t0 + tc0 + i) * 4)), sb);
          }
        }
        if (j == kBlocks - 1 || kb + 1 == kb1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.sempty[si]);
          ++kit;
        }
      }
      if (!ok) break;
      if (n < N) {
        if constexpr (kPar) {
          float* part = reinterpret_cast<float*>(y) + (size_t)(item % n_par) * M * N;
#pragma unroll
          for (int i = 0; i < kTPT; ++i) {
            const int m = m0 + t0 + i;
            if (m < M) part[(size_t)m * N + n] = acc[i];
          }
        } else {
          const float b = bias != nullptr ? to_f32(bias[n]) : 0.0f;
#pragma unroll
          for (int i = 0; i < kTPT; ++i) {
            const int m = m0 + t0 + i;
            if (m < M) {
              float v = acc[i];
              if constexpr (kSplit) v = __fadd_rn(tot[i], acc[i]);
              if (bias != nullptr) v = __fadd_rn(v, b);
              y[(size_t)m * N + n] = from_f32<OutT>(v);
            }
          }
        }
      }
    }
  }

  if (!ok) mirror_device_error(status_host);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == kMmaWarp) tc::tmem_dealloc<1>(tmem, T::kTmemCols);
}

}  // namespace w4a4x

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {



// The reference's split-K plan (binding.cpp:24-43): split only when its
// 64 x 64 output tiles cannot fill 2 work-groups per compute unit; then aim
// for ~2.4 waves, at most 8 splits and at least 8 K-stages of 128 per split.
// The split count is part of the numerics (each split's chain starts at 0),
// so it is computed exactly as the reference computes it on this device.
int reference_auto_splits(int M, int N, int K, int sms) {
  const int tiles = ((M + 63) / 64) * ((N + 63) / 64);
  const int slots = sms * 2;
  if (tiles >= slots) return 1;
  const int k_tiles = (K / 32 + 3) / 4;
  int max_splits = k_tiles / 8;
  if (max_splits < 1) max_splits = 1;
  if (max_splits > 8) max_splits = 8;
  const int wanted = (12 * slots + 5 * tiles - 1) / (5 * tiles);
  return wanted < max_splits ? wanted : max_splits;
}

template <typename OutT, int SUB, int kMode>
int launch_kernel(const void* a8, const float* sat, const void* b_q4, const float* b_scale, const void* bias, void* y,
                  int M, int N, int K, int Mp, int Sp, int split_blocks, int n_par, cudaStream_t st, int sms) {
  using T = w4a4x::Cfg<SUB, kMode == 1>;
  const int S = K * SUB / 32;
  CUtensorMap am, am2, qm, smap;
  int rc = cached_tmap_2d(&am, CU_TENSOR_MAP_DATA_TYPE_UINT8, a8, (uint64_t)K, (uint64_t)M, (uint64_t)K,
                          w4a4x::kStageK, T::kTok, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  am2 = am;
  if (SUB == 2) {
    rc = cached_tmap_2d(&am2, CU_TENSOR_MAP_DATA_TYPE_UINT8, static_cast<const uint8_t*>(a8) + (size_t)M * K,
                        (uint64_t)K, (uint64_t)M, (uint64_t)K, w4a4x::kStageK, T::kTok, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  rc = cached_tmap_2d(&qm, CU_TENSOR_MAP_DATA_TYPE_UINT8, b_q4, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                      w4a4x::kStageK / 2, w4a4x::kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  // dim 0 = the M real tokens (the TMA fills tokens >= M with zeros), rows Mp apart
  rc = cached_tmap_2d(&smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, sat, (uint64_t)M, (uint64_t)S, (uint64_t)Mp * 4,
                      T::kTok, T::kScalesPerStage, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  // weight scales [N, S] (rows Sp floats apart): one box of the stage's scales x 128 rows
  CUtensorMap sbm;
  rc = cached_tmap_2d(&sbm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, b_scale, (uint64_t)S, (uint64_t)N, (uint64_t)Sp * 4,
                      T::kScalesPerStage, w4a4x::kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  auto kern = w4a4x::w4a4x_kernel<OutT, SUB, kMode>;
  static bool attr_set[64] = {false};
  const int dev = current_device();
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T::kSmemBytes);
    if (e != cudaSuccess)
      return set_error(GFX_ERR_CUDA, "w4a4_exact: cannot set %d bytes of shared memory: %s", T::kSmemBytes,
                       cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int tiles = ((M + T::kTok - 1) / T::kTok) * ((N + w4a4x::kRows - 1) / w4a4x::kRows) * n_par;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(tiles < sms ? tiles : sms);
  cfg.blockDim = dim3(w4a4x::kThreads);
  cfg.dynamicSmemBytes = T::kSmemBytes;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, am, am2, qm, smap, sbm, (const OutT*)bias, (OutT*)y, M, N, K,
                                     split_blocks, n_par, host_status_word(dev));
  if (e != cudaSuccess) return set_error(GFX_ERR_CUDA, "w4a4x_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("w4a4x_kernel");
}

template <int SUB, int kMode>
int launch_out(int out_dtype, const void* a8, const float* sat, const void* b_q4, const float* b_scale,
               const void* bias, void* y, int M, int N, int K, int Mp, int Sp, int split_blocks, int n_par,
               cudaStream_t st, int sms) {
  if constexpr (kMode == 2) {  // slice partials are fp32
    return launch_kernel<float, SUB, 2>(a8, sat, b_q4, b_scale, bias, y, M, N, K, Mp, Sp, split_blocks, n_par, st,
                                        sms);
  } else {
    if (out_dtype == GFX_DTYPE_F32)
      return launch_kernel<float, SUB, kMode>(a8, sat, b_q4, b_scale, bias, y, M, N, K, Mp, Sp, split_blocks, n_par,
                                              st, sms);
    if (out_dtype == GFX_DTYPE_F16)
      return launch_kernel<__half, SUB, kMode>(a8, sat, b_q4, b_scale, bias, y, M, N, K, Mp, Sp, split_blocks, n_par,
                                               st, sms);
    return launch_kernel<__nv_bfloat16, SUB, kMode>(a8, sat, b_q4, b_scale, bias, y, M, N, K, Mp, Sp, split_blocks,
                                                    n_par, st, sms);
  }
}

template <typename OutT>
int launch_reduce(const float* part, int P, const void* bias, void* y, int M, int N, cudaStream_t st) {
  const long n = (long)M * N;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3((unsigned)((n + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, w4a4x::split_reduce_kernel<OutT>, part, P, (const OutT*)bias, (OutT*)y, M,
                                     N);
  if (e != cudaSuccess) return set_error(GFX_ERR_CUDA, "split_reduce_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("split_reduce_kernel");
}

// Partial sums of parallel slices are kept when all 8 possible slices fit in this many bytes.
constexpr size_t kMaxPartialBytes = 64ull << 20;

struct Layout {
  // byte offsets: e5m2 A copies, transposed A scales, padded B scales, slice partials
  size_t a8, sat, sbp, part, total;
};

Layout workspace_layout(int M, int N, int K, int qblock, bool pad_b) {
  const int sub = qblock == 16 ? 2 : 1;
  const size_t S = (size_t)K * sub / 32, Sp = (S + 3) / 4 * 4, Mp = (size_t)((M + 3) & ~3);
  Layout l;
  l.a8 = 0;
  l.sat = align_up((size_t)sub * M * K, 1024);
  l.sbp = align_up(l.sat + S * Mp * 4, 1024);
  l.part = align_up(l.sbp + (pad_b ? (size_t)N * Sp * 4 : 0), 1024);
  const size_t part_bytes = (size_t)8 * M * N * 4;
  l.total = l.part + (part_bytes <= kMaxPartialBytes ? part_bytes : 0);
  return l;
}

}  // namespace

size_t w4a4_exact_workspace(int M, int N, int K, int qblock) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int S = K * (qblock == 16 ? 2 : 1) / 32;
  // the padded weight-scale copy is sized in whenever it may be needed
  return workspace_layout(M, N, K, qblock, S % 4 != 0).total;
}

int w4a4_exact_splits(int M, int N, int K, int splits, int sms) {
  return splits == 0 ? reference_auto_splits(M, N, K, sms) : splits;
}

int launch_w4a4_exact(const void* a_q4, const float* a_scale, const void* b_q4, const float* b_scale, int qblock,
                      const void* bias, void* y, int out_dtype, int M, int N, int K, int splits, void* workspace,
                      cudaStream_t st, int sms) {
  const int sub = qblock == 16 ? 2 : 1;
  const int S = K * sub / 32, Sp = (S + 3) / 4 * 4;
  const int Mp = (M + 3) & ~3;
  // TMA needs weight-scale rows of a multiple of 16 bytes; otherwise a padded copy
  const bool pad_b = Sp != S;
  const Layout lay = workspace_layout(M, N, K, qblock, pad_b);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  uint8_t* a8 = base + lay.a8;
  float* sat = reinterpret_cast<float*>(base + lay.sat);
  const long blocks = (long)M * (K / 32);
  const unsigned grid = (unsigned)((blocks + 255) / 256);
  if (sub == 1) {
    w4a4x::e5m2_prepass_kernel<1><<<grid, 256, 0, st>>>((const uint4*)a_q4, (uint4*)a8, nullptr, blocks);
  } else {
    w4a4x::e5m2_prepass_kernel<2><<<grid, 256, 0, st>>>((const uint4*)a_q4, (uint4*)a8, (uint4*)(a8 + (size_t)M * K),
                                                         blocks);
  }
  int rc = check_launch("e5m2_prepass_kernel");
  if (rc) return rc;
  if (pad_b) {
    float* sbp = reinterpret_cast<float*>(base + lay.sbp);
    const long n = (long)N * Sp;
    w4a4x::scale_pad_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(b_scale, sbp, N, S, Sp);
    rc = check_launch("scale_pad_kernel");
    if (rc) return rc;
    b_scale = sbp;
  }
  w4a4x::scale_transpose_kernel<<<dim3((Mp + 31) / 32, (S + 31) / 32), dim3(32, 8), 0, st>>>(a_scale, sat, M, S, Mp);
  rc = check_launch("scale_transpose_kernel");
  if (rc) return rc;
  const int k_tiles = (K / 32 + 3) / 4;
  splits = w4a4_exact_splits(M, N, K, splits, sms);
  const int tps = (k_tiles + splits - 1) / splits;
  if (splits > 1 && tps < k_tiles) {
    const int sb = tps * w4a4x::kBlocks;
    const int n_par = (k_tiles + tps - 1) / tps;  // non-empty slices (an empty one adds +0.0: nothing)
    if (lay.total - lay.part >= (size_t)n_par * M * N * 4) {
      // small problems: slices as parallel work items, then the ordered reduction
      float* part = reinterpret_cast<float*>(base + lay.part);
      rc = sub == 1 ? launch_out<1, 2>(out_dtype, a8, sat, b_q4, b_scale, nullptr, part, M, N, K, Mp, Sp, sb, n_par,
                                       st, sms)
                    : launch_out<2, 2>(out_dtype, a8, sat, b_q4, b_scale, nullptr, part, M, N, K, Mp, Sp, sb, n_par,
                                       st, sms);
      if (rc) return rc;
      if (out_dtype == GFX_DTYPE_F32) return launch_reduce<float>(part, n_par, bias, y, M, N, st);
      if (out_dtype == GFX_DTYPE_F16) return launch_reduce<__half>(part, n_par, bias, y, M, N, st);
      return launch_reduce<__nv_bfloat16>(part, n_par, bias, y, M, N, st);
    }
    if (sub == 1)
      return launch_out<1, 1>(out_dtype, a8, sat, b_q4, b_scale, bias, y, M, N, K, Mp, Sp, sb, 1, st, sms);
    return launch_out<2, 1>(out_dtype, a8, sat, b_q4, b_scale, bias, y, M, N, K, Mp, Sp, sb, 1, st, sms);
  }
  if (sub == 1) return launch_out<1, 0>(out_dtype, a8, sat, b_q4, b_scale, bias, y, M, N, K, Mp, Sp, 0, 1, st, sms);
  return launch_out<2, 0>(out_dtype, a8, sat, b_q4, b_scale, bias, y, M, N, K, Mp, Sp, 0, 1, st, sms);
}

}  // namespace gfx
