// Fused quantized attention on the 5th-generation tensor cores, every Q.K /
// P.V mode (fp16 Q.K keep masks come in 64-row blocks: a CTA visits the union
// of its two blocks' tiles and each warp only its own block's): the arithmetic of attention_kernel
// (nodes/ComfyUI-Gfx906Int4/csrc/attention.hip:83-357) as restated in
// attention.cu, with both products as tcgen05.mma and one thread per query
// row.
//
// CTA = 128 query rows of one head, 4 warps, thread t = TMEM lane t = row t
// of the Q tile (rows permuted so that the 16 lanes of each half-warp hold the
// 16 rows of one 64-lane wave of the reference: its skip groups). Per visited
// 64-key tile:
//   S  = Q K^T     tcgen05.mma.kind::i8 (s8 x s8 -> s32), M 128, N 64, K 4 x 32;
//                  Q (int8, or int4 codes sign-extended once) and K in shared
//                  memory, SWIZZLE_128B K-major; fp16 Q.K: kind::f16, K 8 x 16
//                  over two SWIZZLE_128B halves of the head dimension (rows
//                  grouped in the reference's 64-row fp16 blocks)
//   softmax        each thread loads its row of S (tcgen05.ld), scales,
//                  masks, updates m / l / alpha, decides the skip with its
//                  half-warp, writes its row of P (u8 levels or fp16) to shared
//                  memory in the MMA's SWIZZLE_128B layout
//   O_t = P V      u8: tcgen05.mma.kind::i8 (u8 x u8 -> s32), K 2 x 32;
//                  fp16: kind::f16 -> f32, K 4 x 16; M 128, N 128, in TMEM
//                  columns [128, 256); V tiles are channel-major [128, 64 keys]
//                  (the reference's Vt layout), i.e. K-major for the MMA
//   fold           each thread loads its row of O_t and folds it into its 128
//                  fp32 accumulators: u8 o = fma(rel/255 * v_scale,
//                  (float)acc - 128 sum(pq), o) exactly as the reference;
//                  fp16 o += O_t
// Pipelining: S_{t+1} is issued together with O_t (S double-buffered in TMEM
// columns [0, 64) / [64, 128)), so one block-wide barrier per tile suffices;
// tile t+2's K / V / scales are copied (cp.async; int4 K through registers,
// sign-extended on the way into shared memory) while tile t+1 is processed.
// Two CTAs per SM (256 TMEM columns each) overlap one CTA's CUDA-core
// softmax / fold with the other's MMAs. What bounds it (measured): the
// per-row CUDA-core chain (scale, max, exp2, levels, fold: ~1000
// instructions per row and tile) with two warps per SM sub-partition; the
// MMAs are short. Measured alternatives that were slower: two threads per row
// (halved chains, but an extra exchange barrier per tile and 128-register
// spills). Every mbarrier wait is bounded (common.cuh); a CTA whose
// wait gives up records the error, leaves its loop at the next block-wide
// barrier, frees its TMEM and exits.
#include <stdlib.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace gfx {

GFX_DEFINE_STATUS_READER(attn_tc_device_status)

namespace attn_tc {

constexpr int kD = 128;
constexpr int kTile = 64;
constexpr int kRows = 128;
constexpr int kThreads = 128;
constexpr float kNoScore = -1e30f;
constexpr int kTmemCols = 256;
constexpr int kTmemS = 0;     // S: two buffers of 64 int32 columns
constexpr int kTmemO = 128;   // O_t: 128 columns

template <int QK, int PV>
struct Cfg {
  // int8 Q / K tiles: one SW128 tile [rows][128 B]; fp16: two, one per 64-element half of the
  // head dimension. fp16 K is single-buffered (loaded once the previous S is done) so that two
  // CTAs still fit on an SM.
  static constexpr int kQHalf = kRows * 128;
  static constexpr int kKHalf = kTile * 128;
  static constexpr int kQBytes = QK == 0 ? 2 * kQHalf : kQHalf;
  static constexpr int kKBytes = QK == 0 ? 2 * kKHalf : kKHalf;  // one buffer
  static constexpr int kKBufs = QK == 0 ? 1 : 2;
  static constexpr int kVBytes = kD * 128;         // V tile: 128 channel rows of 128 B (u8 rows use half)
  static constexpr int kPBytes = kRows * 128;      // P tile
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;    // 2 buffers
  static constexpr int kOffV = kOffK + kKBufs * kKBytes;  // 2 buffers
  static constexpr int kOffP = kOffV + 2 * kVBytes;
  static constexpr int kOffKs = kOffP + kPBytes;   // 2 x 64 floats
  static constexpr int kOffVs = kOffKs + 2 * kTile * 4;  // 3 x 128 floats (the fold reads them one tile behind)
  static constexpr int kOffKeep = kOffVs + 3 * kD * 4;
  static constexpr int kOffBar = kOffKeep + 2 * kAttentionMaxTiles / 8;  // 2 mbarriers, TMEM base, fail flag
  static constexpr int kSmem = kOffBar + 64 + 1024;  // + alignment slack
  static constexpr int kVChunks = PV == 0 ? 8 : 4;   // 16-byte chunks per V / P row
};

// kind::i8 instruction descriptor: D s32, A / B s8 (1) or u8 (0), K-major, M 128.
__host__ __device__ constexpr uint32_t idesc_i8(int n, int a_signed, int b_signed) {
  return (2u << 4) | ((uint32_t)a_signed << 7) | ((uint32_t)b_signed << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kRows >> 4) << 24);
}
// kind::f16 instruction descriptor: D f32, A / B f16, K-major, M 128.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Byte offset of 16-byte chunk c of row r in a SWIZZLE_128B K-major tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t s8_from_nibbles(uint32_t nib) {
  return ((nib & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
}
// 16 packed int4 bytes (32 codes) -> 32 int8 bytes, both in the same order
// for Q and K: word w's low nibbles, then its high nibbles.
__device__ __forceinline__ void unpack_chunk(const uint4& p, uint4& a, uint4& b) {
  const uint32_t w[4] = {p.x ^ 0x88888888u, p.y ^ 0x88888888u, p.z ^ 0x88888888u, p.w ^ 0x88888888u};
  a = make_uint4(s8_from_nibbles(w[0]), s8_from_nibbles(w[0] >> 4), s8_from_nibbles(w[1]), s8_from_nibbles(w[1] >> 4));
  b = make_uint4(s8_from_nibbles(w[2]), s8_from_nibbles(w[2] >> 4), s8_from_nibbles(w[3]), s8_from_nibbles(w[3] >> 4));
}

// 2^x by the hardware approximation with subnormal results flushed to zero
// (weights below 2^-126 of the row maximum; the reference's kernel rounds the
// same values to subnormals, a difference far below the fp16 output's ulp).
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 columns of this warp's 32 TMEM lanes, without waiting (tc::tmem_wait_ld waits for all).
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// max(a, b, c): one three-input max (exact, like two two-input ones).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int QK, int PV>
__global__ void __launch_bounds__(kThreads, 2)
    attention_tc_kernel(const uint8_t* __restrict__ Q, const float* __restrict__ q_scale,
                        const uint8_t* __restrict__ K, const float* __restrict__ k_scale,
                        const uint8_t* __restrict__ Vt, const float* __restrict__ v_scale,
                        const uint8_t* __restrict__ keep, __half* __restrict__ out, int H, int KVH, int Lq, int Lk,
                        int n_tiles, float skip_below, int* status_host) {
  using C = Cfg<QK, PV>;
  constexpr int RB = QK == 0 ? 256 : (QK == 1 ? 128 : 64);  // global Q / K row bytes
  constexpr int VROW = PV == 0 ? 128 : 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 2);
  volatile int* s_fail = reinterpret_cast<volatile int*>(bar_s + 3);
  uint8_t* keep_s = smem + C::kOffKeep;

  const int b = blockIdx.z, h = blockIdx.y, qb = blockIdx.x;
  const int kvh = h / (H / KVH);
  const int tid = threadIdx.x, warp = tid >> 5;
  const uint8_t* Qg = Q + (size_t)(b * H + h) * Lq * RB;
  const uint8_t* Kg = K + (size_t)(b * KVH + kvh) * Lk * RB;
  const uint8_t* Vg = Vt + (size_t)(b * KVH + kvh) * n_tiles * kD * VROW;
  const float* ksg = k_scale + (size_t)(b * KVH + kvh) * Lk;
  const float* vsg = PV == 1 ? v_scale + (size_t)(b * KVH + kvh) * n_tiles * kD : nullptr;

  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    *s_fail = 0;
    fence_barrier_init();
  }
  // keep bits: one mask block per CTA (int modes: 128 rows), or two (fp16 Q.K: blocks of 64
  // rows, the second at keep_s + kAttentionMaxTiles / 8, all clear past the last block)
  constexpr int kMaskBlocks = QK == 0 ? 2 : 1;
  if (keep) {
    const int n_qb = QK == 0 ? (Lq + 63) / 64 : (int)gridDim.x;
    for (int mb = 0; mb < kMaskBlocks; ++mb) {
      const int blk = kMaskBlocks * qb + mb;
      const uint8_t* kg = keep + ((size_t)(b * H + h) * n_qb + blk) * n_tiles;
      for (int i = tid; i < (n_tiles + 7) / 8; i += kThreads) {
        uint32_t bits = 0;
        for (int j = 0; j < 8 && i * 8 + j < n_tiles && blk < n_qb; ++j) bits |= (uint32_t)(kg[i * 8 + j] != 0) << j;
        keep_s[mb * (kAttentionMaxTiles / 8) + i] = (uint8_t)bits;
      }
    }
  }
  if (warp == 0) tc::tmem_alloc<1>(tmem_slot, kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_addr = (uint32_t)(32 * warp) << 16;

  // a tile is visited when any of the CTA's mask blocks keeps it; this thread's rows take part
  // when its own block does (fp16: warps 0-1 hold block 0, warps 2-3 block 1: warp-uniform)
  auto kept = [&](int mb, int tt) { return (keep_s[mb * (kAttentionMaxTiles / 8) + (tt >> 3)] >> (tt & 7)) & 1; };
  auto next_tile = [&](int tt) {
    ++tt;
    while (keep && tt < n_tiles && !(kept(0, tt) || (kMaskBlocks == 2 && kept(1, tt)))) ++tt;
    return tt;
  };
  const int my_block = QK == 0 ? (tid >> 6) : 0;

  // This thread's query row: lane t = 16 W + l holds the reference's row
  // ty + TY i of its block, ty = 4 W + (l & 3), i = l >> 2 (int modes: one
  // block of 128 rows, TY = 32; fp16: two blocks of 64 rows, TY = 16).
  const int lrow = QK == 0 ? 64 * (tid >> 6) + 4 * ((tid & 63) >> 4) + (tid & 3) + 16 * ((tid & 15) >> 2)
                           : 4 * (tid >> 4) + (tid & 3) + 32 * ((tid & 15) >> 2);
  const int row = qb * kRows + lrow;
  const bool row_ok = row < Lq;
  const float qsc = (QK != 0 && row_ok) ? q_scale[(size_t)(b * H + h) * Lq + row] : 1.0f;

  // Q tile: this thread's row into SW128 row tid (int4: sign-extended).
  {
    const uint8_t* src = Qg + (size_t)(row_ok ? row : 0) * RB;
    if constexpr (QK == 0) {
#pragma unroll
      for (int c = 0; c < 16; ++c)
        cp_async_16(smem + C::kOffQ + (c >> 3) * C::kQHalf + sw128_off(tid, c & 7), src + 16 * c, row_ok ? 16 : 0);
    } else if constexpr (QK == 1) {
#pragma unroll
      for (int c = 0; c < 8; ++c) cp_async_16(smem + C::kOffQ + sw128_off(tid, c), src + 16 * c, row_ok ? 16 : 0);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 p = row_ok ? ldg_nc_v4(src + 16 * c) : make_uint4(0u, 0u, 0u, 0u);  // padding rows: codes 0
        uint4 lo, hi;
        unpack_chunk(p, lo, hi);
        sts128(sb + C::kOffQ + sw128_off(tid, 2 * c), lo);
        sts128(sb + C::kOffQ + sw128_off(tid, 2 * c + 1), hi);
      }
    }
  }

  // int4 K: this thread's two packed chunks of a tile (row tid / 2, half tid % 2)
  uint4 kpre[2];
  auto load_k4 = [&](int tt) {
    const int r = tid >> 1, k0 = tt * kTile;
    const bool ok = k0 + r < Lk;
    const uint8_t* src = Kg + (size_t)(ok ? k0 + r : 0) * RB + 32 * (tid & 1);
#pragma unroll
    for (int j = 0; j < 2; ++j)
      kpre[j] = ok ? ldg_nc_v4(src + 16 * j) : make_uint4(0u, 0u, 0u, 0u);
  };
  auto store_k4 = [&](int buf) {
    const int r = tid >> 1;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint4 lo, hi;
      unpack_chunk(kpre[j], lo, hi);
      const int c = 4 * (tid & 1) + 2 * j;
      sts128(sb + C::kOffK + buf * C::kKBytes + sw128_off(r, c), lo);
      sts128(sb + C::kOffK + buf * C::kKBytes + sw128_off(r, c + 1), hi);
    }
  };
  // fp16 K tile tt into the single K buffer (its two halves); committed with the next group.
  auto load_k16 = [&](int tt) {
    const int k0 = tt * kTile;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = tid + kThreads * j, r = i >> 4, c = i & 15;
      const bool okr = k0 + r < Lk;
      cp_async_16(smem + C::kOffK + (c >> 3) * C::kKHalf + sw128_off(r, c & 7),
                  Kg + (size_t)(okr ? k0 + r : 0) * RB + 16 * c, okr ? 16 : 0);
    }
  };
  // Copies of tile tt into slot `slot`: K / V / k-scale buffers slot % 2, v-scales slot % 3
  // (fp16 K: only with with_k, into its single buffer).
  auto issue_tile = [&](int tt, int slot, bool with_k) {
    const int k0 = tt * kTile;
    const int buf = slot & 1;
    if constexpr (QK == 0) {
      if (with_k) load_k16(tt);
    } else if constexpr (QK == 1) {
      for (int i = tid; i < kTile * 8; i += kThreads) {
        const int r = i >> 3, c = i & 7;
        const bool ok = k0 + r < Lk;
        cp_async_16(smem + C::kOffK + buf * C::kKBytes + sw128_off(r, c), Kg + (size_t)(ok ? k0 + r : 0) * RB + 16 * c,
                    ok ? 16 : 0);
      }
    } else {
      load_k4(tt);
    }
    const uint8_t* vsrc = Vg + (size_t)tt * kD * VROW;
    for (int i = tid; i < kD * C::kVChunks; i += kThreads) {
      const int d = i / C::kVChunks, c = i % C::kVChunks;
      cp_async_16(smem + C::kOffV + buf * C::kVBytes + sw128_off(d, c), vsrc + (size_t)d * VROW + 16 * c, 16);
    }
    if constexpr (QK != 0) {
      float* kss = reinterpret_cast<float*>(smem + C::kOffKs) + buf * kTile;
      if (tid < kTile) cp_async_4(kss + tid, ksg + (k0 + tid < Lk ? k0 + tid : 0), k0 + tid < Lk ? 4 : 0);
    }
    if constexpr (PV == 1) {
      float* vss = reinterpret_cast<float*>(smem + C::kOffVs) + (slot % 3) * kD;
      cp_async_4(vss + tid, vsg + (size_t)tt * kD + tid, 4);
    }
    cp_async_commit();
  };

  float2 o[kD / 2];  // this row's accumulators, channel pairs
#pragma unroll
  for (int i = 0; i < kD / 2; ++i) o[i] = make_float2(0.0f, 0.0f);
  float m = kNoScore, l = 0.0f;

  __syncthreads();  // keep bits visible
  auto issue_s = [&](int slot) {  // S of the tile in slot `slot`: K buffer and S columns slot % 2
    if constexpr (QK == 0) {  // fp16: 8 x K = 16, two 64-element halves of the head dimension
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint64_t qd = tc::sw128_desc(sb + C::kOffQ + (s >> 2) * C::kQHalf);
        const uint64_t kd = tc::sw128_desc(sb + C::kOffK + (s >> 2) * C::kKHalf);
        tc::umma_f16<1>(tmem + kTmemS + 64 * (slot & 1), qd + (uint64_t)(2 * (s & 3)), kd + (uint64_t)(2 * (s & 3)),
                        idesc_f16(kTile), s > 0);
      }
    } else {
      const uint64_t qd = tc::sw128_desc(sb + C::kOffQ);
      const uint64_t kd = tc::sw128_desc(sb + C::kOffK + (slot & 1) * C::kKBytes);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        umma_i8(tmem + kTmemS + 64 * (slot & 1), qd + (uint64_t)(2 * s), kd + (uint64_t)(2 * s),
                idesc_i8(kTile, 1, 1), s > 0);
    }
    tc::umma_commit<1>(bar_s);
  };
  int tcur = next_tile(-1);
  bool ok = true;
  if (tcur < n_tiles) {
    issue_tile(tcur, 0, true);
    cp_async_wait_all();
    if constexpr (QK == 2) store_k4(0);
    fence_proxy_async();  // Q / K writes -> visible to the tensor core
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (tid == 0) issue_s(0);
    __syncwarp();
    const int t1 = next_tile(tcur);
    if (t1 < n_tiles) issue_tile(t1, 1, false);
  }
  uint32_t it = 0, oit = 0;
  while (tcur < n_tiles) {
    const int nvalid = Lk - tcur * kTile;  // keys of this tile inside Lk (>= 1)
    const int tnext = next_tile(tcur);
    const int buf = it & 1;
    ok = __all_sync(0xffffffffu, mbar_wait(bar_s, it & 1, kDevErrMmaBarrierTimeout)) && ok;  // warp-uniform
    tc::tc_fence_after();
    if constexpr (QK == 0) {  // S_t is done with the single fp16 K buffer: bring in K_{t+1}
      if (tnext < n_tiles && ok) {
        load_k16(tnext);
        cp_async_commit();
      }
    }

    float p[kTile];
    bool skip = true;
    float pscale = 0.0f, pqsum = 0.0f;
    // rows whose mask block does not keep this tile leave it out entirely (m, l, o unchanged,
    // no fold), as the reference's block that never visits it
    const bool visit = !keep || kept(my_block, tcur);
    if (ok && visit) {
      // scores: ((float)dot * q_scale) * k_scale, each product rounded as the
      // reference; |dot| <= 128^3 < 2^22, so 1.5 * 2^23 + dot is exact and
      // its float bits minus 1.5 * 2^23 give (float)dot without a conversion
      uint32_t sraw[32];
      const float* kss = reinterpret_cast<const float*>(smem + C::kOffKs) + buf * kTile;
      const float2 qsc2 = make_float2(qsc, qsc);
      const float2 kMagicS = make_float2(-12582912.0f, -12582912.0f);
      float tm[4] = {kNoScore, kNoScore, kNoScore, kNoScore};
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        tc::tmem_ld32(tmem + lane_addr + kTmemS + 64 * buf + 32 * hf, sraw);
        if constexpr (QK == 0) {  // fp16 Q.K: the fp32 dot is the score (the scale is folded into Q)
#pragma unroll
          for (int j = 0; j < 32; ++j) p[32 * hf + j] = __uint_as_float(sraw[j]);
        } else {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 ks4 = *reinterpret_cast<const float4*>(kss + 32 * hf + j);
          float2 a = __fadd2_rn(make_float2(__int_as_float((int)sraw[j] + 0x4B400000),
                                            __int_as_float((int)sraw[j + 1] + 0x4B400000)), kMagicS);
          float2 c = __fadd2_rn(make_float2(__int_as_float((int)sraw[j + 2] + 0x4B400000),
                                            __int_as_float((int)sraw[j + 3] + 0x4B400000)), kMagicS);
          a = __fmul2_rn(__fmul2_rn(a, qsc2), make_float2(ks4.x, ks4.y));
          c = __fmul2_rn(__fmul2_rn(c, qsc2), make_float2(ks4.z, ks4.w));
          const int key = 32 * hf + j;
          p[key] = a.x;
          p[key + 1] = a.y;
          p[key + 2] = c.x;
          p[key + 3] = c.y;
        }
        }
      }
      if (nvalid < kTile) {  // the last tile only (uniform over the CTA): keys past Lk score -1e30
#pragma unroll
        for (int key = 0; key < kTile; ++key)
          if (key >= nvalid) p[key] = kNoScore;
      }
#pragma unroll
      for (int key = 0; key < kTile; key += 2) tm[(key >> 1) & 3] = max3f(tm[(key >> 1) & 3], p[key], p[key + 1]);
      const float tmax = fmaxf(fmaxf(tm[0], tm[1]), fmaxf(tm[2], tm[3]));
      const float m_new = fmaxf(m, tmax);
      const float alpha = ex2_ftz(m - m_new);
      m = m_new;
      if (alpha != 1.0f) {  // (x * 1 = x: skipping it changes nothing)
        l *= alpha;
        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
        for (int i = 0; i < kD / 2; ++i) o[i] = __fmul2_rn(o[i], a2);
      }
      const float rel = ex2_ftz(tmax - m_new);
      float grel = rel;
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) grel = fmaxf(grel, __shfl_xor_sync(0xffffffffu, grel, off));
      skip = grel < skip_below;  // uniform over the half-warp (the reference's wave)
      pscale = rel * (1.0f / 255.0f);
      const float inv = rel > 1e-30f ? __fdiv_rn(255.0f, rel) : 0.0f;
      const float2 mm = make_float2(-m, -m);
      float2 ls = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int key = 0; key < kTile; key += 2) {
        const float2 d = __fadd2_rn(make_float2(p[key], p[key + 1]), mm);
        p[key] = ex2_ftz(d.x);
        p[key + 1] = ex2_ftz(d.y);
        ls = __fadd2_rn(ls, make_float2(p[key], p[key + 1]));
      }
      l += ls.x + ls.y;
      // P row (skipped rows store whatever: their O_t row is not folded)
      const uint32_t prow = sb + C::kOffP;
      if constexpr (PV == 1) {
        // level = rint(p * 255 / rel): t + 2^23 rounds t (< 2^23) to the
        // nearest integer, ties to even, and leaves it in the low mantissa bits
        const float2 inv2 = make_float2(inv, inv);
        const float2 k23 = make_float2(8388608.0f, 8388608.0f);
        uint32_t lsum = 0;  // sum of the levels, four bytes at a time
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int key = 16 * c + 4 * q;
            const float2 m01 = __fadd2_rn(__fmul2_rn(make_float2(p[key], p[key + 1]), inv2), k23);
            const float2 m23 = __fadd2_rn(__fmul2_rn(make_float2(p[key + 2], p[key + 3]), inv2), k23);
            const uint32_t x = prmt(__float_as_uint(m01.x), __float_as_uint(m01.y), 0x0040u);
            const uint32_t y = prmt(__float_as_uint(m23.x), __float_as_uint(m23.y), 0x0040u);
            w[q] = prmt(x, y, 0x5410u);
            lsum = __dp4a(w[q], 0x01010101u, lsum);
          }
          sts128(prow + sw128_off(tid, c), make_uint4(w[0], w[1], w[2], w[3]));
        }
        pqsum = (float)lsum;  // <= 64 * 255: exact
      } else {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const __half2 hv = __floats2half2_rn(p[8 * c + 2 * q], p[8 * c + 2 * q + 1]);
            w[q] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          sts128(prow + sw128_off(tid, c), make_uint4(w[0], w[1], w[2], w[3]));
        }
      }
    }
    // the next tile's copies (issued one tile ago) must have landed for S_{t+1}
    cp_async_wait_all();
    if constexpr (QK == 2) {
      if (tnext < n_tiles) store_k4((it + 1) & 1);
    }
    fence_proxy_async();  // P, K writes of this thread -> visible to the tensor core
    if (!ok) *s_fail = 1;
    tc::tc_fence_before();
    const int any_run = __syncthreads_or(!skip);
    tc::tc_fence_after();
    if (*s_fail) break;

    // ---- S_{t+1} = Q K_{t+1}^T and O_t = P V_t ----
    if (tid == 0) {
      if (tnext < n_tiles) issue_s(it + 1);
      if (any_run) {
        const uint64_t pd = tc::sw128_desc(sb + C::kOffP);
        const uint64_t vd = tc::sw128_desc(sb + C::kOffV + buf * C::kVBytes);
        if constexpr (PV == 1) {
#pragma unroll
          for (int s = 0; s < 2; ++s)
            umma_i8(tmem + kTmemO, pd + (uint64_t)(2 * s), vd + (uint64_t)(2 * s), idesc_i8(kD, 0, 0), s > 0);
        } else {
#pragma unroll
          for (int s = 0; s < 4; ++s)
            tc::umma_f16<1>(tmem + kTmemO, pd + (uint64_t)(2 * s), vd + (uint64_t)(2 * s), idesc_f16(kD), s > 0);
        }
        tc::umma_commit<1>(bar_o);
      }
    }
    __syncwarp();
    if (any_run) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar_o, oit & 1, kDevErrMmaBarrierTimeout));
      ++oit;
      tc::tc_fence_after();
      if (ok) {  // the whole warp loads (tcgen05.ld is .sync.aligned); skipped half-warps do not fold
        const float* vss = reinterpret_cast<const float*>(smem + C::kOffVs) + (it % 3) * kD;
        // o = fma(rel/255 * v_scale, (float)acc - 128 sum(pq), o): 2^23 + acc
        // (acc < 2^23) minus 2^23 + 128 sum(pq) is that difference, exactly
        const float2 nb = make_float2(-(8388608.0f + 128.0f * pqsum), -(8388608.0f + 128.0f * pqsum));
        const float2 ps2 = make_float2(pscale, pscale);
#pragma unroll
        for (int cp = 0; cp < 4; cp += 2) {
          uint32_t rw[2][32];  // two 32-column chunks in flight, one wait
          tmem_ld32_nowait(tmem + lane_addr + kTmemO + 32 * cp, rw[0]);
          tmem_ld32_nowait(tmem + lane_addr + kTmemO + 32 * cp + 32, rw[1]);
          tc::tmem_wait_ld();
          if (skip) continue;
#pragma unroll
          for (int jj = 0; jj < 64; jj += 4) {
          const int cc = cp + (jj >> 5), j = jj & 31;
          const uint32_t* raw = rw[jj >> 5];
          {
            const int i = 16 * cc + j / 2;  // channel pair index
            if constexpr (PV == 1) {
              const float4 v4 = *reinterpret_cast<const float4*>(vss + 32 * cc + j);
              const float2 d01 = __fadd2_rn(make_float2(__int_as_float((int)raw[j] + 0x4B000000),
                                                        __int_as_float((int)raw[j + 1] + 0x4B000000)), nb);
              const float2 d23 = __fadd2_rn(make_float2(__int_as_float((int)raw[j + 2] + 0x4B000000),
                                                        __int_as_float((int)raw[j + 3] + 0x4B000000)), nb);
              o[i] = __ffma2_rn(__fmul2_rn(ps2, make_float2(v4.x, v4.y)), d01, o[i]);
              o[i + 1] = __ffma2_rn(__fmul2_rn(ps2, make_float2(v4.z, v4.w)), d23, o[i + 1]);
            } else {
              o[i] = __fadd2_rn(o[i], make_float2(__uint_as_float(raw[j]), __uint_as_float(raw[j + 1])));
              o[i + 1] = __fadd2_rn(o[i + 1], make_float2(__uint_as_float(raw[j + 2]), __uint_as_float(raw[j + 3])));
            }
          }
          }
        }
      }
    }
    // tile t+2's copies: K / V / k-scale buffer `buf` (S_t and O_t are done), v-scales (it + 2) % 3
    if (tnext < n_tiles) {
      const int tnn = next_tile(tnext);
      if (tnn < n_tiles) issue_tile(tnn, it + 2, false);
    }
    tcur = tnext;
    ++it;
  }

  cp_async_wait_all();
  if (!ok) {
    mirror_device_error(status_host);
    *s_fail = 1;
  }
  tc::tc_fence_before();
  __syncthreads();  // every thread's failure flag is visible
  tc::tc_fence_after();
  if (row_ok && !*s_fail) {
    __half* dst = out + ((size_t)b * Lq + row) * H * kD + (size_t)h * kD;
#pragma unroll
    for (int c = 0; c < kD / 8; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 v = o[4 * c + q];
        const __half2 hv = __floats2half2_rn(__fdiv_rn(v.x, l), __fdiv_rn(v.y, l));
        w[q] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 0) tc::tmem_dealloc<1>(tmem, kTmemCols);
}

template <int QK, int PV>
static int launch(const void* q, const float* qs, const void* k, const float* ks, const void* vt, const float* vs,
                  const uint8_t* keep, void* out, int B, int H, int KVH, int Lq, int Lk, float skip_below,
                  cudaStream_t st) {
  using C = Cfg<QK, PV>;
  auto kern = attention_tc_kernel<QK, PV>;
  static bool attr_set[64] = {false};
  const int dev = current_device();
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess)
      return set_error(GFX_ERR_CUDA, "attention: cannot set %d bytes of shared memory: %s", C::kSmem,
                       cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int n_tiles = (Lk + kTile - 1) / kTile;
  dim3 grid((Lq + kRows - 1) / kRows, H, B);
  kern<<<grid, kThreads, C::kSmem, st>>>((const uint8_t*)q, qs, (const uint8_t*)k, ks, (const uint8_t*)vt, vs, keep,
                                         (__half*)out, H, KVH, Lq, Lk, n_tiles, skip_below, host_status_word(dev));
  return check_launch("attention_tc_kernel");
}

}  // namespace attn_tc

// The tensor-core kernel for every mode unless GFX906_B200_ATTN_MMA_SYNC is set
// to a nonzero value (then the mma.sync kernel of attention.cu runs).
bool attention_tc_selected(int qk_mode, bool keep) {
  (void)qk_mode;
  (void)keep;
  const char* e = getenv("GFX906_B200_ATTN_MMA_SYNC");
  return !(e && atoi(e) != 0);
}

int launch_attention_tc(int qk_mode, int pv_mode, const void* q, const float* q_scale, const void* k,
                        const float* k_scale, const void* vt, const float* v_scale, const uint8_t* keep, void* out,
                        int B, int H, int KVH, int Lq, int Lk, float skip_below, cudaStream_t st) {
  if (B == 0 || H == 0 || Lq == 0) return GFX_OK;
  if (qk_mode == 0 && pv_mode == 0)
    return attn_tc::launch<0, 0>(q, q_scale, k, k_scale, vt, v_scale, keep, out, B, H, KVH, Lq, Lk, skip_below, st);
  if (qk_mode == 0 && pv_mode == 1)
    return attn_tc::launch<0, 1>(q, q_scale, k, k_scale, vt, v_scale, keep, out, B, H, KVH, Lq, Lk, skip_below, st);
  if (qk_mode == 1 && pv_mode == 0)
    return attn_tc::launch<1, 0>(q, q_scale, k, k_scale, vt, v_scale, keep, out, B, H, KVH, Lq, Lk, skip_below, st);
  if (qk_mode == 1 && pv_mode == 1)
    return attn_tc::launch<1, 1>(q, q_scale, k, k_scale, vt, v_scale, keep, out, B, H, KVH, Lq, Lk, skip_below, st);
  if (qk_mode == 2 && pv_mode == 0)
    return attn_tc::launch<2, 0>(q, q_scale, k, k_scale, vt, v_scale, keep, out, B, H, KVH, Lq, Lk, skip_below, st);
  if (qk_mode == 2 && pv_mode == 1)
    return attn_tc::launch<2, 1>(q, q_scale, k, k_scale, vt, v_scale, keep, out, B, H, KVH, Lq, Lk, skip_below, st);
  return set_error(GFX_ERR_INVALID, "attention: bad modes qk=%d pv=%d", qk_mode, pv_mode);
}

}  // namespace gfx
