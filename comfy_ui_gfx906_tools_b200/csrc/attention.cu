// Fused quantized attention, head dim 128, native GQA: the reference's
// attention_kernel (nodes/ComfyUI-Gfx906Int4/csrc/attention.hip:83-357,
// dispatch :373-382) behind the binding's attention() (binding.cpp:114-170).
//
// out[b, r, h, :] = softmax_2(s[r, :]) V with scores in log2 units (the
// softmax scale times log2(e) is folded into Q or its scale by the prepare
// step), one CTA per block of query rows of one head, looping over the
// 64-key tiles of that head's KV head (all of them, or those the optional
// keep mask marks for the block). Per key tile, as the reference:
//   s        = fp16:  q . k in fp32
//              int8 / int4: ((float)(integer q . k) * q_scale) * k_scale
//              (keys past Lk: -1e30)
//   m_new    = max(m, tile max); alpha = exp2(m - m_new); l *= alpha; o *= alpha
//   rel      = exp2(tile max - m_new)            (the row's largest P in the tile)
//   skip     = max of rel over the warp's 16 rows < skip_below
//   p        = exp2(s - m_new); l += p           (every key, skipped or not)
//   P.V      = fp16: o += (half)p . (half)v      (fp32 accumulation)
//              u8:   pq = rint(p * 255 / rel) in [0, 255], V stored + 128:
//                    o = fma(rel / 255 * v_scale, (float)(pq . vq) - 128 sum(pq), o)
//   (skipped tiles: no P.V)
// and at the end out = (half)(o / l).
//
// B200 design: the reference runs dot2/dot4/dot8 on the CUDA cores of a
// wave64 GPU; here both products run on the tensor cores with mma.sync:
// m16n8k32 s8 x s8 -> s32 for the integer Q.K (int4 codes are sign-extended
// to int8 in registers, exact), m16n8k16 f16 x f16 -> f32 for fp16 Q.K and
// fp16 P.V, m16n8k32 u8 x u8 -> s32 for the u8 P.V (exact integer sums, so the
// reference's fold above is reproduced operation for operation). One warp owns
// 16 query rows: the same 16 rows that one 64-lane wave of the reference owns
// (rows 4w + a + (BQ/4) i, a, i < 4), so the skip decision covers the same
// rows. Q fragments stay in registers for the whole key loop; K and V tiles
// (and their scales) are double-buffered in shared memory with cp.async, the
// next tile's copies in flight during this tile's math; P goes through a
// per-warp shared-memory tile into the P.V operand registers. The K index
// inside every 32-wide (16-wide for f16) MMA step is permuted alike for both
// operands so that each thread's two operand registers are one 8-byte load
// (a dot product does not depend on the order of its terms); row strides
// padded to 32 bytes mod 128 make those loads bank-conflict free.
#include "common.cuh"
#include "kernels.h"

namespace gfx {
namespace attn {

constexpr int kD = 128;
constexpr int kTile = 64;
constexpr float kNoScore = -1e30f;

enum { QK_F16 = 0, QK_I8 = 1, QK_I4 = 2 };
enum { PV_F16 = 0, PV_U8 = 1 };

template <int QK, int PV>
struct Cfg {
  static constexpr int kRows = QK == QK_F16 ? 64 : 128;  // query rows per CTA (= keep-mask block rows)
  static constexpr int kWarps = kRows / 16;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kRowBytes = QK == QK_F16 ? 2 * kD : (QK == QK_I8 ? kD : kD / 2);
  static constexpr int kKStride = kRowBytes + (QK == QK_I4 ? 16 : 32);
  static constexpr int kVRow = PV == PV_F16 ? 2 * kTile : kTile;  // bytes of one channel row of a V tile
  static constexpr int kVStride = kVRow + 32;
  static constexpr int kPStride = kVStride;                       // P rows: 64 keys, same element size as V
  static constexpr int kKSteps = QK == QK_F16 ? kD / 16 : kD / 32;
  static constexpr int kKBytes = kTile * kKStride;
  static constexpr int kVBytes = kD * kVStride;
  static constexpr int kOffV = 2 * kKBytes;
  static constexpr int kOffKs = kOffV + 2 * kVBytes;
  static constexpr int kOffVs = kOffKs + 2 * kTile * 4;
  static constexpr int kOffP = kOffVs + 2 * kD * 4;
  static constexpr int kOffKeep = kOffP + kWarps * 16 * kPStride;
  static constexpr int kSmem = kOffKeep + kAttentionMaxTiles / 8;
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void sts16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Four packed int4 codes of a 32-bit word's low (or high) nibbles -> four
// int8 bytes: n = nibble ^ 8 = code + 8 in [0, 15]; (n + 0x78) ^ 0x80 =
// n - 8 mod 256 per byte (no carry leaves a byte: n + 0x78 <= 0x87).
__device__ __forceinline__ uint32_t s8_from_nibbles(uint32_t nib) {
  return ((nib & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
}
__device__ __forceinline__ uint32_t s8_lo(uint32_t w) { return s8_from_nibbles(w ^ 0x88888888u); }
__device__ __forceinline__ uint32_t s8_hi(uint32_t w) { return s8_from_nibbles((w ^ 0x88888888u) >> 4); }

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

// Q [B, H, Lq, RB] bytes (RB = 256 fp16 / 128 int8 / 64 packed int4), q_scale
// [B, H, Lq] (int modes), K [B, KVH, Lk, RB], k_scale [B, KVH, Lk], Vt [B, KVH,
// n_tiles, 128, 64 * vbytes] (fp16, or u8 + 128), v_scale [B, KVH, n_tiles,
// 128] (u8), keep [B, H, ceil(Lq / kRows), n_tiles] or null, out [B, Lq, H, 128].
template <int QK, int PV>
__global__ void __launch_bounds__(Cfg<QK, PV>::kThreads, 1)
    attention_kernel(const uint8_t* __restrict__ Q, const float* __restrict__ q_scale, const uint8_t* __restrict__ K,
                     const float* __restrict__ k_scale, const uint8_t* __restrict__ Vt,
                     const float* __restrict__ v_scale, const uint8_t* __restrict__ keep, __half* __restrict__ out,
                     int H, int KVH, int Lq, int Lk, int n_tiles, float skip_below) {
  using C = Cfg<QK, PV>;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const int b = blockIdx.z, h = blockIdx.y, qb = blockIdx.x;
  const int kvh = h / (H / KVH);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;

  const uint8_t* Qg = Q + (size_t)(b * H + h) * Lq * C::kRowBytes;
  const uint8_t* Kg = K + (size_t)(b * KVH + kvh) * Lk * C::kRowBytes;
  const uint8_t* Vg = Vt + (size_t)(b * KVH + kvh) * n_tiles * kD * C::kVRow;
  const size_t ks_off = (size_t)(b * KVH + kvh) * Lk;
  const size_t vs_off = (size_t)(b * KVH + kvh) * n_tiles * kD;

  uint8_t* keep_s = smem + C::kOffKeep;
  if (keep) {
    const uint8_t* kg = keep + ((size_t)(b * H + h) * gridDim.x + qb) * n_tiles;
    for (int i = tid; i < (n_tiles + 7) / 8; i += C::kThreads) {
      uint32_t bits = 0;
      for (int j = 0; j < 8 && i * 8 + j < n_tiles; ++j) bits |= (uint32_t)(kg[i * 8 + j] != 0) << j;
      keep_s[i] = (uint8_t)bits;
    }
    __syncthreads();
  }
  auto next_tile = [&](int tt) {
    ++tt;
    while (keep && tt < n_tiles && !((keep_s[tt >> 3] >> (tt & 7)) & 1)) ++tt;
    return tt;
  };

  // Copies of one key tile (K rows, V tile, scales) into buffer `buf`.
  auto issue_tile = [&](int tt, int buf) {
    const int k0 = tt * kTile;
    uint8_t* Ks = smem + buf * C::kKBytes;
    constexpr int kKChunks = kTile * (C::kRowBytes / 16);
    for (int i = tid; i < kKChunks; i += C::kThreads) {
      const int r = i / (C::kRowBytes / 16), c = i % (C::kRowBytes / 16);
      const bool ok = k0 + r < Lk;
      cp_async_16(Ks + r * C::kKStride + c * 16, Kg + (size_t)(ok ? k0 + r : 0) * C::kRowBytes + c * 16, ok ? 16 : 0);
    }
    uint8_t* Vs = smem + C::kOffV + buf * C::kVBytes;
    const uint8_t* Vtile = Vg + (size_t)tt * kD * C::kVRow;
    constexpr int kVChunks = kD * (C::kVRow / 16);
    for (int i = tid; i < kVChunks; i += C::kThreads) {
      const int d = i / (C::kVRow / 16), c = i % (C::kVRow / 16);
      cp_async_16(Vs + d * C::kVStride + c * 16, Vtile + (size_t)d * C::kVRow + c * 16, 16);
    }
    if constexpr (QK != QK_F16) {
      float* kss = reinterpret_cast<float*>(smem + C::kOffKs) + buf * kTile;
      for (int i = tid; i < kTile; i += C::kThreads) {
        const bool ok = k0 + i < Lk;
        cp_async_4(kss + i, k_scale + ks_off + (ok ? k0 + i : 0), ok ? 4 : 0);
      }
    }
    if constexpr (PV == PV_U8) {
      float* vss = reinterpret_cast<float*>(smem + C::kOffVs) + buf * kD;
      for (int i = tid; i < kD; i += C::kThreads) cp_async_4(vss + i, v_scale + vs_off + (size_t)tt * kD + i, 4);
    }
    cp_async_commit();
  };

  int tcur = next_tile(-1);
  if (tcur < n_tiles) issue_tile(tcur, 0);

  // This thread's two query rows (local rows g and g + 8 of the warp's 16):
  // local row l is the reference's row ty + TY * i with ty = 4 * warp + (l & 3)
  // and i = l >> 2.
  constexpr int TY = C::kRows / 4;
  int rows[2];
  float qsc[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    rows[hh] = qb * C::kRows + 4 * warp + (g & 3) + TY * ((g >> 2) + 2 * hh);
    qsc[hh] = 1.0f;
    if constexpr (QK != QK_F16)
      if (rows[hh] < Lq) qsc[hh] = q_scale[(size_t)(b * H + h) * Lq + rows[hh]];
  }
  // Q fragments (A operand, rows g / g + 8), kept for the whole key loop.
  uint32_t qa[C::kKSteps][4];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const bool ok = rows[hh] < Lq;
    const uint8_t* qrow = Qg + (size_t)(ok ? rows[hh] : 0) * C::kRowBytes;
#pragma unroll
    for (int s = 0; s < C::kKSteps; ++s) {
      if constexpr (QK == QK_I4) {
        const uint32_t w = ok ? *reinterpret_cast<const uint32_t*>(qrow + 16 * s + 4 * t4) : 0u;
        qa[s][hh] = s8_lo(w);
        qa[s][2 + hh] = s8_hi(w);
      } else {
        const uint2 v = ok ? *reinterpret_cast<const uint2*>(qrow + 32 * s + 8 * t4) : make_uint2(0u, 0u);
        qa[s][hh] = v.x;
        qa[s][2 + hh] = v.y;
      }
    }
  }

  float o[kD / 8][4];
#pragma unroll
  for (int n = 0; n < kD / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.0f;
  float m[2] = {kNoScore, kNoScore}, l[2] = {0.0f, 0.0f};

  const uint32_t p_base = sbase + C::kOffP + warp * 16 * C::kPStride;
  int buf = 0;
  while (tcur < n_tiles) {
    const int k0 = tcur * kTile;
    const int tnext = next_tile(tcur);
    cp_async_wait_all();
    __syncthreads();  // tile tcur is in buffer buf; every warp is done with the other buffer
    if (tnext < n_tiles) issue_tile(tnext, buf ^ 1);

    // ---- S = Q K^T (16 rows x 64 keys per warp) ----
    float sc[8][4];
    const uint32_t kb = sbase + buf * C::kKBytes;
    if constexpr (QK == QK_F16) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[j][e] = 0.0f;
#pragma unroll
      for (int s = 0; s < C::kKSteps; ++s)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint2 kv = lds64(kb + (8 * j + g) * C::kKStride + 32 * s + 8 * t4);
          mma_f16(sc[j], qa[s], kv.x, kv.y);
        }
    } else {
      int acc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0;
#pragma unroll
      for (int s = 0; s < C::kKSteps; ++s)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if constexpr (QK == QK_I8) {
            const uint2 kv = lds64(kb + (8 * j + g) * C::kKStride + 32 * s + 8 * t4);
            mma_s8(acc[j], qa[s], kv.x, kv.y);
          } else {
            const uint32_t w = lds32(kb + (8 * j + g) * C::kKStride + 16 * s + 4 * t4);
            mma_s8(acc[j], qa[s], s8_lo(w), s8_hi(w));
          }
        }
      const uint32_t kss = sbase + C::kOffKs + buf * kTile * 4;
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float ksc = lds_f32(kss + (8 * j + 2 * t4 + c) * 4);
          sc[j][c] = __fmul_rn(__fmul_rn((float)acc[j][c], qsc[0]), ksc);
          sc[j][2 + c] = __fmul_rn(__fmul_rn((float)acc[j][2 + c], qsc[1]), ksc);
        }
    }
    float tmax[2] = {kNoScore, kNoScore};
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (k0 + 8 * j + 2 * t4 + (e & 1) >= Lk) sc[j][e] = kNoScore;
        tmax[e >> 1] = fmaxf(tmax[e >> 1], sc[j][e]);
      }

    // ---- online softmax ----
    float rel[2], pscale[2], inv[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      tmax[hh] = quad_max(tmax[hh]);
      const float m_new = fmaxf(m[hh], tmax[hh]);
      const float alpha = exp2f(m[hh] - m_new);
      m[hh] = m_new;
      l[hh] *= alpha;
#pragma unroll
      for (int n = 0; n < kD / 8; ++n) {
        o[n][2 * hh] *= alpha;
        o[n][2 * hh + 1] *= alpha;
      }
      rel[hh] = exp2f(tmax[hh] - m_new);
      pscale[hh] = rel[hh] * (1.0f / 255.0f);
      inv[hh] = rel[hh] > 1e-30f ? __fdiv_rn(255.0f, rel[hh]) : 0.0f;
    }
    float wrel = fmaxf(rel[0], rel[1]);
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) wrel = fmaxf(wrel, __shfl_xor_sync(0xffffffffu, wrel, off));
    const bool skip = wrel < skip_below;  // warp-uniform

    float qsum[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float p0 = exp2f(sc[j][2 * hh] - m[hh]);
        const float p1 = exp2f(sc[j][2 * hh + 1] - m[hh]);
        l[hh] += p0;
        l[hh] += p1;
        if (skip) continue;
        const uint32_t prow = p_base + (g + 8 * hh) * C::kPStride;
        if constexpr (PV == PV_F16) {
          const __half2 ph = __floats2half2_rn(p0, p1);
          sts32(prow + (8 * j + 2 * t4) * 2, *reinterpret_cast<const uint32_t*>(&ph));
        } else {
          const float q0 = rintf(p0 * inv[hh]), q1 = rintf(p1 * inv[hh]);
          qsum[hh] += q0;
          qsum[hh] += q1;
          sts16(prow + 8 * j + 2 * t4, (uint16_t)((uint32_t)q0 | ((uint32_t)q1 << 8)));
        }
      }

    // ---- O += P V ----
    if (!skip) {
      __syncwarp();
      const uint32_t vb = sbase + C::kOffV + buf * C::kVBytes;
      if constexpr (PV == PV_F16) {
        uint32_t pa[4][4];
#pragma unroll
        for (int s = 0; s < 4; ++s)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint2 v = lds64(p_base + (g + 8 * hh) * C::kPStride + 32 * s + 8 * t4);
            pa[s][hh] = v.x;
            pa[s][2 + hh] = v.y;
          }
#pragma unroll
        for (int n = 0; n < kD / 8; ++n)
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint2 vv = lds64(vb + (8 * n + g) * C::kVStride + 32 * s + 8 * t4);
            mma_f16(o[n], pa[s], vv.x, vv.y);
          }
      } else {
        const float pqs[2] = {quad_sum(qsum[0]), quad_sum(qsum[1])};
        uint32_t pa[2][4];
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint2 v = lds64(p_base + (g + 8 * hh) * C::kPStride + 32 * s + 8 * t4);
            pa[s][hh] = v.x;
            pa[s][2 + hh] = v.y;
          }
        const uint32_t vss = sbase + C::kOffVs + buf * kD * 4;
#pragma unroll
        for (int n = 0; n < kD / 8; ++n) {
          int acc[4] = {0, 0, 0, 0};
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const uint2 vv = lds64(vb + (8 * n + g) * C::kVStride + 32 * s + 8 * t4);
            mma_u8(acc, pa[s], vv.x, vv.y);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int hh = e >> 1;
            const float vsc = lds_f32(vss + (8 * n + 2 * t4 + (e & 1)) * 4);
            o[n][e] = fmaf(__fmul_rn(pscale[hh], vsc), __fsub_rn((float)acc[e], 128.0f * pqs[hh]), o[n][e]);
          }
        }
      }
      __syncwarp();
    }
    tcur = tnext;
    buf ^= 1;
  }

  // ---- out = o / l ----
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const float lt = quad_sum(l[hh]);
    if (rows[hh] >= Lq) continue;
    __half* dst = out + ((size_t)b * Lq + rows[hh]) * H * kD + (size_t)h * kD;
#pragma unroll
    for (int n = 0; n < kD / 8; ++n) {
      const __half2 v = __floats2half2_rn(__fdiv_rn(o[n][2 * hh], lt), __fdiv_rn(o[n][2 * hh + 1], lt));
      *reinterpret_cast<__half2*>(dst + 8 * n + 2 * t4) = v;
    }
  }
}

template <int QK, int PV>
static int launch(const void* q, const float* qs, const void* k, const float* ks, const void* vt, const float* vs,
                  const uint8_t* keep, void* out, int B, int H, int KVH, int Lq, int Lk, float skip_below,
                  cudaStream_t st) {
  using C = Cfg<QK, PV>;
  auto kern = attention_kernel<QK, PV>;
  static bool attr_set[64] = {false};  // the attribute belongs to the function's instance on each device
  const int dev = current_device();
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess)
      return set_error(GFX_ERR_CUDA, "attention: cannot set %d bytes of shared memory: %s", C::kSmem,
                       cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int n_tiles = (Lk + kTile - 1) / kTile;
  dim3 grid((Lq + C::kRows - 1) / C::kRows, H, B);
  kern<<<grid, C::kThreads, C::kSmem, st>>>((const uint8_t*)q, qs, (const uint8_t*)k, ks, (const uint8_t*)vt, vs, keep,
                                            (__half*)out, H, KVH, Lq, Lk, n_tiles, skip_below);
  return check_launch("attention_kernel");
}

}  // namespace attn

int attention_rows_per_block(int qk_mode) { return qk_mode == attn::QK_F16 ? 64 : 128; }

int launch_attention(int qk_mode, int pv_mode, const void* q, const float* q_scale, const void* k,
                     const float* k_scale, const void* vt, const float* v_scale, const uint8_t* keep, void* out,
                     int B, int H, int KVH, int Lq, int Lk, float skip_below, cudaStream_t st) {
  if (B == 0 || H == 0 || Lq == 0) return GFX_OK;
  if (attention_tc_selected(qk_mode, keep != nullptr))
    return launch_attention_tc(qk_mode, pv_mode, q, q_scale, k, k_scale, vt, v_scale, keep, out, B, H, KVH, Lq, Lk,
                               skip_below, st);
#define GFX_ATT_CASE(QKM, PVM)                                                                                    \
  if (qk_mode == QKM && pv_mode == PVM)                                                                           \
    return attn::launch<QKM, PVM>(q, q_scale, k, k_scale, vt, v_scale, keep, out, B, H, KVH, Lq, Lk, skip_below, \
                                  st);
  GFX_ATT_CASE(0, 0) GFX_ATT_CASE(0, 1) GFX_ATT_CASE(1, 0) GFX_ATT_CASE(1, 1) GFX_ATT_CASE(2, 0) GFX_ATT_CASE(2, 1)
#undef GFX_ATT_CASE
  return set_error(GFX_ERR_INVALID, "attention: bad modes qk=%d pv=%d", qk_mode, pv_mode);
}

}  // namespace gfx
