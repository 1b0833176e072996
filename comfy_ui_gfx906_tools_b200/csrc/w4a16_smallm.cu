// W4A16 small-M GEMM (M <= 64): the HBM-bound weight stream, stream-K.
//
// y[M, N] = x[M, K] @ (code[N, K] * scale[N, K/32])^T (+ bias), x bf16.
//
// Reference counterpart: int4_gemm_kernel + splitk_reduce_kernel
// (nodes/ComfyUI-Gfx906Int4/csrc/int4_gemm_scaled.hip:53-191) as called from
// gemm_int4 (binding.cpp:73-112) with split-K for narrow problems
// (auto_splits, binding.cpp:36-43). Same weight layout and scale format; the
// design is B200-first:
//
//  * Work is a grid of units (128 weight rows x 256 K). CTA c of G takes the
//    contiguous unit range [c*U/G, (c+1)*U/G) in row-block-major order
//    ("stream-K"): every CTA streams the same number of weight bytes, so there
//    is no partial last wave. A split count S is the special case
//    G = row_blocks * S (each row block cut into S equal K segments); the host
//    plan picks it whenever a divisor S of the row block's unit count fills at
//    least 90% of the resident CTA slots (one segment end per CTA), and
//    stream-K otherwise.
//  * One producer warp streams each unit's nibbles (TMA, SWIZZLE_128B), group
//    scales (TMA when the scale row stride is 16-byte aligned, else cp.async)
//    and the matching 256-wide slice of the activations (TMA, SWIZZLE_128B
//    boxes) into a shared-memory ring.
//  * Eight consumer warps = 2 row slices (64 rows, 4 m16 tiles) x 4 K quarters
//    (one pair of 32-groups of the unit each), so one activation fragment feeds
//    64 weight rows (M <= 16; two CTAs per SM for M <= 8, one with 168
//    registers per thread for 8 < M <= 16; M > 16 uses 4 row slices of 2
//    tiles x 2 K halves). A warp reads one 32-bit nibble word per row and group
//    with ldmatrix (conflict-free through the swizzle) and turns each nibble
//    pair into bf16x2 "magic" values 128 + (code + 8) with one LOP3. The MMA
//    (mma.sync m16n8k16, weights = 16-row A, tokens = 8-column B) multiplies
//    those exact values; the +136 offset is removed by starting the group's
//    accumulator at -136 * sum(x) -- one extra MMA with a constant A operand,
//    shared by the warp's four m16 tiles. Each MMA pair covers exactly one
//    32-group, so its fp32 partial is scaled in registers (acc += p * scale).
//    No weight is ever rounded to bf16: products are exact and only the fp32
//    summation order differs from the fp32 dequant-then-matmul.
//  * When a CTA leaves a row block (segment end) the K quarters are summed
//    through shared memory. A row block covered by one CTA is stored directly
//    (+bias). Otherwise each segment writes its fp32 partial to the workspace
//    and bumps the row block's arrival counter; the last arrival (no spinning)
//    sums the segments in segment order -- deterministic -- adds the bias,
//    stores, and re-arms the counter to zero.
//
// Two index permutations keep every operand load a single instruction:
//  * K inside a 16-wide MMA step (both operands alike): k-slot (2t, 2t+1) of
//    step s holds group elements (8t + 2s, 8t + 2s + 4), slot (2t + 8, 2t + 9)
//    holds (8t + 2s + 1, 8t + 2s + 5) -- each A register is two nibbles of one
//    word, each B register two 16-bit halves of one 16-byte activation load.
//  * MMA column n reads token pi(n) = (n >> 1) | ((n & 1) << 2) of its 8-token
//    tile, so the two token rows a quarter-warp reads differ in swizzle bit 2
//    and the 16-byte activation loads are bank-conflict free; the epilogue
//    maps columns back through the same pi.
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace gfx {

namespace smallm {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kRows = 128;                      // weight rows per unit
constexpr int kStageK = 256;                    // K per unit
constexpr int kStageBytesPerRow = kStageK / 2;  // 128 nibble bytes = one SW128 row
constexpr int kGroupsPerStage = kStageK / 32;
constexpr int kConsumerBarrier = 1;             // named barrier id for the 256 consumer threads

// Build-time tuning (defaults are the shipped configuration).
#ifndef GFX_SMALLM_MT_NT1
#define GFX_SMALLM_MT_NT1 4   // m16 tiles per warp when M <= 8
#endif
#ifndef GFX_SMALLM_CTAS_PER_SM
#define GFX_SMALLM_CTAS_PER_SM 2  // resident CTAs per SM for M <= 8
#endif
#ifndef GFX_SMALLM_STAGES_F16
#define GFX_SMALLM_STAGES_F16 4   // smem ring depth, fp16 scales, M <= 8
#endif
#ifndef GFX_SMALLM_MT_NT2
#define GFX_SMALLM_MT_NT2 4       // m16 tiles per warp when 8 < M <= 16
#endif
#ifndef GFX_SMALLM_CTAS_NT2
#define GFX_SMALLM_CTAS_NT2 1     // resident CTAs per SM when 8 < M <= 16 (168 registers)
#endif
#ifndef GFX_SMALLM_STAGES_NT2
#define GFX_SMALLM_STAGES_NT2 4   // smem ring depth, fp16 scales, 8 < M <= 16
#endif
#ifndef GFX_SMALLM_GRID_NT1
#define GFX_SMALLM_GRID_NT1 GFX_SMALLM_CTAS_PER_SM  // CTAs per SM in the grid plan, M <= 8
#endif
#ifndef GFX_SMALLM_GRID_NT2
#define GFX_SMALLM_GRID_NT2 GFX_SMALLM_CTAS_NT2     // CTAs per SM in the grid plan, 8 < M <= 16
#endif
#ifndef GFX_SMALLM_PREWAIT
#define GFX_SMALLM_PREWAIT 0  // 1: load the first stages' weights into the ring before the dependency wait
#endif

// Warp tiling: kMT m16 tiles per warp (rows), the 8 consumer warps split into
// kRowSlices row slices x kKParts K parts (each K part owns kGPW of the 8
// groups of a unit). More m16 tiles per warp amortise the activation
// fragments; fewer keep the accumulators of larger token tiles in registers.
template <int NT, int STAGES, bool kF16Scale>
struct Layout {
  static constexpr int kMT = NT == 1 ? GFX_SMALLM_MT_NT1 : (NT == 2 ? GFX_SMALLM_MT_NT2 : 2);
  static constexpr int kRowSlices = kRows / (16 * kMT);
  static constexpr int kKParts = kConsumerWarps / kRowSlices;
  static constexpr int kGPW = kGroupsPerStage / kKParts;  // groups per warp per unit (even)
  static constexpr int kTok = 8 * NT;
  static constexpr int kNibBytes = kRows * kStageBytesPerRow;
  static constexpr int kScaleRowBytes = kGroupsPerStage * (kF16Scale ? 2 : 4);  // dense [row][group]
  static constexpr int kScaleBytes = (kRows * kScaleRowBytes + 1023) / 1024 * 1024;
  static constexpr int kXBoxBytes = kTok * 128;  // one 64-wide k box (SW128)
  static constexpr int kXBytes = (4 * kXBoxBytes + 1023) / 1024 * 1024;
  static constexpr int kStageBytes = kNibBytes + kScaleBytes + kXBytes;
  static constexpr int kAcc = kMT * NT * 4;      // accumulators per thread
  static constexpr int kRedBytes = kRowSlices * 32 * kAcc * 4;  // one K quarter, aliases the held stage
  static_assert(kRedBytes <= kStageBytes, "a K quarter's reduction buffer must fit in one stage");
  static constexpr int kSmemBytes = 1024 + STAGES * kStageBytes + 2 * STAGES * 8 + 64;
};

__device__ __forceinline__ void ldmatrix_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// A register-only operation: not volatile, so the compiler may interleave the
// MMA chains of different tiles with each other and with the loads.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// Nibbles at bit 0 and bit 16 of w_shifted -> bf16x2 (128 + u) with u = nib ^ 8
// = code + 8: (w & 0x000F000F) ^ 0x43084308 == 0x4300 | (nib ^ 8) per half.
__device__ __forceinline__ uint32_t nib_pair_magic(uint32_t w_shifted) {
  return and_xor(w_shifted, 0x000F000Fu, 0x43084308u);
}

constexpr uint32_t kMinus136x2 = 0xC308C308u;  // bf16x2 (-136, -136)

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kConsumerBarrier), "n"(kConsumerWarps * 32) : "memory");
}

// One output element: into the local y [M, N] (restrict-qualified, so the
// compiler may move the fix-up's loads across these stores), or, for the
// all-gather variant, into every target buffer [M, ldy] at column col0 + n.
template <typename OutT, bool kPeers>
__device__ __forceinline__ void store_out(OutT* __restrict__ y, const OutTargets& out, int N, int tok, int n,
                                          float v) {
  const OutT val = from_f32<OutT>(v);
  if constexpr (!kPeers) {
    y[(size_t)tok * N + n] = val;
  } else {
    const size_t off = (size_t)tok * out.ldy + out.col0 + n;
    for (int q = 0; q < out.count; ++q) reinterpret_cast<OutT*>(out.ptr[q])[off] = val;
  }
}

// Token row of MMA column n within an 8-token tile (conflict-free activation loads).
__device__ __forceinline__ int tok_perm(int n) { return (n >> 1) | ((n & 1) << 2); }

// First CTA whose unit range contains unit t: largest c with floor(c*U/G) <= t.
__device__ __forceinline__ int owner_cta(long long t, long long U, int G) {
  return (int)(((t + 1) * G + U - 1) / U) - 1;
}

template <int NT, int STAGES, bool kF16Scale, typename OutT, bool kCl, bool kPeers>
__global__ void __launch_bounds__(kThreads, NT == 1 ? GFX_SMALLM_CTAS_PER_SM : (NT == 2 ? GFX_SMALLM_CTAS_NT2 : 1))
    w4a16_smallm_kernel(
    const __grid_constant__ CUtensorMap nib_map, const __grid_constant__ CUtensorMap x_map,
    const __grid_constant__ CUtensorMap scale_map, int scale_tma, const void* __restrict__ wscale,
    const OutT* __restrict__ bias, OutT* __restrict__ y, const __grid_constant__ OutTargets out,
    float* __restrict__ partials,
    int* __restrict__ counters, int* status_host,
    int M, int N, int K, int G, int max_segs) {
  using L = Layout<NT, STAGES, kF16Scale>;
  constexpr int kTok = L::kTok;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  uint64_t* empty = full + STAGES;
  int* s_flag = reinterpret_cast<int*>(empty + STAGES);
  uint64_t* cl_go = empty + STAGES + 1;   // cluster split-K: "leader's ring is free" (peers)
  uint64_t* cl_red = empty + STAGES + 2;  // cluster split-K: peers' partials landed (leader)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tb = blockIdx.y;  // token block
  const int tok0 = tb * kTok;
  const int groups = K >> 5;
  const int KS = (K + kStageK - 1) / kStageK;
  const int RB = (N + kRows - 1) / kRows;
  const long long U = (long long)RB * KS;
  const int c = blockIdx.x;
  const long long u_begin = (long long)c * U / G;
  const long long u_end = (long long)(c + 1) * U / G;
  const int n_iters = (int)(u_end - u_begin);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], scale_tma ? 1 : 1 + 32);
      mbar_init(&empty[s], kConsumerWarps);
    }
    if constexpr (kCl) {
      mbar_init(cl_go, 1);
      mbar_init(cl_red, (cluster_nctarank() - 1) * L::kRowSlices * 32);
    }
    fence_barrier_init();
  }
  if constexpr (kCl) {
    cluster_sync_all();  // peers' barriers are initialised before any remote arrive
  } else {
    __syncthreads();
  }
  if (!kCl && n_iters <= 0) return;  // a cluster CTA always has units (classic split)
  pdl_trigger();

  if (warp == kConsumerWarps) {
    // ------------------------------ producer ------------------------------
    // weights (nibbles + scales) of unit it into ring stage it % STAGES,
    // counted on full[stage] together with the activation boxes
    auto load_weights = [&](int it) {
      const int stage = it % STAGES;
      const long long u = u_begin + it;
      const int rb = (int)(u / KS), ks = (int)(u % KS);
      uint8_t* st = smem + stage * L::kStageBytes;
      uint8_t* sc = st + L::kNibBytes;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[stage],
                              L::kNibBytes + 4 * L::kXBoxBytes + (scale_tma ? kRows * L::kScaleRowBytes : 0));
        tma_load_2d(st, &nib_map, &full[stage], ks * kStageBytesPerRow, rb * kRows);
        if (scale_tma) tma_load_2d(sc, &scale_map, &full[stage], ks * kGroupsPerStage, rb * kRows);
      }
      if (!scale_tma) {
        constexpr int kWordsPerRow = L::kScaleRowBytes / 4;
        constexpr int kWords = kRows * kWordsPerRow;
        for (int i = lane; i < kWords; i += 32) {
          const int r = i / kWordsPerRow, wd = i % kWordsPerRow;
          const int n = rb * kRows + r;
          const int g = ks * kGroupsPerStage + wd * (kF16Scale ? 2 : 1);
          const bool valid = (n < N) && (g < groups);
          const uint8_t* src = reinterpret_cast<const uint8_t*>(wscale);
          if (valid) src += ((size_t)n * groups + g) * (kF16Scale ? 2 : 4);
          cp_async_4(sc + 4 * i, src, valid ? 4u : 0u);
        }
        cp_async_mbar_arrive_noinc(&full[stage]);
      }
    };
    // the activation slice of unit it (only after the dependency wait)
    auto load_x = [&](int it) {
      const int stage = it % STAGES;
      const int ks = (int)((u_begin + it) % KS);
      uint8_t* xs = smem + stage * L::kStageBytes + L::kNibBytes + L::kScaleBytes;
      if (lane == 0) {
#pragma unroll
        for (int b = 0; b < 4; ++b)
          tma_load_2d(xs + b * L::kXBoxBytes, &x_map, &full[stage], ks * kStageK + b * 64, tok0);
      }
    };
    const int pre = n_iters < STAGES ? n_iters : STAGES;
    if (lane == 0) {
      tma_prefetch_desc(&nib_map);
      tma_prefetch_desc(&x_map);
      if (scale_tma) tma_prefetch_desc(&scale_map);
      if (!GFX_SMALLM_PREWAIT) {
        // the first stages' weight tiles start streaming into L2 while the
        // previous kernel of the stream finishes
        for (int it = 0; it < pre; ++it) {
          const long long u = u_begin + it;
          tma_prefetch_l2_2d(&nib_map, (int)(u % KS) * kStageBytesPerRow, (int)(u / KS) * kRows);
        }
      }
    }
    // Weights never come from another kernel, so with GFX_SMALLM_PREWAIT the
    // first `pre` stages' weights land in the ring while the previous kernel
    // of the stream still runs; only the activation boxes wait for it.
    if (GFX_SMALLM_PREWAIT)
      for (int it = 0; it < pre; ++it) load_weights(it);  // first use of each stage: no empty wait
    pdl_wait();
    for (int it = 0; it < n_iters; ++it) {
      if (!(GFX_SMALLM_PREWAIT && it < pre)) {
        const int stage = it % STAGES;
        const uint32_t phase = (it / STAGES) & 1;
        if (!mbar_wait(&empty[stage], phase ^ 1, kDevErrEmptyBarrierTimeout)) {
          mirror_device_error(status_host);
          break;
        }
        load_weights(it);
      }
      load_x(it);
    }
    if constexpr (kCl) cluster_sync_all();  // no CTA of the cluster leaves while a peer may address it
    return;
  }

  // ------------------------------ consumers -----------------------------
  pdl_wait();  // outputs, partials and counters are touched only after the previous kernel
  constexpr int kMT = L::kMT, kRowSlices = L::kRowSlices, kKParts = L::kKParts, kGPW = L::kGPW;
  const int rs = warp % kRowSlices;  // row slice: rows rs*16*kMT .. of the row block
  const int kq = warp / kRowSlices;  // K part: groups kq*kGPW .. kq*kGPW + kGPW - 1 of each unit
  const int g_ = lane >> 2, t_ = lane & 3;
  const int lm_j = lane & 7, lm_hi = (lane >> 3) & 1;  // ldmatrix.x2: matrix (lane>>3)&1, row lane&7
  const int xrow_in_tile = tok_perm(g_);
  float acc[kMT][NT][4];
#pragma unroll
  for (int i = 0; i < kMT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;

  for (int it = 0; it < n_iters; ++it) {
    const int stage = it % STAGES;
    const uint32_t phase = (it / STAGES) & 1;
    // A consumer that gives up here leaves early; its peers reach the same
    // wait (they all consume the same stages) and give up the same way.
    if (!mbar_wait(&full[stage], phase, kDevErrFullBarrierTimeout)) {
      mirror_device_error(status_host);
      if constexpr (kCl) cluster_sync_all();
      return;
    }
    // explicit shared-window addresses (generic pointers into shared memory
    // can compile to generic loads, with L1TEX latency)
    const uint32_t st_s = smem_u32(smem) + stage * L::kStageBytes;
    const uint32_t nib_base = st_s;
    const uint32_t sc_s = st_s + L::kNibBytes;
#pragma unroll
    for (int gi = 0; gi < kGPW; ++gi) {
      const int grp = kq * kGPW + gi;
      const int h = grp & 1;  // which 32-group of x box grp/2
      const uint32_t xs_s = sc_s + L::kScaleBytes + (grp >> 1) * L::kXBoxBytes;
      // All shared-memory loads of this group first (volatile ldmatrix keeps
      // source order, so loads written after an MMA could not start earlier):
      // the activation fragments, one nibble word per row and m16 tile, and
      // the two scales per m16 tile.
      uint4 xv[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int row = nt * 8 + xrow_in_tile;
        const int chunk = h * 4 + t_;
        xv[nt] = lds128(xs_s + row * 128 + ((chunk ^ (row & 7)) << 4));
      }
      uint32_t wr[kMT], wr8[kMT];
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt) {
        // word t of group grp for rows rbase+g (matrix 0) and rbase+8+g (matrix 1)
        const int lrow = rs * 16 * kMT + mt * 16 + lm_j + lm_hi * 8;
        ldmatrix_x2(nib_base + lrow * kStageBytesPerRow + ((grp ^ (lrow & 7)) << 4), wr[mt], wr8[mt]);
      }
      float s_r[kMT], s_r8[kMT];
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt) {
        const int r_lo = rs * 16 * kMT + mt * 16 + g_, r_hi = r_lo + 8;
        if (kF16Scale) {
          s_r[mt] = lds_f16_as_f32(sc_s + (r_lo * kGroupsPerStage + grp) * 2);
          s_r8[mt] = lds_f16_as_f32(sc_s + (r_hi * kGroupsPerStage + grp) * 2);
        } else {
          s_r[mt] = lds_f32(sc_s + (r_lo * kGroupsPerStage + grp) * 4);
          s_r8[mt] = lds_f32(sc_s + (r_hi * kGroupsPerStage + grp) * 4);
        }
      }
      // B fragments and the offset correction p0 = -136 * sum_k x (constant A operand).
      uint32_t b[NT][4];
      float p0[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        b[nt][0] = prmt(xv[nt].x, xv[nt].z, 0x5410);  // step 0, slots (2t, 2t+1)
        b[nt][1] = prmt(xv[nt].x, xv[nt].z, 0x7632);  // step 0, slots (2t+8, 2t+9)
        b[nt][2] = prmt(xv[nt].y, xv[nt].w, 0x5410);  // step 1
        b[nt][3] = prmt(xv[nt].y, xv[nt].w, 0x7632);
        const float zero[4] = {0.f, 0.f, 0.f, 0.f};
        mma_bf16_16816(p0[nt], kMinus136x2, kMinus136x2, kMinus136x2, kMinus136x2, b[nt][0], b[nt][1], zero);
        mma_bf16_16816(p0[nt], kMinus136x2, kMinus136x2, kMinus136x2, kMinus136x2, b[nt][2], b[nt][3], p0[nt]);
      }
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt) {
        // step 0: slots (2t,2t+1) <- (n0,n4), (2t+8,2t+9) <- (n1,n5)
        // step 1: slots (2t,2t+1) <- (n2,n6), (2t+8,2t+9) <- (n3,n7)
        const uint32_t w0 = wr[mt], w1 = wr8[mt];
        const uint32_t a00 = nib_pair_magic(w0), a01 = nib_pair_magic(w1);
        const uint32_t a02 = nib_pair_magic(w0 >> 4), a03 = nib_pair_magic(w1 >> 4);
        const uint32_t a10 = nib_pair_magic(w0 >> 8), a11 = nib_pair_magic(w1 >> 8);
        const uint32_t a12 = nib_pair_magic(w0 >> 12), a13 = nib_pair_magic(w1 >> 12);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float p[4];
          mma_bf16_16816(p, a00, a01, a02, a03, b[nt][0], b[nt][1], p0[nt]);
          mma_bf16_16816(p, a10, a11, a12, a13, b[nt][2], b[nt][3], p);
          acc[mt][nt][0] = fmaf(p[0], s_r[mt], acc[mt][nt][0]);
          acc[mt][nt][1] = fmaf(p[1], s_r[mt], acc[mt][nt][1]);
          acc[mt][nt][2] = fmaf(p[2], s_r8[mt], acc[mt][nt][2]);
          acc[mt][nt][3] = fmaf(p[3], s_r8[mt], acc[mt][nt][3]);
        }
      }
    }

    // ---------------- segment end: leaving a row block (or the range) ----------------
    const long long u = u_begin + it;
    const bool seg_end = (((u + 1) % KS) == 0) || (it == n_iters - 1);
    if (!seg_end) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      continue;
    }
    const int rb = (int)(u / KS);
    const long long rb_lo = (long long)rb * KS, rb_hi = rb_lo + KS;
    const long long seg_lo = u_begin > rb_lo ? u_begin : rb_lo;
    const bool single = (seg_lo == rb_lo) && (u + 1 == rb_hi);
    // The stage is still held (not yet released to the producer), so once
    // every consumer is done reading it, it doubles as the reduction buffer.
    // Layout [quarter-1][element][slice*32 + lane]: consecutive lanes write
    // consecutive words (no bank conflicts).
    const uint32_t red_s = st_s;  // float index i at red_s + 4 i
    constexpr int kRedStride = kRowSlices * 32;                     // floats per element row
    constexpr int kRedQuarter = L::kAcc * kRedStride;               // floats per K quarter
    constexpr bool kOneRound = (kKParts - 1) * kRedQuarter * 4 <= L::kStageBytes;
    const int rl = rs * 32 + lane;
    consumer_sync();
    // 1) K parts 1.. -> part 0
    if (kOneRound) {
      if (kq != 0) {
        const uint32_t dst = red_s + 4u * (uint32_t)((kq - 1) * kRedQuarter + rl);
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) sts_f32(dst + 4u * (uint32_t)(((mt * NT + nt) * 4 + e) * kRedStride), acc[mt][nt][e]);
      }
      consumer_sync();
      if (kq == 0) {
#pragma unroll
        for (int q = 0; q < kKParts - 1; ++q) {
          const uint32_t src = red_s + 4u * (uint32_t)(q * kRedQuarter + rl);
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e)
                acc[mt][nt][e] += lds_f32(src + 4u * (uint32_t)(((mt * NT + nt) * 4 + e) * kRedStride));
        }
      }
    } else {
#pragma unroll 1
      for (int q = 1; q < kKParts; ++q) {
        if (kq == q) {
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e)
                sts_f32(red_s + 4u * (uint32_t)(((mt * NT + nt) * 4 + e) * kRedStride + rl), acc[mt][nt][e]);
        }
        consumer_sync();
        if (kq == 0) {
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e)
                acc[mt][nt][e] += lds_f32(red_s + 4u * (uint32_t)(((mt * NT + nt) * 4 + e) * kRedStride + rl));
        }
        consumer_sync();
      }
    }
    const int n0 = rb * kRows;
    if (single) {
      if (kq == 0) {
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int n = n0 + rs * 16 * kMT + mt * 16 + g_ + half * 8;
            if (n >= N) continue;
            const float bv = bias ? to_f32(bias[n]) : 0.0f;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int cc = 0; cc < 2; ++cc) {
                const int tok = tok0 + nt * 8 + tok_perm(2 * t_ + cc);
                if (tok < M) store_out<OutT, kPeers>(y, out, N, tok, n, acc[mt][nt][half * 2 + cc] + bv);
              }
          }
      }
    } else if constexpr (kCl) {
      // 2') cluster split-K: the CTAs of one row block are one cluster; rank 0
      // (the first K segment) takes the peers' fp32 partials into its stage
      // ring (free once its own units are consumed) through distributed shared
      // memory, sums them in rank order (deterministic), adds the bias, stores.
      const uint32_t rank = cluster_ctarank(), csize = cluster_nctarank();
      constexpr int kRecvStride = kRows + 4;  // padded token rows: conflict-free reads
      const int vt = (M - tok0) < kTok ? (M - tok0) : kTok;  // valid tokens of this token block
      float* recv = reinterpret_cast<float*>(smem);
      if (rank != 0) {
        if (kq == 0 && !mbar_wait_acq_cluster(cl_go, 0, kDevErrClusterReduceTimeout)) {
          mirror_device_error(status_host);
        } else if (kq == 0) {
          const uint32_t dst = mapa_shared(smem_u32(recv), 0) + (rank - 1) * (uint32_t)(kTok * kRecvStride * 4);
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const int r = rs * 16 * kMT + mt * 16 + g_ + half * 8;
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                  const int tok = nt * 8 + tok_perm(2 * t_ + cc);
                  if (tok < vt) st_shared_cluster_f32(dst + (uint32_t)(tok * kRecvStride + r) * 4u, acc[mt][nt][half * 2 + cc]);
                }
            }
          mbar_arrive_release_cluster(cl_red, 0);
        }
      } else {
        consumer_sync();  // every consumer is done reading the ring (K-part reduction)
        if (threadIdx.x == 0)
          for (uint32_t q = 1; q < csize; ++q) mbar_arrive_release_cluster(cl_go, q);
        if (kq == 0 && !mbar_wait_acq_cluster(cl_red, 0, kDevErrClusterReduceTimeout)) {
          mirror_device_error(status_host);
        } else if (kq == 0) {
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const int r = rs * 16 * kMT + mt * 16 + g_ + half * 8;
              const int n = n0 + r;
              if (n >= N) continue;
              const float bv = bias ? to_f32(bias[n]) : 0.0f;
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                  const int tok = nt * 8 + tok_perm(2 * t_ + cc);
                  if (tok >= vt) continue;
                  float v = acc[mt][nt][half * 2 + cc];
                  for (uint32_t q = 1; q < csize; ++q) v += recv[((q - 1) * kTok + tok) * kRecvStride + r];
                  store_out<OutT, kPeers>(y, out, N, tok0 + tok, n, v + bv);
                }
            }
        }
      }
    } else {
      // 2) this segment's partial -> workspace slot [tb][rb][seg] ([token][row] order)
      const int seg = c - owner_cta(rb_lo, U, G);
      float* part = partials + (((size_t)tb * RB + rb) * max_segs) * (kTok * kRows);
      if (kq == 0) {
        float* mine = part + (size_t)seg * (kTok * kRows);
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int r = rs * 16 * kMT + mt * 16 + g_ + half * 8;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int cc = 0; cc < 2; ++cc) {
                const int tok = nt * 8 + tok_perm(2 * t_ + cc);
                if (tok0 + tok < M) mine[tok * kRows + r] = acc[mt][nt][half * 2 + cc];  // valid tokens only
              }
          }
        __threadfence();
      }
      consumer_sync();
      int* counter = counters + (size_t)tb * RB + rb;
      const int nsegs = owner_cta(rb_hi - 1, U, G) - owner_cta(rb_lo, U, G) + 1;
      if (warp == 0 && lane == 0) *s_flag = (atomicAdd(counter, 1) == nsegs - 1);
      consumer_sync();
      if (*s_flag) {
        __threadfence();
        // 3) last arrival: fixed-order sum over the segments, + bias, store, re-arm.
        // Items are four consecutive rows of one valid token (float4 loads);
        // each thread issues a batch of eight segments' loads before adding.
        const int tc = threadIdx.x;  // 0..255 (consumers)
        const int vt = (M - tok0) < kTok ? (M - tok0) : kTok;  // valid tokens of this token block
        constexpr int kQuads = kRows / 4;
        for (int item = tc; item < vt * kQuads; item += kConsumerWarps * 32) {
          const int tok = item / kQuads, r = (item % kQuads) * 4;
          const float* src = part + (size_t)tok * kRows + r;
          float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          for (int s0 = 0; s0 < nsegs; s0 += 8) {
            float4 t[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              t[j] = s0 + j < nsegs ? __ldcg(reinterpret_cast<const float4*>(src + (size_t)(s0 + j) * (kTok * kRows)))
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (s0 + j < nsegs) {
                v.x += t[j].x;
                v.y += t[j].y;
                v.z += t[j].z;
                v.w += t[j].w;
              }
          }
          const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int n = n0 + r + e;
            if (n >= N) continue;
            float o = vv[e];
            if (bias) o += to_f32(bias[n]);
            store_out<OutT, kPeers>(y, out, N, tok0 + tok, n, o);
          }
        }
        if (tc == 0) *counter = 0;
      }
    }
    consumer_sync();  // everyone is done with the held stage and s_flag
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
#pragma unroll
    for (int i = 0; i < kMT; ++i)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;
  }
  if constexpr (kPeers) __threadfence_system();  // publish peer-buffer stores before a cross-GPU barrier
  if constexpr (kCl) cluster_sync_all();  // no CTA of the cluster leaves while a peer may address it
}

}  // namespace smallm

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
GFX_DEFINE_STATUS_READER(smallm_device_status)

struct SmallMPlan {
  int nt, tok, tok_blocks, RB, KS, G, max_segs, ctas_per_sm, stages;
  int cl;  // classic split count s when 2 <= s <= 16 (cluster split-K candidate), else 0
};

static int nt_for(int M) { return M <= 8 ? 1 : (M <= 16 ? 2 : 4); }

static SmallMPlan smallm_plan(int M, int N, int K, int splits_req, int sms, bool f16) {
  SmallMPlan p{};
  p.nt = nt_for(M);
  p.tok = 8 * p.nt;
  p.tok_blocks = (M + p.tok - 1) / p.tok;
  p.RB = (N + smallm::kRows - 1) / smallm::kRows;
  p.KS = (K + smallm::kStageK - 1) / smallm::kStageK;
  // resident CTAs per SM follow the stage ring + reduction buffer size
  p.ctas_per_sm = p.nt == 4 ? 1 : (p.nt == 2 ? GFX_SMALLM_GRID_NT2 : GFX_SMALLM_GRID_NT1);
  p.stages = p.nt == 4 ? 6 : ((!f16 && p.nt == 2) ? 3 : 4);
  const long long U = (long long)p.RB * p.KS;
  long long G;
  if (splits_req > 0) {
    const int s = splits_req > p.KS ? p.KS : splits_req;
    G = (long long)p.RB * s;  // classic split-K as a special case of the unit partition
  } else {
    long long slots = (long long)sms * p.ctas_per_sm / p.tok_blocks;
    if (slots < 1) slots = 1;
    // A classic split over a divisor s of KS that fills >= 90% of the resident
    // slots: every CTA then covers one aligned K segment of one row block (one
    // segment end per CTA). Otherwise stream-K over all slots for balance.
    int best_s = 0;
    for (int s = 1; s <= p.KS; ++s) {
      if (p.KS % s) continue;
      if ((long long)p.RB * s > slots) break;
      best_s = s;
    }
    if (best_s > 0 && (long long)p.RB * best_s * 10 >= slots * 9) {
      G = (long long)p.RB * best_s;
    } else {
      G = slots > U ? U : slots;
    }
  }
  p.G = (int)G;
  // a classic split (G = RB * s: every CTA inside one row block) can reduce
  // through distributed shared memory when s CTAs fit in one cluster
  p.cl = (G % p.RB == 0 && G / p.RB >= 2 && G / p.RB <= 16) ? (int)(G / p.RB) : 0;
  // segments per row block: a row block spans KS units and every CTA range
  // holds at least floor(U / G) of them
  const long long min_units = U / G;
  p.max_segs = (int)((p.KS + min_units - 1) / min_units) + 1;
  return p;
}

size_t smallm_workspace_bytes(int M, int N, int K, int splits_req, int sms) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  // sized for the larger of the fp16 / fp32 scale plans
  size_t need = 0;

  for (int f = 0; f < 2; ++f) {
    SmallMPlan p = smallm_plan(M, N, K, splits_req, sms, f == 1);
    const size_t part = (size_t)p.tok_blocks * p.RB * p.max_segs * p.tok * smallm::kRows * sizeof(float);
    const size_t b = kSplitKCounterBytes + align_up(part, 256);
    need = b > need ? b : need;
  }
  return need;
}

int smallm_auto_splits(int M, int N, int K, int sms) {
  SmallMPlan p = smallm_plan(M, N, K, 0, sms, true);
  return (p.G + p.RB - 1) / p.RB;
}

struct SmallMArgs {
  CUtensorMap nib_map, x_map, scale_map;
  int scale_tma;
  const void* ws;
  const void* bias;
  OutTargets out;
  float* part;
  int* cnt;
  int* status_host;
  int M, N, K;
};

template <int NT, int STAGES, bool F16S, typename OutT, bool kCl, bool kPeers>
static int launch_smallm_k(const SmallMPlan& p, const SmallMArgs& a, cudaStream_t st, int cluster) {
  using L = smallm::Layout<NT, STAGES, F16S>;
  auto kern = smallm::w4a16_smallm_kernel<NT, STAGES, F16S, OutT, kCl, kPeers>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.gridDim = dim3(p.G, p.tok_blocks);
  cfg.blockDim = dim3(smallm::kThreads);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (kCl) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a.nib_map, a.x_map, a.scale_map, a.scale_tma, a.ws,
                                     (const OutT*)a.bias, (OutT*)a.out.ptr[0], a.out, a.part, a.cnt, a.status_host, a.M,
                                     a.N, a.K, p.G, p.max_segs);
  if (e != cudaSuccess) return set_error(GFX_ERR_CUDA, "w4a16_smallm_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("w4a16_smallm_kernel");
}

// Cluster split-K (opt-in, GFX906_B200_SMALLM_CLUSTER=1): a classic split s
// (2..16) whose peers' partials fit in the leader's stage ring and whose
// RB * token_blocks clusters can all be resident at once. On B200 it measured
// no faster than the global fix-up at M = 1 (the vectorised fix-up is ~1 us)
// and 2x slower for the 2-CTA clusters of the M = 16 qkv shape, so the global
// fix-up stays the default.
template <int NT, int STAGES, bool F16S, typename OutT>
static bool smallm_use_cluster(const SmallMPlan& p) {
  using L = smallm::Layout<NT, STAGES, F16S>;
  if (p.cl < 2) return false;
  const char* env = getenv("GFX906_B200_SMALLM_CLUSTER");
  if (!(env && env[0] == '1' && env[1] == 0)) return false;
  const size_t recv = (size_t)(p.cl - 1) * L::kTok * (smallm::kRows + 4) * sizeof(float);
  if (recv > (size_t)STAGES * L::kStageBytes) return false;
  static int max_active[64][17];  // per device and cluster size: 0 unknown, -1 impossible, else clusters
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return false;
  int& m = max_active[dev][p.cl];
  if (m == 0) {
    auto kern = smallm::w4a16_smallm_kernel<NT, STAGES, F16S, OutT, true, false>;
    m = -1;
    if (p.cl > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(p.cl * 16);
    cfg.blockDim = dim3(smallm::kThreads);
    cfg.dynamicSmemBytes = L::kSmemBytes;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) m = n;
    (void)cudaGetLastError();
  }
  return m > 0 && (long long)m >= (long long)p.RB * p.tok_blocks;
}

template <int NT, int STAGES, bool F16S, typename OutT>
static int launch_smallm_t(const SmallMPlan& p, const SmallMArgs& a, cudaStream_t st) {
  using L = smallm::Layout<NT, STAGES, F16S>;
  static bool attr_set[64] = {false};  // per device
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    for (auto kern : {smallm::w4a16_smallm_kernel<NT, STAGES, F16S, OutT, false, false>,
                      smallm::w4a16_smallm_kernel<NT, STAGES, F16S, OutT, true, false>,
                      smallm::w4a16_smallm_kernel<NT, STAGES, F16S, OutT, false, true>}) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
      if (e != cudaSuccess)
        return set_error(GFX_ERR_CUDA, "w4a16_smallm: cannot set %d bytes of shared memory: %s", L::kSmemBytes,
                         cudaGetErrorString(e));
    }
    attr_set[dev] = true;
  }
  if (a.out.count > 1 || a.out.fence_sys) return launch_smallm_k<NT, STAGES, F16S, OutT, false, true>(p, a, st, 1);
  if (smallm_use_cluster<NT, STAGES, F16S, OutT>(p))
    return launch_smallm_k<NT, STAGES, F16S, OutT, true, false>(p, a, st, p.cl);
  return launch_smallm_k<NT, STAGES, F16S, OutT, false, false>(p, a, st, 1);
}

template <int NT, int STAGES, bool F16S>
static int launch_smallm_out(int out_dtype, const SmallMPlan& p, const SmallMArgs& a, cudaStream_t st) {
  if (out_dtype == GFX_DTYPE_F32) return launch_smallm_t<NT, STAGES, F16S, float>(p, a, st);
  if (out_dtype == GFX_DTYPE_F16) return launch_smallm_t<NT, STAGES, F16S, __half>(p, a, st);
  return launch_smallm_t<NT, STAGES, F16S, __nv_bfloat16>(p, a, st);
}

int launch_w4a16_smallm(const void* x, const void* wq, const void* ws, int scale_dtype, const void* bias, void* y,
                        int out_dtype, int M, int N, int K, int splits_req, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream, int sms) {
  OutTargets out{};
  out.ptr[0] = y;
  out.count = 1;
  out.ldy = N;
  out.col0 = 0;
  out.fence_sys = 0;
  return launch_w4a16_smallm_targets(x, wq, ws, scale_dtype, bias, out, out_dtype, M, N, K, splits_req, workspace,
                                     workspace_bytes, stream, sms);
}

int launch_w4a16_smallm_targets(const void* x, const void* wq, const void* ws, int scale_dtype, const void* bias,
                                const OutTargets& out, int out_dtype, int M, int N, int K, int splits_req,
                                void* workspace, size_t workspace_bytes, cudaStream_t stream, int sms) {
  const bool f16 = scale_dtype == GFX_SCALE_F16;
  if (M > 64)
    return set_error(GFX_ERR_UNSUPPORTED, "w4a16_gemm: the small-M kernel takes M <= 64 (got M=%d); "
                     "use splits=0 so larger M runs on the tensor-core kernel", M);
  SmallMPlan p = smallm_plan(M, N, K, splits_req, sms, f16);
  SmallMArgs a{};
  const size_t need = smallm_workspace_bytes(M, N, K, splits_req, sms);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(GFX_ERR_WORKSPACE, "w4a16_gemm: workspace of %zu bytes required, got %zu (ptr %p)", need,
                     workspace_bytes, workspace);
  if ((size_t)p.tok_blocks * p.RB * sizeof(int) > kSplitKCounterBytes)
    return set_error(GFX_ERR_UNSUPPORTED, "w4a16_gemm: %d x %d row blocks exceed the %zu-byte counter region",
                     p.tok_blocks, p.RB, kSplitKCounterBytes);
  // Counters live at a fixed offset (the first kSplitKCounterBytes) so that
  // calls of any shape sharing one workspace always find them re-armed to
  // zero; the fp32 partials follow and need no initial value.
  a.cnt = reinterpret_cast<int*>(workspace);
  a.status_host = host_status_word(current_device());
  a.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + kSplitKCounterBytes);
  int rc = cached_tmap_2d(&a.nib_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                        smallm::kStageBytesPerRow, smallm::kRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&a.x_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, 64,
                    (uint32_t)p.tok, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const uint64_t elem = f16 ? 2 : 4;
  const uint64_t groups = (uint64_t)K / 32;
  a.scale_tma = ((groups * elem) % 16 == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0) ? 1 : 0;
  if (a.scale_tma) {
    rc = cached_tmap_2d(&a.scale_map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ws,
                      groups, (uint64_t)N, groups * elem, smallm::kGroupsPerStage, smallm::kRows,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    memset(&a.scale_map, 0, sizeof(a.scale_map));
  }
  a.ws = ws;
  a.bias = bias;
  a.out = out;
  a.M = M;
  a.N = N;
  a.K = K;
  // stage counts: two resident CTAs per SM for NT <= 2 (<= ~110 KB each), one for NT = 4
  if (f16) {
    if (p.nt == 1) return launch_smallm_out<1, GFX_SMALLM_STAGES_F16, true>(out_dtype, p, a, stream);
    if (p.nt == 2) return launch_smallm_out<2, GFX_SMALLM_STAGES_NT2, true>(out_dtype, p, a, stream);
    return launch_smallm_out<4, 6, true>(out_dtype, p, a, stream);
  }
  if (p.nt == 1) return launch_smallm_out<1, 4, false>(out_dtype, p, a, stream);
  if (p.nt == 2) return launch_smallm_out<2, 3, false>(out_dtype, p, a, stream);
  return launch_smallm_out<4, 6, false>(out_dtype, p, a, stream);
}

// ---------------------------------------------------------------------------
// cross-GPU flag barrier for the all-gather epilogue
// ---------------------------------------------------------------------------
// flags[q] is rank q's array of n_ranks + 1 ints (symmetric memory, reachable
// from every rank); slot n_ranks of a rank's own array counts the barriers it
// passed, so the epoch needs no host argument (graph-capturable). With e = that
// count + 1, lane q of rank r stores e into flags[q][r] with release at system
// scope, then waits -- bounded -- until flags[r][q] >= e with acquire at system
// scope: after it, every store rank q made before its own release (its GEMM's
// writes into this rank's y) is visible here. Only peers write flags[r][0..n),
// only rank r writes flags[r][n], and the next barrier on this stream reads the
// counter after this kernel ends.
struct FlagTable {
  int* p[kMaxOutTargets];
};

__global__ void peer_barrier_kernel(const __grid_constant__ FlagTable flags, int n_ranks, int rank,
                                    int* status_host) {
  const int q = threadIdx.x;
  int* own = flags.p[rank];
  const int epoch = own[n_ranks] + 1;
  __syncwarp();
  if (q < n_ranks) {
    __threadfence_system();
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(flags.p[q] + rank), "r"(epoch) : "memory");
    const unsigned long long t0 = global_timer_ns();
    for (;;) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(own + q) : "memory");
      if (v - epoch >= 0) break;
      if (global_timer_ns() - t0 > kWaitTimeoutNs) {
        record_device_error(kDevErrPeerBarrierTimeout);
        mirror_device_error(status_host);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();
  if (q == 0) own[n_ranks] = epoch;
}

int launch_peer_barrier(int* const* flags, int n_ranks, int rank, cudaStream_t stream) {
  FlagTable t{};
  for (int q = 0; q < n_ranks; ++q) t.p[q] = flags[q];
  peer_barrier_kernel<<<1, 32, 0, stream>>>(t, n_ranks, rank, host_status_word(current_device()));
  return check_launch("peer_barrier_kernel");
}

}  // namespace gfx
