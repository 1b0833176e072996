// C ABI of the library (declared in include/gfx906_b200.h): argument checks
// mirroring the reference binding (nodes/ComfyUI-Gfx906Int4/csrc/binding.cpp),
// per-device caches, TMA descriptor encoding, dispatch to the kernels.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace gfx {

static thread_local char t_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(GFX_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return GFX_OK;
}

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

int sm_count(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
    cache[device] = v;
  }
  return cache[device];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(GFX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the CUDA driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(GFX_ERR_INVALID, "TMA base address %p is not 16-byte aligned", base);
  if (row_stride_bytes % 16 != 0)
    return set_error(GFX_ERR_INVALID, "TMA row stride %llu bytes is not a multiple of 16",
                     (unsigned long long)row_stride_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(GFX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu, box %u x %u", (int)r,
                     (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
  return GFX_OK;
}

static bool valid_dtype(int d) { return d == GFX_DTYPE_F32 || d == GFX_DTYPE_F16 || d == GFX_DTYPE_BF16; }

// ---------------------------------------------------------------------------
// tensor-map cache: a model's weight maps are encoded once per (device, args)
// ---------------------------------------------------------------------------
namespace {
struct TmapKey {
  int dev;
  int dtype;
  const void* base;
  uint64_t inner, outer, stride;
  uint32_t box_inner, box_outer;
  int swizzle;
  bool operator==(const TmapKey& o) const {
    return dev == o.dev && dtype == o.dtype && base == o.base && inner == o.inner && outer == o.outer &&
           stride == o.stride && box_inner == o.box_inner && box_outer == o.box_outer && swizzle == o.swizzle;
  }
};
constexpr int kTmapSlots = 512;  // direct-mapped by a hash of the key; a collision re-encodes
struct TmapSlot {
  bool valid = false;
  TmapKey key{};
  CUtensorMap map;
};
std::mutex g_tmap_mu;
TmapSlot g_tmap[kTmapSlots];
}  // namespace

int cached_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  const TmapKey key{current_device(), (int)dtype, base, inner, outer, row_stride_bytes, box_inner, box_outer,
                    (int)swizzle};
  uint64_t h = reinterpret_cast<uintptr_t>(base) >> 4;
  h ^= inner * 0x9E3779B97F4A7C15ull ^ outer * 0xC2B2AE3D27D4EB4Full ^ ((uint64_t)key.dev << 40) ^
       ((uint64_t)box_inner << 20) ^ ((uint64_t)box_outer << 8) ^ (uint64_t)key.swizzle ^ ((uint64_t)dtype << 4);
  h ^= h >> 29;
  TmapSlot& slot = g_tmap[h % kTmapSlots];
  {
    std::lock_guard<std::mutex> lock(g_tmap_mu);
    if (slot.valid && slot.key == key) {
      *map = slot.map;
      return GFX_OK;
    }
  }
  int rc = make_tmap_2d(map, dtype, base, inner, outer, row_stride_bytes, box_inner, box_outer, swizzle);
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(g_tmap_mu);
  slot.valid = true;
  slot.key = key;
  slot.map = *map;
  return GFX_OK;
}

// ---------------------------------------------------------------------------
// host-visible status words: one page of host memory, pinned and mapped into
// every device's address space, one 64-byte slot per device
// ---------------------------------------------------------------------------
namespace {
constexpr int kMaxDevices = 64;
alignas(4096) int g_status_page[kMaxDevices * 16];
std::once_flag g_status_once;
bool g_status_mapped = false;
unsigned g_fail_epoch[kMaxDevices] = {};
std::mutex g_status_mu;
}  // namespace

int* host_status_word(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_status_once, [] {
    g_status_mapped = cudaHostRegister(g_status_page, sizeof(g_status_page),
                                       cudaHostRegisterPortable | cudaHostRegisterMapped) == cudaSuccess;
    if (!g_status_mapped) (void)cudaGetLastError();
  });
  if (!g_status_mapped) return nullptr;
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, g_status_page, 0) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  return reinterpret_cast<int*>(d) + dev * 16;
}

int host_status_read(int dev) {
  if (dev < 0 || dev >= kMaxDevices || !g_status_mapped) return 0;
  return *reinterpret_cast<volatile int*>(&g_status_page[dev * 16]);
}

void host_status_clear(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return;
  std::lock_guard<std::mutex> lock(g_status_mu);
  volatile int* w = reinterpret_cast<volatile int*>(&g_status_page[dev * 16]);
  if (*w != 0) {
    *w = 0;
    ++g_fail_epoch[dev];
  }
}

unsigned failure_epoch(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return 0;
  std::lock_guard<std::mutex> lock(g_status_mu);
  return g_fail_epoch[dev];
}

int check_device_health(const char* fn, int dev, void* workspace, size_t counter_bytes, cudaStream_t stream) {
  const int v = host_status_read(dev);
  if (v == 0) return GFX_OK;
  bool rearmed = false;
  if (workspace != nullptr && counter_bytes > 0)
    rearmed = cudaMemsetAsync(workspace, 0, counter_bytes, stream) == cudaSuccess;
  (void)cudaGetLastError();
  return set_error(GFX_ERR_DEVICE,
                   "%s: device %d reports status %d: an earlier kernel gave up in a bounded wait, so results "
                   "computed since then are not valid%s; read and clear it with gfx_device_status(1)",
                   fn, dev, v, rearmed ? " (the split-K counters of this call's workspace were re-zeroed)" : "");
}

int check_gemm_common(const char* fn, const void* x, int x_dtype, const void* w, const void* ws, int scale_dtype,
                      void* y, int out_dtype, int M, int N, int K, int splits) {
  if (M < 0 || N <= 0 || K <= 0)
    return set_error(GFX_ERR_INVALID, "%s: expected M >= 0, N > 0, K > 0; got M=%d N=%d K=%d", fn, M, N, K);
  if (K % 32 != 0)
    return set_error(GFX_ERR_INVALID, "%s: expected K %% 32 == 0 (one scale per 32 elements), got K=%d", fn, K);
  if (!valid_dtype(out_dtype))
    return set_error(GFX_ERR_INVALID, "%s: unsupported out dtype code %d, expected 0 (f32) / 1 (f16) / 2 (bf16)", fn,
                     out_dtype);
  if (x_dtype != GFX_DTYPE_BF16)
    return set_error(GFX_ERR_UNSUPPORTED, "%s: activations must be bfloat16 (dtype code 2), got code %d", fn, x_dtype);
  if (scale_dtype != GFX_SCALE_F32 && scale_dtype != GFX_SCALE_F16)
    return set_error(GFX_ERR_INVALID, "%s: scale dtype must be 0 (f32) or 1 (f16), got %d", fn, scale_dtype);
  if (splits < 0 || splits > kMaxSplits)
    return set_error(GFX_ERR_INVALID, "%s: splits must be in [0, %d], got %d", fn, kMaxSplits, splits);
  if (M > 0 && (!x || !w || !ws || !y))
    return set_error(GFX_ERR_INVALID, "%s: null pointer among x=%p w=%p scale=%p y=%p", fn, x, w, ws, y);
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return set_error(GFX_ERR_INVALID, "%s: x (%p) and weights (%p) must be 16-byte aligned", fn, x, w);
  if (scale_dtype == GFX_SCALE_F16 && (K % 64 != 0 || (reinterpret_cast<uintptr_t>(ws) & 3)))
    return set_error(GFX_ERR_UNSUPPORTED, "%s: float16 scales need K %% 64 == 0 and 4-byte alignment (K=%d)", fn, K);
  if (scale_dtype == GFX_SCALE_F32 && (reinterpret_cast<uintptr_t>(ws) & 3))
    return set_error(GFX_ERR_INVALID, "%s: float32 scales must be 4-byte aligned", fn);
  return GFX_OK;
}

}  // namespace gfx

using namespace gfx;

extern "C" {

const char* gfx_last_error(void) { return t_last_error; }

int gfx_version(void) { return 100; }

int gfx_device_status(int clear) {
  int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return -set_error(GFX_ERR_CUDA, "gfx_device_status: %s", cudaGetErrorString(e));
  const int parts[5] = {smallm_device_status(clear), tc_device_status(clear), selftest_device_status(clear),
                         w4a4x_device_status(clear), attn_tc_device_status(clear)};
  for (int p : parts) {
    if (p < 0) return -set_error(GFX_ERR_CUDA, "gfx_device_status: reading a status word failed");
    if (p && !v) v = p;
  }
  const int dev = current_device();
  const int h = host_status_read(dev);
  if (h && !v) v = h;
  if (clear) host_status_clear(dev);
  return v;
}

size_t w4a16_workspace_bytes(int M, int N, int K, int splits) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (w4a16_tc_supported(M, N, K, GFX_SCALE_F32)) return 0;  // the tensor-core path needs no scratch
  return smallm_workspace_bytes(M, N, K, splits, sm_count(current_device()));
}

int w4a16_auto_splits(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 1;
  if (w4a16_tc_supported(M, N, K, GFX_SCALE_F32)) return 1;
  return smallm_auto_splits(M, N, K, sm_count(current_device()));
}

int w4a16_gemm(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype, const void* bias,
               void* y, int out_dtype, int M, int N, int K, int splits, void* workspace, size_t workspace_bytes,
               gfx_stream_t stream) {
  int rc = check_gemm_common("w4a16_gemm", x, x_dtype, w_q4, w_scale, scale_dtype, y, out_dtype, M, N, K, splits);
  if (rc) return rc;
  if (M == 0) return GFX_OK;
  const int dev = current_device();
  const int sms = sm_count(dev);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = check_device_health("w4a16_gemm", dev, workspace,
                           workspace_bytes >= kSplitKCounterBytes ? kSplitKCounterBytes : 0, st);
  if (rc) return rc;
  // M > 64 always runs on the tcgen05 kernel (its tiles cover K whole, so a
  // requested split count only matters for the small-M kernel, as for the
  // reference where `splits` changes speed, not the result's definition).
  if (w4a16_tc_supported(M, N, K, scale_dtype))
    return launch_w4a16_tc(x, w_q4, w_scale, scale_dtype, bias, y, out_dtype, M, N, K, st, sms);
  return launch_w4a16_smallm(x, w_q4, w_scale, scale_dtype, bias, y, out_dtype, M, N, K, splits, workspace,
                             workspace_bytes, st, sms);
}

int w4a16_gemm_qblock(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype, int qblock,
                      const void* bias, void* y, int out_dtype, int M, int N, int K, int splits, void* workspace,
                      size_t workspace_bytes, gfx_stream_t stream) {
  if (qblock == 32)
    return w4a16_gemm(x, x_dtype, w_q4, w_scale, scale_dtype, bias, y, out_dtype, M, N, K, splits, workspace,
                      workspace_bytes, stream);
  if (qblock != 16)
    return set_error(GFX_ERR_INVALID, "w4a16_gemm_qblock: qblock must be 32 or 16, got %d", qblock);
  int rc = check_gemm_common("w4a16_gemm_qblock", x, x_dtype, w_q4, w_scale, scale_dtype, y, out_dtype, M, N, K,
                             splits);
  if (rc) return rc;
  if (scale_dtype != GFX_SCALE_F32)
    return set_error(GFX_ERR_UNSUPPORTED, "w4a16_gemm_qblock: qblock=16 takes float32 scales [N, K/16], got scale "
                     "dtype %d", scale_dtype);
  if (M == 0) return GFX_OK;
  const int dev = current_device();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = check_device_health("w4a16_gemm_qblock", dev, nullptr, 0, st);
  if (rc) return rc;
  // 16-element groups run on the tensor-core kernel for every M (the
  // reference's qblock=16 GEMMs are its training GEMMs, large M)
  return launch_w4a16_tc(x, w_q4, w_scale, GFX_SCALE_F32, bias, y, out_dtype, M, N, K, st, sm_count(dev), 16);
}

size_t w4a4_gemm_exact_workspace_bytes(int M, int N, int K, int qblock) {
  return w4a4_exact_workspace(M, N, K, qblock);
}

int w4a4_gemm_exact_splits(int M, int N, int K, int splits) {
  const int dev = current_device();
  return w4a4_exact_splits(M, N, K, splits, sm_count(dev < 0 ? 0 : dev));
}

int w4a4_gemm_exact(const void* a_q4, const float* a_scale, const void* b_q4, const float* b_scale, int qblock,
                    const void* bias, void* y, int out_dtype, int M, int N, int K, int splits, void* workspace,
                    size_t workspace_bytes, gfx_stream_t stream) {
  const char* fn = "w4a4_gemm_exact";
  if (!a_q4 || !a_scale || !b_q4 || !b_scale || !y)
    return set_error(GFX_ERR_INVALID, "%s: A, A_scale, B, B_scale and C must be device pointers", fn);
  if (M < 0 || N <= 0 || K <= 0 || K % 32 != 0)
    return set_error(GFX_ERR_INVALID, "%s: expected A [M, K/2], B [N, K/2], K %% 32 == 0; got M=%d N=%d K=%d", fn, M,
                     N, K);
  if (qblock != 32 && qblock != 16)
    return set_error(GFX_ERR_INVALID, "%s: qblock must be 32 or 16, got %d", fn, qblock);
  if (splits < 0 || splits > 8) return set_error(GFX_ERR_INVALID, "%s: splits must be in [0, 8], got %d", fn, splits);
  if (out_dtype != GFX_DTYPE_F32 && out_dtype != GFX_DTYPE_F16 && out_dtype != GFX_DTYPE_BF16)
    return set_error(GFX_ERR_INVALID, "%s: unsupported out dtype %d, expected float32/float16/bfloat16", fn, out_dtype);
  if ((reinterpret_cast<uintptr_t>(a_q4) & 15) || (reinterpret_cast<uintptr_t>(b_q4) & 15) ||
      (reinterpret_cast<uintptr_t>(b_scale) & 15))
    return set_error(GFX_ERR_INVALID, "%s: packed A, packed B and B_scale must be 16-byte aligned", fn);
  if (M == 0) return GFX_OK;
  const size_t need = w4a4_exact_workspace(M, N, K, qblock);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return set_error(GFX_ERR_INVALID, "%s: needs a 16-byte aligned workspace of %zu bytes (w4a4_gemm_exact_workspace_"
                     "bytes), got %zu", fn, need, workspace ? workspace_bytes : (size_t)0);
  const int dev = current_device();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = check_device_health(fn, dev, nullptr, 0, st);
  if (rc) return rc;
  return launch_w4a4_exact(a_q4, a_scale, b_q4, b_scale, qblock, bias, y, out_dtype, M, N, K, splits, workspace, st,
                           sm_count(dev));
}

int attention_block_rows(int qk_mode) {
  if (qk_mode < 0 || qk_mode > 2) {
    set_error(GFX_ERR_INVALID, "attention_block_rows: qk_mode must be 0 fp16 / 1 int8 / 2 int4, got %d", qk_mode);
    return -1;
  }
  return attention_rows_per_block(qk_mode);
}

int attention_max_tiles(void) { return kAttentionMaxTiles; }

int attention(int qk_mode, int pv_mode, const void* q, const float* q_scale, const void* k, const float* k_scale,
              const void* vt, const float* v_scale, const uint8_t* keep, void* out, int B, int H, int KVH, int Lq,
              int Lk, float skip_below, gfx_stream_t stream) {
  const char* fn = "attention";
  if (qk_mode < 0 || qk_mode > 2)
    return set_error(GFX_ERR_INVALID, "%s: qk_mode must be 0 fp16 / 1 int8 / 2 int4, got %d", fn, qk_mode);
  if (pv_mode < 0 || pv_mode > 1)
    return set_error(GFX_ERR_INVALID, "%s: pv_mode must be 0 fp16 / 1 u8, got %d", fn, pv_mode);
  if (B < 0 || H < 0 || Lq < 0 || KVH <= 0 || Lk <= 0 || H % KVH != 0)
    return set_error(GFX_ERR_INVALID, "%s: need B, H, Lq >= 0, Lk >= 1 and H (%d) a multiple of KVH (%d); got B=%d "
                     "Lq=%d Lk=%d", fn, H, KVH, B, Lq, Lk);
  if (!q || !k || !vt || !out)
    return set_error(GFX_ERR_INVALID, "%s: Q, K, Vt and out must be device pointers", fn);
  if (qk_mode != 0 && (!q_scale || !k_scale))
    return set_error(GFX_ERR_INVALID, "%s: the int Q.K modes need q_scale and k_scale", fn);
  if (pv_mode == 1 && !v_scale) return set_error(GFX_ERR_INVALID, "%s: the u8 P.V mode needs v_scale", fn);
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(k) & 15) ||
      (reinterpret_cast<uintptr_t>(vt) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(q_scale) & 3) || (reinterpret_cast<uintptr_t>(k_scale) & 3) ||
      (reinterpret_cast<uintptr_t>(v_scale) & 3))
    return set_error(GFX_ERR_INVALID, "%s: Q, K, Vt and out must be 16-byte aligned, the scales 4-byte aligned", fn);
  const long long n_tiles = (Lk + 63) / 64;
  if (keep && n_tiles > kAttentionMaxTiles)
    return set_error(GFX_ERR_INVALID, "%s: keep supports at most %d key tiles, got %lld", fn, kAttentionMaxTiles,
                     n_tiles);
  if (H > 65535 || B > 65535)
    return set_error(GFX_ERR_UNSUPPORTED, "%s: at most 65535 heads and batches, got H=%d B=%d", fn, H, B);
  return launch_attention(qk_mode, pv_mode, q, q_scale, k, k_scale, vt, v_scale, keep, out, B, H, KVH, Lq, Lk,
                          skip_below, reinterpret_cast<cudaStream_t>(stream));
}

static int check_train_quant(const char* fn, const void* x, int64_t row_stride, int R, int C, int mult_r, int mult_c,
                             const void* packed, const void* scale) {
  if (!x || !packed || !scale) return set_error(GFX_ERR_INVALID, "%s: x, packed and scale must be device pointers", fn);
  if (R < 0 || C < 0 || R % mult_r != 0 || C % mult_c != 0)
    return set_error(GFX_ERR_INVALID, "%s: x must be [R %% %d == 0, C %% %d == 0], got [%d, %d]", fn, mult_r, mult_c, R,
                     C);
  if (row_stride < C || row_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return set_error(GFX_ERR_INVALID, "%s: x rows must be 16-byte aligned, got row stride %lld", fn,
                     (long long)row_stride);
  if ((reinterpret_cast<uintptr_t>(packed) & 15) != 0 || (reinterpret_cast<uintptr_t>(scale) & 7) != 0)
    return set_error(GFX_ERR_INVALID, "%s: packed must be 16-byte and scale 8-byte aligned", fn);
  return GFX_OK;
}

int quantize_int4_rows(const void* x, int64_t row_stride, int R, int C, int sr, uint32_t seed, void* packed,
                       float* scale, gfx_stream_t stream) {
  int rc = check_train_quant("quantize_int4_rows", x, row_stride, R, C, 1, 32, packed, scale);
  if (rc) return rc;
  return launch_quantize_int4_rows(x, row_stride, R, C, sr, seed, packed, scale, reinterpret_cast<cudaStream_t>(stream));
}

int quantize_int4_cols(const void* x, int64_t row_stride, int R, int C, const float* signs, int sr, uint32_t seed,
                       void* packed, float* scale, gfx_stream_t stream) {
  int rc = check_train_quant("quantize_int4_cols", x, row_stride, R, C, 32, 1, packed, scale);
  if (rc) return rc;
  return launch_quantize_int4_cols(x, row_stride, R, C, signs, sr, seed, packed, scale,
                                   reinterpret_cast<cudaStream_t>(stream));
}

int w4a16_gemm_allgather(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype,
                         const void* bias, void* const* y_ranks, int n_ranks, int rank, int out_dtype, int M,
                         int N_local, int K, int splits, void* workspace, size_t workspace_bytes,
                         gfx_stream_t stream) {
  if (n_ranks < 1 || n_ranks > gfx::kMaxOutTargets || rank < 0 || rank >= n_ranks || !y_ranks)
    return set_error(GFX_ERR_INVALID, "w4a16_gemm_allgather: need 1 <= n_ranks <= %d, 0 <= rank < n_ranks and the "
                     "ranks' output pointers (got n_ranks=%d rank=%d)", gfx::kMaxOutTargets, n_ranks, rank);
  for (int q = 0; q < n_ranks; ++q)
    if (!y_ranks[q]) return set_error(GFX_ERR_INVALID, "w4a16_gemm_allgather: output pointer of rank %d is null", q);
  int rc = check_gemm_common("w4a16_gemm_allgather", x, x_dtype, w_q4, w_scale, scale_dtype, y_ranks[0], out_dtype,
                             M, N_local, K, splits);
  if (rc) return rc;
  if (M > 64)
    return set_error(GFX_ERR_UNSUPPORTED, "w4a16_gemm_allgather: M <= 64 only (the HBM-bound case), got M=%d", M);
  if (M == 0) return GFX_OK;
  rc = check_device_health("w4a16_gemm_allgather", current_device(), workspace,
                           workspace_bytes >= kSplitKCounterBytes ? kSplitKCounterBytes : 0,
                           reinterpret_cast<cudaStream_t>(stream));
  if (rc) return rc;
  gfx::OutTargets t{};
  for (int q = 0; q < n_ranks; ++q) t.ptr[q] = y_ranks[q];
  t.count = n_ranks;
  t.ldy = N_local * n_ranks;
  t.col0 = rank * N_local;
  t.fence_sys = 1;
  return launch_w4a16_smallm_targets(x, w_q4, w_scale, scale_dtype, bias, t, out_dtype, M, N_local, K, splits,
                                     workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream),
                                     sm_count(current_device()));
}

int w4a16_gemm_rows_allgather(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype,
                              const void* bias, void* const* y_ranks, int n_ranks, int row0, int out_dtype, int M,
                              int N, int K, int splits, void* workspace, size_t workspace_bytes, gfx_stream_t stream) {
  const char* fn = "w4a16_gemm_rows_allgather";
  if (n_ranks < 1 || n_ranks > gfx::kMaxOutTargets || row0 < 0 || !y_ranks)
    return set_error(GFX_ERR_INVALID, "%s: need 1 <= n_ranks <= %d, row0 >= 0 and the ranks' output pointers "
                     "(got n_ranks=%d row0=%d)", fn, gfx::kMaxOutTargets, n_ranks, row0);
  for (int q = 0; q < n_ranks; ++q)
    if (!y_ranks[q]) return set_error(GFX_ERR_INVALID, "%s: output pointer of rank %d is null", fn, q);
  int rc = check_gemm_common(fn, x, x_dtype, w_q4, w_scale, scale_dtype, y_ranks[0], out_dtype, M, N, K, splits);
  if (rc) return rc;
  if (M == 0) return GFX_OK;
  const int dev = current_device();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = check_device_health(fn, dev, workspace, workspace_bytes >= kSplitKCounterBytes ? kSplitKCounterBytes : 0, st);
  if (rc) return rc;
  const size_t elem = out_dtype == GFX_DTYPE_F32 ? 4 : 2;
  gfx::OutTargets t{};
  for (int q = 0; q < n_ranks; ++q) t.ptr[q] = static_cast<char*>(y_ranks[q]) + (size_t)row0 * N * elem;
  t.count = n_ranks;
  t.ldy = N;
  t.col0 = 0;
  t.fence_sys = 1;
  if (M > 64) {
    if (!w4a16_tc_supported(M, N, K, scale_dtype))
      return set_error(GFX_ERR_UNSUPPORTED, "%s: K=%d with scale dtype %d is not supported for M > 64", fn, K,
                       scale_dtype);
    return launch_w4a16_tc_targets(x, w_q4, w_scale, scale_dtype, bias, t, out_dtype, M, N, K, st, sm_count(dev));
  }
  return launch_w4a16_smallm_targets(x, w_q4, w_scale, scale_dtype, bias, t, out_dtype, M, N, K, splits, workspace,
                                     workspace_bytes, st, sm_count(dev));
}

int gfx_peer_barrier(int* const* flags_ranks, int n_ranks, int rank, gfx_stream_t stream) {
  if (n_ranks < 1 || n_ranks > gfx::kMaxOutTargets || rank < 0 || rank >= n_ranks || !flags_ranks)
    return set_error(GFX_ERR_INVALID, "gfx_peer_barrier: need 1 <= n_ranks <= %d and 0 <= rank < n_ranks",
                     gfx::kMaxOutTargets);
  for (int q = 0; q < n_ranks; ++q)
    if (!flags_ranks[q]) return set_error(GFX_ERR_INVALID, "gfx_peer_barrier: flag pointer of rank %d is null", q);
  return gfx::launch_peer_barrier(flags_ranks, n_ranks, rank, reinterpret_cast<cudaStream_t>(stream));
}

int w8a16_gemm(const void* x, int x_dtype, const void* w_q8, const void* w_scale, int scale_per_channel,
               const void* bias, void* y, int out_dtype, int M, int N, int K, int splits, void* workspace,
               size_t workspace_bytes, gfx_stream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  int rc = check_gemm_common("w8a16_gemm", x, x_dtype, w_q8, w_scale, GFX_SCALE_F32, y, out_dtype, M, N, K, splits);
  if (rc) return rc;
  if (scale_per_channel != 0 && scale_per_channel != 1)
    return set_error(GFX_ERR_INVALID, "w8a16_gemm: scale_per_channel must be 0 or 1, got %d", scale_per_channel);
  if (scale_per_channel && (reinterpret_cast<uintptr_t>(w_scale) & 1))
    return set_error(GFX_ERR_INVALID, "w8a16_gemm: float16 channel scales must be 2-byte aligned");
  if (M == 0) return GFX_OK;
  rc = check_device_health("w8a16_gemm", current_device(), nullptr, 0, reinterpret_cast<cudaStream_t>(stream));
  if (rc) return rc;
  // Every M runs on the tensor-core kernel (the int8 path has no small-M kernel yet).
  return launch_w8a16_tc(x, w_q8, w_scale, scale_per_channel, bias, y, out_dtype, M, N, K,
                         reinterpret_cast<cudaStream_t>(stream), sm_count(current_device()));
}

size_t w8a16_workspace_bytes(int M, int N, int K, int splits) {
  (void)M; (void)N; (void)K; (void)splits;
  return 0;
}

int quantize_pack_int4(const void* x, int x_dtype, void* packed, float* scale, int64_t rows, int K, int div_mode,
                       gfx_stream_t stream) {
  if (rows < 0 || K <= 0 || K % 32 != 0)
    return set_error(GFX_ERR_INVALID, "quantize_pack_int4: x must be [rows, K] with K %% 32 == 0, got [%lld, %d]",
                     (long long)rows, K);
  if (!valid_dtype(x_dtype)) return set_error(GFX_ERR_INVALID, "quantize_pack_int4: bad x dtype code %d", x_dtype);
  if (div_mode != 0 && div_mode != 1)
    return set_error(GFX_ERR_INVALID, "quantize_pack_int4: div_mode must be 0 or 1, got %d", div_mode);
  if (rows == 0) return GFX_OK;
  if (!x || !packed || !scale) return set_error(GFX_ERR_INVALID, "quantize_pack_int4: null pointer");
  if ((reinterpret_cast<uintptr_t>(packed) & 15))
    return set_error(GFX_ERR_INVALID, "quantize_pack_int4: packed output must be 16-byte aligned");
  return launch_quantize_pack_int4(x, x_dtype, packed, scale, rows, K, div_mode,
                                   reinterpret_cast<cudaStream_t>(stream));
}

int quantize_int8(const void* x, int x_dtype, void* q, float* scale, int64_t rows, int K, gfx_stream_t stream) {
  if (rows < 0 || K <= 0 || K % 32 != 0)
    return set_error(GFX_ERR_INVALID, "quantize_int8: x must be [rows, K] with K %% 32 == 0, got [%lld, %d]",
                     (long long)rows, K);
  if (!valid_dtype(x_dtype)) return set_error(GFX_ERR_INVALID, "quantize_int8: bad x dtype code %d", x_dtype);
  if (rows == 0) return GFX_OK;
  if (!x || !q || !scale) return set_error(GFX_ERR_INVALID, "quantize_int8: null pointer");
  if ((reinterpret_cast<uintptr_t>(q) & 15))
    return set_error(GFX_ERR_INVALID, "quantize_int8: q output must be 16-byte aligned");
  return launch_quantize_int8(x, x_dtype, q, scale, rows, K, reinterpret_cast<cudaStream_t>(stream));
}

int repack_q4_0(const void* raw, void* packed, float* scale, void* scale_f16, int N, int K, gfx_stream_t stream) {
  if (N < 0 || K <= 0 || K % 32 != 0)
    return set_error(GFX_ERR_INVALID, "repack_q4_0: expected N >= 0 and K %% 32 == 0, got N=%d K=%d", N, K);
  if (N == 0) return GFX_OK;
  if (!raw || !packed) return set_error(GFX_ERR_INVALID, "repack_q4_0: null pointer");
  if ((reinterpret_cast<uintptr_t>(packed) & 15) || (reinterpret_cast<uintptr_t>(raw) & 1))
    return set_error(GFX_ERR_INVALID, "repack_q4_0: packed must be 16-byte and raw 2-byte aligned");
  return launch_repack_q4_0(raw, packed, scale, scale_f16, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int int4_dequant_qblock(const void* w_q4, const void* w_scale, int scale_dtype, int qblock, void* out, int out_dtype,
                        int N, int K, gfx_stream_t stream) {
  if (qblock != 32 && qblock != 16)
    return set_error(GFX_ERR_INVALID, "int4_dequant_qblock: qblock must be 32 or 16, got %d", qblock);
  if (N < 0 || K <= 0 || K % 32 != 0)
    return set_error(GFX_ERR_INVALID, "int4_dequant_qblock: expected N >= 0 and K %% 32 == 0, got N=%d K=%d", N, K);
  if (!valid_dtype(out_dtype)) return set_error(GFX_ERR_INVALID, "int4_dequant_qblock: bad out dtype code %d", out_dtype);
  if (scale_dtype != GFX_SCALE_F32 && scale_dtype != GFX_SCALE_F16)
    return set_error(GFX_ERR_INVALID, "int4_dequant_qblock: scale dtype must be 0 or 1, got %d", scale_dtype);
  if (N == 0) return GFX_OK;
  if (!w_q4 || !w_scale || !out) return set_error(GFX_ERR_INVALID, "int4_dequant_qblock: null pointer");
  if ((reinterpret_cast<uintptr_t>(w_q4) & 3) || (reinterpret_cast<uintptr_t>(out) & 15))
    return set_error(GFX_ERR_INVALID, "int4_dequant_qblock: weights must be 4-byte and out 16-byte aligned");
  return launch_int4_dequant(w_q4, w_scale, scale_dtype, out, out_dtype, N, K, reinterpret_cast<cudaStream_t>(stream),
                             qblock);
}

int int4_dequant(const void* w_q4, const void* w_scale, int scale_dtype, void* out, int out_dtype, int N, int K,
                 gfx_stream_t stream) {
  if (N < 0 || K <= 0 || K % 32 != 0)
    return set_error(GFX_ERR_INVALID, "int4_dequant: expected N >= 0 and K %% 32 == 0, got N=%d K=%d", N, K);
  if (!valid_dtype(out_dtype)) return set_error(GFX_ERR_INVALID, "int4_dequant: bad out dtype code %d", out_dtype);
  if (scale_dtype != GFX_SCALE_F32 && scale_dtype != GFX_SCALE_F16)
    return set_error(GFX_ERR_INVALID, "int4_dequant: scale dtype must be 0 or 1, got %d", scale_dtype);
  if (N == 0) return GFX_OK;
  if (!w_q4 || !w_scale || !out) return set_error(GFX_ERR_INVALID, "int4_dequant: null pointer");
  if ((reinterpret_cast<uintptr_t>(w_q4) & 3) || (reinterpret_cast<uintptr_t>(out) & 15))
    return set_error(GFX_ERR_INVALID, "int4_dequant: weights must be 4-byte and out 16-byte aligned");
  return launch_int4_dequant(w_q4, w_scale, scale_dtype, out, out_dtype, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int scales_to_f16(const float* scale, void* scale_f16, int64_t n, int* inexact, gfx_stream_t stream) {
  if (n < 0 || !inexact || (n > 0 && (!scale || !scale_f16)))
    return set_error(GFX_ERR_INVALID, "scales_to_f16: bad arguments");
  return launch_scales_to_f16(scale, scale_f16, n, inexact, reinterpret_cast<cudaStream_t>(stream));
}

int repack_q8_0(const void* raw, void* q, float* scale, int N, int K, gfx_stream_t stream) {
  if (N < 0 || K <= 0 || K % 32 != 0)
    return set_error(GFX_ERR_INVALID, "repack_q8_0: expected N >= 0 and K a positive multiple of 32, got [%d, %d]", N,
                     K);
  if (N == 0) return GFX_OK;
  if (!raw || !q || !scale) return set_error(GFX_ERR_INVALID, "repack_q8_0: null pointer");
  if (((uintptr_t)raw & 1) || ((uintptr_t)q & 15))
    return set_error(GFX_ERR_INVALID, "repack_q8_0: raw must be 2-byte and q 16-byte aligned");
  return gfx::launch_repack_q8_0(raw, q, scale, N, K, (cudaStream_t)stream);
}

int hadamard_rotate(const void* x, int x_dtype, const float* sign, void* out, int out_dtype, int64_t rows, int K,
                    int group, gfx_stream_t stream) {
  if (group != 32 && group != 64 && group != 128)
    return set_error(GFX_ERR_INVALID, "hadamard_rotate: group must be 32, 64 or 128, got %d", group);
  if (rows < 0 || K <= 0 || K % group != 0)
    return set_error(GFX_ERR_INVALID, "hadamard_rotate: K (%d) must be a positive multiple of group %d", K, group);
  if (x_dtype < 0 || x_dtype > 2 || out_dtype < 0 || out_dtype > 2)
    return set_error(GFX_ERR_INVALID, "hadamard_rotate: dtype codes must be 0, 1 or 2");
  if (rows == 0) return GFX_OK;
  if (!x || !sign || !out) return set_error(GFX_ERR_INVALID, "hadamard_rotate: null pointer");
  return gfx::launch_hadamard_rotate(x, x_dtype, sign, out, out_dtype, rows, K, group, (cudaStream_t)stream);
}

}  // extern "C"
