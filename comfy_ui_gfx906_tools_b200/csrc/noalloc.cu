// W4A16 GEMM for callers that cannot allocate device memory (w4a16_gemm_noalloc).
//
// w4a16_gemm needs a caller-provided, zero-initialised scratch buffer for
// M <= 64 (split-K arrival counters and fp32 partials). Some callers cannot
// provide one: a plugin host that hands the library only its input and output
// device pointers and owns the device's memory budget itself, or code that
// runs while other work on the device forbids a synchronising cudaMalloc /
// cudaFree. For them this entry point runs the same small-M kernel with its
// scratch in a fixed array in the library's own device memory.
//
// The array below is a file-scope __device__ variable: every GPU that loads
// the library holds its kNoAllocScratchBytes until the process exits. In host
// code the array's name only stands for the symbol, so its device address is
// looked up with cudaGetSymbolAddress, once per device, with that device
// current. The first call on a device does that set-up (and clears the
// counter region, which must start at zero); make that first call before any
// stream capture. Every call shares the one array and leaves its counters at
// zero: calls whose kernels overlap on the GPU (different streams, or the
// same graph launched concurrently) race on it, so serialise them.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace gfx {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB: counters + fp32 partials
static_assert(kNoAllocScratchBytes > kSplitKCounterBytes, "scratch must hold the counter region");

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {};

// Device address of the scratch array on `dev` (the current device).
int noalloc_scratch(int dev, void** out) {
  if (dev < 0 || dev >= 64) return set_error(GFX_ERR_CUDA, "w4a16_gemm_noalloc: no current CUDA device (%d)", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(GFX_ERR_CUDA, "w4a16_gemm_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                       cudaGetErrorString(e));
    e = cudaMemset(p, 0, kSplitKCounterBytes);  // arrival counters start at zero; calls re-arm them
    if (e != cudaSuccess)
      return set_error(GFX_ERR_CUDA, "w4a16_gemm_noalloc: clearing the scratch counters failed: %s",
                       cudaGetErrorString(e));
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess)
      return set_error(GFX_ERR_CUDA, "w4a16_gemm_noalloc: set-up failed: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return GFX_OK;
}

}  // namespace
}  // namespace gfx

using namespace gfx;

extern "C" int w4a16_gemm_noalloc(const void* x, int x_dtype, const void* w_q4, const void* w_scale, int scale_dtype,
                                  const void* bias, void* y, int out_dtype, int M, int N, int K, int splits,
                                  gfx_stream_t stream) {
  if (M < 0 || N <= 0 || K <= 0 || K % 32 != 0)
    return set_error(GFX_ERR_INVALID, "w4a16_gemm_noalloc: expected M >= 0, N > 0, K > 0, K %% 32 == 0; got M=%d N=%d K=%d",
                     M, N, K);
  if (M > 64)
    return set_error(GFX_ERR_UNSUPPORTED,
                     "w4a16_gemm_noalloc: M=%d > 64; for M > 64 call w4a16_gemm with a NULL workspace (that kernel "
                     "needs no scratch)", M);
  if (x_dtype != GFX_DTYPE_BF16)
    return set_error(GFX_ERR_UNSUPPORTED, "w4a16_gemm_noalloc: activations must be bfloat16 (dtype code 2), got %d",
                     x_dtype);
  if (out_dtype != GFX_DTYPE_F32 && out_dtype != GFX_DTYPE_F16 && out_dtype != GFX_DTYPE_BF16)
    return set_error(GFX_ERR_INVALID, "w4a16_gemm_noalloc: bad out dtype code %d", out_dtype);
  if (scale_dtype != GFX_SCALE_F32 && scale_dtype != GFX_SCALE_F16)
    return set_error(GFX_ERR_INVALID, "w4a16_gemm_noalloc: scale dtype must be 0 (f32) or 1 (f16), got %d", scale_dtype);
  if (scale_dtype == GFX_SCALE_F16 && K % 64 != 0)
    return set_error(GFX_ERR_UNSUPPORTED, "w4a16_gemm_noalloc: float16 scales need K %% 64 == 0 (K=%d)", K);
  if (splits < 0 || splits > kMaxSplits)
    return set_error(GFX_ERR_INVALID, "w4a16_gemm_noalloc: splits must be in [0, %d], got %d", kMaxSplits, splits);
  if (M == 0) return GFX_OK;
  if (!x || !w_q4 || !w_scale || !y) return set_error(GFX_ERR_INVALID, "w4a16_gemm_noalloc: null pointer");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w_q4) & 15) ||
      (reinterpret_cast<uintptr_t>(w_scale) & 3))
    return set_error(GFX_ERR_INVALID, "w4a16_gemm_noalloc: x and weights must be 16-byte, scales 4-byte aligned");
  const int dev = current_device();
  const int sms = sm_count(dev);
  const size_t need = smallm_workspace_bytes(M, N, K, splits, sms);
  if (need > kNoAllocScratchBytes)
    return set_error(GFX_ERR_UNSUPPORTED,
                     "w4a16_gemm_noalloc: M=%d N=%d K=%d needs %zu bytes of scratch, more than the fixed %zu; "
                     "use w4a16_gemm with a workspace", M, N, K, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  int rc = noalloc_scratch(dev, &scratch);
  if (rc) return rc;
  return launch_w4a16_smallm(x, w_q4, w_scale, scale_dtype, bias, y, out_dtype, M, N, K, splits, scratch,
                             kNoAllocScratchBytes, reinterpret_cast<cudaStream_t>(stream), sms);
}
