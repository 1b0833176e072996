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
// current. The first call on a device does that look-up and enqueues the
// clearing of the counter region (which must start at zero) on the caller's
// stream, ahead of its kernel; make that first call before any stream
// capture. Nothing here synchronises the device. Every call shares the one
// array and leaves its counters at zero: calls whose kernels overlap on the
// GPU (different streams, or the same graph launched concurrently) race on
// it, so serialise them. After a device-side wait gave up (the call returns
// GFX_ERR_DEVICE, see gfx_device_status), the next call once the status has
// been cleared re-zeroes the counters on its stream before its kernel.
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
unsigned g_scratch_epoch[64] = {};  // failure epoch at which the counters were last zeroed

// Device address of the scratch array on `dev` (the current device). The
// counter region is (re-)zeroed on `stream` at the first call and after every
// cleared device failure.
int noalloc_scratch(int dev, cudaStream_t stream, void** out) {
  if (dev < 0 || dev >= 64) return set_error(GFX_ERR_CUDA, "w4a16_gemm_noalloc: no current CUDA device (%d)", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  const unsigned epoch = failure_epoch(dev);
  bool zero = false;
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(GFX_ERR_CUDA, "w4a16_gemm_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                       cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
    zero = true;
  } else if (g_scratch_epoch[dev] != epoch) {
    zero = true;
  }
  if (zero) {
    cudaError_t e = cudaMemsetAsync(g_scratch_ptr[dev], 0, kSplitKCounterBytes, stream);
    if (e != cudaSuccess)
      return set_error(GFX_ERR_CUDA, "w4a16_gemm_noalloc: clearing the scratch counters failed: %s",
                       cudaGetErrorString(e));
    g_scratch_epoch[dev] = epoch;
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
  int rc = check_gemm_common("w4a16_gemm_noalloc", x, x_dtype, w_q4, w_scale, scale_dtype, y, out_dtype, M, N, K,
                             splits);
  if (rc) return rc;
  if (M > 64)
    return set_error(GFX_ERR_UNSUPPORTED,
                     "w4a16_gemm_noalloc: M=%d > 64; for M > 64 call w4a16_gemm with a NULL workspace (that kernel "
                     "needs no scratch)", M);
  if (M == 0) return GFX_OK;
  const int dev = current_device();
  const int sms = sm_count(dev);
  const size_t need = smallm_workspace_bytes(M, N, K, splits, sms);
  if (need > kNoAllocScratchBytes)
    return set_error(GFX_ERR_UNSUPPORTED,
                     "w4a16_gemm_noalloc: M=%d N=%d K=%d needs %zu bytes of scratch, more than the fixed %zu; "
                     "use w4a16_gemm with a workspace", M, N, K, need, kNoAllocScratchBytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  rc = noalloc_scratch(dev, st, &scratch);
  if (rc) return rc;
  rc = check_device_health("w4a16_gemm_noalloc", dev, scratch, kSplitKCounterBytes, st);
  if (rc) return rc;
  return launch_w4a16_smallm(x, w_q4, w_scale, scale_dtype, bias, y, out_dtype, M, N, K, splits, scratch,
                             kNoAllocScratchBytes, st, sms);
}
