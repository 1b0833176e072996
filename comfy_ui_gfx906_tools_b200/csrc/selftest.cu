// Failure detection check for the bounded device-side waits.
//
// Every spin-wait of the GEMM kernels (mbarrier phases fed by TMA, MMA
// commits, peer CTAs) gives up after a wall-clock budget, records the code of
// the wait in a device status word and returns, so a pipeline that can never
// complete ends the launch with an error status instead of a hang, and the CUDA
// context stays usable. gfx_selftest_wait_timeout exercises exactly that path
// on the GPU: one CTA waits on an mbarrier that nothing ever arrives on, with a
// short budget, and mirrors the code into the host-visible status word as the
// GEMM kernels do. No fault, trap or endless loop is involved.
#include "common.cuh"
#include "kernels.h"

namespace gfx {

GFX_DEFINE_STATUS_READER(selftest_device_status)

__global__ void wait_timeout_selftest_kernel(unsigned long long timeout_ns, int* status_host) {
  __shared__ __align__(8) uint64_t never_arrived;
  if (threadIdx.x == 0) {
    mbar_init(&never_arrived, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_for(&never_arrived, 0, kDevErrSelfTestTimeout, timeout_ns))
    mirror_device_error(status_host);
}

}  // namespace gfx

extern "C" int gfx_selftest_wait_timeout(int timeout_us, void* stream) {
  using namespace gfx;
  if (timeout_us <= 0 || timeout_us > 1000000)
    return set_error(GFX_ERR_INVALID, "gfx_selftest_wait_timeout: timeout_us must be in (0, 1e6], got %d",
                     timeout_us);
  wait_timeout_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((unsigned long long)timeout_us * 1000ull,
                                                                   host_status_word(current_device()));
  return check_launch("wait_timeout_selftest_kernel");
}
