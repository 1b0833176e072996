// W4A16 large-M GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
// Placeholder until the tcgen05 kernel lands: reports "unsupported" so the
// dispatcher keeps every shape on the split-K kernel.
#include "common.cuh"
#include "kernels.h"

namespace gfx {

GFX_DEFINE_STATUS_READER(tc_device_status)

bool w4a16_tc_supported(int M, int N, int K, int scale_dtype) {
  (void)M; (void)N; (void)K; (void)scale_dtype;
  return false;
}

int launch_w4a16_tc(const void*, const void*, const void*, int, const void*, void*, int, int, int, int, cudaStream_t,
                    int) {
  return set_error(GFX_ERR_UNSUPPORTED, "w4a16 tcgen05 kernel not built");
}

}  // namespace gfx
