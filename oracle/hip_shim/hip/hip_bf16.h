/* Stand-in for HIP's bf16 header (see hip_runtime.h here): HIP's
 * __hip_bfloat16 is CUDA's __nv_bfloat16 (same bits, same RNE conversions). */
#pragma once
#include <cuda_bf16.h>
typedef __nv_bfloat16 __hip_bfloat16;
