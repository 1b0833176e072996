/* Stand-in for HIP's fp16 header (see hip_runtime.h here): CUDA's __half. */
#pragma once
#include <cuda_fp16.h>
