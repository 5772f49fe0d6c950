// HIP -> CUDA shim: __hip_bfloat16 is CUDA's __nv_bfloat16 (same RNE conversions).
#pragma once
#include <cuda_bf16.h>
using __hip_bfloat16 = __nv_bfloat16;
