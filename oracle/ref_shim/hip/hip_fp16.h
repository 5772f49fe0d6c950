// HIP -> CUDA shim: __half and its conversions come from CUDA's cuda_fp16.h.
#pragma once
#include <cuda_fp16.h>
