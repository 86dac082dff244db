// Stand-in for <hip/hip_runtime.h> when the reference's C++ headers (heteromega/gpu_ffn.hpp,
// hipkernels/w4a16_gemm_packed.hpp) are compiled for B200: those headers only name the stream type,
// and a HIP stream handle becomes a CUDA stream handle.
#pragma once
#include <cuda_runtime.h>
typedef cudaStream_t hipStream_t;
