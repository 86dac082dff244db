// Stand-in for <hip/hip_runtime.h>, only so that the reference's CPU AVX GEMV
// (src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp) compiles unchanged on a host
// without ROCm. That file only needs an event type whose query reports
// completion: the oracle harness always passes a null event.
#pragma once
#include <immintrin.h>

typedef struct hmb_shim_event *hipEvent_t;
typedef enum { hipSuccess = 0 } hipError_t;
static inline hipError_t hipEventQuery(hipEvent_t) { return hipSuccess; }
