// Shared helpers of libhmb: status handling, bf16/fp16 bit conversions, small PTX wrappers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hmb.h"

namespace hmb {

constexpr int kTileK = HMB_TILE_K;
constexpr int kTileN = HMB_TILE_N;
constexpr int kTileBytes = HMB_TILE_BYTES;

// Last CUDA error seen by an entry point of this thread.
void set_cuda_error(cudaError_t e);

// Returns HMB_OK, or HMB_ERR_CUDA after recording the launch error.
inline int launch_status() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    return HMB_OK;
}

inline bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

// Unique id of the current CUDA context (cuCtxGetId; 0 if it cannot be read). Device addresses that the
// library caches per device are cached together with it and looked up again when it changes, since a
// device's primary context (and every module address in it) is replaced after cudaDeviceReset.
unsigned long long current_context_id();

// Device address of the status word on the current device (cached per device and context; nullptr on
// error). A kernel that gives up a bounded wait ORs 1 into it; hmb_device_status() reads and clears it.
int *device_status_word();

// Programmatic dependent launch. A kernel launched with launch_pdl() may start while the previous
// kernel of the stream is still running: it reads only its constant weights before pdl_wait(),
// which returns once the previous kernel has completed and its writes are visible (at once when
// there is no such kernel). pdl_launch_dependents() lets the next kernel start early.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Position of tile (c, r) in a packed tiles_k x tiles_n matrix: tiles ordered by column modulo 8,
// then column, then row.
__host__ __device__ inline int64_t tile_index(int64_t c, int64_t r, int64_t tiles_k, int64_t tiles_n) {
    int64_t before = c >> 3;
    const int64_t g = c & 7;
    // Column groups 0 .. g-1 hold ceil((tiles_n - j) / 8) columns each.
    for (int64_t j = 0; j < g; ++j) before += (tiles_n - j + 7) >> 3;
    return before * tiles_k + r;
}

__device__ __forceinline__ float bf16_to_f32(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// fp32 -> bf16 / fp16 bits, round to nearest even (NaN kept as NaN).
__device__ __forceinline__ uint32_t f32_to_bf16(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
__device__ __forceinline__ uint32_t f32_to_f16(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float f16_to_f32(uint32_t h) { return __half2float(__ushort_as_half(static_cast<unsigned short>(h))); }

// Round a float to the 16-bit activation type and back.
template <bool F16>
__device__ __forceinline__ float round16(float f) {
    if constexpr (F16) {
        return f16_to_f32(f32_to_f16(f));
    } else {
        return bf16_to_f32(f32_to_bf16(f));
    }
}
template <bool F16>
__device__ __forceinline__ uint32_t to16(float f) {
    if constexpr (F16) {
        return f32_to_f16(f);
    } else {
        return f32_to_bf16(f);
    }
}
template <bool F16>
__device__ __forceinline__ float from16(uint32_t b) {
    if constexpr (F16) {
        return f16_to_f32(b);
    } else {
        return bf16_to_f32(b);
    }
}

// 16-byte load that bypasses L1 (weights are read once).
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ld_stream8(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

}  // namespace hmb
