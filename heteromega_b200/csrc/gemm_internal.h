// Internal interface between the GEMM entry point (gemm_w4a16_tc.cu) and the CTA-pair kernel
// (gemm_w4a16_pair.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hmb {

struct PairArgs {
    const uint8_t *packed;
    void *y;
    int64_t ldy;
    int tiles_k_total, tiles_n_total;
    int col_tile0;
    int k_tiles;     // K / 128
    int m;
    int m_blocks;    // ceil(M / 256)
    int n_blocks;    // N / 256
    int num_tiles;   // m_blocks x n_blocks
    int cols_fastest;  // tile order: column blocks fastest (x larger than the weights) or row blocks
    int col_stride;  // SwiGLU blocked layout: tile columns from gate to up; 1 = interleaved
    int y_f32;       // HMB_EPI_STORE: write the fp32 sums instead of rounding them
    int *status;     // device status word (1 after a wait gave up)
};

// Launches the CTA-pair kernel; `map` is x as a 2D tensor map with 64 x 128 boxes (SWIZZLE_128B).
int launch_gemm_pair(const CUtensorMap &map, const PairArgs &a, bool f16, int epilogue, cudaStream_t stream);

}  // namespace hmb
