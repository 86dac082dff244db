// Internal interface between the GEMM entry point (gemm_w4a16_tc.cu) and the CTA-pair kernel
// (gemm_w4a16_pair.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm_internal.h"

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
    int band_rows;   // tile order: bands of `band` row blocks (1) or of `band` column blocks (0)
    int band;
    int col_stride;  // SwiGLU blocked layout: tile columns from gate to up; 1 = interleaved
    int y_f32;       // HMB_EPI_STORE: write the fp32 sums instead of rounding them
    int *status;     // device status word (1 after a wait gave up)
    int k_splits;    // splits of K per tile (1: none)
    int k_per_split; // K steps (of 64) per split
    float *split_ws;      // k_splits > 1: [tile][split][CTA] 128 x 256 fp32 sums
    unsigned *split_cnt;  // k_splits > 1: [tile][CTA] arrival and completion counters (self-resetting)
    int scatter;          // HMB_EPI_STORE, 16-bit output: rows go to the communicator's receive slots `sc`
    ScatterTarget sc;
    const unsigned *x_ready;  // non-null: row block mb of x is complete once x_ready[mb] = min(256, m - 256 mb)
    int mb_rot;               // row blocks visited from this one on (a rank's own rows first)
};

// The band order of an m x k x n problem (m_blocks x n_blocks tiles of 256 x 256): the direction
// and width that read the fewest bytes from DRAM when a band of one operand stays in L2.
void pair_band_order(int64_t m, int64_t k, int64_t n, int *band_rows, int *band);

// CTA pairs the pair kernel keeps resident on the current device.
int pair_clusters();
// K splits for an m x n output with k/64 K steps (1 when the tiles already fill the GPU), and the
// workspace bytes they need.
int pair_k_splits(int64_t m, int64_t k, int64_t n);
size_t pair_split_bytes(int64_t m, int64_t k, int64_t n);

// Arguments of the swap-AB kernel for 17 to 128 rows (gemm_w4a16_skinny.cu).
struct SkinnyArgs {
    const uint8_t *packed;
    void *y;
    int64_t ldy;
    int tiles_k_total, tiles_n_total;
    int col_tile0;
    int col_stride;      // SwiGLU blocked layout: tile columns from gate to up; 1 = interleaved
    int tiles;           // K / 128 (packed tile rows; two steps of 64 each)
    int blocks;          // column blocks of 128 weight columns (SwiGLU: 64 channels)
    int m, nt;           // rows of x; the MMA's N (a multiple of 16, >= m, <= 128)
    int y_f32;           // HMB_EPI_STORE: write the fp32 sums instead of rounding them
    int streamk;         // 1: equal shares of the (block, step) units, split blocks summed in `partial`
    float *partial;      // streamk: 2 slots per CTA of 128 x 128 fp32
    unsigned *counters;  // streamk: one per block, zero before the call, left zero
    int *status;         // device status word (1 after a wait gave up)
    int scatter;         // HMB_EPI_STORE only: rows go to the receive slots of `sc` instead of y
    ScatterTarget sc;
};

// Whether the swap-AB kernel takes an m x k x n problem, its grid, and the workspace bytes of its
// stream-K partial sums.
bool skinny_supported(int64_t m, int64_t k, int64_t n);
int skinny_ctas(int64_t m, int64_t k, int64_t n, bool streamk);
size_t skinny_split_bytes(int64_t m, int64_t k, int64_t n);
// Launches it; `map` is x as a 2D tensor map with 64 x nt boxes (SWIZZLE_128B).
int launch_gemm_skinny(const CUtensorMap &map, const SkinnyArgs &a, bool f16, int epilogue, cudaStream_t stream);

// How gemm_run schedules an m x k x n problem: the swap-AB kernel (skinny, 17 to 128 rows), the
// CTA-pair kernel (pair) or the one-CTA kernel; the pair kernel's band order and its K splits
// (split_ws: the caller gives a large enough workspace); the skinny kernel's stream-K mode.
struct GemmPlan {
    bool skinny, streamk;
    bool pair;
    int band_rows, band;
    int k_splits, k_per_split;
};
// Workspace bytes that gemm_run's split-K and stream-K modes use for an m x k x n problem.
size_t gemm_split_bytes(int64_t m, int64_t k, int64_t n);
GemmPlan gemm_plan(int64_t m, int64_t k, int64_t n, bool split_ws, bool scatter);

// hmb_w4a16_gemm with an optional split-K workspace: split_ws (pair_split_bytes(m, k, n) bytes of
// fp32 sums) and split_cnt (4 KB of counters, zero before the first call; the kernel leaves them
// zero). Without them (nullptr) no K splits are used. With a scatter target (HMB_EPI_STORE, 16-bit
// output, n == sc->h, m == sc->m) the output rows go to a communicator's receive slots instead of y,
// always through the CTA-pair kernel.
// x_ready / x_rot (the CTA-pair kernel only, ignored by the others): wait per row block of x on the
// counters of a chained boundary before loading it, and start at row block x_rot.
int gemm_run(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype, void *y, int64_t ldy,
             int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue, int layout, void *split_ws, size_t split_ws_bytes,
             unsigned *split_cnt, cudaStream_t stream, const ScatterTarget *sc = nullptr, const unsigned *x_ready = nullptr,
             int x_rot = 0);
constexpr size_t kSplitCounterBytes = 4096;

// Launches the CTA-pair kernel; `map` is x as a 2D tensor map with 64 x 128 boxes (SWIZZLE_128B).
int launch_gemm_pair(const CUtensorMap &map, const PairArgs &a, bool f16, int epilogue, cudaStream_t stream);

}  // namespace hmb
