// Internal interface of the tensor-parallel communicator (allreduce.cu) to the kernels that write
// their outputs straight into its receive slots: the down GEMM of a tensor-parallel layer stores its
// partial rows over NVLink into the slots that the next boundary reads, so the reduce-scatter
// overlaps the GEMM tile by tile.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "hmb.h"

namespace hmb {

constexpr int kCommMaxRanks = 8;

// Where the rows of an m x h bf16 partial go before a boundary call. Slot of data from this rank in
// rank c's buffer for the call of parity p: base[c] + slot0 + (p * world + rank) * slot_bytes.
//   all = 1 (one-shot size): every row to every rank, at row * h.
//   all = 0: row r to its owner c (rows [c*m/P, (c+1)*m/P)), at (r - c*m/P) * h.
// The parity is that of the next boundary call: (epochs[0] + 1) & 1, read on the device once the
// previous calls have completed.
struct ScatterTarget {
    uint8_t *base[kCommMaxRanks];
    int64_t slot0;
    int64_t slot_bytes;
    int world, rank, all;
    int64_t m, h;
    const unsigned *epochs;
};

__host__ __device__ __forceinline__ int64_t comm_share_row(int64_t m, int world, int c) { return m * c / world; }

// The rank that owns row r of m: rows [m*c/P, m*(c+1)/P) belong to rank c.
__host__ __device__ __forceinline__ int comm_row_owner(int64_t m, int world, int64_t r) {
    return static_cast<int>(((r + 1) * world + m - 1) / m - 1);
}

#ifdef __CUDACC__
// Destination d (of scatter_count) of output row r: a bf16 row of h values in a receive slot.
__device__ __forceinline__ int scatter_count(const ScatterTarget &t) { return t.all ? t.world : 1; }
__device__ __forceinline__ uint16_t *scatter_row(const ScatterTarget &t, int par, int64_t r, int d) {
    const int c = t.all ? d : comm_row_owner(t.m, t.world, r);
    const int64_t row = t.all ? r : r - comm_share_row(t.m, t.world, c);
    return reinterpret_cast<uint16_t *>(t.base[c] + t.slot0 + (static_cast<int64_t>(par) * t.world + t.rank) * t.slot_bytes) + row * t.h;
}
__device__ __forceinline__ int scatter_parity(const ScatterTarget &t) { return (*reinterpret_cast<const volatile unsigned *>(t.epochs) + 1) & 1; }
#endif

// Ranks in the communicator's group (0 for null).
int comm_world(const hmb_comm *c);

// The scatter target of an m x h boundary on this communicator (HMB_ERR_WORKSPACE if it does not fit).
int comm_scatter_target(const hmb_comm *c, int64_t m, int64_t h, ScatterTarget *t);

// hmb_allreduce_residual_norm; with `prefilled` the partials are already in the slots (written by
// a scatter to comm_scatter_target, bf16) and y is not read. `chained` (taken where comm_chains):
// the call ends once this rank's rows are stored, and every rank's row-block counters (comm_ready)
// count the rows as they land; the next reader of the output region waits on them.
int comm_boundary(hmb_comm *c, const void *y, int y_dtype, void *x, const void *weight, int64_t m, int64_t h, float eps,
                  bool prefilled, cudaStream_t stream, uint64_t spin_limit_ns, bool chained = false);

// Whether an m x h boundary on this communicator can be chained (two-shot, two or more ranks).
bool comm_chains(const hmb_comm *c, int64_t m, int64_t h);
// This rank's row-block counters (row block mb = rows [256 mb, 256 mb + 256) of the output region
// holds all its rows once counter mb = min(256, m - 256 mb)) and the output region itself.
const unsigned *comm_ready(const hmb_comm *c);
const void *comm_out_region(const hmb_comm *c);

}  // namespace hmb
