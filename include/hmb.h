/*
 * heteromega-b200: C ABI of the B200-native W4A16 SwiGLU FFN engine (libhmb.so).
 *
 * The entry points replace the kernel interfaces of glassescrab/HeteroMega's FFN hot
 * path; each declaration names the reference interface it stands in for
 * (file:line inside that project). Conventions, shared by every entry point:
 *
 *   - Plain pointers and sizes only. Device entry points take device pointers and
 *     enqueue on `stream` (0 = the legacy default stream); they never synchronize and
 *     never allocate. Host entry points (hmb_pack_*, hmb_slice_*) run on the CPU.
 *   - Return 0 (HMB_OK) or a negative hmb_status. Nothing calls exit() or throws.
 *     After HMB_ERR_CUDA, hmb_last_cuda_error() gives the cudaError_t of the call.
 *   - Packed weights use the reference's tile layout unchanged: 128 (K) x 64 (N)
 *     tiles of 4352 bytes (4096 nibble bytes, 64 bf16 scales, 64 zeros stored
 *     twice), ordered by tile column modulo 8, tile column, tile row
 *     (kernels/gpu/include/heteromega/gpu_ffn.hpp:18-20, kernels/gpu/src/pack_w4a16.cpp:30-61).
 *     A packed [packed_k, packed_n] matrix can be used through its leading [k, n] block.
 *   - Activations are row-major bf16 (or fp16 where x_dtype allows it) with a row stride
 *     in elements. Alignment: packed 16 bytes; x, y 16 bytes; strides multiples of 8.
 *   - Entry points that take `workspace` use it for split-K partial sums. It is owned by
 *     the caller, must be zero-filled once before its first use, and is left with its
 *     counter words zero after every call. Calls that run at the same time on different
 *     streams need different workspaces. hmb_*_workspace() gives the size.
 */
#ifndef HMB_H
#define HMB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *hmb_stream_t; /* a cudaStream_t */
typedef struct hmb_comm hmb_comm;         /* opaque: one rank of a tensor-parallel group */

enum { HMB_TILE_K = 128, HMB_TILE_N = 64, HMB_TILE_BYTES = 4352 };

typedef enum hmb_status {
    HMB_OK = 0,
    HMB_ERR_ARG = -1,         /* null pointer, bad size or bad enum value */
    HMB_ERR_ALIGN = -2,       /* pointer or stride alignment */
    HMB_ERR_VALUE = -3,       /* a weight or zero point outside 0..15 */
    HMB_ERR_WORKSPACE = -4,   /* workspace missing or too small */
    HMB_ERR_UNSUPPORTED = -5, /* a shape this build does not handle */
    HMB_ERR_CUDA = -6,        /* a CUDA call failed; see hmb_last_cuda_error() */
    HMB_ERR_TIMEOUT = -7      /* a bounded device-side wait gave up */
} hmb_status;

typedef enum hmb_dtype { HMB_BF16 = 0, HMB_FP16 = 1, HMB_FP32 = 2 } hmb_dtype;

/* Column order of a packed gate_up matrix of n channels (gpu_ffn.hpp:50-54). */
typedef enum hmb_gate_up_layout {
    HMB_GATE_UP_BLOCKED = 0,    /* [gate 0..n | up 0..n] */
    HMB_GATE_UP_INTERLEAVED = 1 /* per 64 channels: 64 gate columns, then 64 up columns */
} hmb_gate_up_layout;

typedef enum hmb_epilogue {
    HMB_EPI_STORE = 0, /* y = x @ W */
    HMB_EPI_SWIGLU = 1 /* W is gate_up [k, 2c] in `layout` order; y[:, j] = SiLU(gate_j) * up_j, c columns */
} hmb_epilogue;

const char *hmb_status_string(int status);
int hmb_version(void);
int hmb_last_cuda_error(void);

/* ---- packed layout, host side ------------------------------------------------------------- */

/* Bytes of a packed [k, n] matrix: (k/128) * (n/64) * 4352. -1 if k % 128 or n % 64. */
int64_t hmb_packed_bytes(int64_t k, int64_t n);

/* Position of tile (column c, row r) in a packed tiles_k x tiles_n matrix.
 * Replaces heteromega::packed_tile_index (kernels/gpu/src/pack_w4a16.cpp:100-107). */
int64_t hmb_packed_tile_index(int64_t c, int64_t r, int64_t tiles_k, int64_t tiles_n);

/* Packs q [k, n] (0..15), scales [k/128, n] (bf16 bits) and zeros [k/128, n] (0..15) into `out`
 * (hmb_packed_bytes(k, n) bytes). HMB_ERR_VALUE if a value exceeds 15.
 * Replaces heteromega::pack_w4a16 (gpu_ffn.hpp:34; pack_w4a16.cpp:9-66) and HeteroMosaic's
 * _pack_weights_packed without padding (py/unified_llm_w4a16/llama3_8b_w4a16_model.py:546-656). */
int hmb_pack_w4a16(const uint8_t *q, const uint16_t *scales_bf16, const uint8_t *zeros, int64_t k, int64_t n, uint8_t *out);

/* Tile counts of the channel slice [begin, end) of an FFN layer with `hidden` rows and `inter`
 * channels: gate_up [hidden, 2(end-begin)] and down [end-begin, hidden]. */
int hmb_slice_tile_counts(int64_t hidden, int64_t inter, int64_t begin, int64_t end, int64_t *gate_up_tiles,
                          int64_t *down_tiles);

/* For each tile of the slice, the source tile it copies: gate_up_src indexes the concatenation
 * [gate tiles | up tiles] of the packed gate [hidden, inter] and up [hidden, inter]; down_src
 * indexes the packed down [inter, hidden]. begin and end are multiples of 128.
 * Replaces the index computation of heteromega::slice_packed_ffn (pack_w4a16.cpp:109-165). */
int hmb_slice_tile_map(int64_t hidden, int64_t inter, int64_t begin, int64_t end, int layout, int64_t *gate_up_src,
                       int64_t *down_src);

/* ---- device ------------------------------------------------------------------------------- */

/* dst tile i = (idx[i] < src0_tiles ? src0 tile idx[i] : src1 tile idx[i] - src0_tiles).
 * idx is a device array of `count` int64. The tile gather of slice_packed_ffn
 * (pack_w4a16.cpp:124-128, 143, 158) on the device. src1 may be null when every idx < src0_tiles. */
int hmb_gather_tiles(const uint8_t *src0, int64_t src0_tiles, const uint8_t *src1, const int64_t *idx, int64_t count,
                     uint8_t *dst, hmb_stream_t stream);

/* The packer of hmb_pack_w4a16 on device pointers. Values above 15 are masked to 4 bits and make
 * the kernel set *bad_flag (a device int, may be null) to 1. */
int hmb_pack_w4a16_device(const uint8_t *q, const uint16_t *scales_bf16, const uint8_t *zeros, int64_t k, int64_t n,
                          uint8_t *out, int *bad_flag, hmb_stream_t stream);

/* out[r][c] (fp32, row stride ldo) = (q - zero) * scale for the leading [k, n] block. Exact.
 * The dequantization the reference's kernels and oracle apply
 * (src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp:255-281; gpu_ffn_test dequant, kernels/gpu/tests/test_gpu_ffn.cpp:75-80). */
int hmb_w4a16_dequant(const uint8_t *packed, int64_t packed_k, int64_t packed_n, int64_t k, int64_t n, float *out, int64_t ldo,
                      hmb_stream_t stream);

/* Decode GEMV / skinny GEMM (in-register dequantization, mma.sync tensor-core fragments), for m <= 16
 * per launch (larger m is processed in chunks of 16 rows):
 *   HMB_EPI_STORE:  y[m, n] = x[m, k] @ W[:k, start_col : start_col + n]
 *   HMB_EPI_SWIGLU: W[:k, start_col : start_col + n] is gate_up of n/2 channels in `layout` order and
 *                   y[m, n/2] = bf16(SiLU(g) * u) with g, u the bf16-rounded gate and up sums.
 * x_dtype: HMB_BF16 or HMB_FP16; y_dtype: x_dtype or HMB_FP32 (unrounded sums, HMB_EPI_STORE only).
 * split_k <= 0 picks the split from the shape; a split > 1 needs the workspace.
 * Replaces hipkernels::w4a16_gemv_fused_packed (include/hipkernels/w4a16_gemm_packed.hpp:52-53) and
 * heteromega::gemv_w4a16 (gpu_ffn.hpp:98-99), plus the SiLU*up that the model runs after gate/up
 * (kernels/gpu/src/silu_mul.cu; unified_llm_w4a16.cpp:2881-2883). */
int hmb_w4a16_gemv(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype, void *y,
                   int64_t ldy, int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue, int layout,
                   int split_k, void *workspace, size_t workspace_bytes, hmb_stream_t stream);
size_t hmb_w4a16_gemv_workspace(int64_t m, int64_t k, int64_t n, int epilogue, int split_k);

/* hmb_w4a16_gemv without a workspace argument, for callers that cannot allocate device memory (a host
 * runtime that owns the device memory pool and exposes no scratch API, or a plugin ABI that hands over
 * only input and output buffers). No counterpart in the reference: its kernels take scratch from the
 * PyTorch caching allocator. The split-K scratch lives in a fixed 16 MiB + 64 KiB array in device
 * memory that every GPU loading libhmb.so keeps until the process exits; a call that would need more
 * (see hmb_w4a16_gemv_workspace) returns HMB_ERR_WORKSPACE before touching the device. The call
 * itself allocates nothing. The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress), and so does the first call after the device's context was replaced
 * (cudaDeviceReset), so make that first call before any stream capture. All calls share the one
 * array: each clears its counters first, and calls whose kernels overlap on the GPU (different
 * streams, or different host threads) race on it and give wrong results. */
int hmb_w4a16_gemv_noalloc(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype,
                           void *y, int64_t ldy, int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue,
                           int layout, int split_k, hmb_stream_t stream);

/* Prefill GEMM on the tcgen05 tensor cores (TMA-fed, TMEM accumulator), same operands and epilogues
 * as hmb_w4a16_gemv (y_dtype: x_dtype, or HMB_FP32 for HMB_EPI_STORE): the weights are dequantized to bf16((q - z) * s) in shared memory, products
 * accumulate in fp32, the output rounds once. For 17 to 128 rows and n % 128 == 0 the weights are the MMA's
 * A operand in TMEM (the batch range where the weight stream, not the MMA, sets the pace).
 * Needs n % 256 == 0, or n % 128 == 0 for 17 to 128 rows (HMB_ERR_UNSUPPORTED otherwise,
 * see hmb_w4a16_gemm_supports); any m. Replaces hipkernels::w4a16_gemm_fused_packed and
 * w4a16_gemm_fused_packed_tiles with fuse_activation (include/hipkernels/w4a16_gemm_packed.hpp:38-48) and
 * heteromega::gemm_w4a16 (gpu_ffn.hpp:101-107). */
int hmb_w4a16_gemm(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype, void *y,
                   int64_t ldy, int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue, int layout,
                   hmb_stream_t stream);
int hmb_w4a16_gemm_supports(int64_t m, int64_t k, int64_t n, int epilogue);
/* How hmb_w4a16_gemm (with_workspace 0) or the GEMMs of hmb_w4a16_ffn (with_workspace 1) schedule an
 * m x k x n problem on the current device, for diagnostics and tests. plan[5] receives:
 *   [0] kernel: 1 = one CTA per 128 x 256 tile, 2 = CTA pairs (tcgen05 cta_group::2) on 256 x 256 tiles,
 *       3 = the swap-AB kernel of 17 to 128 rows (dequantized weights as the MMA's A operand in TMEM);
 *   [1] kernel 2: the tile order, 1 = bands of [2] row blocks (x kept in L2 while the weight column
 *       blocks stream past), 0 = bands of [2] weight column blocks; kernel 3: 1 = stream-K shares of
 *       the (column block, K step) units (needs the workspace), 0 = whole column blocks;
 *   [2] kernel 2: that band width in blocks; [3] K splits per tile (1 = none);
 *   [4] CTAs (kernels 1 and 3) or CTA pairs (kernel 2) the launch keeps busy.
 * No counterpart in the reference (its GEMMs have a fixed grid). */
int hmb_w4a16_gemm_plan(int64_t m, int64_t k, int64_t n, int epilogue, int with_workspace, int *plan);

/* One SwiGLU FFN (or the FFN slice of one rank) end to end: y[m, h] = (SiLU(x Wg) * (x Wu)) Wd over
 * channels [0, n). gate_up is the packed [h x 2 stored] matrix in `layout` order (HMB_GATE_UP_BLOCKED
 * with n < stored: up columns start at tile column stored / 64), down the packed [stored x h] matrix
 * whose first n rows are used. y_dtype: x_dtype, or HMB_FP32 for the unrounded partial sums that a
 * tensor-parallel rank reduces. m <= 16 (decode) runs the gate/up GEMV with the SwiGLU epilogue and the
 * down GEMV per 16 rows, the second launched as a programmatic dependent of the first (it requests its
 * weights while gate/up finishes). Larger m runs the two tcgen05 GEMMs. act lives in the workspace
 * (hmb_w4a16_ffn_workspace bytes, 256-byte aligned, zero-filled once before the first call and then
 * left to the library: it resets what it uses). h, n and stored are multiples of 128.
 * Replaces heteromega::gemm_w4a16_ffn (kernels/gpu/include/heteromega/gpu_ffn.hpp:113-114,
 * kernels/gpu/src/gemm_w4a16.cu:463-502) and the GPU part of gpu_ffn_slice_forward (gpu_ffn.hpp:182-183). */
int hmb_w4a16_ffn(const uint8_t *gate_up, const uint8_t *down, int64_t h, int64_t n, int64_t stored, int layout, const void *x,
                  int64_t ldx, int x_dtype, void *y, int64_t ldy, int y_dtype, int64_t m, void *workspace, size_t workspace_bytes,
                  hmb_stream_t stream);
size_t hmb_w4a16_ffn_workspace(int64_t m, int64_t h, int64_t n);

/* Self-test of failure detection: launches one warp that waits on an mbarrier nothing arrives on and
 * gives up after limit_ns (at most 100 ms), exactly as the GEMM and GEMV waits do; afterwards
 * hmb_device_status reports HMB_ERR_TIMEOUT and the context stays usable. No counterpart in the
 * reference (its kernels have no bounded waits). */
int hmb_selftest_bounded_wait(int64_t limit_ns, hmb_stream_t stream);

/* Tensor-parallel boundary sum over NVLink peer memory (the counterpart of the per-layer partial sum:
 * heteromega::residual_add2, kernels/gpu/src/residual_add.cu:55-73; MergedFfn::add_out,
 * src/unified_llm_w4a16_hetero/merged_ffn.cpp:417). One communicator per rank of a P-rank group
 * (P <= 8, one GPU each): hmb_comm_create allocates this rank's flag words, receive slots and the
 * output region of hmb_allreduce_residual_norm (about 5 x max_bytes in all; max_bytes must be the same
 * on every rank) and writes its CUDA IPC handle (hmb_comm_handle_bytes bytes); after the handles of
 * all ranks are exchanged (rank order), hmb_comm_connect opens the peers'. The communicator's kernels
 * keep 128 CTAs resident while they run and must not share the GPU with another kernel that waits
 * on them. hmb_allreduce_partials then replaces
 * y (bf16, fp16 or fp32; elems * size a multiple of 16 bytes, at most max_bytes) on every rank by
 * the sum over the ranks: fp32 sums in rank order, one rounding, the same bits everywhere. Every
 * rank must make the same calls in the same order. Waits give up after spin_limit_ns (0: one
 * second) with HMB_ERR_TIMEOUT in the device status word. No multicast: plain stores over NVLink. */
size_t hmb_comm_handle_bytes(void);
int hmb_comm_create(int rank, int world, size_t max_bytes, hmb_comm **comm, void *handle);
int hmb_comm_connect(hmb_comm *comm, const void *handles);
int hmb_allreduce_partials(void *y, int64_t elems, int dtype, hmb_comm *comm, hmb_stream_t stream, uint64_t spin_limit_ns);
int hmb_comm_destroy(hmb_comm *comm);

/* The whole layer boundary of a tensor-parallel stack in one launch: the rank sum of hmb_allreduce_partials
 * fused with residual_norm_bf16 (kernels/gpu/include/heteromega/gpu_ffn.hpp:131-138,
 * kernels/gpu/src/residual_norm.cu:38-87; called between layers at
 * src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:2533-2540 with the GPU and NPU partials as its
 * two addends). For every row owned by this rank:
 *   x   = bf16(((x + y_0) + y_1) + ... + y_{P-1})            y_r = rank r's partial, fp32, one rounding
 *   out = bf16((x * rsqrt(sum(x^2) / h + eps)) * weight)     weight null: out = x
 * and `out`, the communicator's output region (hmb_comm_out), holds all m rows on every rank when the
 * call completes, the same bits everywhere; it is the next layer's input. y: [m, h] partials of
 * y_dtype (HMB_BF16 as the reference's GPU partial, or HMB_FP32 for unrounded sums); x: bf16 [m, h];
 * both with ld = h;
 * weight bf16 [h]; h a multiple of 8, at most 16384; m * h * 2 at most the communicator's max_bytes
 * (which must be the same on every rank). Messages up to 512 KB run one-shot: every rank owns every
 * row, so x stays whole on every rank. Larger ones reduce-scatter by rows: rank c owns rows
 * [c*m/P, (c+1)*m/P) (hmb_comm_rows), reads and updates only those rows of x, and stores its normed
 * rows into every rank's output region; the other rows of x are neither read nor written. Every rank
 * must make the same calls in the same order; waits give up after spin_limit_ns (0: one second) with
 * HMB_ERR_TIMEOUT in the device status word. A group of one runs hmb_residual_norm into the output. */
int hmb_allreduce_residual_norm(const void *y, int y_dtype, void *x, const void *weight, int64_t m, int64_t h, float eps,
                                hmb_comm *comm, hmb_stream_t stream, uint64_t spin_limit_ns);
/* One tensor-parallel FFN layer with its boundary, end to end on this rank: this rank's channel slice
 * of the layer (as hmb_w4a16_ffn: gate_up, down, h, n, stored, layout) for x[m, h] (bf16, ld = h;
 * normally the output region holding the previous boundary's result), then the boundary of
 * hmb_allreduce_residual_norm on resid[m, h] with norm_weight (null: no norm) into the output region.
 * For m > 16 on two or more ranks the down GEMM stores its partial rows over NVLink straight into
 * the receive slots the boundary reads (the owner's rows, or every rank's for one-shot sizes), so
 * the reduce-scatter overlaps the GEMM tile by tile and the boundary only sums, normalises and
 * gathers; otherwise (decode) the partial goes to the workspace, in fp32 on two or more ranks, and the
 * boundary exchanges it. workspace:
 * hmb_tp_ffn_layer_workspace(m, h, n) bytes, 256-byte aligned, zero-filled once before the first call.
 * Replaces, per layer, GpuFfnModel::forward plus the boundary of the model loop
 * (kernels/gpu/src/gpu_ffn.cpp:142-156; src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:2533-2540,
 * 2852-2865) with the partner device's partial coming from the other ranks. */
int hmb_tp_ffn_layer(hmb_comm *comm, const uint8_t *gate_up, const uint8_t *down, int64_t h, int64_t n, int64_t stored, int layout,
                     const void *x, void *resid, const void *norm_weight, float eps, int64_t m, void *workspace, size_t workspace_bytes,
                     hmb_stream_t stream, uint64_t spin_limit_ns);
size_t hmb_tp_ffn_layer_workspace(int64_t m, int64_t h, int64_t n);
/* hmb_tp_ffn_layer for the layers of a stack, overlapping each boundary's gather with the next layer's
 * gate/up GEMM (no reference counterpart: the reference has no tensor parallelism). chain is a set of
 * HMB_TP_CHAIN_* bits, taken where the boundary is two-shot and gate/up runs on CTA pairs (m > 128):
 *   HMB_TP_CHAIN_OUT  the boundary returns once this rank's rows are stored; the output region is
 *                     complete only for a following HMB_TP_CHAIN_IN call on the same communicator, which
 *                     must come next (same m, h, n), before anything else reads the region;
 *   HMB_TP_CHAIN_IN   x is the output region of the previous call, made with HMB_TP_CHAIN_OUT: the gate/up
 *                     GEMM waits per 256-row block until its rows have landed, starting at this rank's
 *                     own rows.
 * The results are the same bits as unchained calls. Any other bit is HMB_ERR_ARG. */
#define HMB_TP_CHAIN_IN 1
#define HMB_TP_CHAIN_OUT 2
int hmb_tp_ffn_layer_chained(hmb_comm *comm, const uint8_t *gate_up, const uint8_t *down, int64_t h, int64_t n, int64_t stored,
                             int layout, const void *x, void *resid, const void *norm_weight, float eps, int64_t m, void *workspace,
                             size_t workspace_bytes, hmb_stream_t stream, uint64_t spin_limit_ns, int chain);
/* The output region of hmb_allreduce_residual_norm: *ptr (256-byte aligned), *bytes = max_bytes. */
int hmb_comm_out(hmb_comm *comm, void **ptr, size_t *bytes);
/* Rows [*begin, *end) of an m x h boundary whose residual this rank keeps (all rows when one-shot). */
int hmb_comm_rows(const hmb_comm *comm, int64_t m, int64_t h, int64_t *begin, int64_t *end);

/* Reads and clears the device status word of the current device: *status = HMB_ERR_TIMEOUT if a kernel
 * gave up a bounded wait since the last call, else HMB_OK. Synchronizes `stream`. A kernel that gave up
 * can leave split-K counters raised in the workspace it was given: after HMB_ERR_TIMEOUT, zero-fill
 * every workspace (hmb_w4a16_gemv, hmb_w4a16_ffn, hmb_tp_ffn_layer) again before its next use, or its
 * next call may pick the wrong last contributor and write wrong sums without an error. */
int hmb_device_status(int *status, hmb_stream_t stream);

/* act[m, n] = bf16(SiLU(g) * u), fp32 math, one rounding; gate_up [m, 2n] in `layout` order.
 * Replaces heteromega::silu_mul (gpu_ffn.hpp:92-93; silu_mul.cu:34-57). */
int hmb_silu_mul(const void *gate_up, int64_t ld_in, void *act, int64_t ld_out, int64_t m, int64_t n, int layout,
                 hmb_stream_t stream);

/* The layer boundary on one GPU: x[m, h] = bf16((x + a) + b) (fp32, one rounding; a and b may be null,
 * b only with a; without a, x is not written), then normed = bf16((x * rsqrt(sum(x^2) / h + eps)) * weight)
 * with the mean over the rounded x. weight null: no norm, normed (if not null) receives x. normed may be
 * null. bf16 rows; h a multiple of 8, at most 16384; strides multiples of 8 elements; 16-byte aligned
 * pointers. Replaces heteromega::residual_norm_bf16 (kernels/gpu/include/heteromega/gpu_ffn.hpp:131-138,
 * kernels/gpu/src/residual_norm.cu:24-97) without its prepared-input side output: the GEMMs here read
 * x in row order and form their own row sums. */
int hmb_residual_norm(void *x, int64_t ldx, const void *a, int64_t lda, const void *b, int64_t ldb, const void *weight, void *normed,
                      int64_t ldn, int64_t m, int64_t h, float eps, hmb_stream_t stream);

/* x[m, cols] += y_g + y_n (partials first, fp32 math, one bf16 rounding); y_g, y_n bf16 or fp32.
 * Replaces heteromega::residual_add2 (gpu_ffn.hpp:159; residual_add.cu:55-73). */
int hmb_residual_add2(void *x, int64_t ldx, const void *y_g, int64_t ldg, int g_dtype, const void *y_n, int64_t ldn,
                      int n_dtype, int64_t m, int64_t cols, hmb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* HMB_H */
