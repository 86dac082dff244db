// W4A16 prefill GEMM over CTA pairs (tcgen05.mma cta_group::2), persistent, sm_100a.
//
// Same contract and arithmetic as the one-CTA kernel (gemm_w4a16_tc.cu): weights dequantized to
// bf16((q - z) * s) per 128-row group (src/hipkernels/w4a16_gemm_packed.cu:491-497), fp32
// accumulation, one rounding of the output, optional SwiGLU epilogue.
//
// A cluster of two CTAs (two SMs) computes 256 x 256 output tiles: CTA r holds rows 128 r .. 128 r
// + 127 of x and columns 128 r .. 128 r + 127 of the dequantized weights in its shared memory, and
// rows 128 r .. 128 r + 127 of the fp32 result (all 256 columns) in its TMEM. The pair walks the
// tiles round robin (tile = cluster + i * clusters; the larger operand stays in L2). Per CTA:
//   warp 0      TMA of its 128 x 64 tile of x; the completion bytes of both CTAs count on the even
//               CTA's barrier, which the even CTA arms with both tiles' bytes;
//   warp 1      allocates 512 TMEM columns (two 256-column accumulators) for the pair; in the even
//               CTA one thread issues tcgen05.mma M=256 N=256 K=16 for the pair and commits each
//               stage to the barriers of both CTAs;
//   warp 2      cp.async.bulk of the 64-row halves of its two packed tiles with scales and zeros;
//   warps 3-10  dequantize into the B operand (MN-major, SWIZZLE_128B), then arrive on the even
//               CTA's barrier; they form groups that work on successive K steps concurrently;
//   warps 11-14 epilogue: tcgen05.ld of one accumulator while the other one is being computed,
//               SwiGLU or plain store, then release the accumulator on the even CTA's barrier.
// x, packed and B stages have separate rings, so a stage of packed weights is refilled as soon as
// it is dequantized and a tile of x as soon as the MMA has read it.
//
// Every wait is bounded (one second); a wait that gives up records HMB_ERR_TIMEOUT in the status
// word and the CTA winds down. Before leaving, each role waits (bounded) for the arrivals that
// the peer CTA still owes it, so that no arrival targets a CTA that has exited.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "gemm_internal.h"
#include "tcgen05.cuh"

namespace hmb {
namespace {

using namespace tc;

constexpr int BK = 64;
constexpr int kXBytes = 128 * BK * 2;  // this CTA's 128 rows of x for one K step
constexpr int kPHalf = 2048 + 256;     // half a packed tile + its scales and zeros
constexpr int kPBytes = 2 * kPHalf;    // this CTA's two tile columns
constexpr int kBBytes = 128 * BK * 2;  // this CTA's 128 columns of the dequantized B
#ifndef HMB_PAIR_DQ_GROUPS
#define HMB_PAIR_DQ_GROUPS 4
#endif
// The dequant warps form kDqGroups groups that take successive K steps round robin: the latency of
// one step (waits, shared loads, stores, proxy fence, arrivals) overlaps across groups instead of
// bounding the step rate. A group can only start a step whose B stage the MMA has released, so the
// B ring holds one stage per group plus the one the MMA is reading.
constexpr int kDqGroups = HMB_PAIR_DQ_GROUPS;
constexpr int kDequantWarps = 8, kEpiWarps = 4;
constexpr int kDqWarpsPerGroup = kDequantWarps / kDqGroups;
constexpr int kChunksPerWarp = 8 / kDqWarpsPerGroup;  // 512-byte chunks of the CTA's packed half tiles per step
constexpr int kBStages = kDqGroups + 1, kAccStages = 2;
constexpr int kXStages = kDqGroups >= 4 ? 6 : 7, kPStages = 8;
static_assert(kDequantWarps % kDqGroups == 0 && kChunksPerWarp <= 4, "dequant groups");
constexpr int kWarpX = 0, kWarpMma = 1, kWarpP = 2, kWarpDq0 = 3, kWarpEpi0 = kWarpDq0 + kDequantWarps;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;
constexpr int kXOff = 0;
constexpr int kBOff = kXOff + kXStages * kXBytes;  // 1024-aligned stages (SWIZZLE_128B atoms)
constexpr int kPOff = kBOff + kBStages * kBBytes;
constexpr int kBarOff = kPOff + kPStages * kPBytes;
constexpr int kNumBars = 2 * (kXStages + kPStages + kAccStages) + kBStages;
static_assert(kXStages >= kBStages, "the done ring serves both the x and the B ring");
// Scatter epilogue: each epilogue warp stages 16 rows x 64 columns (bf16, 2 KB) at a time here, so its
// NVLink stores go out as 128-byte row pieces instead of one 16-byte piece per row.
constexpr int kStgOff = (kBarOff + 8 * kNumBars + 64 + 127) / 128 * 128;
constexpr int kStgBytes = 16 * 128;
constexpr int kSmemBytes = 1024 + kBarOff + 8 * kNumBars + 16;              // local output
constexpr int kSmemBytesSc = 1024 + kStgOff + kEpiWarps * kStgBytes;         // scattering (SC)
constexpr int kTmemCols = 256 * kAccStages;
static_assert(kSmemBytes <= kSmemBytesSc && kSmemBytesSc <= 227 * 1024, "shared memory plan");
static_assert(kBOff % 1024 == 0 && kPOff % 1024 == 0, "stage alignment");

// 8 outputs (16 bytes) at column col of output row tok: into y, or over NVLink into the receive slots
// of a tensor-parallel communicator (every rank's, or the row owner's).
__device__ __forceinline__ void store_out16(const PairArgs &a, int par, int64_t tok, int64_t col, uint4 v) {
    if (!a.scatter) {
        *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.y) + tok * a.ldy + col) = v;
        return;
    }
    const int nd = scatter_count(a.sc);
    for (int d = 0; d < nd; ++d) *reinterpret_cast<uint4 *>(scatter_row(a.sc, par, tok, d) + col) = v;
}

// Epilogue of one split of a split-K tile, run by the 4 epilogue warps of a CTA (thread = row
// 32 q + lane of this CTA's 128 rows). The split's fp32 sums go to its slot of the workspace and the
// accumulator is released; the splits of the tile meet at a counter (all of them are resident); then
// each split adds the slots, in split order, for its share of the rows and writes the outputs.
template <bool F16, int EPI>
__device__ __forceinline__ void split_epilogue(const PairArgs &a, uint32_t taddr, int unit, int tile, int mb, int nb, int rank,
                                               int q, int lane, volatile int *abort, uint32_t release_bar, int par) {
    const int S = a.k_splits, ks = unit % S, row = 32 * q + lane;
    constexpr int kRowFloats = 256, kSlotFloats = 128 * kRowFloats;
    float *part = a.split_ws + (static_cast<int64_t>(tile * S + ks) * 2 + rank) * kSlotFloats;
    for (int cb = 0; cb < 8; ++cb) {
        uint32_t v[32];
        tmem_ld32(taddr + 32 * cb, v);
        float *dst = part + row * kRowFloats + 32 * cb;
#pragma unroll
        for (int g8 = 0; g8 < 4; ++g8) {
            float o[8];
#pragma unroll
            for (int p = 0; p < 8; ++p) o[p] = __uint_as_float(v[8 * g8 + perm_pos(p)]);
            __stcg(reinterpret_cast<float4 *>(dst + 8 * g8), make_float4(o[0], o[1], o[2], o[3]));
            __stcg(reinterpret_cast<float4 *>(dst + 8 * g8 + 4), make_float4(o[4], o[5], o[6], o[7]));
        }
    }
    fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(release_bar);  // the accumulator is free
    unsigned *cnt = a.split_cnt + 2 * (tile * 2 + rank);
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (q == 0 && lane == 0) {
        __threadfence();
        atomicAdd(cnt, 1u);
        const uint64_t start = global_ns();
        for (uint32_t i = 0;; ++i) {
            unsigned c;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(c) : "l"(cnt) : "memory");
            if (static_cast<int>(c) >= S) break;
            if ((i & 15) == 15 && (*abort || global_ns() - start > kWaitLimitNs)) {
                *abort = 1;
                atomicOr(a.status, 1);
                break;
            }
            __nanosleep(64);
        }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!*abort) {
        // This split's rows [r0, r1) of the CTA's 128; work items of 8 outputs, spread over 128 threads.
        const int r0 = 128 * ks / S, r1 = 128 * (ks + 1) / S;
        const float *slot0 = a.split_ws + (static_cast<int64_t>(tile * S) * 2 + rank) * kSlotFloats;
        const int64_t split_stride = 2 * static_cast<int64_t>(kSlotFloats);
        constexpr int kItemsPerRow = EPI == HMB_EPI_SWIGLU ? 16 : 32;  // 128 channels or 256 columns, 8 each
        for (int item = row; item < (r1 - r0) * kItemsPerRow; item += 128) {
            const int rr = r0 + item / kItemsPerRow, c8 = item % kItemsPerRow;
            const int tk = 256 * mb + 128 * rank + rr;
            if (tk >= a.m) continue;
            if constexpr (EPI == HMB_EPI_SWIGLU) {
                // channels 8 c8 .. + 7 of block pair chb = c8 / 8: gate columns 128 chb + 8 (c8 % 8), up + 64
                const int chb = c8 >> 3, j8 = c8 & 7;
                const int gc = 128 * chb + 8 * j8;
                float g[8], u[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) g[e] = u[e] = 0.0f;
                for (int sp = 0; sp < S; ++sp) {
                    const float *src = slot0 + sp * split_stride + rr * kRowFloats;
                    const float4 g0 = __ldcg(reinterpret_cast<const float4 *>(src + gc));
                    const float4 g1 = __ldcg(reinterpret_cast<const float4 *>(src + gc + 4));
                    const float4 u0 = __ldcg(reinterpret_cast<const float4 *>(src + gc + 64));
                    const float4 u1 = __ldcg(reinterpret_cast<const float4 *>(src + gc + 68));
                    g[0] += g0.x; g[1] += g0.y; g[2] += g0.z; g[3] += g0.w; g[4] += g1.x; g[5] += g1.y; g[6] += g1.z; g[7] += g1.w;
                    u[0] += u0.x; u[1] += u0.y; u[2] += u0.z; u[3] += u0.w; u[4] += u1.x; u[5] += u1.y; u[6] += u1.z; u[7] += u1.w;
                }
                uint32_t o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    uint32_t pr = 0;
#pragma unroll
                    for (int hl = 0; hl < 2; ++hl) {
                        const float gg = round16<F16>(g[2 * e + hl]), uu = round16<F16>(u[2 * e + hl]);
                        pr |= to16<F16>(gg / (1.0f + __expf(-gg)) * uu) << (16 * hl);
                    }
                    o[e] = pr;
                }
                uint16_t *y = static_cast<uint16_t *>(a.y) + static_cast<int64_t>(tk) * a.ldy + (2 * nb + chb) * kTileN + 8 * j8;
                *reinterpret_cast<uint4 *>(y) = make_uint4(o[0], o[1], o[2], o[3]);
            } else {
                float acc8[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) acc8[e] = 0.0f;
                for (int sp = 0; sp < S; ++sp) {
                    const float *src = slot0 + sp * split_stride + rr * kRowFloats + 8 * c8;
                    const float4 v0 = __ldcg(reinterpret_cast<const float4 *>(src));
                    const float4 v1 = __ldcg(reinterpret_cast<const float4 *>(src + 4));
                    acc8[0] += v0.x; acc8[1] += v0.y; acc8[2] += v0.z; acc8[3] += v0.w;
                    acc8[4] += v1.x; acc8[5] += v1.y; acc8[6] += v1.z; acc8[7] += v1.w;
                }
                if (a.y_f32) {
                    float *y = static_cast<float *>(a.y) + static_cast<int64_t>(tk) * a.ldy + nb * 256 + 8 * c8;
                    *reinterpret_cast<float4 *>(y) = make_float4(acc8[0], acc8[1], acc8[2], acc8[3]);
                    *reinterpret_cast<float4 *>(y + 4) = make_float4(acc8[4], acc8[5], acc8[6], acc8[7]);
                } else {
                    uint32_t o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[e] = to16<F16>(acc8[2 * e]) | (to16<F16>(acc8[2 * e + 1]) << 16);
                    store_out16(a, par, tk, nb * 256 + 8 * c8, make_uint4(o[0], o[1], o[2], o[3]));
                }
            }
        }
    }
    // The last split to finish resets the tile's counters for the next call.
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (q == 0 && lane == 0 && atomicAdd(cnt + 1, 1u) == static_cast<unsigned>(S - 1)) {
        atomicExch(cnt, 0u);
        atomicExch(cnt + 1, 0u);
    }
}

template <bool F16, int EPI, bool SC = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ PairArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + kBarOff;
    // done(j % kXStages) completes when the pair MMA of K step j has finished reading its x and B
    // stages (one commit per step; kXStages >= kBStages, so neither ring can lap it).
    auto full_x = [&](int s) { return bars + 8 * s; };
    auto done = [&](int s) { return bars + 8 * (kXStages + s); };
    auto full_p = [&](int s) { return bars + 8 * (2 * kXStages + s); };
    auto empty_p = [&](int s) { return bars + 8 * (2 * kXStages + kPStages + s); };
    auto full_b = [&](int s) { return bars + 8 * (2 * kXStages + 2 * kPStages + s); };
    auto tmem_full = [&](int s) { return bars + 8 * (2 * kXStages + 2 * kPStages + kBStages + s); };
    auto tmem_empty = [&](int s) { return bars + 8 * (2 * kXStages + 2 * kPStages + kBStages + kAccStages + s); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kBarOff + 8 * kNumBars);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster = static_cast<int>(cluster_id_x()), nclusters = static_cast<int>(nclusters_x());
    const int num_k = 2 * a.k_tiles;
    // Work unit u = (tile u / k_splits, K steps [k0, k1) of split u % k_splits). With k_splits > 1 all
    // units are resident at once (units <= clusters), and the splits of a tile add up in the epilogue.
    const int num_units = a.num_tiles * a.k_splits;
    auto unit_k0 = [&](int u) { return (u % a.k_splits) * a.k_per_split; };
    auto unit_k1 = [&](int u) { return min(num_k, unit_k0(u) + a.k_per_split); };
    // Tile t -> (row block, column block) in bands: a band of `band` row blocks (band_rows) whose x
    // stays in L2 while the column blocks of the weights stream past it, row blocks fastest inside
    // the band; or the mirror image with a band of column blocks. The pairs working at one time hold
    // consecutive tiles, so each weight (or x) block comes from DRAM about once per band.
    // Row blocks from a.mb_rot on. Scattering to row owners, every rank starts at its own offset
    // (rank * m_blocks / P): at any moment rank r stores to a different owner than the other ranks,
    // instead of all ranks pouring their rows into the same one or two GPUs. Reading x from a chained
    // boundary, a rank starts at its own rows, which it stored itself.
    const int mb_shift = a.mb_rot;
    auto tile_mb = [&](int t) {
        const int per = a.band * (a.band_rows ? a.n_blocks : a.m_blocks), b = t / per, i = t - b * per;
        const int g = min(a.band, (a.band_rows ? a.m_blocks : a.n_blocks) - b * a.band);
        const int mb = a.band_rows ? b * a.band + i % g : i / g;
        return mb_shift ? (mb + mb_shift) % a.m_blocks : mb;
    };
    auto tile_nb = [&](int t) {
        const int per = a.band * (a.band_rows ? a.n_blocks : a.m_blocks), b = t / per, i = t - b * per;
        const int g = min(a.band, (a.band_rows ? a.m_blocks : a.n_blocks) - b * a.band);
        return a.band_rows ? i / g : b * a.band + i % g;
    };

    // Tile column d (0..3) of pair tile column nb, relative to the packed matrix. SwiGLU keeps them
    // as [gate, up, gate, up] of two 64-channel blocks.
    auto tile_col = [&](int nb, int d) {
        if (EPI == HMB_EPI_SWIGLU && a.col_stride != 1) return a.col_tile0 + 2 * nb + (d >> 1) + (d & 1) * a.col_stride;
        return a.col_tile0 + 4 * nb + d;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kXStages; ++s) {
            mbar_init(full_x(s), 1);  // even CTA: its producer's arrive.expect_tx (both CTAs' bytes)
            mbar_init(done(s), 1);    // the pair MMA's commit
        }
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(full_p(s), 1);
            mbar_init(empty_p(s), kDqWarpsPerGroup);
        }
        for (int s = 0; s < kBStages; ++s) mbar_init(full_b(s), 2 * kDqWarpsPerGroup);  // even CTA: one dequant group of each CTA
        for (int s = 0; s < kAccStages; ++s) {
            mbar_init(tmem_full(s), 1);
            mbar_init(tmem_empty(s), 2 * kEpiWarps);  // even CTA: epilogue warps of both CTAs
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    cluster_sync();  // the peer's barriers are initialised before anyone arrives on them
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    // Programmatic dependent launch: the packed weights (constant) stream in at once; x, which the
    // previous kernel may write, and y, which it may read, wait for it to complete.
    pdl_launch_dependents();

    if (warp == kWarpX) {
        if (lane == 0) {
            prefetch_tensormap(&tmap_x);
            pdl_wait();
            int it = 0;
            bool ok = true;
            for (int unit = cluster; ok && unit < num_units; unit += nclusters) {
                const int mb = tile_mb(unit / a.k_splits);
                const int row0 = 256 * mb + 128 * static_cast<int>(rank);
                // x from a chained boundary: the row block's rows have all landed (bounded wait), then
                // the TMA (async proxy) reads what the peers stored.
                if (a.x_ready && !wait_rows(a.x_ready + mb, static_cast<unsigned>(min(256, a.m - 256 * mb)), abort, a.status)) break;
                for (int i = unit_k0(unit); i < unit_k1(unit); ++i, ++it) {
                    const int s = it % kXStages, u = it / kXStages;
                    if (u > 0 && !mbar_wait(done(s), (u - 1) & 1, abort, a.status)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_expect_tx(full_x(s), 2 * kXBytes);
                    tma_load_2d_pair(sbase + kXOff + s * kXBytes, &tmap_x, i * BK, row0, mapa(full_x(s), 0));
                }
            }
            // The pair MMA's last commits to this CTA, one per barrier of the done ring (bounded).
            for (int j = std::max(0, it - kXStages); j < it; ++j) mbar_wait(done(j % kXStages), (j / kXStages) & 1, abort, a.status);
        }
    } else if (warp == kWarpP) {
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int unit = cluster; ok && unit < num_units; unit += nclusters) {
                const int nb = tile_nb(unit / a.k_splits);
                const uint8_t *col_base[2];
                for (int d = 0; d < 2; ++d)
                    col_base[d] = a.packed + tile_index(tile_col(nb, 2 * static_cast<int>(rank) + d), 0, a.tiles_k_total, a.tiles_n_total) * kTileBytes;
                for (int i = unit_k0(unit); i < unit_k1(unit); ++i, ++it) {
                    const int s = it % kPStages, u = it / kPStages;
                    if (u > 0 && !mbar_wait(empty_p(s), (u - 1) & 1, abort, a.status)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full_p(s), kPBytes);
                    const int kt = i >> 1, h = i & 1;
                    for (int d = 0; d < 2; ++d) {
                        const uint8_t *t = col_base[d] + static_cast<int64_t>(kt) * kTileBytes;
                        const uint32_t pd = sbase + kPOff + s * kPBytes + d * kPHalf;
                        bulk_load(pd, t + h * 2048, 2048, full_p(s));
                        bulk_load(pd + 2048, t + 4096, 256, full_p(s));
                    }
                }
            }
            // Copies still in flight land before the CTA leaves (bounded).
            for (int j = std::max(0, it - kPStages); j < it; ++j) mbar_wait(empty_p(j % kPStages), (j / kPStages) & 1, abort, a.status);
        }
    } else if (warp == kWarpMma) {
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_f16(F16, 256, 256);
            // x: K-major, 128-byte rows, 8-row groups 1 KB apart. B: MN-major, two 64-column atoms
            // 1 KB apart, 8-row K groups 2 KB apart. Per MMA (K = 16) x advances 32 bytes, B 4 KB.
            const uint32_t a_lo0 = smem_desc_lo(sbase + kXOff, 16), b_lo0 = smem_desc_lo(sbase + kBOff, 1024);
            constexpr uint32_t a_hi = smem_desc_hi(1024), b_hi = smem_desc_hi(2048);
            int it = 0, t = 0;
            bool ok = true;
            for (int unit = cluster; ok && unit < num_units; unit += nclusters, ++t) {
                const int acc = t % kAccStages, ua = t / kAccStages;
                const int k0 = unit_k0(unit);
                if (ua > 0 && !mbar_wait(tmem_empty(acc), (ua - 1) & 1, abort, a.status)) break;
                fence_after_sync();
                const uint32_t d = tmem + 256 * acc;
                for (int i = k0; i < unit_k1(unit); ++i, ++it) {
                    const int sx = it % kXStages, sb = it % kBStages;
                    // full_b implies full_x: the even CTA's dequant warps wait for both CTAs' x tiles
                    // before they arrive.
                    if (!mbar_wait(full_b(sb), (it / kBStages) & 1, abort, a.status)) {
                        ok = false;
                        break;
                    }
                    fence_after_sync();
                    const uint32_t a_lo = a_lo0 + sx * (kXBytes >> 4), b_lo = b_lo0 + sb * (kBBytes >> 4);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        umma_f16_pair_lohi(d, a_lo + kk * 2, a_hi, b_lo + kk * 256, b_hi, idesc, i != k0 || kk != 0);
                    umma_commit_pair(done(sx), 3);
                }
                if (ok) umma_commit_pair(tmem_full(acc), 3);
            }
            // The last releases of each accumulator by the epilogues of both CTAs (bounded).
            for (int j = std::max(0, t - kAccStages); j < t; ++j) mbar_wait(tmem_empty(j % kAccStages), (j / kAccStages) & 1, abort, a.status);
        }
    } else if (warp < kWarpEpi0) {
        // Dequantization: warp j belongs to group g = j / kDqWarpsPerGroup, which takes the K steps
        // with it % kDqGroups == g, and handles kChunksPerWarp of the step's eight 512-byte chunks
        // (chunk ch: tile column dl = ch / 4 of this CTA, quarter c = ch % 4 of its 64-row half tile).
        // Lane L of chunk c takes the 16 bytes at 16 L: K rows 8 ga + 4 (L & 1) .. + 3
        // (ga = 2 c + L / 16) of column group cc = (L / 2) % 8.
        const int j = warp - kWarpDq0, g = j / kDqWarpsPerGroup, w = j % kDqWarpsPerGroup;
        const int dl = (w * kChunksPerWarp) >> 2, c0 = (w * kChunksPerWarp) & 3;
        const int cc = (lane >> 1) & 7;
        uint32_t st_off[kChunksPerWarp][4];
#pragma unroll
        for (int r = 0; r < kChunksPerWarp; ++r) {
            const int ga = 2 * (c0 + r) + (lane >> 4);
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                const int rr = 4 * (lane & 1) + wi;
                st_off[r][wi] = ga * 2048 + dl * 1024 + rr * 128 + ((cc ^ rr) << 4);
            }
        }
        const uint32_t ld_off = dl * kPHalf + 16 * lane + 512 * c0;
        int it = 0;
        bool ok = true;
        for (int unit = cluster; ok && unit < num_units; unit += nclusters) {
            for (int i = unit_k0(unit); i < unit_k1(unit); ++i, ++it) {
                if (it % kDqGroups != g) continue;
                const int s = it % kPStages, sb = it % kBStages, jb = it - kBStages;
                if (!mbar_wait(full_p(s), (it / kPStages) & 1, abort, a.status) ||
                    (jb >= 0 && !mbar_wait(done(jb % kXStages), (jb / kXStages) & 1, abort, a.status)) ||
                    (leader && !mbar_wait(full_x(it % kXStages), (it / kXStages) & 1, abort, a.status))) {
                    ok = false;
                    break;
                }
                const uint8_t *pk = smem + kPOff + s * kPBytes + dl * kPHalf;
                uint32_t sp[4], zp[4];
                group_consts<F16>(pk + 2048, pk + 2048 + 128, cc, sp, zp);
                uint4 wv[kChunksPerWarp];
#pragma unroll
                for (int r = 0; r < kChunksPerWarp; ++r) wv[r] = *reinterpret_cast<const uint4 *>(smem + kPOff + s * kPBytes + ld_off + 512 * r);
                uint8_t *bt = smem + kBOff + sb * kBBytes;
#pragma unroll
                for (int r = 0; r < kChunksPerWarp; ++r) {
                    *reinterpret_cast<uint4 *>(bt + st_off[r][0]) = dequant_word<F16>(wv[r].x, sp, zp);
                    *reinterpret_cast<uint4 *>(bt + st_off[r][1]) = dequant_word<F16>(wv[r].y, sp, zp);
                    *reinterpret_cast<uint4 *>(bt + st_off[r][2]) = dequant_word<F16>(wv[r].z, sp, zp);
                    *reinterpret_cast<uint4 *>(bt + st_off[r][3]) = dequant_word<F16>(wv[r].w, sp, zp);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_cluster(mapa(full_b(sb), 0));
                    mbar_arrive(empty_p(s));
                }
            }
        }
    } else {
        // Epilogue: warp q = warp % 4 reads TMEM lanes 32 q .. 32 q + 31 (rows of this CTA).
        const int q = warp & 3;
        pdl_wait();
        // With a scatter target: the parity of the boundary call that will read the slots (the
        // communicator's earlier calls have completed once pdl_wait returns).
        const int par = a.scatter ? scatter_parity(a.sc) : 0;
        int t = 0;
        for (int unit = cluster; unit < num_units; unit += nclusters, ++t) {
            const int acc = t % kAccStages;
            if (!mbar_wait(tmem_full(acc), (t / kAccStages) & 1, abort, a.status)) break;
            fence_after_sync();
            const int tile = unit / a.k_splits;
            const int mb = tile_mb(tile), nb = tile_nb(tile);
            const int tok = 256 * mb + 128 * static_cast<int>(rank) + 32 * q + lane;
            const uint32_t taddr = tmem + 256 * acc + (static_cast<uint32_t>(32 * q) << 16);
            if (a.k_splits > 1) {
                split_epilogue<F16, EPI>(a, taddr, unit, tile, mb, nb, static_cast<int>(rank), q, lane, abort,
                                         mapa(tmem_empty(acc), 0), par);
                continue;
            }
            if constexpr (EPI == HMB_EPI_SWIGLU) {
                for (int ch = 0; ch < 2; ++ch) {
                    // Block pair ch: gate = columns 128 ch .. + 63, up = 128 ch + 64 .. + 127.
                    for (int hh = 0; hh < 2; ++hh) {
                        uint32_t gv[32], uv[32];
                        tmem_ld32_nowait(taddr + 128 * ch + 32 * hh, gv);
                        tmem_ld32_nowait(taddr + 128 * ch + 64 + 32 * hh, uv);
                        tmem_wait_ld();
                        if (tok < a.m) {
                            uint16_t *y = static_cast<uint16_t *>(a.y) + static_cast<int64_t>(tok) * a.ldy + (2 * nb + ch) * kTileN + 32 * hh;
#pragma unroll
                            for (int g8 = 0; g8 < 4; ++g8) {
                                uint32_t o[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    uint32_t pr = 0;
#pragma unroll
                                    for (int hl = 0; hl < 2; ++hl) {
                                        const int pp = perm_pos(2 * e + hl);
                                        const float g = round16<F16>(__uint_as_float(gv[8 * g8 + pp]));
                                        const float uu = round16<F16>(__uint_as_float(uv[8 * g8 + pp]));
                                        pr |= to16<F16>(g / (1.0f + __expf(-g)) * uu) << (16 * hl);
                                    }
                                    o[e] = pr;
                                }
                                *reinterpret_cast<uint4 *>(y + 8 * g8) = make_uint4(o[0], o[1], o[2], o[3]);
                            }
                        }
                    }
                }
            } else if constexpr (SC) {
                // Over NVLink: 64 columns of the warp's 32 rows at a time, each half of the rows staged
                // in shared memory (16 rows x 128 bytes, 16-byte chunks swizzled by row), then every
                // store instruction writes 4 rows x 128 contiguous bytes.
                uint8_t *stg = smem + kStgOff + q * kStgBytes;
                const int tok0 = tok - lane;
                for (int cp = 0; cp < 4; ++cp) {
                    uint4 o[8];
#pragma unroll
                    for (int hv = 0; hv < 2; ++hv) {
                        uint32_t v[32];
                        tmem_ld32(taddr + 64 * cp + 32 * hv, v);
#pragma unroll
                        for (int g8 = 0; g8 < 4; ++g8) {
                            uint32_t w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                w[e] = to16<F16>(__uint_as_float(v[8 * g8 + perm_pos(2 * e)])) |
                                       (to16<F16>(__uint_as_float(v[8 * g8 + perm_pos(2 * e + 1)])) << 16);
                            o[4 * hv + g8] = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    }
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        if ((lane >> 4) == half) {
                            const int rl = lane & 15;
#pragma unroll
                            for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4 *>(stg + 128 * rl + 16 * (c ^ (rl & 7))) = o[c];
                        }
                        __syncwarp();
#pragma unroll
                        for (int s4 = 0; s4 < 4; ++s4) {
                            const int rl = 4 * s4 + (lane >> 3), c = lane & 7;
                            const uint4 w = *reinterpret_cast<const uint4 *>(stg + 128 * rl + 16 * (c ^ (rl & 7)));
                            const int row = tok0 + 16 * half + rl;
                            if (row < a.m) store_out16(a, par, row, nb * 256 + 64 * cp + 8 * c, w);
                        }
                        __syncwarp();
                    }
                }
            } else {
                for (int cb = 0; cb < 8; ++cb) {
                    uint32_t v[32];
                    tmem_ld32(taddr + 32 * cb, v);
                    if (tok < a.m && a.y_f32) {
                        float *y = static_cast<float *>(a.y) + static_cast<int64_t>(tok) * a.ldy + nb * 256 + 32 * cb;
#pragma unroll
                        for (int g8 = 0; g8 < 4; ++g8) {
                            float o[8];
#pragma unroll
                            for (int p = 0; p < 8; ++p) o[p] = __uint_as_float(v[8 * g8 + perm_pos(p)]);
                            *reinterpret_cast<float4 *>(y + 8 * g8) = make_float4(o[0], o[1], o[2], o[3]);
                            *reinterpret_cast<float4 *>(y + 8 * g8 + 4) = make_float4(o[4], o[5], o[6], o[7]);
                        }
                    } else if (tok < a.m) {
#pragma unroll
                        for (int g8 = 0; g8 < 4; ++g8) {
                            uint32_t o[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                o[e] = to16<F16>(__uint_as_float(v[8 * g8 + perm_pos(2 * e)])) |
                                       (to16<F16>(__uint_as_float(v[8 * g8 + perm_pos(2 * e + 1)])) << 16);
                            store_out16(a, par, tok, nb * 256 + 32 * cb + 8 * g8, make_uint4(o[0], o[1], o[2], o[3]));
                        }
                    }
                }
            }
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa(tmem_empty(acc), 0));
        }
        // Stores into peers' slots are visible at system scope before the boundary kernel that
        // follows this grid raises its flags.
        if (a.scatter) __threadfence_system();
    }

    fence_before_sync();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while the other may still address its shared memory or TMEM
    if (warp == kWarpMma) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

template <bool F16, int EPI, bool SC = false>
int launch(const CUtensorMap &map, const PairArgs &a, cudaStream_t stream) {
    auto kernel = gemm_pair_kernel<F16, EPI, SC>;
    constexpr int kSmem = SC ? kSmemBytesSc : kSmemBytes;
    static std::mutex mu;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64) return HMB_ERR_UNSUPPORTED;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
            if (e != cudaSuccess) {
                set_cuda_error(e);
                return HMB_ERR_CUDA;
            }
            configured[dev] = true;
        }
    }
    const int max_clusters = pair_clusters();
    if (max_clusters <= 0) return HMB_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const int clusters = std::min(a.num_tiles * a.k_splits, max_clusters);
    cfg.gridDim = dim3(2 * clusters);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, map, a);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    return launch_status();
}

}  // namespace

int pair_clusters() {
    static std::mutex mu;
    static int n_clusters[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (n_clusters[dev] == 0) {
        // Every instantiation has the same resources; ask for one of them.
        auto kernel = gemm_pair_kernel<false, HMB_EPI_STORE>;
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2 * sm_count());
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = kSmemBytes;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
        if (e != cudaSuccess || n <= 0) {
            set_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidConfiguration);
            return 0;
        }
        n_clusters[dev] = n;
    }
    return n_clusters[dev];
}

int pair_k_splits(int64_t m, int64_t k, int64_t n) {
    const int64_t tiles = (m + 255) / 256 * (n / 256), steps = k / BK;
    const int clusters = pair_clusters();
    if (tiles <= 0 || clusters <= 0 || 2 * tiles > clusters || steps < 16) return 1;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(clusters / tiles, steps / 8)));
}

size_t pair_split_bytes(int64_t m, int64_t k, int64_t n) {
    const int splits = pair_k_splits(m, k, n);
    if (splits <= 1) return 0;
    const int64_t tiles = (m + 255) / 256 * (n / 256);
    return static_cast<size_t>(tiles * splits * 2) * 128 * 256 * sizeof(float) + static_cast<size_t>(tiles * 2 * 2) * 4 + 256;
}

void pair_band_order(int64_t m, int64_t k, int64_t n, int *band_rows, int *band) {
    // A band of one operand kept in L2 (budget well under the 126 MB: the other operand streams
    // through the same cache); DRAM bytes ~ that operand once + the other once per band.
    constexpr double kBudget = 48.0 * 1024 * 1024;
    const int64_t mb = (m + 255) / 256, nb = n / 256;
    const double xrow = 256.0 * k * 2, wcol = static_cast<double>(k) * 256 * kTileBytes / (kTileK * kTileN);
    const int64_t gm = std::max<int64_t>(1, std::min<int64_t>(mb, static_cast<int64_t>(kBudget / xrow)));
    const int64_t gn = std::max<int64_t>(1, std::min<int64_t>(nb, static_cast<int64_t>(kBudget / wcol)));
    const double rows = mb * xrow + static_cast<double>((mb + gm - 1) / gm) * nb * wcol;
    const double cols = nb * wcol + static_cast<double>((nb + gn - 1) / gn) * mb * xrow;
    *band_rows = rows <= cols;
    *band = static_cast<int>(rows <= cols ? gm : gn);
}

int launch_gemm_pair(const CUtensorMap &map, const PairArgs &a, bool f16, int epilogue, cudaStream_t stream) {
    // Scattering (HMB_EPI_STORE only): its own instantiation, so the staged NVLink epilogue adds no
    // registers to the local kernels.
    if (a.scatter) return f16 ? launch<true, HMB_EPI_STORE, true>(map, a, stream) : launch<false, HMB_EPI_STORE, true>(map, a, stream);
    if (f16) return epilogue == HMB_EPI_SWIGLU ? launch<true, HMB_EPI_SWIGLU>(map, a, stream) : launch<true, HMB_EPI_STORE>(map, a, stream);
    return epilogue == HMB_EPI_SWIGLU ? launch<false, HMB_EPI_SWIGLU>(map, a, stream) : launch<false, HMB_EPI_STORE>(map, a, stream);
}

}  // namespace hmb
