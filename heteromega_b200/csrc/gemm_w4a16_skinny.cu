// W4A16 GEMM for batches of 17 to 128 rows on sm_100a: the dequantized weights are the MMA's A
// operand in tensor memory.
//
// Same contract and arithmetic as the other GEMMs (gemm_w4a16_tc.cu): weights dequantized to
// bf16((q - z) * s) per 128-row group (src/hipkernels/w4a16_gemm_packed.cu:491-497), fp32
// accumulation, one rounding of the output, optional SwiGLU epilogue.
//
// With at most 128 rows of x the work is the weight stream: 0.53 bytes of packed weights per weight
// from HBM, and little arithmetic per weight. The kernels with weights as the B operand stage every
// dequantized weight in shared memory (a 2-byte store and a 2-byte tensor-core read per weight), which
// makes shared-memory bandwidth, not HBM, the limit. Here the products are computed transposed,
//     D[weight column, token] = A[weight column, K] . x[token, K]^T,
// A = the dequantized weights, written by the dequant warps straight into TMEM (tcgen05.st), and
// B = the x tile, staged by TMA in shared memory (K-major, SWIZZLE_128B). Shared memory then carries
// only the packed tiles and x.
//
// Work: a column block is 128 weight columns (two tile columns; for SwiGLU the gate and the up tile
// column of 64 channels) over all of K, one packed tile (128 rows) = two steps of 64 rows. With a
// workspace the (block, K tile) units are cut into equal contiguous shares, one per SM ("stream-K"): a
// block split between CTAs is finished by the last one to arrive, which adds the fp32 partial sums of
// every part in part order (results do not depend on timing). Without a workspace each CTA takes whole
// blocks round robin.
//
// Copies are few and large and come from two threads: per K tile one 4352-byte bulk copy per tile
// column (the whole tile with its scales and zeros), and per step one TMA of x. Measured per 64-row
// step of a 70B gate/up launch at 64 rows (clock64 per role in CTA 0): the x tile arrives about 3,700
// cycles after its TMA and the ring holds 8 steps, which sets a step to about 750 cycles; the MMA
// thread needs about 320 cycles to issue a step's 4 MMAs and commit, and a dequant warp about 630.
// The x tile is re-read from L2 by every SM for each of its blocks (at 64 rows about twice the weight
// bytes). Variants that cut that stream (up to four blocks per x tile, or CTA pairs that each stage half
// of every x tile and share M = 256 MMAs) were at most 15% faster per launch: neither the x stream nor
// MMA issue, and not HBM, sets the pace, but the latency of each step's chain from packed tile to MMA.
//
// Roles in a CTA of 15 warps:
//   warp 0      TMA of the x tile [nt tokens x 64] of each step;
//   warp 14     bulk copies of the block's two packed tiles of each K tile;
//   warp 1      allocates TMEM (8 A stages at columns 0..255, two accumulators at 256..511); one thread
//               issues tcgen05.mma (A from TMEM, M = 128, N = nt, K = 16) and commits each stage;
//   warps 2-9   dequantize, two groups of four warps (one per TMEM lane quadrant), group h taking the
//               64-row half h of every K tile: a lane reads 16 bytes of a packed tile (4 K rows x 8
//               columns), pairs the K rows with PRMT, ORs nibbles into the mantissa of bf16 128.0
//               (exact 128 + q), subtracts 128 + z (exact) and multiplies by the scale (one rounding),
//               then tcgen05.st.16x256b writes the K pairs of four weight columns into their lanes;
//   warps 10-13 epilogue: tcgen05.ld of the accumulator (one lane = one weight column), the stream-K
//               fix-up when the block was split, SwiGLU (gate and up lanes meet through shared
//               memory) or a plain store, then release the accumulator.
// TMEM lane L of quadrant q holds weight column 8 g + 2 byte + h of tile column q / 2, with
// L = 16 s + 8 h + g, byte = 2 (q % 2) + s: the lanes a tcgen05.st.16x256b of one thread reaches.
// Every wait is bounded (one second); a wait that gives up records HMB_ERR_TIMEOUT in the status word
// and the CTA winds down.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "gemm_internal.h"
#include "tcgen05.cuh"

namespace hmb {
namespace {

using namespace tc;

constexpr int BK = 64;
constexpr int kMaxNt = 128;
constexpr int kStages = 8;                 // x ring, one stage per step
constexpr int kPStages = 4;                // packed ring, one stage per K tile
constexpr int kXBytes = kMaxNt * BK * 2;   // x tile of one step (nt rows used)
constexpr int kPBytes = 2 * kTileBytes;    // the block's two packed tiles of one K tile
constexpr int kAStages = 8, kAccStages = 2;
constexpr int kACols = BK / 2;             // TMEM columns of one A stage: 64 K values as bf16 pairs
constexpr int kAccCol0 = kAStages * kACols;
constexpr int kTmemCols = 512;
constexpr int kDqWarps = 8, kEpiWarps = 4;
constexpr int kWarpDq0 = 2, kWarpEpi0 = kWarpDq0 + kDqWarps, kWarpP = kWarpEpi0 + kEpiWarps;
constexpr int kThreads = (kWarpP + 1) * 32;
constexpr int kXOff = 0;
constexpr int kPOff = kXOff + kStages * kXBytes;
constexpr int kUpOff = kPOff + kPStages * kPBytes;      // SwiGLU: up values of 64 lanes x kMaxNt tokens, bf16
constexpr int kBarOff = kUpOff + 64 * kMaxNt * 2;
constexpr int kNumBars = 2 * kStages + 2 * kPStages + kAStages + 2 * kAccStages;
constexpr int kSmemBytes = 1024 + kBarOff + 8 * kNumBars + 64;
static_assert(kSmemBytes <= 227 * 1024, "shared memory plan");
static_assert(kXBytes % 1024 == 0 && kPOff % 1024 == 0, "stage alignment");
static_assert(kAccCol0 + kAccStages * kMaxNt <= kTmemCols, "TMEM plan");

// Global column (within the 128 of a block) of TMEM lane L of quadrant q.
__host__ __device__ constexpr int lane_column(int q, int L) {
    const int s = L >> 4, h = (L >> 3) & 1, g = L & 7;
    return 64 * (q >> 1) + 8 * g + 2 * (2 * (q & 1) + s) + h;
}

// The segment i of a CTA's share: block b, K tiles [t0, t1). False when the share has no segment i.
__device__ __forceinline__ bool segment(const SkinnyArgs &a, int i, int &b, int &t0, int &t1) {
    const int P = gridDim.x, c = blockIdx.x;
    if (!a.streamk) {
        b = c + i * P;
        t0 = 0;
        t1 = a.tiles;
        return b < a.blocks;
    }
    const int64_t total = static_cast<int64_t>(a.blocks) * a.tiles;
    const int64_t u0 = total * c / P, u1 = total * (c + 1) / P;
    if (u0 >= u1) return false;
    b = static_cast<int>(u0 / a.tiles) + i;
    const int64_t base = static_cast<int64_t>(b) * a.tiles;
    if (base >= u1) return false;
    t0 = static_cast<int>(std::max<int64_t>(u0 - base, 0));
    t1 = static_cast<int>(std::min<int64_t>(u1 - base, a.tiles));
    return true;
}

// The CTA whose share holds unit u (the last c with total * c / P <= u).
__device__ __forceinline__ int owner_of(int64_t u, int64_t total, int P) { return static_cast<int>(((u + 1) * P + total - 1) / total - 1); }

template <bool F16>
__device__ __forceinline__ uint32_t dq2(uint32_t h, uint32_t zc, uint32_t s) {
    return sub_mul2<F16>(h, zc, s);
}

__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]),
        "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// tcgen05.mma with A in TMEM: D[128 x nt] (+)= A[128 x 16] . B[nt x 16]^T.
__device__ __forceinline__ void umma_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor, kind::f16: fp32 accumulate, A and B bf16 (or fp16), both K-major, N, M = 128.
__host__ __device__ constexpr uint32_t idesc_swap(bool f16, int n) {
    return (1u << 4) | ((f16 ? 0u : 1u) << 7) | ((f16 ? 0u : 1u) << 10) | (static_cast<uint32_t>(n >> 3) << 17) | ((128u >> 4) << 24);
}

template <bool F16>
__device__ __forceinline__ float round_out(float v) {
    return round16<F16>(v);
}

// One output (HMB_EPI_STORE) at column col of row tok: into y (fp32 or rounded), or rounded over
// NVLink into the receive slots of a tensor-parallel communicator (every rank's, or the row owner's).
template <bool F16>
__device__ __forceinline__ void store_out(const SkinnyArgs &a, int par, int tok, int col, float v) {
    if (a.scatter) {
        const uint16_t h = static_cast<uint16_t>(to16<F16>(v));
        const int nd = scatter_count(a.sc);
        for (int d = 0; d < nd; ++d) scatter_row(a.sc, par, tok, d)[col] = h;
    } else if (a.y_f32) {
        static_cast<float *>(a.y)[static_cast<int64_t>(tok) * a.ldy + col] = v;
    } else {
        static_cast<uint16_t *>(a.y)[static_cast<int64_t>(tok) * a.ldy + col] = static_cast<uint16_t>(to16<F16>(v));
    }
}

template <bool F16, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ SkinnyArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + kBarOff;
    // full_x / done: x of step it landed / the MMA of step it has completed (x and its A stage are free).
    // full_p / empty_p: the packed tiles of K tile j landed / both dequant groups have read them.
    auto full_x = [&](int s) { return bars + 8 * s; };
    auto done = [&](int s) { return bars + 8 * (kStages + s); };
    auto full_p = [&](int s) { return bars + 8 * (2 * kStages + s); };
    auto empty_p = [&](int s) { return bars + 8 * (2 * kStages + kPStages + s); };
    auto a_full = [&](int s) { return bars + 8 * (2 * kStages + 2 * kPStages + s); };
    auto acc_full = [&](int s) { return bars + 8 * (2 * kStages + 2 * kPStages + kAStages + s); };
    auto acc_empty = [&](int s) { return bars + 8 * (2 * kStages + 2 * kPStages + kAStages + kAccStages + s); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kBarOff + 8 * kNumBars);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *last_flag = reinterpret_cast<volatile int *>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nt = a.nt;

    // Tile column d (0, 1) of block b, relative to the packed matrix.
    auto tile_col = [&](int b, int d) {
        if (EPI == HMB_EPI_SWIGLU && a.col_stride != 1) return a.col_tile0 + b + d * a.col_stride;
        return a.col_tile0 + 2 * b + d;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full_x(s), 1);
            mbar_init(done(s), 1);
        }
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(full_p(s), 1);
            mbar_init(empty_p(s), kDqWarps);
        }
        for (int s = 0; s < kAStages; ++s) mbar_init(a_full(s), 4);
        for (int s = 0; s < kAccStages; ++s) {
            mbar_init(acc_full(s), 1);
            mbar_init(acc_empty(s), kEpiWarps);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // x of every step.
            prefetch_tensormap(&tmap_x);
            pdl_wait();
            int it = 0;
            bool ok = true;
            int b, t0, t1;
            for (int i = 0; ok && segment(a, i, b, t0, t1); ++i) {
                for (int s = 2 * t0; s < 2 * t1; ++s, ++it) {
                    const int st = it % kStages, u = it / kStages;
                    if (u > 0 && !mbar_wait(done(st), (u - 1) & 1, abort, a.status)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full_x(st), nt * BK * 2);
                    tma_load_2d(sbase + kXOff + st * kXBytes, &tmap_x, s * BK, 0, full_x(st));
                }
            }
            // Copies still in flight land before the CTA leaves (bounded).
            for (int j = std::max(0, it - kStages); j < it; ++j) mbar_wait(done(j % kStages), (j / kStages) & 1, abort, a.status);
        }
    } else if (warp == kWarpP) {
        if (lane == 0) {
            // The block's two packed tiles of every K tile (constant data: no wait for the previous kernel).
            int jt = 0;
            bool ok = true;
            int b, t0, t1;
            for (int i = 0; ok && segment(a, i, b, t0, t1); ++i) {
                const uint8_t *col_base[2];
                for (int d = 0; d < 2; ++d) col_base[d] = a.packed + tile_index(tile_col(b, d), 0, a.tiles_k_total, a.tiles_n_total) * kTileBytes;
                for (int kt = t0; kt < t1; ++kt, ++jt) {
                    const int ps = jt % kPStages, u = jt / kPStages;
                    if (u > 0 && !mbar_wait(empty_p(ps), (u - 1) & 1, abort, a.status)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full_p(ps), kPBytes);
                    for (int d = 0; d < 2; ++d)
                        bulk_load(sbase + kPOff + ps * kPBytes + d * kTileBytes, col_base[d] + static_cast<int64_t>(kt) * kTileBytes, kTileBytes,
                                  full_p(ps));
                }
            }
            for (int j = std::max(0, jt - kPStages); j < jt; ++j) mbar_wait(empty_p(j % kPStages), (j / kPStages) & 1, abort, a.status);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_swap(F16, nt);
            const uint64_t bhi = static_cast<uint64_t>(1024 >> 4) << 32 | (1ull << 46) | (2ull << 61);
            int it = 0, t = 0;
            bool ok = true;
            int b, t0, t1;
            for (int i = 0; ok && segment(a, i, b, t0, t1); ++i, ++t) {
                const int acc = t % kAccStages, ua = t / kAccStages;
                if (ua > 0 && !mbar_wait(acc_empty(acc), (ua - 1) & 1, abort, a.status)) break;
                fence_after_sync();
                const uint32_t d = tmem + kAccCol0 + kMaxNt * acc;
                for (int s = 2 * t0; s < 2 * t1; ++s, ++it) {
                    const int as = it % kAStages, st = it % kStages;
                    if (!mbar_wait(a_full(as), (it / kAStages) & 1, abort, a.status) ||
                        !mbar_wait(full_x(st), (it / kStages) & 1, abort, a.status)) {
                        ok = false;
                        break;
                    }
                    fence_after_sync();
                    const uint32_t xa = sbase + kXOff + st * kXBytes;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t bdesc = static_cast<uint64_t>(((xa + 32 * kk) & 0x3FFFF) >> 4) | (static_cast<uint64_t>(16 >> 4) << 16) | bhi;
                        umma_tmem_a(d, tmem + kACols * as + 8 * kk, bdesc, idesc, (s != 2 * t0 || kk != 0) ? 1u : 0u);
                    }
                    umma_commit(done(st));
                }
                if (ok) umma_commit(acc_full(acc));
            }
            // The epilogue's last releases (bounded).
            for (int j = std::max(0, t - kAccStages); j < t; ++j) mbar_wait(acc_empty(j % kAccStages), (j / kAccStages) & 1, abort, a.status);
        }
    } else if (warp < kWarpEpi0) {
        // Dequantization. Quadrant q = warp % 4 covers tile column d = q / 2, bytes 2 (q % 2) and
        // 2 (q % 2) + 1 of every 8-column group. Lane (g = lane / 4, t = lane % 4) reads the 16 bytes of
        // K rows 16 j + 4 t .. + 3, column group g, for each 16-row chunk j of the step.
        const int q = warp & 3, grp = (warp - kWarpDq0) >> 2;
        const int d = q >> 1, bp = q & 1;
        const int g = lane >> 2, tq = lane & 3;
        constexpr uint32_t kMagic = F16 ? 0x64006400u : 0x43004300u;
        constexpr uint32_t kMask = 0x000F000Fu;
        // This lane's load offset inside a half tile for chunk j: ((2 j + t / 2) * 8 + g) * 32 + 16 (t % 2).
        const uint32_t ld0 = static_cast<uint32_t>(((tq >> 1) * 8 + g) * 32 + 16 * (tq & 1));
        const uint32_t sel[2] = {static_cast<uint32_t>((2 * bp) | ((2 * bp) << 4) | ((4 + 2 * bp) << 8) | ((4 + 2 * bp) << 12)),
                                 static_cast<uint32_t>((2 * bp + 1) | ((2 * bp + 1) << 4) | ((5 + 2 * bp) << 8) | ((5 + 2 * bp) << 12))};
        int it = 0, jt = 0;
        bool ok = true;
        int b, t0, t1;
        for (int i = 0; ok && segment(a, i, b, t0, t1); ++i) {
            for (int kt = t0; kt < t1; ++kt, ++jt, it += 2) {
                // Group grp takes half grp of the tile: step it + grp.
                const int sit = it + grp;
                const int ps = jt % kPStages, as = sit % kAStages;
                // The packed tiles have landed; the MMA has finished reading this A stage (step sit - 4).
                if (!mbar_wait(full_p(ps), (jt / kPStages) & 1, abort, a.status) ||
                    (sit >= kAStages && !mbar_wait(done((sit - kAStages) % kStages), ((sit - kAStages) / kStages) & 1, abort, a.status))) {
                    ok = false;
                    break;
                }
                const uint8_t *tile = smem + kPOff + ps * kPBytes + d * kTileBytes;
                const uint8_t *ph = tile + grp * 2048;
                // Scales and zeros of this lane's four columns 8 g + 4 bp .. + 3 (bf16 scales at 4096 + 2 c,
                // zeros at 4224 + (c / 8) * 16 + c % 8).
                const uint2 sv = *reinterpret_cast<const uint2 *>(tile + 4096 + 2 * (8 * g + 4 * bp));
                const uint32_t zv = *reinterpret_cast<const uint32_t *>(tile + 4224 + 16 * g + 4 * bp);
                uint32_t sc[4], zc[4];  // column 8 g + 4 bp + e: (byte 2 bp + e / 2, nibble e % 2)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t s16 = ((e < 2 ? sv.x : sv.y) >> (16 * (e & 1))) & 0xFFFFu;
                    if constexpr (F16) {
                        const uint32_t h16 = f32_to_f16(__uint_as_float(s16 << 16));
                        sc[e] = h16 | (h16 << 16);
                    } else {
                        sc[e] = s16 | (s16 << 16);
                    }
                    const uint32_t z8 = (zv >> (8 * e)) & 0xFFu;
                    zc[e] = kMagic | z8 | (z8 << 16);
                }
                uint32_t r[2][16];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(ph + ld0 + 512 * j);
#pragma unroll
                    for (int sb = 0; sb < 2; ++sb) {
                        const uint32_t p01 = prmt(w.x, w.y, sel[sb]);  // K rows 4t, 4t+1 of byte 2 bp + sb
                        const uint32_t p23 = prmt(w.z, w.w, sel[sb]);  // K rows 4t+2, 4t+3
                        const int e_lo = 2 * sb, e_hi = 2 * sb + 1;
                        r[sb][4 * j + 0] = dq2<F16>(and_or(p01, kMask, kMagic), zc[e_lo], sc[e_lo]);
                        r[sb][4 * j + 1] = dq2<F16>(and_or(p23, kMask, kMagic), zc[e_lo], sc[e_lo]);
                        r[sb][4 * j + 2] = dq2<F16>(and_or(p01 >> 4, kMask, kMagic), zc[e_hi], sc[e_hi]);
                        r[sb][4 * j + 3] = dq2<F16>(and_or(p23 >> 4, kMask, kMagic), zc[e_hi], sc[e_hi]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_p(ps));  // this warp's reads of the packed stage are done
#pragma unroll
                for (int sb = 0; sb < 2; ++sb)
                    tmem_st_16x256b_x4(tmem + (static_cast<uint32_t>(32 * q + 16 * sb) << 16) + kACols * as, r[sb]);
                tmem_wait_st();
                fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full(as));
            }
        }
    } else {
        // Epilogue: warp q = warp % 4 reads TMEM lanes 32 q .. 32 q + 31 (weight columns lane_column(q, L)).
        const int q = warp & 3;
        const int col = lane_column(q, lane);
        pdl_wait();
        // With a scatter target: the parity of the boundary call that will read the slots (the
        // communicator's earlier calls have completed once pdl_wait returns).
        const int par = a.scatter ? scatter_parity(a.sc) : 0;
        const int P = gridDim.x, c = blockIdx.x;
        const int64_t total = static_cast<int64_t>(a.blocks) * a.tiles;
        int t = 0;
        int b, t0, t1;
        for (int i = 0; segment(a, i, b, t0, t1); ++i, ++t) {
            const int acc = t % kAccStages;
            if (!mbar_wait(acc_full(acc), (t / kAccStages) & 1, abort, a.status)) break;
            fence_after_sync();
            const uint32_t taddr = tmem + kAccCol0 + kMaxNt * acc + (static_cast<uint32_t>(32 * q) << 16);
            const bool whole = t0 == 0 && t1 == a.tiles;
            // Partial blocks: this part's sums go to its slot, and the last part to arrive adds all of them.
            int c_first = c, parts = 1;
            float *slot = nullptr;
            if (!whole) {
                c_first = owner_of(static_cast<int64_t>(b) * a.tiles, total, P);
                const int c_last = owner_of(static_cast<int64_t>(b + 1) * a.tiles - 1, total, P);
                parts = c_last - c_first + 1;
                const int first_block = static_cast<int>(total * c / P / a.tiles);
                slot = a.partial + (static_cast<int64_t>(2 * c + (b == first_block ? 0 : 1)) * 128 + 32 * q + lane) * kMaxNt;
            }
            // Pass over the tokens in chunks of 32 TMEM columns.
            for (int c0 = 0; c0 < nt; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                if (!whole) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        __stcg(reinterpret_cast<float4 *>(slot + c0 + e),
                               make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]), __uint_as_float(v[e + 2]), __uint_as_float(v[e + 3])));
                    continue;
                }
                if constexpr (EPI == HMB_EPI_SWIGLU) {
                    uint16_t *up = reinterpret_cast<uint16_t *>(smem + kUpOff);
                    if (q >= 2) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) up[(32 * (q - 2) + lane) * kMaxNt + c0 + e] = static_cast<uint16_t>(to16<F16>(__uint_as_float(v[e])));
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    if (q < 2) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const int tok = c0 + e;
                            if (tok >= a.m) break;
                            const float gg = round16<F16>(__uint_as_float(v[e]));
                            const float uu = from16<F16>(up[(32 * q + lane) * kMaxNt + tok]);
                            static_cast<uint16_t *>(a.y)[static_cast<int64_t>(tok) * a.ldy + 64 * b + col] =
                                static_cast<uint16_t>(to16<F16>(gg / (1.0f + __expf(-gg)) * uu));
                        }
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const int tok = c0 + e;
                        if (tok >= a.m) break;
                        store_out<F16>(a, par, tok, 128 * b + col, __uint_as_float(v[e]));
                    }
                }
            }
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty(acc));  // the accumulator is free
            if (whole) continue;

            // Stream-K fix-up: count this part in; the last part adds every part's slot in part order.
            __threadfence();
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (q == 0 && lane == 0) {
                const unsigned prev = atomicAdd(a.counters + b, 1u);
                *last_flag = prev == static_cast<unsigned>(parts - 1);
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (!*last_flag) continue;
            __threadfence();
            const int c_last = c_first + parts - 1;
            for (int c0 = 0; c0 < nt; c0 += 32) {
                float sum[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) sum[e] = 0.0f;
                for (int pc = c_first; pc <= c_last; ++pc) {
                    const int pc_first_block = static_cast<int>(total * pc / P / a.tiles);
                    const float *src = a.partial + (static_cast<int64_t>(2 * pc + (b == pc_first_block ? 0 : 1)) * 128 + 32 * q + lane) * kMaxNt + c0;
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        const float4 f = __ldcg(reinterpret_cast<const float4 *>(src + e));
                        sum[e] += f.x;
                        sum[e + 1] += f.y;
                        sum[e + 2] += f.z;
                        sum[e + 3] += f.w;
                    }
                }
                if constexpr (EPI == HMB_EPI_SWIGLU) {
                    uint16_t *up = reinterpret_cast<uint16_t *>(smem + kUpOff);
                    if (q >= 2) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) up[(32 * (q - 2) + lane) * kMaxNt + c0 + e] = static_cast<uint16_t>(to16<F16>(sum[e]));
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    if (q < 2) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const int tok = c0 + e;
                            if (tok >= a.m) break;
                            const float gg = round16<F16>(sum[e]);
                            const float uu = from16<F16>(up[(32 * q + lane) * kMaxNt + tok]);
                            static_cast<uint16_t *>(a.y)[static_cast<int64_t>(tok) * a.ldy + 64 * b + col] =
                                static_cast<uint16_t>(to16<F16>(gg / (1.0f + __expf(-gg)) * uu));
                        }
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const int tok = c0 + e;
                        if (tok >= a.m) break;
                        store_out<F16>(a, par, tok, 128 * b + col, sum[e]);
                    }
                }
            }
            if (q == 0 && lane == 0) atomicExch(a.counters + b, 0u);  // ready for the next call
        }
        // Stores into peers' slots are visible at system scope before the boundary kernel that
        // follows this grid raises its flags.
        if (a.scatter) __threadfence_system();
    }

    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

template <bool F16, int EPI>
int launch(const CUtensorMap &map, const SkinnyArgs &a, int grid, cudaStream_t stream) {
    auto kernel = gemm_skinny_kernel<F16, EPI>;
    static std::mutex mu;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64) return HMB_ERR_UNSUPPORTED;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
            if (e != cudaSuccess) {
                set_cuda_error(e);
                return HMB_ERR_CUDA;
            }
            configured[dev] = true;
        }
    }
    const cudaError_t e = launch_pdl(kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, map, a);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    return launch_status();
}

}  // namespace

bool skinny_supported(int64_t m, int64_t k, int64_t n) { return m > 16 && m <= kMaxNt && k % kTileK == 0 && n % 128 == 0 && n > 0; }

int skinny_ctas(int64_t m, int64_t k, int64_t n, bool streamk) {
    const int64_t blocks = n / 128, tiles = k / kTileK;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(sm_count(), streamk ? blocks * tiles : blocks)));
}

size_t skinny_split_bytes(int64_t m, int64_t k, int64_t n) {
    if (!skinny_supported(m, k, n)) return 0;
    return static_cast<size_t>(2 * skinny_ctas(m, k, n, true)) * 128 * kMaxNt * sizeof(float);
}

int launch_gemm_skinny(const CUtensorMap &map, const SkinnyArgs &a, bool f16, int epilogue, cudaStream_t stream) {
    const int grid = skinny_ctas(a.m, static_cast<int64_t>(a.tiles) * kTileK, static_cast<int64_t>(a.blocks) * 128, a.streamk != 0);
    if (f16) return epilogue == HMB_EPI_SWIGLU ? launch<true, HMB_EPI_SWIGLU>(map, a, grid, stream) : launch<true, HMB_EPI_STORE>(map, a, grid, stream);
    return epilogue == HMB_EPI_SWIGLU ? launch<false, HMB_EPI_SWIGLU>(map, a, grid, stream) : launch<false, HMB_EPI_STORE>(map, a, grid, stream);
}

}  // namespace hmb
