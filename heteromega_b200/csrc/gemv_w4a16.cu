// W4A16 decode GEMV / skinny GEMM (m <= 16 rows per launch) on the packed tile layout.
//
// What it computes is the reference's GEMV definition (src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp:83-289,
// kernels/gpu/src/gemv_w4a16.cu:27-28): for each 128-row tile and column,
//     s * (sum_r q_r * x_r - z * sum_r x_r)     in fp32,
// summed over the tiles of a column, then rounded once. How it computes it is B200-specific:
//
//   * Work is the stream of packed tiles. The tiles of a "column set" (one tile column, or the gate
//     and up tile columns of 64 channels for the SwiGLU epilogue) form consecutive items, and the
//     whole item range is cut into equal contiguous chunks, one per warp of a grid of one CTA per
//     SM. Every warp streams its chunk through a private ring in shared memory: each tile arrives
//     as one 4352-byte cp.async.bulk (the tensor-memory-access engine, not per-lane requests) on a
//     per-stage mbarrier, and the tile's rows of x as 16-byte cp.async copies. A small matrix is
//     requested from HBM at once and a large one keeps the memory system full.
//   * The kernel is launched as a programmatic dependent of the previous kernel in the stream: it
//     requests its first weight tiles before waiting for that kernel (weights are constant), so
//     the launch and the first HBM round trip overlap the previous kernel's tail.
//   * The weights go through the tensor cores as exact integers. A nibble q becomes the bf16
//     (fp16) number 128 + q (1024 + q) by OR-ing it into the mantissa of 0x4300 (0x6400), so one
//     PRMT and two LOP3 turn 4 bytes into MMA operand registers. The MMA multiplies them with x and
//     accumulates in fp32; an extra MMA with an all-ones operand yields sum_r x_r in the same
//     fragment positions. Per tile and column: s * (acc - (C + z) * sum_x) = s * (sum q*x - z*sum x).
//   * The MMA is m16n8k16 with the weights on the M side ("swap AB"): 16 output columns x 8 rows of
//     x. The packed layout stores, per K row, 8 consecutive columns in one 32-bit word. A lane with
//     g = lane/4, t = lane%4 takes column group g and K rows 4t..4t+3 of each 16-row chunk; K inside
//     a chunk is permuted so that these rows form the lane's operand pairs, and x is read with the
//     same permutation, so the dot products are unchanged. Column 2b/2b+1 of the group feed MMA
//     block b.
//   * A column set that lies inside one warp's chunk is finished from that warp's registers. One
//     that crosses chunks is finished by the last warp to contribute (an atomic counter per column
//     set): every contributor stores the fp32 sums of its valid rows, and the last one adds them in
//     chunk order with all lanes (batches of loads in flight), so results do not depend on timing.
//   * The SwiGLU epilogue writes bf16(SiLU(g) * u) from the bf16-rounded gate and up sums of the
//     same lane, so gate/up never reach HBM.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm_internal.h"

namespace hmb {
namespace {

constexpr int kSmemBudget = 227 * 1024;
constexpr int kXRowBytes = 288;  // 256 bytes of x per row and tile, padded so 4 rows hit distinct banks

// Per-warp ring stage: [the packed tile as stored: 4096 weight bytes, 128 scale bytes, 128 zero
// bytes][m x 288 x bytes]. The ring's mbarriers follow all rings (8 bytes per warp and stage).
__host__ __device__ constexpr int stage_bytes(int m) { return 4352 + kXRowBytes * m; }

struct GemvArgs {
    const uint8_t *packed;
    const uint16_t *x;
    void *y;
    float *partial;  // contributor slots of column sets that cross warp chunks
    int *counters;   // [column sets]
    int64_t ldx, ldy;
    int tiles_k_total, tiles_n_total;  // the whole packed matrix
    int col_tile0;                     // first tile column used
    int k_tiles;                       // tile rows used
    int colsets;
    int col_stride;  // tile columns between slot 0 and slot 1 of a column set (pairs only)
    int m;
    int y_f32;
    int items;  // colsets * NCOL * k_tiles
    int warps;  // warps that share the items
    int *status;  // device status word: 1 after a bounded wait gave up
};

template <bool F16>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    if constexpr (F16) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

__device__ __forceinline__ void cp_async16(uint32_t smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src),
                 "r"(bytes), "r"(bar)
                 : "memory");
}
// Wait for phase `parity` of a ring barrier; false after one second (the warp then stops and the
// status word reports HMB_ERR_TIMEOUT).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    uint64_t start = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t done;
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done)
                     : "r"(bar), "r"(parity)
                     : "memory");
        if (done) return true;
        if ((i & 63) == 63) {
            uint64_t now;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (start == 0) {
                start = now;
            } else if (now - start > 1000000000ull) {
                return false;
            }
        }
    }
}
// Shared-memory loads as plain C++ accesses: ordered after cp.async.wait_group (its "memory" clobber)
// and otherwise free for the compiler to schedule early. a is an offset from the dynamic smem base.
extern __shared__ __align__(128) uint8_t g_smem[];
__device__ __forceinline__ uint4 lds128(uint32_t a) { return *reinterpret_cast<const uint4 *>(g_smem + a); }
__device__ __forceinline__ uint2 lds64(uint32_t a) { return *reinterpret_cast<const uint2 *>(g_smem + a); }

// (a & b) | c in one LOP3 (0xEA is the truth table of that expression).
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}



template <bool F16>
__device__ __forceinline__ void mma16816_zc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                            uint32_t b1) {
    const float z = 0.0f;
    if constexpr (F16) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
    } else {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
    }
}

// Accumulates one staged tile into acc: acc += s * (sum (C+q) x - (C+z) sum x) for the lane's fragment.
// wlane: offset of the lane's 16 bytes in each 512-byte weight chunk of the tile.
// xrow[mt]: shared address of this lane's x row for token block mt (rows past m repeat row m-1; their
// results are never stored).
template <int MT, bool F16>
__device__ __forceinline__ void tile_mma(uint32_t st, uint32_t wlane, const uint32_t (&xrow)[MT], int g,
                                         float (&acc)[MT][4][4]) {
    constexpr uint32_t kMagic = F16 ? 0x64006400u : 0x43004300u;
    constexpr uint32_t kOnes = F16 ? 0x3C003C00u : 0x3F803F80u;
    constexpr float kOffset = F16 ? 1024.0f : 128.0f;
    constexpr uint32_t kMask = 0x000F000Fu;
    constexpr uint32_t kMaskHi = 0x00F000F0u;
    float d[MT][4][4];
    float sx[MT][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t bx[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const uint2 v = lds64(st + xrow[mt] + 32 * j);
            bx[mt][0] = v.x;
            bx[mt][1] = v.y;
            if (j == 0) {
                mma16816_zc<F16>(sx[mt], kOnes, kOnes, kOnes, kOnes, bx[mt][0], bx[mt][1]);
            } else {
                mma16816<F16>(sx[mt], kOnes, kOnes, kOnes, kOnes, bx[mt][0], bx[mt][1]);
            }
        }
        const uint4 w = lds128(st + wlane + 512 * j);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            // Byte b of rows (4t, 4t+1) and of rows (4t+2, 4t+3), side by side in 16-bit halves.
            const uint32_t sel = static_cast<uint32_t>(b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12));
            const uint32_t p = prmt(w.x, w.y, sel);
            const uint32_t q = prmt(w.z, w.w, sel);
            const uint32_t a0 = and_or(p, kMask, kMagic);  // column 2b, rows 4t, 4t+1
            const uint32_t a2 = and_or(q, kMask, kMagic);  // column 2b, rows 4t+2, 4t+3
            // Column 2b+1 (high nibbles). fp16 keeps them in place: 1024 + 16 q is exact in its 10-bit
            // mantissa, and the fold divides by 16. bf16 has 7 mantissa bits, so the nibble moves down.
            const uint32_t a1 = F16 ? and_or(p, kMaskHi, kMagic) : and_or(p >> 4, kMask, kMagic);
            const uint32_t a3 = F16 ? and_or(q, kMaskHi, kMagic) : and_or(q >> 4, kMask, kMagic);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                if (j == 0) {
                    mma16816_zc<F16>(d[mt][b], a0, a1, a2, a3, bx[mt][0], bx[mt][1]);
                } else {
                    mma16816<F16>(d[mt][b], a0, a1, a2, a3, bx[mt][0], bx[mt][1]);
                }
            }
        }
    }
    const uint4 sv = lds128(st + 4096 + 16 * g);
    const uint2 zv = lds64(st + 4224 + 16 * g);
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
    const uint32_t zw[2] = {zv.x, zv.y};
    // High-nibble columns of the fp16 path carry 1024 + 16 q: scale 1/16, offset 1024 + 16 z.
    constexpr float kHiScale = F16 ? 0.0625f : 1.0f;
    constexpr float kHiZ = F16 ? 16.0f : 1.0f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const float s_lo = bf16_to_f32(sw[b] & 0xFFFFu);
        const float s_hi = bf16hi_to_f32(sw[b]) * kHiScale;
        // 2^23 + z as float bits: zero byte 2b (2b+1) of the group under an exponent byte 0x4B.
        const uint32_t zsel_lo = static_cast<uint32_t>(((2 * b) & 3) | 0x7440), zsel_hi = zsel_lo + 1;
        const float zc_lo = __uint_as_float(prmt(zw[b >> 1], 0x4B000000u, zsel_lo)) - (8388608.0f - kOffset);
        const float zc_hi = fmaf(__uint_as_float(prmt(zw[b >> 1], 0x4B000000u, zsel_hi)) - 8388608.0f, kHiZ, kOffset);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            acc[mt][b][0] = fmaf(s_lo, fmaf(-zc_lo, sx[mt][0], d[mt][b][0]), acc[mt][b][0]);
            acc[mt][b][1] = fmaf(s_lo, fmaf(-zc_lo, sx[mt][1], d[mt][b][1]), acc[mt][b][1]);
            acc[mt][b][2] = fmaf(s_hi, fmaf(-zc_hi, sx[mt][2], d[mt][b][2]), acc[mt][b][2]);
            acc[mt][b][3] = fmaf(s_hi, fmaf(-zc_hi, sx[mt][3], d[mt][b][3]), acc[mt][b][3]);
        }
    }
}

template <bool F16>
__device__ __forceinline__ float silu_mul_rounded(float g, float u) {
    const float gr = round16<F16>(g), ur = round16<F16>(u);
    return gr / (1.0f + __expf(-gr)) * ur;
}

// Warp chunk that holds item x: the last gw with floor(gw * items / warps) <= x.
__device__ __forceinline__ int chunk_of(int x, int items, int warps) {
    return static_cast<int>(((static_cast<int64_t>(x) + 1) * warps + items - 1) / items - 1);
}

// Writes the finished sums of column set j from one lane's fragment (tok 2t + (i&1), column 8g + 2b + (i>>1)).
// v0 holds slot 0 (gate, or the only column), v1 slot 1 (up).
template <int MT, bool F16, int EPI>
__device__ __forceinline__ void epilogue(const GemvArgs &a, int j, int g, int t, const float (&v0)[MT][4][4],
                                         const float (&v1)[MT][4][4]) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int tok = mt * 8 + 2 * t + h;
            if (tok >= a.m) continue;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int c = 8 * g + 2 * b;  // columns c and c + 1 of the tile
                if constexpr (EPI == HMB_EPI_SWIGLU) {
                    const float lo = silu_mul_rounded<F16>(v0[mt][b][h], v1[mt][b][h]);
                    const float hi = silu_mul_rounded<F16>(v0[mt][b][2 + h], v1[mt][b][2 + h]);
                    uint16_t *y = static_cast<uint16_t *>(a.y) + tok * a.ldy + j * kTileN + c;
                    *reinterpret_cast<uint32_t *>(y) = to16<F16>(lo) | (to16<F16>(hi) << 16);
                } else {
                    const int col = j * kTileN + c;
                    if (a.y_f32) {
                        *reinterpret_cast<float2 *>(static_cast<float *>(a.y) + tok * a.ldy + col) =
                            make_float2(v0[mt][b][h], v0[mt][b][2 + h]);
                    } else {
                        uint16_t *y = static_cast<uint16_t *>(a.y) + tok * a.ldy + col;
                        *reinterpret_cast<uint32_t *>(y) = to16<F16>(v0[mt][b][h]) | (to16<F16>(v0[mt][b][2 + h]) << 16);
                    }
                }
            }
        }
    }
}

template <int MT>
__device__ __forceinline__ void zero(float (&v)[MT][4][4]) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[mt][b][i] = 0.0f;
}

// Walks the items of a warp chunk in order: column set j, slot s (gate/up), tile row kt.
struct Cursor {
    int j, s, kt;
    __device__ __forceinline__ void next(int k_tiles, int ncol) {
        if (++kt == k_tiles) {
            kt = 0;
            if (++s == ncol) {
                s = 0;
                ++j;
            }
        }
    }
};

// One warp's share of a GEMV: its contiguous chunk of items, streamed through its private ring.
// prefetch() requests the weight tiles of the first S - 1 items (they never depend on an earlier
// kernel); start() requests their rows of x; run() consumes the chunk and finishes its column sets.
// Ring stages have the size of the kernel's largest m (a compile-time constant), and the ring position
// and barrier phase are wrap-around counters, so the per-tile address arithmetic needs no division.
template <int NCOL, int MT, int W, int S, int MAXM, bool F16, int EPI>
struct GemvWarp {
    static constexpr int kSb = stage_bytes(MAXM);
    const GemvArgs &a;
    int lane, g, t, gw, b, e, per_set;
    uint32_t smem_base, ring, wlane, bars;
    int64_t x_src[(16 * MAXM + 31) / 32];
    uint32_t x_dst[(16 * MAXM + 31) / 32];
    uint32_t xrow[MT];
    Cursor in;
    const uint8_t *in_col;
    int in_slot;  // ring stage of the next copy

    __device__ __forceinline__ GemvWarp(const GemvArgs &args) : a(args), in_slot(0) {
        const int warp = threadIdx.x >> 5;
        lane = threadIdx.x & 31;
        g = lane >> 2;
        t = lane & 3;
        gw = blockIdx.x * W + warp;
        // a.warps <= items: every chunk below it holds at least one tile; warps past it sit out.
        b = gw < a.warps ? static_cast<int>(static_cast<int64_t>(gw) * a.items / a.warps) : 0;
        e = gw < a.warps ? static_cast<int>(static_cast<int64_t>(gw + 1) * a.items / a.warps) : 0;
        per_set = NCOL * a.k_tiles;
        smem_base = static_cast<uint32_t>(__cvta_generic_to_shared(g_smem));
        ring = warp * S * kSb;
        // This lane's 16 bytes of weight chunk c are at tile + 512 c + wlane: K rows 16c + 4t .. +3, column group g.
        wlane = 256 * (t >> 1) + 32 * g + 16 * (t & 1);
        bars = smem_base + W * S * kSb + warp * S * 8;
        // x rows of a tile: 16 m copies of 16 bytes, taken by the lanes in turn (copy lane + 32 r).
#pragma unroll
        for (int r = 0; r < (16 * MAXM + 31) / 32; ++r) {
            const int c = lane + 32 * r;
            const int tok = c >> 4, piece = c & 15;
            x_dst[r] = 4352 + tok * kXRowBytes + piece * 16;
            x_src[r] = (static_cast<int64_t>(tok) * a.ldx + piece * 8) * 2;
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) xrow[mt] = 4352 + min(mt * 8 + g, a.m - 1) * kXRowBytes + 8 * t;
        in = Cursor{b / per_set, (b % per_set) / a.k_tiles, b % a.k_tiles};
        in_col = column(in);
    }

    __device__ __forceinline__ const uint8_t *column(const Cursor &c) const {
        const int base = (NCOL == 2 && a.col_stride == 1) ? 2 * c.j : c.j;
        return a.packed + tile_index(a.col_tile0 + base + c.s * a.col_stride, 0, a.tiles_k_total, a.tiles_n_total) * kTileBytes;
    }
    __device__ __forceinline__ uint32_t stage_addr(int slot) const { return ring + slot * kSb; }

    // The weight tile of the item at `in`, as one bulk copy (lane 0) onto its stage's barrier.
    __device__ __forceinline__ void issue_w(int slot) {
        if (lane == 0) {
            const uint32_t bar = bars + 8 * slot;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // after this warp's reads of the stage
            mbar_expect_tx(bar, kTileBytes);
            bulk_load(smem_base + stage_addr(slot), in_col + static_cast<int64_t>(in.kt) * kTileBytes, kTileBytes, bar);
        }
    }
    // Rows of x of the item at `in` (cp.async, one commit group per tile), then advance `in`.
    __device__ __forceinline__ void issue_x(int slot) {
        const uint8_t *xsrc = reinterpret_cast<const uint8_t *>(a.x + in.kt * kTileK);
        const uint32_t dst = smem_base + stage_addr(slot);
#pragma unroll
        for (int r = 0; r < (16 * MAXM + 31) / 32; ++r)
            if (lane + 32 * r < 16 * a.m) cp_async16(dst + x_dst[r], xsrc + x_src[r]);
        advance();
    }
    __device__ __forceinline__ void advance() {
        const int j0 = in.j, s0 = in.s;
        in.next(a.k_tiles, NCOL);
        if (in.j != j0 || in.s != s0) in_col = column(in);
    }

    __device__ __forceinline__ void prefetch() {
        const Cursor in0 = in;
        const uint8_t *in_col0 = in_col;
        for (int p = 0; p < S - 1 && b + p < e; ++p) {
            issue_w(p);
            advance();
        }
        in = in0;
        in_col = in_col0;
    }
    __device__ __forceinline__ void start() {
#pragma unroll
        for (int p = 0; p < S - 1; ++p) {
            if (b + p < e) issue_x(p);
            cp_async_commit();
        }
        in_slot = S - 1;
    }

    // Finishes column set j from acc (slot NCOL-1) and gate (slot 0 when NCOL == 2): from registers
    // if this chunk holds all of it, else as a contributor.
    __device__ __forceinline__ void finish(int j, const float (&gate)[MT][4][4], const float (&acc)[MT][4][4]) {
        const float(&v0)[MT][4][4] = NCOL == 2 ? gate : acc;
        const int first = j * per_set, last = first + per_set - 1;
        if (first >= b && last < e) {
            epilogue<MT, F16, EPI>(a, j, g, t, v0, acc);
            return;
        }
        const int c0 = chunk_of(first, a.items, a.warps), c1 = chunk_of(last, a.items, a.warps);
        // Contributor slot (one per warp and column set it shares): the valid rows only, as
        // [slot s][token][64 columns] fp32, so small m moves little data.
        constexpr int kSlot = NCOL * MT * 16 * 32;
        float *slot = a.partial + static_cast<int64_t>(gw + j) * kSlot;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int tok = mt * 8 + 2 * t + h;
                if (tok >= a.m) continue;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int col = 8 * g + 2 * q;
                    __stcg(reinterpret_cast<float2 *>(slot + tok * kTileN + col), make_float2(v0[mt][q][h], v0[mt][q][2 + h]));
                    if (NCOL == 2)
                        __stcg(reinterpret_cast<float2 *>(slot + (a.m + tok) * kTileN + col), make_float2(acc[mt][q][h], acc[mt][q][2 + h]));
                }
            }
        __threadfence();
        __syncwarp();
        int last_one = 0;
        if (lane == 0) last_one = atomicAdd(a.counters + j, 1) == c1 - c0;
        last_one = __shfl_sync(0xffffffffu, last_one, 0);
        if (!last_one) return;
        __threadfence();
        // Last contributor: lane L sums the (token, column) pairs L, L + 32, ... over the contributors in
        // chunk order (the order does not depend on timing). Two pairs and up to kC contributors are
        // loaded at once, so the reduction costs few L2 round trips.
        constexpr int kC = 12;
        const int pairs = a.m * kTileN;
        for (int p = lane; p < pairs; p += 64) {
            const bool two = p + 32 < pairs;
            float s0[2] = {0.0f, 0.0f}, s1[2] = {0.0f, 0.0f};
            for (int c = c0; c <= c1; c += kC) {
                float l0[2][kC], l1[2][kC];
#pragma unroll
                for (int u = 0; u < kC; ++u)
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const bool ok = c + u <= c1 && (q == 0 || two);
                        const float *src = a.partial + static_cast<int64_t>(c + u + j) * kSlot + p + 32 * q;
                        l0[q][u] = ok ? __ldcg(src) : 0.0f;
                        l1[q][u] = (ok && NCOL == 2) ? __ldcg(src + pairs) : 0.0f;
                    }
#pragma unroll
                for (int u = 0; u < kC; ++u)
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        s0[q] += l0[q][u];
                        s1[q] += l1[q][u];
                    }
            }
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                if (q == 1 && !two) break;
                const int tok = (p + 32 * q) / kTileN, ycol = j * kTileN + (p + 32 * q) % kTileN;
                if constexpr (EPI == HMB_EPI_SWIGLU) {
                    static_cast<uint16_t *>(a.y)[static_cast<int64_t>(tok) * a.ldy + ycol] =
                        static_cast<uint16_t>(to16<F16>(silu_mul_rounded<F16>(s0[q], s1[q])));
                } else if (a.y_f32) {
                    static_cast<float *>(a.y)[static_cast<int64_t>(tok) * a.ldy + ycol] = s0[q];
                } else {
                    static_cast<uint16_t *>(a.y)[static_cast<int64_t>(tok) * a.ldy + ycol] = static_cast<uint16_t>(to16<F16>(s0[q]));
                }
            }
        }
        if (lane == 0) a.counters[j] = 0;
    }

    // Consumes the chunk; returns the warp's ring use count afterwards.
    __device__ __forceinline__ int run() {
        float acc[MT][4][4], gate[MT][4][4];
        zero(acc);
        zero(gate);
        Cursor cur{b / per_set, (b % per_set) / a.k_tiles, b % a.k_tiles};
        int slot = 0;
        uint32_t phase = 0;
        for (int it = b; it < e; ++it) {
            cp_async_wait<S - 2>();
            if (!mbar_wait(bars + 8 * slot, phase)) {
                if (lane == 0) atomicOr(a.status, 1);
                break;
            }
            __syncwarp();
            if (it + S - 1 < e) {
                issue_w(in_slot);
                issue_x(in_slot);
                in_slot = in_slot + 1 == S ? 0 : in_slot + 1;
            }
            cp_async_commit();
            tile_mma<MT, F16>(stage_addr(slot), wlane, xrow, g, acc);
            if (++slot == S) {
                slot = 0;
                phase ^= 1;
            }
            const int j0 = cur.j, s0 = cur.s;
            cur.next(a.k_tiles, NCOL);
            const bool set_done = cur.j != j0 || it + 1 == e;
            // acc holds the slot in progress; gate sums move aside when the up tiles start or the chunk ends on them.
            if (NCOL == 2 && s0 == 0 && (set_done || cur.s == 1)) {
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int q = 0; q < 4; ++q)
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            gate[mt][q][i] = acc[mt][q][i];
                            acc[mt][q][i] = 0.0f;
                        }
            }
            if (set_done) {
                finish(j0, gate, acc);
                zero(acc);
                zero(gate);
            }
        }
        cp_async_wait<0>();
        return e - b;
    }
};

// Initialises this warp's S ring barriers (one expected arrival each: the bulk copy's arrive.expect_tx).
template <int W, int S>
__device__ __forceinline__ void init_ring_barriers(int sb) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        const uint32_t bars = static_cast<uint32_t>(__cvta_generic_to_shared(g_smem)) + W * S * sb + warp * S * 8;
        for (int q = 0; q < S; ++q) mbar_init(bars + 8 * q, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
}

template <int NCOL, int MT, int W, int S, int MAXM, bool F16, int EPI>
__global__ void __launch_bounds__(W * 32, 1) gemv_kernel(const GemvArgs a) {
    if (static_cast<int>(blockIdx.x * W + (threadIdx.x >> 5)) >= a.warps) return;
    pdl_launch_dependents();
    init_ring_barriers<W, S>(stage_bytes(MAXM));
    GemvWarp<NCOL, MT, W, S, MAXM, F16, EPI> w(a);
    // Weights of the first S - 1 items before the previous kernel has finished; everything that
    // kernel may write (x) or read (y, the workspace) only after pdl_wait().
    w.prefetch();
    pdl_wait();
    w.start();
    w.run();
}

template <int NCOL, int MT, int W, int S, int MAXM, bool F16, int EPI>
int launch(const GemvArgs &a, cudaStream_t stream) {
    auto kernel = gemv_kernel<NCOL, MT, W, S, MAXM, F16, EPI>;
    constexpr int smem = W * S * stage_bytes(MAXM) + W * S * 8;
    static_assert(smem <= kSmemBudget, "ring too large");
    static std::mutex mu;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 64 && !configured[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) {
                set_cuda_error(e);
                return HMB_ERR_CUDA;
            }
            configured[dev] = true;
        }
    }
    const cudaError_t e = launch_pdl(kernel, dim3((a.warps + W - 1) / W), dim3(W * 32), smem, stream, a);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    return launch_status();
}

// Warps and ring depth by rows of x: stage_bytes grows with m, the rings stay within the shared-memory
// budget. The kernel is latency-bound, so more warps beat deeper rings: at 2-4 rows 12 warps x 3 stages
// (x staged for 4 rows) took 91.7 / 97.0 us per 70B layer against 101.5 / 105.2 with 8 warps x 5 / 4.
template <int NCOL, bool F16, int EPI>
int by_rows(const GemvArgs &a, cudaStream_t stream) {
    if (a.m == 1) return launch<NCOL, 1, 16, 3, 1, F16, EPI>(a, stream);
    if (a.m <= 4) return launch<NCOL, 1, 12, 3, 4, F16, EPI>(a, stream);
    if (a.m <= 8) return launch<NCOL, 1, 8, 4, 8, F16, EPI>(a, stream);
    return launch<NCOL, 2, 8, 3, 16, F16, EPI>(a, stream);
}

template <bool F16>
int dispatch(const GemvArgs &a, int epilogue, cudaStream_t stream) {
    if (epilogue == HMB_EPI_SWIGLU) return by_rows<2, F16, HMB_EPI_SWIGLU>(a, stream);
    return by_rows<1, F16, HMB_EPI_STORE>(a, stream);
}

// Warps per CTA for m rows of x (the kernel variant by_rows() picks).
int warps_per_cta(int64_t m) { return m == 1 ? 16 : (m <= 4 ? 12 : 8); }

// Warps that share the tile stream: those of one CTA per SM (split_k > 0 caps the CTAs), never more
// than there are tiles.
int64_t grid_warps(int64_t items, int split_k, int64_t m) {
    int64_t ctas = sm_count();
    if (split_k > 0) ctas = std::min<int64_t>(ctas, split_k);
    return std::max<int64_t>(1, std::min<int64_t>(ctas * warps_per_cta(m), items));
}

constexpr size_t kCounterBytes = 64 * 1024;  // room for 16384 column sets

size_t partial_bytes(int64_t m, int64_t colsets, int ncol, int64_t warps) {
    const int mt = m <= 8 ? 1 : 2;
    return static_cast<size_t>(warps + colsets) * ncol * mt * 16 * 32 * sizeof(float);
}

// Validates a GEMV over [k x n] of a [packed_k x packed_n] matrix and fills every field of `a` but x,
// y, m, counters and partial; `partial` receives the bytes of contributor slots it needs. For the
// SwiGLU blocked layout the up columns start up_tiles tile columns after the gate ones (0: n / 2).
int gemv_args(GemvArgs &a, size_t &partial, const uint8_t *packed, int64_t packed_k, int64_t packed_n, int64_t ldx, int x_dtype,
              int64_t ldy, int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue, int layout, int split_k,
              int64_t up_tiles) {
    if (!packed || m <= 0) return HMB_ERR_ARG;
    if (k <= 0 || n <= 0 || k % kTileK || n % kTileN || packed_k % kTileK || packed_n % kTileN || start_col < 0 ||
        start_col % kTileN || k > packed_k || start_col + n > packed_n)
        return HMB_ERR_ARG;
    if (x_dtype != HMB_BF16 && x_dtype != HMB_FP16) return HMB_ERR_ARG;
    if (epilogue != HMB_EPI_STORE && epilogue != HMB_EPI_SWIGLU) return HMB_ERR_ARG;
    if (y_dtype != x_dtype && !(y_dtype == HMB_FP32 && epilogue == HMB_EPI_STORE)) return HMB_ERR_ARG;
    if (epilogue == HMB_EPI_SWIGLU) {
        if (layout != HMB_GATE_UP_BLOCKED && layout != HMB_GATE_UP_INTERLEAVED) return HMB_ERR_ARG;
        if (n % (2 * kTileN)) return HMB_ERR_ARG;
    }
    const int64_t out_cols = epilogue == HMB_EPI_SWIGLU ? n / 2 : n;
    if (ldx < k || ldy < out_cols || ldx % 8 || ldy % 8) return ldx < k || ldy < out_cols ? HMB_ERR_ARG : HMB_ERR_ALIGN;
    if (!aligned(packed, 16)) return HMB_ERR_ALIGN;
    if (packed_k / kTileK > (1 << 30) || packed_n / kTileN > (1 << 30)) return HMB_ERR_UNSUPPORTED;
    a = GemvArgs{};
    a.packed = packed;
    a.tiles_k_total = static_cast<int>(packed_k / kTileK);
    a.tiles_n_total = static_cast<int>(packed_n / kTileN);
    a.col_tile0 = static_cast<int>(start_col / kTileN);
    a.k_tiles = static_cast<int>(k / kTileK);
    const int n_tiles = static_cast<int>(n / kTileN);
    a.ldx = ldx;
    a.ldy = ldy;
    a.y_f32 = y_dtype == HMB_FP32;
    const int ncol = epilogue == HMB_EPI_SWIGLU ? 2 : 1;
    a.colsets = n_tiles / ncol;
    a.col_stride = epilogue == HMB_EPI_SWIGLU
                       ? (layout == HMB_GATE_UP_INTERLEAVED ? 1 : static_cast<int>(up_tiles > 0 ? up_tiles : n_tiles / 2))
                       : 0;
    if (epilogue == HMB_EPI_SWIGLU && layout == HMB_GATE_UP_BLOCKED && a.col_tile0 + a.col_stride + a.colsets > a.tiles_n_total)
        return HMB_ERR_ARG;
    const int64_t items = static_cast<int64_t>(a.colsets) * ncol * a.k_tiles;
    if (items > (1LL << 30)) return HMB_ERR_UNSUPPORTED;
    a.items = static_cast<int>(items);
    a.warps = static_cast<int>(grid_warps(items, split_k, std::min<int64_t>(m, 16)));
    if (a.colsets > static_cast<int>(kCounterBytes / sizeof(int))) return HMB_ERR_UNSUPPORTED;
    partial = partial_bytes(std::min<int64_t>(m, 16), a.colsets, ncol, a.warps);
    a.status = device_status_word();
    if (!a.status) return HMB_ERR_CUDA;
    return HMB_OK;
}

// Workspace of hmb_w4a16_ffn: [gate/up GEMV counters][down GEMV counters][gate/up GEMM split counters]
// [down GEMM split counters][act][scratch]. Counters are never written by another path (each is left
// zero by its own); the scratch holds the GEMV contributor slots on the decode path and the GEMMs'
// split-K sums on the prefill path (gate/up and down run one after the other, so they share it).
size_t round256(size_t b) { return (b + 255) / 256 * 256; }
constexpr size_t kFfnControlBytes = 2 * kCounterBytes + 2 * kSplitCounterBytes;

}  // namespace
}  // namespace hmb

using namespace hmb;

extern "C" {

size_t hmb_w4a16_gemv_workspace(int64_t m, int64_t k, int64_t n, int epilogue, int split_k) {
    if (m <= 0 || k <= 0 || n <= 0 || k % kTileK || n % kTileN) return 0;
    const int ncol = epilogue == HMB_EPI_SWIGLU ? 2 : 1;
    const int64_t colsets = (n / kTileN) / ncol;
    const int64_t items = colsets * ncol * (k / kTileK);
    return kCounterBytes + partial_bytes(std::min<int64_t>(m, 16), colsets, ncol, grid_warps(items, split_k, std::min<int64_t>(m, 16)));
}

int hmb_w4a16_gemv(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype, void *y,
                   int64_t ldy, int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue, int layout,
                   int split_k, void *workspace, size_t workspace_bytes, hmb_stream_t stream) {
    if (!x || !y) return HMB_ERR_ARG;
    GemvArgs a;
    size_t partial = 0;
    int rc = gemv_args(a, partial, packed, packed_k, packed_n, ldx, x_dtype, ldy, y_dtype, m, k, n, start_col, epilogue, layout, split_k, 0);
    if (rc != HMB_OK) return rc;
    if (!aligned(x, 16) || !aligned(y, 16)) return HMB_ERR_ALIGN;
    if (!workspace || workspace_bytes < kCounterBytes + partial || !aligned(workspace, 16)) return HMB_ERR_WORKSPACE;
    a.counters = static_cast<int *>(workspace);
    a.partial = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + kCounterBytes);

    const size_t y_elem = y_dtype == HMB_FP32 ? 4 : 2;
    for (int64_t r0 = 0; r0 < m; r0 += 16) {
        a.m = static_cast<int>(std::min<int64_t>(16, m - r0));
        a.x = static_cast<const uint16_t *>(x) + r0 * ldx;
        a.y = static_cast<uint8_t *>(y) + r0 * ldy * y_elem;
        rc = x_dtype == HMB_FP16 ? dispatch<true>(a, epilogue, stream) : dispatch<false>(a, epilogue, stream);
        if (rc != HMB_OK) return rc;
    }
    return HMB_OK;
}

size_t hmb_w4a16_ffn_workspace(int64_t m, int64_t h, int64_t n) {
    if (m <= 0 || h <= 0 || n <= 0 || h % kTileK || n % kTileK) return 0;
    const int64_t rows = std::min<int64_t>(m, 16);
    const int64_t gu_items = (2 * n / kTileN) * (h / kTileK), dn_items = (h / kTileN) * (n / kTileK);
    const size_t decode = round256(partial_bytes(rows, n / kTileN, 2, grid_warps(gu_items, 0, rows))) +
                          round256(partial_bytes(rows, h / kTileN, 1, grid_warps(dn_items, 0, rows)));
    size_t prefill = 0;
    if (m > 16) prefill = std::max(gemm_split_bytes(m, h, 2 * n), gemm_split_bytes(m, n, h));
    return kFfnControlBytes + round256(static_cast<size_t>(m) * n * 2) + std::max(decode, prefill);
}

int hmb_w4a16_ffn(const uint8_t *gate_up, const uint8_t *down, int64_t h, int64_t n, int64_t stored, int layout, const void *x,
                  int64_t ldx, int x_dtype, void *y, int64_t ldy, int y_dtype, int64_t m, void *workspace, size_t workspace_bytes,
                  hmb_stream_t stream) {
    if (!gate_up || !down || !x || !y || m <= 0 || h <= 0 || n <= 0 || stored <= 0) return HMB_ERR_ARG;
    if (h % kTileK || n % kTileK || stored % kTileK || n > stored) return HMB_ERR_ARG;
    if (layout != HMB_GATE_UP_BLOCKED && layout != HMB_GATE_UP_INTERLEAVED) return HMB_ERR_ARG;
    if (!aligned(x, 16) || !aligned(y, 16) || !workspace || !aligned(workspace, 256)) return workspace ? HMB_ERR_ALIGN : HMB_ERR_WORKSPACE;
    if (workspace_bytes < hmb_w4a16_ffn_workspace(m, h, n)) return HMB_ERR_WORKSPACE;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    unsigned *gu_split_cnt = reinterpret_cast<unsigned *>(ws + 2 * kCounterBytes);
    unsigned *dn_split_cnt = reinterpret_cast<unsigned *>(ws + 2 * kCounterBytes + kSplitCounterBytes);
    uint8_t *act_p = ws + kFfnControlBytes;
    uint8_t *scratch = act_p + round256(static_cast<size_t>(m) * n * 2);
    const size_t scratch_bytes = workspace_bytes - (scratch - ws);

    // Prefill: the tcgen05 GEMMs (K split where the tiles alone would leave the GPU idle), gate/up with
    // the SwiGLU epilogue into act, then down.
    const bool same_up = layout == HMB_GATE_UP_INTERLEAVED || n == stored;
    if (m > 16 && same_up && hmb_w4a16_gemm_supports(m, h, 2 * n, HMB_EPI_SWIGLU) && hmb_w4a16_gemm_supports(m, n, h, HMB_EPI_STORE)) {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        int rc = gemm_run(gate_up, h, 2 * stored, x, ldx, x_dtype, act_p, n, x_dtype, m, h, 2 * n, 0, HMB_EPI_SWIGLU, layout, scratch,
                          scratch_bytes, gu_split_cnt, s);
        if (rc != HMB_OK) return rc;
        return gemm_run(down, stored, h, act_p, n, x_dtype, y, ldy, y_dtype, m, n, h, 0, HMB_EPI_STORE, 0, scratch, scratch_bytes,
                        dn_split_cnt, s);
    }

    // Decode: the gate/up GEMV with the SwiGLU epilogue into act, then the down GEMV, per 16 rows. The
    // down GEMV is a programmatic dependent of the first: it requests its weights while gate/up ends.
    GemvArgs gu, dn;
    size_t gu_partial = 0, dn_partial = 0;
    int rc = gemv_args(gu, gu_partial, gate_up, h, 2 * stored, ldx, x_dtype, n, x_dtype, m, h, 2 * n, 0, HMB_EPI_SWIGLU, layout, 0,
                       stored / kTileN);
    if (rc != HMB_OK) return rc;
    rc = gemv_args(dn, dn_partial, down, stored, h, n, x_dtype, ldy, y_dtype, m, n, h, 0, HMB_EPI_STORE, 0, 0, 0);
    if (rc != HMB_OK) return rc;
    gu.counters = reinterpret_cast<int *>(ws);
    dn.counters = reinterpret_cast<int *>(ws + kCounterBytes);
    uint16_t *act = reinterpret_cast<uint16_t *>(act_p);
    gu.partial = reinterpret_cast<float *>(scratch);
    dn.partial = reinterpret_cast<float *>(scratch + round256(gu_partial));
    const size_t y_elem = y_dtype == HMB_FP32 ? 4 : 2;
    for (int64_t r0 = 0; r0 < m; r0 += 16) {
        gu.m = dn.m = static_cast<int>(std::min<int64_t>(16, m - r0));
        gu.x = static_cast<const uint16_t *>(x) + r0 * ldx;
        gu.y = act;
        dn.x = act;
        dn.y = static_cast<uint8_t *>(y) + r0 * ldy * y_elem;
        rc = x_dtype == HMB_FP16 ? dispatch<true>(gu, HMB_EPI_SWIGLU, stream) : dispatch<false>(gu, HMB_EPI_SWIGLU, stream);
        if (rc != HMB_OK) return rc;
        rc = x_dtype == HMB_FP16 ? dispatch<true>(dn, HMB_EPI_STORE, stream) : dispatch<false>(dn, HMB_EPI_STORE, stream);
        if (rc != HMB_OK) return rc;
    }
    return HMB_OK;
}

size_t hmb_tp_ffn_layer_workspace(int64_t m, int64_t h, int64_t n) {
    const size_t ffn = hmb_w4a16_ffn_workspace(m, h, n);
    return ffn ? ffn + round256(static_cast<size_t>(m) * h * 4) : 0;
}

int hmb_tp_ffn_layer(hmb_comm *comm, const uint8_t *gate_up, const uint8_t *down, int64_t h, int64_t n, int64_t stored, int layout,
                     const void *x, void *resid, const void *norm_weight, float eps, int64_t m, void *workspace, size_t workspace_bytes,
                     hmb_stream_t stream, uint64_t spin_limit_ns) {
    return hmb_tp_ffn_layer_chained(comm, gate_up, down, h, n, stored, layout, x, resid, norm_weight, eps, m, workspace, workspace_bytes,
                                    stream, spin_limit_ns, 0);
}

int hmb_tp_ffn_layer_chained(hmb_comm *comm, const uint8_t *gate_up, const uint8_t *down, int64_t h, int64_t n, int64_t stored,
                             int layout, const void *x, void *resid, const void *norm_weight, float eps, int64_t m, void *workspace,
                             size_t workspace_bytes, hmb_stream_t stream, uint64_t spin_limit_ns, int chain) {
    if (!comm || !gate_up || !down || !x || !resid || m <= 0) return HMB_ERR_ARG;
    const size_t ffn_bytes = hmb_w4a16_ffn_workspace(m, h, n);
    if (!ffn_bytes) return HMB_ERR_ARG;
    if (!workspace || workspace_bytes < hmb_tp_ffn_layer_workspace(m, h, n)) return HMB_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return HMB_ERR_ALIGN;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    void *y = ws + ffn_bytes;  // this rank's partial, when it is not scattered (fp32 on two or more ranks)

    // Prefill on two or more ranks: gate/up GEMM with SwiGLU, then the down GEMM storing its partial
    // rows over NVLink into the receive slots of the boundary, which then only sums and normalises.
    ScatterTarget t;
    const bool same_up = layout == HMB_GATE_UP_INTERLEAVED || n == stored;
    const bool fused = m > 16 && same_up && hmb_w4a16_gemm_supports(m, h, 2 * n, HMB_EPI_SWIGLU) &&
                       hmb_w4a16_gemm_supports(m, n, h, HMB_EPI_STORE) && comm_scatter_target(comm, m, h, &t) == HMB_OK && t.world > 1;
    if (chain & ~(HMB_TP_CHAIN_IN | HMB_TP_CHAIN_OUT)) return HMB_ERR_ARG;
    if (fused) {
        if (h % kTileK || n % kTileK || stored % kTileK || n > stored) return HMB_ERR_ARG;
        if (layout != HMB_GATE_UP_BLOCKED && layout != HMB_GATE_UP_INTERLEAVED) return HMB_ERR_ARG;
        if (!aligned(x, 16)) return HMB_ERR_ALIGN;
        // Chaining (two-shot boundaries read by the CTA-pair gate/up GEMM): the same condition in
        // consecutive calls of one stack, so a chained boundary's counters meet a waiting GEMM.
        const bool chain_ok = comm_chains(comm, m, h) && gemm_plan(m, h, 2 * n, false, false).pair;
        const bool chain_in = chain_ok && (chain & HMB_TP_CHAIN_IN), chain_out = chain_ok && (chain & HMB_TP_CHAIN_OUT);
        if (chain_in && x != comm_out_region(comm)) return HMB_ERR_ARG;
        unsigned *gu_split_cnt = reinterpret_cast<unsigned *>(ws + 2 * kCounterBytes);
        unsigned *dn_split_cnt = reinterpret_cast<unsigned *>(ws + 2 * kCounterBytes + kSplitCounterBytes);
        uint8_t *act_p = ws + kFfnControlBytes;
        uint8_t *scratch = act_p + round256(static_cast<size_t>(m) * n * 2);
        const size_t scratch_bytes = ffn_bytes - (scratch - ws);
        // Chained in: the rows of x land while this GEMM runs; it starts at this rank's own rows.
        const int own_block = static_cast<int>(comm_share_row(m, t.world, t.rank) / 256);
        int rc = gemm_run(gate_up, h, 2 * stored, x, h, HMB_BF16, act_p, n, HMB_BF16, m, h, 2 * n, 0, HMB_EPI_SWIGLU, layout, scratch,
                          scratch_bytes, gu_split_cnt, s, nullptr, chain_in ? comm_ready(comm) : nullptr, own_block);
        if (rc != HMB_OK) return rc;
        rc = gemm_run(down, stored, h, act_p, n, HMB_BF16, nullptr, h, HMB_BF16, m, n, h, 0, HMB_EPI_STORE, 0, scratch, scratch_bytes,
                      dn_split_cnt, s, &t);
        if (rc != HMB_OK) return rc;
        return comm_boundary(comm, nullptr, HMB_BF16, resid, norm_weight, m, h, eps, true, s, spin_limit_ns, chain_out);
    }
    // Decode (and a group of one): the FFN into y, then the boundary with its own exchange. Across
    // ranks the partials stay fp32 (unrounded sums): the messages are small, and P rounded partials
    // would add P roundings to every layer's sum.
    const int y_dtype = comm_world(comm) > 1 ? HMB_FP32 : HMB_BF16;
    int rc = hmb_w4a16_ffn(gate_up, down, h, n, stored, layout, x, h, HMB_BF16, y, h, y_dtype, m, workspace, ffn_bytes, stream);
    if (rc != HMB_OK) return rc;
    return comm_boundary(comm, y, y_dtype, resid, norm_weight, m, h, eps, false, s, spin_limit_ns);
}

}  // extern "C"

// ---- the GEMV without caller workspace ------------------------------------------------------------------
//
// Some callers cannot hand this library a device allocation: a host runtime whose memory pool is owned
// elsewhere and offers no scratch API, or a plugin ABI that only passes input and output buffers. For
// them, hmb_w4a16_gemv_noalloc keeps the split-K scratch of the GEMV in a fixed array in device memory
// that the library reserves when it is loaded, so a call allocates nothing.

namespace hmb {
namespace {

constexpr size_t kStaticPartialBytes = 16u << 20;  // fp32 partial sums of column sets that cross warp chunks
constexpr size_t kStaticScratchBytes = kCounterBytes + kStaticPartialBytes;

// Every GPU that loads libhmb.so keeps this array until the process exits. In host code the name is a
// stand-in, not a device address: only the pointer from cudaGetSymbolAddress may reach a kernel.
static __device__ __align__(256) uint8_t g_gemv_scratch[kStaticScratchBytes];

// Device address of g_gemv_scratch for the current device, looked up once per device and context:
// after cudaDeviceReset the device gets a new primary context, the module is loaded again and the
// array has a new address, so a change of context id triggers a new lookup.
int static_scratch(uint8_t **out) {
    static std::mutex mu;
    static uint8_t *addr[64] = {};
    static unsigned long long ctx[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    if (dev >= 64) return HMB_ERR_UNSUPPORTED;
    const unsigned long long id = current_context_id();
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev] || ctx[dev] != id || id == 0) {  // id 0: no context id to key on, look it up again
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gemv_scratch);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return HMB_ERR_CUDA;
        }
        addr[dev] = static_cast<uint8_t *>(p);
        ctx[dev] = id;
    }
    *out = addr[dev];
    return HMB_OK;
}

}  // namespace
}  // namespace hmb

extern "C" {

int hmb_w4a16_gemv_noalloc(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype,
                           void *y, int64_t ldy, int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue,
                           int layout, int split_k, hmb_stream_t stream) {
    // The size check comes first, so an oversized call fails before touching the device.
    const size_t need = hmb_w4a16_gemv_workspace(m, k, n, epilogue, split_k);
    if (need == 0) return HMB_ERR_ARG;
    if (need > hmb::kStaticScratchBytes) return HMB_ERR_WORKSPACE;
    uint8_t *scratch = nullptr;
    int rc = hmb::static_scratch(&scratch);
    if (rc != HMB_OK) return rc;
    // The counters must start at zero; a completed call leaves them so, but a call that failed on the
    // device may not have.
    const cudaError_t e = cudaMemsetAsync(scratch, 0, hmb::kCounterBytes, stream);
    if (e != cudaSuccess) {
        hmb::set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    return hmb_w4a16_gemv(packed, packed_k, packed_n, x, ldx, x_dtype, y, ldy, y_dtype, m, k, n, start_col, epilogue, layout,
                          split_k, scratch, hmb::kStaticScratchBytes, stream);
}

}  // extern "C"
