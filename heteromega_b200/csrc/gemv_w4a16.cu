// W4A16 decode GEMV / skinny GEMM (m <= 16 rows) on the packed tile layout.
//
// What it computes is the reference's GEMV definition (src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp:83-289,
// kernels/gpu/src/gemv_w4a16.cu:27-28): for each 128-row tile and column,
//     s * (sum_r q_r * x_r - z * sum_r x_r)     in fp32,
// summed over the tiles of a column, then rounded once. How it computes it is B200-specific:
//
//   * One warp consumes one whole 4352-byte tile per step: eight 16-byte streaming loads per lane,
//     512 contiguous bytes per warp load, no shared memory and no __syncthreads in the K loop.
//   * The weights go through the tensor cores as exact integers. A nibble q becomes the bf16
//     (fp16) number 128 + q (1024 + q) by OR-ing it into the mantissa of 0x4300 (0x6400), so one
//     PRMT and two LOP3 turn 4 bytes into 4 MMA operand registers. The MMA multiplies them with
//     x and accumulates in fp32; an extra MMA with an all-ones operand yields sum_r x_r in the
//     same fragment positions. Per tile and column:
//         s * (acc - (C + z) * sum_x) = s * (sum q*x - z * sum x)        (C = 128 or 1024).
//   * The MMA is m16n8k16 with the weights on the M side ("swap AB"): 16 output columns x 8 rows
//     of x. The packed layout stores, per K row, 8 consecutive columns in one 32-bit word. A lane
//     with group g = lane/4 and t = lane%4 takes column group g and K rows 4t..4t+3 of each
//     16-row chunk; K inside a chunk is permuted so that these 4 rows form the lane's operand
//     pairs, and x is read with the same permutation, so the dot products are unchanged. Of the
//     8 columns of its group, the lane feeds columns 2b and 2b+1 to MMA block b (b = 0..3).
//   * Split-K over CTAs writes fp32 partial sums to the workspace; the last CTA of a column set
//     (an atomic counter) adds them in split order, so results do not depend on timing.
//   * The SwiGLU epilogue pairs the gate and up tile columns of 64 channels in one CTA and
//     writes bf16(SiLU(g) * u) from the bf16-rounded g and u, so gate/up never reach HBM.
#include <algorithm>

#include "common.cuh"

namespace hmb {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

struct GemvArgs {
    const uint8_t *packed;
    const uint16_t *x;
    void *y;
    float *partial;   // [splits][m][n] fp32, n = computed columns
    int *counters;    // [column sets]
    int64_t ldx, ldy;
    int tiles_k_total, tiles_n_total;  // the whole packed matrix
    int col_tile0;                     // first tile column used
    int k_tiles;                       // tile rows used
    int n_tiles;                       // tile columns used
    int m;
    int splits, tiles_per_split;
    int col_stride;  // tile columns between slot 0 and slot 1 of a column set (pairs only)
    int y_f32;
};

template <bool F16>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    if constexpr (F16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

struct TileRegs {
    uint4 w[8];  // chunk j: K rows 16j + 4t .. +3 of column group g
    uint4 s;     // 8 bf16 scales of column group g
    uint2 z;     // 8 zeros of column group g
};

__device__ __forceinline__ void load_tile(TileRegs &r, const uint8_t *tile, int lane_off, int g) {
#pragma unroll
    for (int j = 0; j < 8; ++j) r.w[j] = ld_stream16(tile + 512 * j + lane_off);
    r.s = ld_stream16(tile + 4096 + 16 * g);
    r.z = ld_stream8(tile + 4224 + 16 * g);
}

// Accumulates one tile into tot. MT token blocks of 8 rows of x.
template <int MT, bool F16>
__device__ __forceinline__ void tile_mma(const TileRegs &r, const uint16_t *__restrict__ x, int64_t ldx, int m, int64_t krow0,
                                         int g, int t, float (&tot)[MT][4][4]) {
    constexpr uint32_t kMagic = F16 ? 0x64006400u : 0x43004300u;
    constexpr uint32_t kOnes = F16 ? 0x3C003C00u : 0x3F803F80u;
    constexpr float kOffset = F16 ? 1024.0f : 128.0f;
    constexpr uint32_t kMask = 0x000F000Fu;
    float acc[MT][4][4];
    float sx[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            sx[mt][i] = 0.0f;
#pragma unroll
            for (int b = 0; b < 4; ++b) acc[mt][b][i] = 0.0f;
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t bx[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int tok = mt * 8 + g;
            if (tok < m) {
                const uint2 v = *reinterpret_cast<const uint2 *>(x + tok * ldx + krow0 + 16 * j + 4 * t);
                bx[mt][0] = v.x;
                bx[mt][1] = v.y;
            } else {
                bx[mt][0] = 0u;
                bx[mt][1] = 0u;
            }
            mma16816<F16>(sx[mt], kOnes, kOnes, kOnes, kOnes, bx[mt][0], bx[mt][1]);
        }
        const uint4 w = r.w[j];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            // Byte b of rows (4t, 4t+1) and of rows (4t+2, 4t+3), side by side in 16-bit halves.
            const uint32_t sel = static_cast<uint32_t>(b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12));
            const uint32_t p = prmt(w.x, w.y, sel);
            const uint32_t q = prmt(w.z, w.w, sel);
            const uint32_t a0 = (p & kMask) | kMagic;         // column 2b, rows 4t, 4t+1
            const uint32_t a1 = ((p >> 4) & kMask) | kMagic;  // column 2b+1
            const uint32_t a2 = (q & kMask) | kMagic;         // column 2b, rows 4t+2, 4t+3
            const uint32_t a3 = ((q >> 4) & kMask) | kMagic;  // column 2b+1
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) mma16816<F16>(acc[mt][b], a0, a1, a2, a3, bx[mt][0], bx[mt][1]);
        }
    }
    const uint32_t sw[4] = {r.s.x, r.s.y, r.s.z, r.s.w};
    const uint32_t zw[2] = {r.z.x, r.z.y};
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const float s_lo = bf16_to_f32(sw[b] & 0xFFFFu);
        const float s_hi = bf16hi_to_f32(sw[b]);
        const uint32_t zz = zw[b >> 1] >> (16 * (b & 1));
        const float zc_lo = kOffset + static_cast<float>(zz & 0xFFu);
        const float zc_hi = kOffset + static_cast<float>((zz >> 8) & 0xFFu);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            tot[mt][b][0] = fmaf(s_lo, fmaf(-zc_lo, sx[mt][0], acc[mt][b][0]), tot[mt][b][0]);
            tot[mt][b][1] = fmaf(s_lo, fmaf(-zc_lo, sx[mt][1], acc[mt][b][1]), tot[mt][b][1]);
            tot[mt][b][2] = fmaf(s_hi, fmaf(-zc_hi, sx[mt][2], acc[mt][b][2]), tot[mt][b][2]);
            tot[mt][b][3] = fmaf(s_hi, fmaf(-zc_hi, sx[mt][3], acc[mt][b][3]), tot[mt][b][3]);
        }
    }
}

template <bool F16>
__device__ __forceinline__ float silu_mul_rounded(float g, float u) {
    const float gr = round16<F16>(g), ur = round16<F16>(u);
    return gr / (1.0f + __expf(-gr)) * ur;
}

// Grid: (column sets, splits). A column set is 1 tile column, or 2 (gate and up of 64 channels).
template <int NCOL, int MT, bool F16, int EPI>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvArgs a) {
    __shared__ float red[kWarps][NCOL][MT * 8][kTileN];
    __shared__ int s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int lane_off = 256 * (t >> 1) + 32 * g + 16 * (t & 1);
    const int cs = blockIdx.x;
    const int base = (NCOL == 2 && a.col_stride == 1) ? 2 * cs : cs;
    const int kb = blockIdx.y * a.tiles_per_split;
    const int nk = min(kb + a.tiles_per_split, a.k_tiles) - kb;
    const int items = NCOL * nk;

    for (int i = threadIdx.x; i < kWarps * NCOL * MT * 8 * kTileN; i += kThreads) (&red[0][0][0][0])[i] = 0.0f;
    __syncthreads();

    int64_t col_base[NCOL];
#pragma unroll
    for (int s = 0; s < NCOL; ++s) {
        col_base[s] = tile_index(a.col_tile0 + base + s * a.col_stride, 0, a.tiles_k_total, a.tiles_n_total);
    }

    float tot[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) tot[mt][b][i] = 0.0f;

    auto flush = [&](int slot) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int b = 0; b < 4; ++b)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    red[warp][slot][mt * 8 + 2 * t + (i & 1)][8 * g + 2 * b + (i >> 1)] = tot[mt][b][i];
                    tot[mt][b][i] = 0.0f;
                }
    };

    int it = warp;
    int cur_slot = nk > 0 ? it / nk : 0;
    TileRegs cur, nxt;
    auto tile_ptr = [&](int item) {
        const int slot = item / nk;
        const int kt = kb + item - slot * nk;
        int64_t cb = col_base[0];
#pragma unroll
        for (int s = 1; s < NCOL; ++s)
            if (slot == s) cb = col_base[s];
        return a.packed + (cb + kt) * kTileBytes;
    };
    if (it < items) load_tile(cur, tile_ptr(it), lane_off, g);
    while (it < items) {
        const int nit = it + kWarps;
        if (nit < items) load_tile(nxt, tile_ptr(nit), lane_off, g);
        const int slot = it / nk;
        if (slot != cur_slot) {
            flush(cur_slot);
            cur_slot = slot;
        }
        const int kt = kb + it - slot * nk;
        tile_mma<MT, F16>(cur, a.x, a.ldx, a.m, static_cast<int64_t>(kt) * kTileK, g, t, tot);
        cur = nxt;
        it = nit;
    }
    if (warp < items) flush(cur_slot);
    __syncthreads();

    const int n = a.n_tiles * kTileN;
    const int total = NCOL * a.m * kTileN;
    // Column index (within the computed n) of slot s, lane column c.
    auto out_col = [&](int s, int c) { return (base + s * a.col_stride) * kTileN + c; };

    if (a.splits > 1) {
        for (int e = threadIdx.x; e < total; e += kThreads) {
            const int s = e / (a.m * kTileN), tok = (e / kTileN) % a.m, c = e % kTileN;
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v += red[w][s][tok][c];
            a.partial[(static_cast<int64_t>(blockIdx.y) * a.m + tok) * n + out_col(s, c)] = v;
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const int prev = atomicAdd(&a.counters[cs], 1);
            s_last = prev == a.splits - 1;
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
    }

    // Sum of slot s, row tok, lane column c: from shared memory, or from all splits in order.
    auto value = [&](int s, int tok, int c) {
        if (a.splits == 1) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v += red[w][s][tok][c];
            return v;
        }
        float v = 0.0f;
        for (int sp = 0; sp < a.splits; ++sp) v += __ldcg(a.partial + (static_cast<int64_t>(sp) * a.m + tok) * n + out_col(s, c));
        return v;
    };

    if constexpr (EPI == HMB_EPI_SWIGLU) {
        uint16_t *y = static_cast<uint16_t *>(a.y);
        for (int e = threadIdx.x; e < a.m * kTileN; e += kThreads) {
            const int tok = e / kTileN, c = e % kTileN;
            const float act = silu_mul_rounded<F16>(value(0, tok, c), value(1, tok, c));
            y[tok * a.ldy + cs * kTileN + c] = static_cast<uint16_t>(to16<F16>(act));
        }
    } else {
        for (int e = threadIdx.x; e < total; e += kThreads) {
            const int s = e / (a.m * kTileN), tok = (e / kTileN) % a.m, c = e % kTileN;
            const float v = value(s, tok, c);
            if (a.y_f32) {
                static_cast<float *>(a.y)[tok * a.ldy + out_col(s, c)] = v;
            } else {
                static_cast<uint16_t *>(a.y)[tok * a.ldy + out_col(s, c)] = static_cast<uint16_t>(to16<F16>(v));
            }
        }
    }
    if (a.splits > 1 && threadIdx.x == 0) a.counters[cs] = 0;
}

constexpr size_t kCounterBytes = 64 * 1024;  // room for 16384 column sets

int pick_splits(int colsets, int k_tiles, int ncol) {
    const int target = 4 * sm_count();
    int splits = (target + colsets - 1) / colsets;
    // Keep at least one tile per warp in every split.
    splits = std::min(splits, std::max(1, ncol * k_tiles / kWarps));
    return std::max(1, std::min(splits, k_tiles));
}

template <int NCOL, int MT, bool F16, int EPI>
int launch(const GemvArgs &a, int colsets, cudaStream_t stream) {
    gemv_kernel<NCOL, MT, F16, EPI><<<dim3(colsets, a.splits), kThreads, 0, stream>>>(a);
    return launch_status();
}

template <bool F16>
int dispatch(const GemvArgs &a, int colsets, int epilogue, cudaStream_t stream) {
    if (epilogue == HMB_EPI_SWIGLU) {
        return a.m <= 8 ? launch<2, 1, F16, HMB_EPI_SWIGLU>(a, colsets, stream)
                        : launch<2, 2, F16, HMB_EPI_SWIGLU>(a, colsets, stream);
    }
    return a.m <= 8 ? launch<1, 1, F16, HMB_EPI_STORE>(a, colsets, stream) : launch<1, 2, F16, HMB_EPI_STORE>(a, colsets, stream);
}

}  // namespace
}  // namespace hmb

using namespace hmb;

extern "C" {

size_t hmb_w4a16_gemv_workspace(int64_t m, int64_t k, int64_t n, int epilogue, int split_k) {
    if (m <= 0 || k <= 0 || n <= 0 || k % kTileK || n % kTileN) return 0;
    const int ncol = epilogue == HMB_EPI_SWIGLU ? 2 : 1;
    const int k_tiles = static_cast<int>(k / kTileK);
    const int colsets = static_cast<int>(n / kTileN) / ncol;
    const int splits = split_k > 0 ? std::min(split_k, k_tiles) : pick_splits(colsets, k_tiles, ncol);
    const int64_t rows = std::min<int64_t>(m, 16);
    return kCounterBytes + static_cast<size_t>(splits) * rows * n * sizeof(float);
}

int hmb_w4a16_gemv(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype, void *y,
                   int64_t ldy, int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue, int layout,
                   int split_k, void *workspace, size_t workspace_bytes, hmb_stream_t stream) {
    if (!packed || !x || !y || m <= 0) return HMB_ERR_ARG;
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
    if (ldx < k || ldy < out_cols) return HMB_ERR_ARG;
    if (!aligned(packed, 16) || !aligned(x, 16) || !aligned(y, 16) || ldx % 8 || ldy % 8) return HMB_ERR_ALIGN;
    if (packed_k / kTileK > (1 << 30) || packed_n / kTileN > (1 << 30)) return HMB_ERR_UNSUPPORTED;

    GemvArgs a{};
    a.packed = packed;
    a.tiles_k_total = static_cast<int>(packed_k / kTileK);
    a.tiles_n_total = static_cast<int>(packed_n / kTileN);
    a.col_tile0 = static_cast<int>(start_col / kTileN);
    a.k_tiles = static_cast<int>(k / kTileK);
    a.n_tiles = static_cast<int>(n / kTileN);
    a.ldx = ldx;
    a.ldy = ldy;
    a.y_f32 = y_dtype == HMB_FP32;
    const int ncol = epilogue == HMB_EPI_SWIGLU ? 2 : 1;
    const int colsets = a.n_tiles / ncol;
    a.col_stride = epilogue == HMB_EPI_SWIGLU ? (layout == HMB_GATE_UP_INTERLEAVED ? 1 : a.n_tiles / 2) : 0;
    a.splits = split_k > 0 ? std::min<int>(split_k, a.k_tiles) : pick_splits(colsets, a.k_tiles, ncol);
    a.tiles_per_split = (a.k_tiles + a.splits - 1) / a.splits;
    a.splits = (a.k_tiles + a.tiles_per_split - 1) / a.tiles_per_split;
    if (colsets > static_cast<int>(kCounterBytes / sizeof(int))) return HMB_ERR_UNSUPPORTED;
    if (a.splits > 1) {
        const size_t need = kCounterBytes + static_cast<size_t>(a.splits) * std::min<int64_t>(m, 16) * n * sizeof(float);
        if (!workspace || workspace_bytes < need || !aligned(workspace, 16)) return HMB_ERR_WORKSPACE;
        a.counters = static_cast<int *>(workspace);
        a.partial = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + kCounterBytes);
    }
    const size_t y_elem = y_dtype == HMB_FP32 ? 4 : 2;
    for (int64_t r0 = 0; r0 < m; r0 += 16) {
        a.m = static_cast<int>(std::min<int64_t>(16, m - r0));
        a.x = static_cast<const uint16_t *>(x) + r0 * ldx;
        a.y = static_cast<uint8_t *>(y) + r0 * ldy * y_elem;
        const int rc = x_dtype == HMB_FP16 ? dispatch<true>(a, colsets, epilogue, stream)
                                           : dispatch<false>(a, colsets, epilogue, stream);
        if (rc != HMB_OK) return rc;
    }
    return HMB_OK;
}

}  // extern "C"
