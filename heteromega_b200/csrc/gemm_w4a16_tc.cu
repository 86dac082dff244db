// W4A16 prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a: the C-ABI entry
// point and the one-CTA kernel used for M <= 128 (M > 128 runs on CTA pairs, gemm_w4a16_pair.cu).
//
//   y[m, n] = x[m, k] @ W[:k, cols]          (HMB_EPI_STORE)
//   y[m, c] = SiLU(g) * u over gate/up pairs (HMB_EPI_SWIGLU)
//
// W is the reference's packed int4 layout (128 x 64 tiles of 4352 bytes, kernels/gpu/src/pack_w4a16.cpp:30-61).
// The result is the reference GEMM's (src/hipkernels/w4a16_gemm_packed.cu:380-613): weights
// dequantized to bf16((q - z) * s) per 128-row group, fp32 accumulation, one rounding of the output.
//
// One CTA computes a 128 x 256 output tile (4 tile columns of W) over K in steps of 64:
//   warp 0      TMA: the 128 x 64 bf16 tile of x (SWIZZLE_128B) and cp.async.bulk copies of the
//               four 64-row halves of packed tiles with their scales and zeros, on one mbarrier;
//   warp 1      allocates 256 TMEM columns; one thread issues tcgen05.mma M=128 N=256 K=16 into
//               them and tcgen05.commit releases each stage;
//   warps 2-9   dequantize: a 32-bit word of a packed tile is one K row and 8 columns; OR-ing its
//               nibbles into the mantissa of bf16 128.0 gives 128 + q exactly, sub.bf16x2 takes
//               128 + z off (exact) and mul.bf16x2 applies the scale (one rounding). The 8 values go
//               to the B operand as one 16-byte store in the MN-major SWIZZLE_128B layout, in the
//               column order (0,4,1,5,2,6,3,7) that the nibble masks give; the epilogue undoes it.
//               After the K loop the same warps read the accumulator (tcgen05.ld) and write y.
// Every mbarrier wait is bounded; a wait that gives up records HMB_ERR_TIMEOUT in the status word
// and the CTA winds down (waiting, again bounded, for its own copies in flight) instead of hanging.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "gemm_internal.h"
#include "tcgen05.cuh"

namespace hmb {
namespace {

using namespace tc;

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kLoadStages = 5;         // x tile + packed halves, ahead of the MMA
constexpr int kBStages = 2;            // dequantized B tiles
constexpr int kABytes = BM * BK * 2;   // 16384
constexpr int kBBytes = BN * BK * 2;   // 32768
constexpr int kPHalf = 2048 + 256;     // half a packed tile + its scales and zeros
constexpr int kPBytes = 4 * kPHalf;    // 9216
constexpr int kDequantWarps = 8;
constexpr int kThreads = (2 + kDequantWarps) * 32;
constexpr int kAOff = 0;
constexpr int kPOff = kAOff + kLoadStages * kABytes;
constexpr int kBOff = kPOff + kLoadStages * kPBytes;  // 1024-aligned: 9216 = 9 x 1024
constexpr int kBarOff = kBOff + kBStages * kBBytes;
constexpr int kTmemCols = 256;
constexpr int kSmemBytes = 1024 + kBarOff + 256;
static_assert(kBOff % 1024 == 0, "stage alignment");

// Set to 1 by a kernel (GEMM or GEMV) that gave up a bounded wait; read and cleared by hmb_device_status().
__device__ int g_gemm_status = 0;

struct GemmArgs {
    const uint8_t *packed;
    void *y;
    int64_t ldy;
    int tiles_k_total, tiles_n_total;
    int col_tile0;
    int k_tiles;     // K / 128
    int n_tiles;     // tile columns computed (multiple of 4)
    int m;
    int col_stride;  // SwiGLU blocked layout: tile columns from gate to up; 1 = interleaved
    int y_f32;       // HMB_EPI_STORE: write the fp32 sums instead of rounding them
};

template <bool F16, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + kBarOff;
    // barriers: full_load, empty_load (per load stage), full_b, empty_b (per B stage), acc_full;
    // then the TMEM address and the abort flag
    auto full_load = [&](int s) { return bars + 8 * s; };
    auto empty_load = [&](int s) { return bars + 8 * (kLoadStages + s); };
    auto full_b = [&](int s) { return bars + 8 * (2 * kLoadStages + s); };
    auto empty_b = [&](int s) { return bars + 8 * (2 * kLoadStages + kBStages + s); };
    const uint32_t acc_full = bars + 8 * (2 * kLoadStages + 2 * kBStages);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kBarOff + 8 * (2 * kLoadStages + 2 * kBStages + 1));
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *status = &g_gemm_status;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM;
    const int nb = blockIdx.y;
    const int num_k = 2 * a.k_tiles;

    // Tile column d (0..3) of this CTA, relative to the packed matrix. SwiGLU keeps them as
    // [gate, up, gate, up] of two 64-channel blocks.
    auto tile_col = [&](int d) {
        if (EPI == HMB_EPI_SWIGLU && a.col_stride != 1) return a.col_tile0 + 2 * nb + (d >> 1) + (d & 1) * a.col_stride;
        return a.col_tile0 + 4 * nb + d;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kLoadStages; ++s) {
            mbar_init(full_load(s), 1);
            mbar_init(empty_load(s), 1 + kDequantWarps);  // the MMA commit (x read) and every dequant warp (packed read)
        }
        for (int s = 0; s < kBStages; ++s) {
            mbar_init(full_b(s), kDequantWarps);
            mbar_init(empty_b(s), 1);
        }
        mbar_init(acc_full, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
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
            // Producer. x (and the y the epilogue writes) wait for the previous kernel to complete.
            prefetch_tensormap(&tmap_x);
            pdl_wait();
            const uint8_t *col_base[4];
            for (int d = 0; d < 4; ++d) col_base[d] = a.packed + tile_index(tile_col(d), 0, a.tiles_k_total, a.tiles_n_total) * kTileBytes;
            int issued = 0;
            for (int i = 0; i < num_k; ++i) {
                const int s = i % kLoadStages, u = i / kLoadStages;
                if (u > 0 && !mbar_wait(empty_load(s), (u - 1) & 1, abort, status)) break;
                mbar_expect_tx(full_load(s), kABytes + kPBytes);
                tma_load_2d(sbase + kAOff + s * kABytes, &tmap_x, i * BK, m0, full_load(s));
                const int kt = i >> 1, h = i & 1;
                for (int d = 0; d < 4; ++d) {
                    const uint8_t *tile = col_base[d] + static_cast<int64_t>(kt) * kTileBytes;
                    const uint32_t pd = sbase + kPOff + s * kPBytes + d * kPHalf;
                    bulk_load(pd, tile + h * 2048, 2048, full_load(s));
                    bulk_load(pd + 2048, tile + 4096, 256, full_load(s));
                }
                issued = i + 1;
            }
            // Do not leave while copies of this CTA are in flight (bounded).
            for (int i = std::max(0, issued - kLoadStages); i < issued; ++i) {
                mbar_wait(full_load(i % kLoadStages), (i / kLoadStages) & 1, abort, status);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: fp32 accumulate, A K-major, B MN-major, M = 128, N = 256.
            constexpr uint32_t idesc = idesc_f16(F16, BM, BN);
            for (int i = 0; i < num_k; ++i) {
                const int sb = i % kBStages, ub = i / kBStages;
                if (!mbar_wait(full_b(sb), ub & 1, abort, status)) break;
                fence_after_sync();
                const uint32_t sa = sbase + kAOff + (i % kLoadStages) * kABytes;
                const uint32_t sbb = sbase + kBOff + sb * kBBytes;
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    // x: K-major, 128-byte rows, 8-row groups 1 KB apart. B: MN-major, four 64-column
                    // atoms 1 KB apart, 8-row K groups 4 KB apart.
                    umma_f16(tmem, smem_desc(sa + kk * 32, 16, 1024), smem_desc(sbb + kk * 2 * 4096, 1024, 4096), idesc, (i | kk) != 0);
                }
                umma_commit(empty_b(sb));
                umma_commit(empty_load(i % kLoadStages));
            }
            umma_commit(acc_full);
        }
    } else {
        // Dequantization: warp dw handles packed tile column d = dw / 2, chunks {2 hc, 2 hc + 1} x 32.
        const int dw = warp - 2, d = dw >> 1, hc = dw & 1;
        const int cc = (lane >> 1) & 7;  // column group of every chunk this lane takes
        // Byte offsets of the lane's 8 output chunks in a B stage (K row r = 8 ga + 4 (lane & 1) + wi).
        uint32_t st_off[2][4];
#pragma unroll
        for (int r2 = 0; r2 < 2; ++r2) {
            const int ga = (lane >> 4) + 2 * (2 * hc + r2);
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                const int rr = 4 * (lane & 1) + wi;
                st_off[r2][wi] = ga * 4096 + d * 1024 + rr * 128 + ((cc ^ rr) << 4);
            }
        }
        const uint32_t ld_off = d * kPHalf + 16 * lane + 512 * (2 * hc);
        bool ok = true;
        uint32_t sp[4], zp[4];
        for (int i = 0; i < num_k; ++i) {
            const int sl = i % kLoadStages, ul = i / kLoadStages;
            const int sb = i % kBStages, ub = i / kBStages;
            if (!mbar_wait(full_load(sl), ul & 1, abort, status) || (ub > 0 && !mbar_wait(empty_b(sb), (ub - 1) & 1, abort, status))) {
                ok = false;
                break;
            }
            const uint8_t *pk = smem + kPOff + sl * kPBytes + d * kPHalf;
            const uint8_t *pw = smem + kPOff + sl * kPBytes + ld_off;
            if ((i & 1) == 0) group_consts<F16>(pk + 2048, pk + 2048 + 128, cc, sp, zp);  // one 128-row group per two steps
            const uint4 wv2[2] = {*reinterpret_cast<const uint4 *>(pw), *reinterpret_cast<const uint4 *>(pw + 512)};
            uint8_t *bt = smem + kBOff + sb * kBBytes;
#pragma unroll
            for (int r2 = 0; r2 < 2; ++r2) {
                const uint32_t ws[4] = {wv2[r2].x, wv2[r2].y, wv2[r2].z, wv2[r2].w};
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) *reinterpret_cast<uint4 *>(bt + st_off[r2][wi]) = dequant_word<F16>(ws[wi], sp, zp);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(full_b(sb));
                mbar_arrive(empty_load(sl));
            }
        }

        // Epilogue: warp q = warp % 4 reads TMEM lanes 32q .. 32q + 31; warps 2-5 take columns 0-127
        // and warps 6-9 columns 128-255.
        const int q = warp & 3, half = dw >> 2;
        const int row = 32 * q + lane, tok = m0 + row;
        pdl_wait();
        if (ok && mbar_wait(acc_full, 0, abort, status)) {
            fence_after_sync();
            const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * q) << 16) + 128 * half;
            if constexpr (EPI == HMB_EPI_SWIGLU) {
                // Block pair `half`: gate = accumulator columns 128 half .. + 63, up = the next 64.
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t gv[32], uv[32];
                    tmem_ld32_nowait(taddr + 32 * hh, gv);
                    tmem_ld32_nowait(taddr + 64 + 32 * hh, uv);
                    tmem_wait_ld();
                    if (tok < a.m) {
                        uint16_t *y = static_cast<uint16_t *>(a.y) + static_cast<int64_t>(tok) * a.ldy + (2 * nb + half) * kTileN + 32 * hh;
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
            } else {
                for (int cb = 0; cb < 4; ++cb) {
                    uint32_t v[32];
                    tmem_ld32(taddr + 32 * cb, v);
                    if (tok < a.m && a.y_f32) {
                        float *y = static_cast<float *>(a.y) + static_cast<int64_t>(tok) * a.ldy + nb * BN + 128 * half + 32 * cb;
#pragma unroll
                        for (int g8 = 0; g8 < 4; ++g8) {
                            float o[8];
#pragma unroll
                            for (int p = 0; p < 8; ++p) o[p] = __uint_as_float(v[8 * g8 + perm_pos(p)]);
                            *reinterpret_cast<float4 *>(y + 8 * g8) = make_float4(o[0], o[1], o[2], o[3]);
                            *reinterpret_cast<float4 *>(y + 8 * g8 + 4) = make_float4(o[4], o[5], o[6], o[7]);
                        }
                    } else if (tok < a.m) {
                        uint16_t *y = static_cast<uint16_t *>(a.y) + static_cast<int64_t>(tok) * a.ldy + nb * BN + 128 * half + 32 * cb;
#pragma unroll
                        for (int g8 = 0; g8 < 4; ++g8) {
                            uint32_t o[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                o[e] = to16<F16>(__uint_as_float(v[8 * g8 + perm_pos(2 * e)])) |
                                       (to16<F16>(__uint_as_float(v[8 * g8 + perm_pos(2 * e + 1)])) << 16);
                            *reinterpret_cast<uint4 *>(y + 8 * g8) = make_uint4(o[0], o[1], o[2], o[3]);
                        }
                    }
                }
            }
        }
    }

    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---- host ---------------------------------------------------------------------------------------------

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *, const cuuint64_t *,
                                 const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

template <bool F16, int EPI>
int launch(const CUtensorMap &map, const GemmArgs &a, cudaStream_t stream) {
    auto kernel = gemm_kernel<F16, EPI>;
    static std::mutex mu;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 64 && !configured[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
            if (e != cudaSuccess) {
                set_cuda_error(e);
                return HMB_ERR_CUDA;
            }
            configured[dev] = true;
        }
    }
    const cudaError_t e = launch_pdl(kernel, dim3((a.m + BM - 1) / BM, a.n_tiles / 4), dim3(kThreads), kSmemBytes, stream, map, a);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    return launch_status();
}

}  // namespace

unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext *);
    using GetId = CUresult (*)(CUcontext, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

int *device_status_word() {
    static std::mutex mu;
    static int *addr[64] = {};
    static unsigned long long ctx[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return nullptr;
    const unsigned long long id = current_context_id();
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev] || ctx[dev] != id || id == 0) {  // id 0: no context id to key on, look it up again
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_gemm_status) != cudaSuccess) return nullptr;
        addr[dev] = static_cast<int *>(p);
        ctx[dev] = id;
    }
    return addr[dev];
}

size_t gemm_split_bytes(int64_t m, int64_t k, int64_t n) { return std::max(pair_split_bytes(m, k, n), skinny_split_bytes(m, k, n)); }

GemmPlan gemm_plan(int64_t m, int64_t k, int64_t n, bool split_ws, bool scatter) {
    GemmPlan p{};
    // 17 to 128 rows: the swap-AB kernel (weights as the MMA's A operand in TMEM); stream-K shares
    // with a workspace (and at most one counter per block in the 4 KB counter area).
    if (skinny_supported(m, k, n)) {
        p.skinny = true;
        p.streamk = split_ws && n / 128 <= static_cast<int64_t>(kSplitCounterBytes / sizeof(unsigned));
        p.k_splits = 1;
        p.k_per_split = static_cast<int>(k / BK);
        return p;
    }
    // CTA pairs for m > 128, and for smaller m when K splits (which need the caller's workspace) can
    // fill a GPU that one-CTA tiles would leave mostly idle.
    const int splits = split_ws ? pair_k_splits(m, k, n) : 1;
    const bool split_ok = splits > 1;
    const bool small_grid = (m + BM - 1) / BM * (n / BN) * 2 < sm_count();
    // or when the pair tiles fit in one round: two SMs per tile, each dequantizing half of it
    const bool one_round = (m + 255) / 256 * (n / 256) <= pair_clusters();
    p.pair = m > BM || (split_ok && small_grid) || (small_grid && one_round) || scatter;
    p.k_splits = 1;
    p.k_per_split = static_cast<int>(k / BK);
    if (!p.pair) return p;
    pair_band_order(m, k, n, &p.band_rows, &p.band);
    p.k_splits = split_ok ? splits : 1;
    const int steps = static_cast<int>(k / BK);
    p.k_per_split = ((steps + p.k_splits - 1) / p.k_splits + 1) / 2 * 2;
    p.k_splits = (steps + p.k_per_split - 1) / p.k_per_split;  // no empty split
    return p;
}

int gemm_run(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype, void *y, int64_t ldy,
             int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue, int layout, void *split_ws, size_t split_ws_bytes,
             unsigned *split_cnt, cudaStream_t stream, const ScatterTarget *sc, const unsigned *x_ready, int x_rot) {
    if (!packed || !x || (!y && !sc) || m <= 0) return HMB_ERR_ARG;
    if (sc && (epilogue != HMB_EPI_STORE || y_dtype == HMB_FP32 || sc->h != n || sc->m != m)) return HMB_ERR_ARG;
    if (sc) {
        y = const_cast<void *>(x);  // never written (the rows go to the scatter target); passes the checks below
        ldy = n;
    }
    if (k <= 0 || n <= 0 || k % kTileK || n % kTileN || packed_k % kTileK || packed_n % kTileN || start_col < 0 ||
        start_col % kTileN || k > packed_k || start_col + n > packed_n)
        return HMB_ERR_ARG;
    if (x_dtype != HMB_BF16 && x_dtype != HMB_FP16) return HMB_ERR_ARG;
    if (epilogue != HMB_EPI_STORE && epilogue != HMB_EPI_SWIGLU) return HMB_ERR_ARG;
    if (y_dtype != x_dtype && !(y_dtype == HMB_FP32 && epilogue == HMB_EPI_STORE)) return HMB_ERR_ARG;
    if (epilogue == HMB_EPI_SWIGLU && layout != HMB_GATE_UP_BLOCKED && layout != HMB_GATE_UP_INTERLEAVED) return HMB_ERR_ARG;
    if (!hmb_w4a16_gemm_supports(m, k, n, epilogue)) return HMB_ERR_UNSUPPORTED;
    // Blocked SwiGLU: the CTA-pair tiles take two gate tile columns at a time; the swap-AB kernel one.
    if (epilogue == HMB_EPI_SWIGLU && layout == HMB_GATE_UP_BLOCKED && (n / 2) % (2 * kTileN) && !skinny_supported(m, k, n))
        return HMB_ERR_UNSUPPORTED;
    const int64_t out_cols = epilogue == HMB_EPI_SWIGLU ? n / 2 : n;
    if (ldx < k || ldy < out_cols) return HMB_ERR_ARG;
    if (!aligned(packed, 16) || !aligned(x, 16) || !aligned(y, 16) || ldx % 8 || ldy % 8) return HMB_ERR_ALIGN;

    EncodeTiled encode = encode_fn();
    int *status = device_status_word();
    if (!encode || !status) return HMB_ERR_CUDA;
    // Both kernels load x in 64 x 128 boxes: the one-CTA kernel its 128-row tile, each CTA of a pair
    // its half of a 256-row tile.
    CUtensorMap map;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(m)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldx) * 2};
    const cuuint32_t box[2] = {BK, 128};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = encode(&map, x_dtype == HMB_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                               const_cast<void *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return HMB_ERR_ARG;

    const int col_stride = (epilogue == HMB_EPI_SWIGLU && layout == HMB_GATE_UP_BLOCKED) ? static_cast<int>(n / kTileN / 2) : 1;
    const bool f16 = x_dtype == HMB_FP16, swiglu = epilogue == HMB_EPI_SWIGLU;
    const GemmPlan plan = gemm_plan(m, k, n, split_ws && split_cnt && split_ws_bytes >= gemm_split_bytes(m, k, n), sc != nullptr);
    if (plan.skinny) {
        SkinnyArgs sa{};
        sa.packed = packed;
        sa.y = y;
        sa.ldy = ldy;
        sa.tiles_k_total = static_cast<int>(packed_k / kTileK);
        sa.tiles_n_total = static_cast<int>(packed_n / kTileN);
        sa.col_tile0 = static_cast<int>(start_col / kTileN);
        sa.col_stride = col_stride;
        sa.tiles = static_cast<int>(k / kTileK);
        sa.blocks = static_cast<int>(n / 128);
        sa.m = static_cast<int>(m);
        sa.nt = static_cast<int>((m + 15) / 16 * 16);
        sa.y_f32 = y_dtype == HMB_FP32;
        sa.streamk = plan.streamk ? 1 : 0;
        sa.partial = static_cast<float *>(split_ws);
        sa.counters = split_cnt;
        sa.status = status;
        if (sc) {
            sa.scatter = 1;
            sa.sc = *sc;
        }
        // x in 64 x nt boxes: rows past m read as zeros.
        CUtensorMap smap;
        const cuuint32_t sbox[2] = {BK, static_cast<cuuint32_t>(sa.nt)};
        const CUresult scr = encode(&smap, x_dtype == HMB_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                    const_cast<void *>(x), dims, strides, sbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (scr != CUDA_SUCCESS) return HMB_ERR_ARG;
        return launch_gemm_skinny(smap, sa, f16, epilogue, stream);
    }
    if (plan.pair) {
        PairArgs p{};
        p.packed = packed;
        p.y = y;
        p.ldy = ldy;
        p.tiles_k_total = static_cast<int>(packed_k / kTileK);
        p.tiles_n_total = static_cast<int>(packed_n / kTileN);
        p.col_tile0 = static_cast<int>(start_col / kTileN);
        p.k_tiles = static_cast<int>(k / kTileK);
        p.m = static_cast<int>(m);
        p.m_blocks = static_cast<int>((m + 255) / 256);
        p.n_blocks = static_cast<int>(n / 256);
        p.num_tiles = p.m_blocks * p.n_blocks;
        p.band_rows = plan.band_rows;
        p.band = plan.band;
        p.col_stride = col_stride;
        p.y_f32 = y_dtype == HMB_FP32;
        p.status = status;
        p.k_splits = plan.k_splits;
        p.k_per_split = plan.k_per_split;
        p.split_ws = static_cast<float *>(split_ws);
        p.split_cnt = split_cnt;
        if (sc) {
            p.scatter = 1;
            p.sc = *sc;
            // Scattering to row owners, every rank starts its row blocks at its own offset: at any
            // moment rank r stores to a different owner than the other ranks.
            if (!sc->all) p.mb_rot = static_cast<int>(static_cast<int64_t>(sc->rank) * p.m_blocks / sc->world);
        }
        p.x_ready = x_ready;
        if (x_ready) p.mb_rot = ((x_rot % p.m_blocks) + p.m_blocks) % p.m_blocks;
        return launch_gemm_pair(map, p, f16, epilogue, stream);
    }
    GemmArgs a{};
    a.packed = packed;
    a.y = y;
    a.ldy = ldy;
    a.tiles_k_total = static_cast<int>(packed_k / kTileK);
    a.tiles_n_total = static_cast<int>(packed_n / kTileN);
    a.col_tile0 = static_cast<int>(start_col / kTileN);
    a.k_tiles = static_cast<int>(k / kTileK);
    a.n_tiles = static_cast<int>(n / kTileN);
    a.m = static_cast<int>(m);
    a.col_stride = col_stride;
    a.y_f32 = y_dtype == HMB_FP32;
    if (f16) return swiglu ? launch<true, HMB_EPI_SWIGLU>(map, a, stream) : launch<true, HMB_EPI_STORE>(map, a, stream);
    return swiglu ? launch<false, HMB_EPI_SWIGLU>(map, a, stream) : launch<false, HMB_EPI_STORE>(map, a, stream);
}

}  // namespace hmb

using namespace hmb;

extern "C" {

int hmb_w4a16_gemm_supports(int64_t m, int64_t k, int64_t n, int epilogue) {
    if (m <= 0 || k <= 0 || n <= 0 || k % kTileK) return 0;
    return (n % BN == 0 || skinny_supported(m, k, n)) && (epilogue == HMB_EPI_STORE || epilogue == HMB_EPI_SWIGLU) &&
           m < (int64_t(1) << 30);
}

int hmb_w4a16_gemm_plan(int64_t m, int64_t k, int64_t n, int epilogue, int with_workspace, int *plan) {
    if (!plan || !hmb_w4a16_gemm_supports(m, k, n, epilogue)) return HMB_ERR_ARG;
    if (pair_clusters() <= 0) return HMB_ERR_CUDA;
    const GemmPlan p = gemm_plan(m, k, n, with_workspace != 0, false);
    if (p.skinny) {
        plan[0] = 3;
        plan[1] = p.streamk ? 1 : 0;
        plan[2] = 0;
        plan[3] = 1;
        plan[4] = skinny_ctas(m, k, n, p.streamk);
        return HMB_OK;
    }
    plan[0] = p.pair ? 2 : 1;
    plan[1] = p.pair ? p.band_rows : 0;
    plan[2] = p.pair ? p.band : 0;
    plan[3] = p.k_splits;
    plan[4] = p.pair ? pair_clusters() : static_cast<int>((m + BM - 1) / BM * (n / BN));
    return HMB_OK;
}

int hmb_w4a16_gemm(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype, void *y,
                   int64_t ldy, int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue, int layout,
                   hmb_stream_t stream) {
    return gemm_run(packed, packed_k, packed_n, x, ldx, x_dtype, y, ldy, y_dtype, m, k, n, start_col, epilogue, layout, nullptr, 0,
                    nullptr, static_cast<cudaStream_t>(stream));
}

int hmb_device_status(int *status, hmb_stream_t stream) {
    if (!status) return HMB_ERR_ARG;
    int v = 0;
    const int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_gemm_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && v) e = cudaMemcpyToSymbolAsync(g_gemm_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    *status = v ? HMB_ERR_TIMEOUT : HMB_OK;
    return HMB_OK;
}

}  // extern "C"
