// W4A16 prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
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

#include "common.cuh"

namespace hmb {
namespace {

constexpr int BN = 256, BK = 64;
constexpr int kBStages = 2;            // dequantized B tiles
constexpr int kBBytes = BN * BK * 2;   // 32768
constexpr int kPHalf = 2048 + 256;     // half a packed tile + its scales and zeros
constexpr int kPBytes = 4 * kPHalf;    // 9216
constexpr int kDequantWarps = 8;
constexpr int kThreads = (2 + kDequantWarps) * 32;

// Shared-memory plan for a CTA of BM rows (BM = 128: one accumulator, BM = 256: two that share each
// dequantized B tile, so the dequantization work per MMA halves).
template <int BM>
struct Plan {
    static constexpr int kAcc = BM / 128;
    static constexpr int kLoadStages = BM == 128 ? 5 : 3;  // x tile + packed halves, ahead of the MMA
    static constexpr int kABytes = BM * BK * 2;
    static constexpr int kAOff = 0;
    static constexpr int kPOff = kAOff + kLoadStages * kABytes;
    static constexpr int kBOff = kPOff + kLoadStages * kPBytes;  // 1024-aligned: 9216 = 9 x 1024
    static constexpr int kBarOff = kBOff + kBStages * kBBytes;
    static constexpr int kTmemCols = 256 * kAcc;
    static constexpr int kSmemBytes = 1024 + kBarOff + 256;
};
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // a barrier wait gives up after one second

// Set to 1 by a kernel that gave up a bounded wait; read and cleared by hmb_device_status().
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
    int f16;         // activations (and a 16-bit output) are fp16, else bf16
    int y_f32;       // HMB_EPI_STORE: write the fp32 sums instead of rounding them
};

// ---- PTX wrappers ----------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for phase `parity` of a barrier: false if another thread of the CTA gave up, or if
// one second passes (then this thread sets the CTA's abort flag and the device status word).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort) {
    uint64_t start = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 63) == 63) {
            if (*abort) return false;
            const uint64_t now = global_ns();
            if (start == 0) {
                start = now;
            } else if (now - start > kWaitLimitNs) {
                *abort = 1;
                atomicOr(&g_gemm_status, 1);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src),
                 "r"(bytes), "r"(bar)
                 : "memory");
}

// Shared-memory matrix descriptors (tcgen05 format: start >> 4 at bit 0, leading byte offset >> 4
// at bit 16, stride byte offset >> 4 at bit 32, version 1 at bit 46, layout at bit 61: 2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return static_cast<uint64_t>((addr & 0x3FFFF) >> 4) | (static_cast<uint64_t>(lbo_bytes >> 4) << 16) |
           (static_cast<uint64_t>(sbo_bytes >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p; }" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// (h - zc) * s on bf16 (fp16) pairs: the subtraction is exact, the product rounds once.
template <bool F16>
__device__ __forceinline__ uint32_t sub_mul2(uint32_t h, uint32_t zc, uint32_t s) {
    uint32_t d;
    if constexpr (F16) {
        asm("{ .reg .b32 t; sub.rn.f16x2 t, %1, %2; mul.rn.f16x2 %0, t, %3; }" : "=r"(d) : "r"(h), "r"(zc), "r"(s));
    } else {
        asm("{ .reg .b32 t; sub.rn.bf16x2 t, %1, %2; mul.rn.bf16x2 %0, t, %3; }" : "=r"(d) : "r"(h), "r"(zc), "r"(s));
    }
    return d;
}

// ---- the kernel -----------------------------------------------------------------------------------

template <int BM, bool F16, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmArgs a) {
    using P = Plan<BM>;
    constexpr int kLoadStages = P::kLoadStages, kABytes = P::kABytes, kAOff = P::kAOff, kPOff = P::kPOff, kBOff = P::kBOff,
                  kBarOff = P::kBarOff, kTmemCols = P::kTmemCols, kAcc = P::kAcc;
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
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // Producer.
            const uint8_t *col_base[4];
            for (int d = 0; d < 4; ++d) col_base[d] = a.packed + tile_index(tile_col(d), 0, a.tiles_k_total, a.tiles_n_total) * kTileBytes;
            int issued = 0;
            for (int i = 0; i < num_k; ++i) {
                const int s = i % kLoadStages, u = i / kLoadStages;
                if (u > 0 && !mbar_wait(empty_load(s), (u - 1) & 1, abort)) break;
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
                mbar_wait(full_load(i % kLoadStages), (i / kLoadStages) & 1, abort);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer. idesc: fp32 accumulate, bf16 (fp16) A and B, A K-major, B MN-major, N = 256, M = 128.
            const uint32_t fmt = F16 ? 0u : 1u;
            const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) | ((BN >> 3) << 17) | ((128 >> 4) << 24);
            for (int i = 0; i < num_k; ++i) {
                const int sb = i % kBStages, ub = i / kBStages;
                if (!mbar_wait(full_b(sb), ub & 1, abort)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t sa = sbase + kAOff + (i % kLoadStages) * kABytes;
                const uint32_t sbb = sbase + kBOff + sb * kBBytes;
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t bd = smem_desc(sbb + kk * 2 * 4096, 1024, 4096);
#pragma unroll
                    for (int h = 0; h < kAcc; ++h) {
                        // Rows 128 h .. 128 h + 127 of the x tile (16 KB apart) into accumulator h.
                        const uint64_t ad = smem_desc(sa + h * 16384 + kk * 32, 16, 1024);
                        umma_f16(tmem + 256 * h, ad, bd, idesc, (i | kk) != 0);
                    }
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
        constexpr uint32_t kMagic = F16 ? 0x64006400u : 0x43004300u;
        constexpr uint32_t kMask = 0x000F000Fu;
        bool ok = true;
        for (int i = 0; i < num_k; ++i) {
            const int sl = i % kLoadStages, ul = i / kLoadStages;
            const int sb = i % kBStages, ub = i / kBStages;
            if (!mbar_wait(full_load(sl), ul & 1, abort) || (ub > 0 && !mbar_wait(empty_b(sb), (ub - 1) & 1, abort))) {
                ok = false;
                break;
            }
            const uint8_t *pk = smem + kPOff + sl * kPBytes + d * kPHalf;
            const uint8_t *pw = smem + kPOff + sl * kPBytes + ld_off;
            // Scales and offset zeros of columns (p, p + 4) of the group, as 16-bit pairs.
            const uint4 sv = *reinterpret_cast<const uint4 *>(pk + 2048 + 16 * cc);
            const uint2 zv = *reinterpret_cast<const uint2 *>(pk + 2048 + 128 + 16 * cc);
            const uint4 wv2[2] = {*reinterpret_cast<const uint4 *>(pw), *reinterpret_cast<const uint4 *>(pw + 512)};
            uint32_t sp[4], zp[4];
            {
                const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};  // scale of column p at half p%2 of word p/2
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const uint32_t lo = (sw[p >> 1] >> (16 * (p & 1))) & 0xFFFFu;          // column p
                    const uint32_t hi = (sw[2 + (p >> 1)] >> (16 * (p & 1))) & 0xFFFFu;    // column p + 4
                    uint32_t s_pair;
                    if constexpr (F16) {
                        // Scales are stored as bf16; the fp16 path converts them (one rounding).
                        const float flo = __uint_as_float(lo << 16), fhi = __uint_as_float(hi << 16);
                        s_pair = f32_to_f16(flo) | (f32_to_f16(fhi) << 16);
                    } else {
                        s_pair = lo | (hi << 16);
                    }
                    sp[p] = s_pair;
                    const uint32_t zlo = (zv.x >> (8 * p)) & 0xFFu;  // zero of column p
                    const uint32_t zhi = (zv.y >> (8 * p)) & 0xFFu;  // zero of column p + 4
                    zp[p] = kMagic | zlo | (zhi << 16);             // 128 + z (1024 + z) in both halves
                }
            }
            uint8_t *bt = smem + kBOff + sb * kBBytes;
#pragma unroll
            for (int r2 = 0; r2 < 2; ++r2) {
                // Chunk lane + 32 (2 hc + r2) of the half tile: K rows 8 ga + 4 (lane & 1) .. +3, column group cc.
                const uint32_t ws[4] = {wv2[r2].x, wv2[r2].y, wv2[r2].z, wv2[r2].w};
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    const uint32_t w = ws[wi];
                    uint4 o;
                    o.x = sub_mul2<F16>(and_or(w, kMask, kMagic), zp[0], sp[0]);        // columns 0, 4
                    o.y = sub_mul2<F16>(and_or(w >> 4, kMask, kMagic), zp[1], sp[1]);   // columns 1, 5
                    o.z = sub_mul2<F16>(and_or(w >> 8, kMask, kMagic), zp[2], sp[2]);   // columns 2, 6
                    o.w = sub_mul2<F16>(and_or(w >> 12, kMask, kMagic), zp[3], sp[3]);  // columns 3, 7
                    *reinterpret_cast<uint4 *>(bt + st_off[r2][wi]) = o;
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(full_b(sb));
                mbar_arrive(empty_load(sl));
            }
        }

        // Epilogue: warp q = warp % 4 reads TMEM lanes 32q .. 32q + 31. With one accumulator, warps
        // 2-5 take its columns 0-127 and warps 6-9 columns 128-255; with two, warps 2-5 take
        // accumulator 0 (rows 0-127 of the tile) and warps 6-9 accumulator 1, all 256 columns.
        const int q = warp & 3, half = dw >> 2;
        const int acc = kAcc == 2 ? half : 0;
        const int row = 128 * acc + 32 * q + lane, tok = m0 + row;
        if (ok && mbar_wait(acc_full, 0, abort)) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t taddr = tmem + 256 * acc + (static_cast<uint32_t>(32 * q) << 16);
            // Column j = 8 cc + p' of a 64-wide block holds physical column 8 cc + perm[p'].
            constexpr int kPerm[8] = {0, 4, 1, 5, 2, 6, 3, 7};
            if constexpr (EPI == HMB_EPI_SWIGLU) {
              for (int ch = kAcc == 2 ? 0 : half; ch < (kAcc == 2 ? 2 : half + 1); ++ch) {
                // Block pair ch: gate = accumulator block 2 ch, up = block 2 ch + 1 (64 channels).
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t gv[32], uv[32];
                    tmem_ld32(taddr + 128 * ch + 32 * hh, gv);
                    tmem_ld32(taddr + 128 * ch + 64 + 32 * hh, uv);
                    if (tok < a.m) {
                        uint16_t *y = static_cast<uint16_t *>(a.y) + static_cast<int64_t>(tok) * a.ldy +
                                      (2 * nb + ch) * kTileN + 32 * hh;
#pragma unroll
                        for (int g8 = 0; g8 < 4; ++g8) {
                            uint32_t o[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                uint32_t pr = 0;
#pragma unroll
                                for (int hl = 0; hl < 2; ++hl) {
                                    int pp = 0;  // position p' holding physical column 2e + hl
#pragma unroll
                                    for (int t = 0; t < 8; ++t)
                                        if (kPerm[t] == 2 * e + hl) pp = t;
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
            } else {
              for (int ch = kAcc == 2 ? 0 : half; ch < (kAcc == 2 ? 2 : half + 1); ++ch) {
                for (int cb = 0; cb < 4; ++cb) {
                    uint32_t v[32];
                    tmem_ld32(taddr + 128 * ch + 32 * cb, v);
                    if (tok < a.m && a.y_f32) {
                        float *y = static_cast<float *>(a.y) + static_cast<int64_t>(tok) * a.ldy + nb * BN + 128 * ch + 32 * cb;
#pragma unroll
                        for (int g8 = 0; g8 < 4; ++g8) {
                            float o[8];
#pragma unroll
                            for (int t = 0; t < 8; ++t) o[kPerm[t]] = __uint_as_float(v[8 * g8 + t]);
                            *reinterpret_cast<float4 *>(y + 8 * g8) = make_float4(o[0], o[1], o[2], o[3]);
                            *reinterpret_cast<float4 *>(y + 8 * g8 + 4) = make_float4(o[4], o[5], o[6], o[7]);
                        }
                    } else if (tok < a.m) {
                        uint16_t *y = static_cast<uint16_t *>(a.y) + static_cast<int64_t>(tok) * a.ldy + nb * BN + 128 * ch + 32 * cb;
#pragma unroll
                        for (int g8 = 0; g8 < 4; ++g8) {
                            uint32_t o[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                int p0 = 0, p1 = 0;
#pragma unroll
                                for (int t = 0; t < 8; ++t) {
                                    if (kPerm[t] == 2 * e) p0 = t;
                                    if (kPerm[t] == 2 * e + 1) p1 = t;
                                }
                                o[e] = to16<F16>(__uint_as_float(v[8 * g8 + p0])) | (to16<F16>(__uint_as_float(v[8 * g8 + p1])) << 16);
                            }
                            *reinterpret_cast<uint4 *>(y + 8 * g8) = make_uint4(o[0], o[1], o[2], o[3]);
                        }
                    }
                }
              }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
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

template <int BM, bool F16, int EPI>
int launch(const CUtensorMap &map, const GemmArgs &a, cudaStream_t stream) {
    auto kernel = gemm_kernel<BM, F16, EPI>;
    constexpr int kSmemBytes = Plan<BM>::kSmemBytes;
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
    dim3 grid((a.m + BM - 1) / BM, a.n_tiles / 4);
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(map, a);
    return launch_status();
}

}  // namespace
}  // namespace hmb

using namespace hmb;

extern "C" {

int hmb_w4a16_gemm_supports(int64_t m, int64_t k, int64_t n, int epilogue) {
    if (m <= 0 || k <= 0 || n <= 0 || k % kTileK) return 0;
    return n % BN == 0 && (epilogue == HMB_EPI_STORE || epilogue == HMB_EPI_SWIGLU) && m < (int64_t(1) << 30);
}

int hmb_w4a16_gemm(const uint8_t *packed, int64_t packed_k, int64_t packed_n, const void *x, int64_t ldx, int x_dtype, void *y,
                   int64_t ldy, int y_dtype, int64_t m, int64_t k, int64_t n, int64_t start_col, int epilogue, int layout,
                   hmb_stream_t stream) {
    if (!packed || !x || !y || m <= 0) return HMB_ERR_ARG;
    if (k <= 0 || n <= 0 || k % kTileK || n % kTileN || packed_k % kTileK || packed_n % kTileN || start_col < 0 ||
        start_col % kTileN || k > packed_k || start_col + n > packed_n)
        return HMB_ERR_ARG;
    if (x_dtype != HMB_BF16 && x_dtype != HMB_FP16) return HMB_ERR_ARG;
    if (epilogue != HMB_EPI_STORE && epilogue != HMB_EPI_SWIGLU) return HMB_ERR_ARG;
    if (y_dtype != x_dtype && !(y_dtype == HMB_FP32 && epilogue == HMB_EPI_STORE)) return HMB_ERR_ARG;
    if (epilogue == HMB_EPI_SWIGLU && layout != HMB_GATE_UP_BLOCKED && layout != HMB_GATE_UP_INTERLEAVED) return HMB_ERR_ARG;
    if (!hmb_w4a16_gemm_supports(m, k, n, epilogue)) return HMB_ERR_UNSUPPORTED;
    if (epilogue == HMB_EPI_SWIGLU && layout == HMB_GATE_UP_BLOCKED && (n / 2) % (2 * kTileN)) return HMB_ERR_UNSUPPORTED;
    const int64_t out_cols = epilogue == HMB_EPI_SWIGLU ? n / 2 : n;
    if (ldx < k || ldy < out_cols) return HMB_ERR_ARG;
    if (!aligned(packed, 16) || !aligned(x, 16) || !aligned(y, 16) || ldx % 8 || ldy % 8) return HMB_ERR_ALIGN;

    EncodeTiled encode = encode_fn();
    if (!encode) return HMB_ERR_CUDA;
    CUtensorMap map;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(m)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldx) * 2};
    // 256-row tiles (two accumulators per dequantized B tile) once there are more than 128 rows.
    const int bm = m > 128 ? 256 : 128;
    const cuuint32_t box[2] = {BK, static_cast<cuuint32_t>(bm)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = encode(&map, x_dtype == HMB_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                               const_cast<void *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return HMB_ERR_ARG;

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
    a.col_stride = (epilogue == HMB_EPI_SWIGLU && layout == HMB_GATE_UP_BLOCKED) ? a.n_tiles / 2 : 1;
    a.f16 = x_dtype == HMB_FP16;
    a.y_f32 = y_dtype == HMB_FP32;
    const bool swiglu = epilogue == HMB_EPI_SWIGLU;
    if (bm == 256) {
        if (x_dtype == HMB_FP16) return swiglu ? launch<256, true, HMB_EPI_SWIGLU>(map, a, stream) : launch<256, true, HMB_EPI_STORE>(map, a, stream);
        return swiglu ? launch<256, false, HMB_EPI_SWIGLU>(map, a, stream) : launch<256, false, HMB_EPI_STORE>(map, a, stream);
    }
    if (x_dtype == HMB_FP16) return swiglu ? launch<128, true, HMB_EPI_SWIGLU>(map, a, stream) : launch<128, true, HMB_EPI_STORE>(map, a, stream);
    return swiglu ? launch<128, false, HMB_EPI_SWIGLU>(map, a, stream) : launch<128, false, HMB_EPI_STORE>(map, a, stream);
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
