// PTX wrappers for the tcgen05 GEMMs (sm_100a): mbarriers (bounded waits), TMA and bulk copies,
// shared-memory matrix descriptors, tcgen05.mma / commit / ld, cluster addressing, and the nibble
// dequantization arithmetic shared by the one-CTA and the CTA-pair kernels.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace hmb {
namespace tc {

constexpr uint64_t kWaitLimitNs = 1000000000ull;  // a barrier wait gives up after one second

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
// Arrive on a barrier given by its shared::cluster address (this CTA's or the peer's), with the
// instruction's default semantics (release, CTA scope). A release at cluster scope here costs about
// a microsecond per arrival and serialises the producer warps; the data it publishes is this CTA's
// own shared memory, made visible to the tensor core by fence.proxy.async before the arrival.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// All threads of both CTAs of the cluster (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for phase `parity` of a barrier of this CTA. Returns false if another thread of the
// CTA gave up (abort flag set) or if one second passes; then this thread sets the abort flag and
// ORs 1 into the device status word.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort, int *status) {
    uint64_t start = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t done;
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
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
                atomicOr(status, 1);
                return false;
            }
        }
    }
}

// Spins (bounded like mbar_wait) until the counter at p reaches `need` (acquire at system scope: it is
// raised by other GPUs after their stores), then orders this thread's later bulk-tensor copies, which
// read through the async proxy, after what it acquired.
__device__ __forceinline__ bool wait_rows(const unsigned *p, unsigned need, volatile int *abort, int *status) {
    uint64_t start = 0;
    for (uint32_t i = 0;; ++i) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (v >= need) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            return true;
        }
        if ((i & 15) == 15) {
            if (*abort) return false;
            const uint64_t now = global_ns();
            if (start == 0) {
                start = now;
            } else if (now - start > kWaitLimitNs) {
                *abort = 1;
                atomicOr(status, 1);
                return false;
            }
        }
        __nanosleep(64);
    }
}

// 2D TMA tile load into this CTA's shared memory, completing on a barrier of this CTA.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// 2D TMA tile load into this CTA's shared memory whose completion is signalled on a barrier of
// either CTA of the pair (`cluster_bar` is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t cluster_bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(cluster_bar)
        : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
// Contiguous copy global -> this CTA's shared memory (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src),
                 "r"(bytes), "r"(bar)
                 : "memory");
}

// Shared-memory matrix descriptor (tcgen05 format: start >> 4 at bit 0, leading byte offset >> 4
// at bit 16, stride byte offset >> 4 at bit 32, version 1 at bit 46, layout at bit 61: 2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return static_cast<uint64_t>((addr & 0x3FFFF) >> 4) | (static_cast<uint64_t>(lbo_bytes >> 4) << 16) |
           (static_cast<uint64_t>(sbo_bytes >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulate, A and B both bf16 (fmt 1) or both fp16
// (fmt 0), A K-major, B MN-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_f16(bool f16, int m, int n) {
    return (1u << 4) | ((f16 ? 0u : 1u) << 7) | ((f16 ? 0u : 1u) << 10) | (1u << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p; }" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// MMA over a CTA pair (issued by the even CTA): A rows and B columns split between the two CTAs'
// shared memory at the same offsets, D rows split between their TMEM.
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p; }" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// The same with the descriptors given as 32-bit halves (the issuing loop only adds offsets to the
// low halves: start address >> 4 lives in bits 0-13).
__device__ __forceinline__ void umma_f16_pair_lohi(uint32_t tmem_d, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo, uint32_t b_hi, uint32_t idesc,
                                                   uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; .reg .b64 da, db;\n"
        "mov.b64 da, {%1, %2}; mov.b64 db, {%3, %4}; setp.ne.b32 p, %6, 0;\n"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %5, {%7, %7, %7, %7, %7, %7, %7, %7}, p; }" ::"r"(tmem_d),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// Low / high 32 bits of smem_desc().
__device__ __forceinline__ uint32_t smem_desc_lo(uint32_t addr, uint32_t lbo_bytes) { return ((addr & 0x3FFFF) >> 4) | ((lbo_bytes >> 4) << 16); }
__host__ __device__ constexpr uint32_t smem_desc_hi(uint32_t sbo_bytes) { return (sbo_bytes >> 4) | (1u << 14) | (2u << 29); }
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// Arrive on the barrier at shared offset `bar` of every CTA in `mask` once this thread's earlier
// pair MMAs have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar, uint16_t mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
                 "h"(mask)
                 : "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes (one fp32 per lane and column).
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    tmem_ld32_nowait(taddr, v);
    tmem_wait_ld();
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

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

// Dequantization constants of one 8-column group of a packed tile: the scale and 128 + z (1024 + z
// for fp16) of columns (p, p + 4) as 16-bit pairs, p = 0..3. `sc` points at the tile's 64 bf16
// scales, `zr` at its zero bytes (column c at (c / 8) * 16 + c % 8), `cc` is the column group.
template <bool F16>
__device__ __forceinline__ void group_consts(const uint8_t *sc, const uint8_t *zr, int cc, uint32_t (&sp)[4], uint32_t (&zp)[4]) {
    constexpr uint32_t kMagic = F16 ? 0x64006400u : 0x43004300u;
    const uint4 sv = *reinterpret_cast<const uint4 *>(sc + 16 * cc);
    const uint2 zv = *reinterpret_cast<const uint2 *>(zr + 16 * cc);
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};  // scale of column p at half p % 2 of word p / 2
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t lo = (sw[p >> 1] >> (16 * (p & 1))) & 0xFFFFu;        // column p
        const uint32_t hi = (sw[2 + (p >> 1)] >> (16 * (p & 1))) & 0xFFFFu;  // column p + 4
        if constexpr (F16) {
            // Scales are stored as bf16; the fp16 path converts them (one rounding).
            sp[p] = f32_to_f16(__uint_as_float(lo << 16)) | (f32_to_f16(__uint_as_float(hi << 16)) << 16);
        } else {
            sp[p] = lo | (hi << 16);
        }
        const uint32_t zlo = (zv.x >> (8 * p)) & 0xFFu;  // zero of column p
        const uint32_t zhi = (zv.y >> (8 * p)) & 0xFFu;  // zero of column p + 4
        zp[p] = kMagic | zlo | (zhi << 16);
    }
}

// One 32-bit word of a packed tile (one K row, 8 columns) to 8 dequantized 16-bit values in the
// column order (0,4,1,5,2,6,3,7): OR-ing a nibble into the mantissa of bf16 128.0 (fp16 1024.0)
// gives 128 + q exactly, and (128 + q) - (128 + z) is exact before the one rounding by the scale.
template <bool F16>
__device__ __forceinline__ uint4 dequant_word(uint32_t w, const uint32_t (&sp)[4], const uint32_t (&zp)[4]) {
    constexpr uint32_t kMagic = F16 ? 0x64006400u : 0x43004300u;
    constexpr uint32_t kMask = 0x000F000Fu;
    uint4 o;
    o.x = sub_mul2<F16>(and_or(w, kMask, kMagic), zp[0], sp[0]);        // columns 0, 4
    o.y = sub_mul2<F16>(and_or(w >> 4, kMask, kMagic), zp[1], sp[1]);   // columns 1, 5
    o.z = sub_mul2<F16>(and_or(w >> 8, kMask, kMagic), zp[2], sp[2]);   // columns 2, 6
    o.w = sub_mul2<F16>(and_or(w >> 12, kMask, kMagic), zp[3], sp[3]);  // columns 3, 7
    return o;
}

// Position p' (0..7) inside an 8-column group of the dequantized B operand that holds physical
// column c: the inverse of the order (0,4,1,5,2,6,3,7).
__host__ __device__ constexpr int perm_pos(int c) { return (c & 3) * 2 + (c >> 2); }

}  // namespace tc
}  // namespace hmb
