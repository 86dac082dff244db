// Tensor-parallel boundary over NVLink peer memory, two kernels on one communicator:
//   allreduce_kernel: y = the sum over the P ranks of each rank's y, in place, identical bits on
//     every rank (fp32 sums in rank order, one rounding to the output type). It replaces the
//     per-layer all-reduce of the rank partials and the reference's boundary sum residual_add2 /
//     MergedFfn::add_out (kernels/gpu/src/residual_add.cu:55-73,
//     src/unified_llm_w4a16_hetero/merged_ffn.cpp:417).
//   boundary_kernel: the whole layer boundary in one launch: x += the rank partials, then RMSNorm
//     of x into the next layer's input, which lands in every rank's output region. It replaces
//     residual_norm_bf16 on the summed partials (kernels/gpu/src/residual_norm.cu:38-87,
//     src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:2533-2540).
//
// Every rank allocates one symmetric buffer (cudaMalloc) and opens its peers' through CUDA IPC
// handles; the buffer holds flag words, receive slots and the output region. Plain stores and loads
// over NVLink only: no multicast, no library kernel on peer memory.
//
// The grid is always kCtas CTAs. Byte block i (4 KB) of a message or slot belongs to CTA i % kCtas
// on every rank and in every call, whatever the message size, so a CTA only ever copies its own
// blocks, and it synchronizes with the same CTA of the other ranks through flag words that carry a
// per-CTA epoch (incremented at every call of either kernel, the same on all ranks because every
// rank makes the same calls). Receive slots are double-buffered by epoch parity: a CTA cannot be
// two calls ahead of the same CTA of a peer, because finishing a call needs every peer's
// contribution to it.
//   one-shot (small messages): each rank stores its message into every rank's slot[parity][me],
//     raises its flag there, waits for every rank's flag, and sums the P slots in rank order.
//   two-shot (large): the message is cut into P chunks; rank c owns chunk c. Reduce-scatter: each
//     rank stores its part of chunk c into rank c's slot; rank c sums them in rank order. Gather: rank
//     c stores the rounded sum into every rank's gather slot; each rank copies the chunks into y.
// The boundary kernel cuts by rows instead (a row needs all its values for the norm): rank c owns
// rows [c*m/P, (c+1)*m/P). Its CTAs process whole rows, so they wait for the flags of every CTA.
// Chained (two-shot): instead of waiting at its end until every rank's rows have arrived, each CTA
// counts the rows it stored into row-block counters (256 rows a block) on every rank and leaves; the
// next layer's gate/up GEMM waits per row block on this rank's counters before it loads x, so the
// gather overlaps that GEMM. A chained call zeroes this rank's counters before its first flags.
// Every wait gives up after spin_limit_ns (default one second) and ORs 1 into the device status word.
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "comm_internal.h"
#include "common.cuh"
#include "norm_internal.h"
#include "rownorm.cuh"

namespace hmb {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kCtas = 128;
constexpr int kThreads = 256;    // 16 bytes each: one 4 KB block per pass
constexpr int64_t kBlock = 4096;
constexpr size_t kFlagBytes = 2 * 2 * kMaxRanks * kCtas * 4;  // [phase][parity][rank][cta]
constexpr int64_t kReadyBlocks = 4096;                         // row-block counters of a chained boundary
constexpr size_t kHeadBytes = kFlagBytes + kReadyBlocks * 4;   // flags and counters, then the slots
constexpr int64_t kOneShotBytes = 512 * 1024;
constexpr size_t kRowSlack = 2 * kRowMaxH;  // a row-cut chunk can exceed 1/P of a message by one row
static_assert(kThreads == kRowThreads, "the boundary kernel processes rows with the whole CTA");
static_assert(kMaxRanks == kCommMaxRanks, "one rank limit");

struct Peers {
    uint8_t *base[kMaxRanks];  // every rank's symmetric buffer (this rank's included)
};

// What both kernels need to reach the peers and to synchronize with them.
struct Link {
    Peers p;
    int rank, world;
    int64_t slot_bytes;  // bytes of one receive slot
    unsigned *epochs;    // this rank's per-CTA call counters (device memory)
    int *status;
    uint64_t limit_ns;
};

struct ArArgs {
    Link l;
    void *y;
    int64_t elems;
    int two_shot;
};

struct BnArgs {
    Link l;
    const void *y;      // this rank's partial [m, h]: bf16, or fp32 (AT of the kernel)
    uint16_t *x;        // the residual [m, h]
    const uint16_t *w;  // norm weight [h], or null
    int64_t m;
    int h;
    float eps;
    int two_shot;
    int prefilled;       // the partials are already in the slots (a scatter wrote them); y unused
    int64_t out_offset;  // of the output region in every symmetric buffer
    int chained;         // two-shot: count rows into the ready counters instead of waiting for them
};

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys(unsigned *p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Flag word (phase, parity, from-rank, cta) in the buffer of rank `owner`.
__device__ __forceinline__ unsigned *flag(const Link &l, int owner, int phase, int parity, int from, int cta) {
    return reinterpret_cast<unsigned *>(l.p.base[owner]) + ((phase * 2 + parity) * kMaxRanks + from) * kCtas + cta;
}
// Receive slot (phase 0: reduce-scatter / one-shot, phase 1: gather) for data from rank `from`.
__device__ __forceinline__ uint8_t *slot(const Link &l, int owner, int phase, int parity, int from) {
    return l.p.base[owner] + kHeadBytes + ((static_cast<int64_t>(phase) * 2 + parity) * l.world + from) * l.slot_bytes;
}
// Row-block counter mb of a chained boundary in the buffer of rank `owner`.
__device__ __forceinline__ unsigned *ready(const Link &l, int owner, int64_t mb) {
    return reinterpret_cast<unsigned *>(l.p.base[owner] + kFlagBytes) + mb;
}

// Spins (bounded) until the flag reaches `epoch`.
__device__ __forceinline__ bool wait_flag(const Link &l, const unsigned *f, unsigned epoch) {
    const uint64_t start = now_ns();
    for (uint32_t i = 0;; ++i) {
        if (static_cast<int>(ld_acquire_sys(f) - epoch) >= 0) return true;
        if ((i & 15) == 15 && now_ns() - start > l.limit_ns) {
            atomicOr(l.status, 1);
            return false;
        }
        __nanosleep(32);
    }
}

// This CTA's call number (the same on every rank); *ok = 1.
__device__ __forceinline__ unsigned begin_call(const Link &l, unsigned *s_epoch, int *ok) {
    if (threadIdx.x == 0) {
        *s_epoch = ++l.epochs[blockIdx.x];
        *ok = 1;
    }
    __syncthreads();
    return *s_epoch;
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// 16-byte copies of this CTA's blocks of [0, bytes): dst + o <- src + o. Each thread loads its
// granule of kU blocks before storing them, so kU loads per thread are in flight.
__device__ __forceinline__ void copy_blocks(uint8_t *dst, const uint8_t *src, int64_t bytes) {
    constexpr int kU = 8;
    const int64_t t16 = 16 * static_cast<int64_t>(threadIdx.x);
    for (int64_t blk = blockIdx.x; blk * kBlock < bytes; blk += kU * kCtas) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int64_t o = (blk + u * kCtas) * kBlock + t16;
            if (o < bytes) v[u] = *reinterpret_cast<const uint4 *>(src + o);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int64_t o = (blk + u * kCtas) * kBlock + t16;
            if (o < bytes) *reinterpret_cast<uint4 *>(dst + o) = v[u];
        }
    }
}

// For this CTA's blocks of [0, bytes): out + o = sum over ranks r, in rank order, of in[r] + o
// (fp32 sums, one rounding to T); kU blocks per thread step, every load issued before the sums.
template <typename T>
__device__ __forceinline__ void sum_blocks(int world, uint8_t *out, const uint8_t *const *in, int64_t bytes) {
    constexpr int kV = 16 / sizeof(T), kU = 4;
    const int64_t t16 = 16 * static_cast<int64_t>(threadIdx.x);
    for (int64_t blk = blockIdx.x; blk * kBlock < bytes; blk += kU * kCtas) {
        float acc[kU][kV];
#pragma unroll
        for (int u = 0; u < kU; ++u)
#pragma unroll
            for (int v = 0; v < kV; ++v) acc[u][v] = 0.0f;
        for (int r = 0; r < world; ++r) {
            uint4 raw[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t o = (blk + u * kCtas) * kBlock + t16;
                if (o < bytes) raw[u] = *reinterpret_cast<const uint4 *>(in[r] + o);
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const T *vals = reinterpret_cast<const T *>(&raw[u]);
#pragma unroll
                for (int v = 0; v < kV; ++v) acc[u][v] += to_f32<T>(vals[v]);
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int64_t o = (blk + u * kCtas) * kBlock + t16;
            if (o >= bytes) continue;
            uint4 res;
            T *rv = reinterpret_cast<T *>(&res);
#pragma unroll
            for (int v = 0; v < kV; ++v) rv[v] = from_f32<T>(acc[u][v]);
            *reinterpret_cast<uint4 *>(out + o) = res;
        }
    }
}

// Raises this CTA's flag `phase` on every rank (after the CTA's stores of the phase).
__device__ __forceinline__ void raise_flags(const Link &l, int phase, int par, unsigned epoch) {
    __syncthreads();  // this CTA's stores of the phase are issued
    // release at system scope after the CTA barrier: this CTA's stores (to peers too) are visible
    // to whoever acquires the flag
    if (threadIdx.x < l.world) st_release_sys(flag(l, threadIdx.x, phase, par, l.rank, blockIdx.x), epoch);
}

// Raises this CTA's flag `phase` on every rank, then waits (bounded) for every rank's flag of the
// same CTA here.
__device__ __forceinline__ bool exchange_flags(const Link &l, int phase, int par, unsigned epoch, int *ok) {
    raise_flags(l, phase, par, epoch);
    if (threadIdx.x < l.world && !wait_flag(l, flag(l, l.rank, phase, par, threadIdx.x, blockIdx.x), epoch)) *ok = 0;
    __syncthreads();
    return *ok != 0;
}

// Waits (bounded) until every CTA of every rank has raised its flag `phase` here.
__device__ __forceinline__ bool wait_all_ctas(const Link &l, int phase, int par, unsigned epoch, int *ok) {
    for (int i = threadIdx.x; i < l.world * kCtas; i += blockDim.x)
        if (!wait_flag(l, flag(l, l.rank, phase, par, i / kCtas, i % kCtas), epoch)) {
            *ok = 0;
            break;
        }
    __syncthreads();
    return *ok != 0;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) allreduce_kernel(const ArArgs a) {
    __shared__ unsigned s_epoch;
    __shared__ int s_ok;
    const Link &l = a.l;
    const unsigned epoch = begin_call(l, &s_epoch, &s_ok);
    const int par = epoch & 1;
    uint8_t *y = static_cast<uint8_t *>(a.y);
    const int64_t bytes = a.elems * static_cast<int64_t>(sizeof(T));
    const uint8_t *in[kMaxRanks];

    if (!a.two_shot) {
        // One-shot: this rank's message into every rank's slot[me]; then sum the P slots here. Each
        // rank visits the peers starting after itself, so no GPU receives from all ranks at once.
        for (int j = 0; j < l.world; ++j) {
            const int r = (l.rank + j) % l.world;
            copy_blocks(slot(l, r, 0, par, l.rank), y, bytes);
        }
        if (!exchange_flags(l, 0, par, epoch, &s_ok)) return;
        for (int r = 0; r < l.world; ++r) in[r] = slot(l, l.rank, 0, par, r);
        sum_blocks<T>(l.world, y, in, bytes);
        return;
    }

    // Two-shot. Chunk c = bytes [c * chunk, (c + 1) * chunk) of the message; rank c owns it.
    const int64_t chunk = ((bytes + l.world - 1) / l.world + 15) / 16 * 16;
    auto chunk_bytes = [&](int c) { return std::max<int64_t>(0, std::min<int64_t>(chunk, bytes - c * chunk)); };
    // Reduce-scatter: chunk c of this rank's message into rank c's slot[me].
    for (int j = 0; j < l.world; ++j) {
        const int c = (l.rank + j) % l.world;
        copy_blocks(slot(l, c, 0, par, l.rank), y + c * chunk, chunk_bytes(c));
    }
    if (!exchange_flags(l, 0, par, epoch, &s_ok)) return;
    // The sum of this rank's chunk, in rank order, into this rank's gather slot[me], then into every
    // other rank's gather slot[me].
    uint8_t *mine = slot(l, l.rank, 1, par, l.rank);
    for (int r = 0; r < l.world; ++r) in[r] = slot(l, l.rank, 0, par, r);
    sum_blocks<T>(l.world, mine, in, chunk_bytes(l.rank));
    __syncthreads();
    for (int j = 1; j < l.world; ++j) copy_blocks(slot(l, (l.rank + j) % l.world, 1, par, l.rank), mine, chunk_bytes(l.rank));
    if (!exchange_flags(l, 1, par, epoch, &s_ok)) return;
    // Gather: chunk c from gather slot[c] into y.
    for (int c = 0; c < l.world; ++c) copy_blocks(y + c * chunk, slot(l, l.rank, 1, par, c), chunk_bytes(c));
}

// The layer boundary. One-shot: every rank gets every partial and computes every row (the residual
// stays whole on every rank). Two-shot: rank c receives the rows it owns from every rank, computes
// them, keeps x for those rows, and stores the normed rows into every rank's output region.
template <int V, int NW, typename AT>
__global__ void __launch_bounds__(kThreads, 1) boundary_kernel(const BnArgs a) {
    __shared__ unsigned s_epoch;
    __shared__ int s_ok;
    __shared__ float red[kRowThreads / 32];
    const Link &l = a.l;
    // The next kernel may start its prologue; it waits for this grid before it reads the output.
    pdl_launch_dependents();
    pdl_wait();  // y comes from the previous kernel
    const unsigned epoch = begin_call(l, &s_epoch, &s_ok);
    const int par = epoch & 1;
    const int64_t row_bytes = static_cast<int64_t>(sizeof(AT)) * a.h;  // a partial row, in y and in the slots
    const uint8_t *y = static_cast<const uint8_t *>(a.y);
    const AT *ya = static_cast<const AT *>(a.y);
    const AT *in[kMaxRanks];
    uint16_t *out[kMaxRanks];

    // This rank's own partial: y, or (prefilled) its own slot like every other rank's.
    const bool own_y = !a.prefilled;
    if (!a.two_shot) {
        if (!a.prefilled)
            for (int j = 1; j < l.world; ++j) copy_blocks(slot(l, (l.rank + j) % l.world, 0, par, l.rank), y, a.m * row_bytes);
        raise_flags(l, 0, par, epoch);
        if (!wait_all_ctas(l, 0, par, epoch, &s_ok)) return;
        for (int64_t row = blockIdx.x; row < a.m; row += kCtas) {
#pragma unroll
            for (int r = 0; r < NW; ++r)
                in[r] = r == l.rank && own_y ? ya + row * a.h
                                             : reinterpret_cast<const AT *>(slot(l, l.rank, 0, par, r) + row * row_bytes);
            out[0] = reinterpret_cast<uint16_t *>(l.p.base[l.rank] + a.out_offset) + row * a.h;
            boundary_row<V, NW, AT>(in, a.x + row * a.h, true, a.w, a.h, a.eps, out, 1, red);
        }
        return;
    }

    // Chained: this rank's counters start from zero; the flags below publish that before any rank
    // counts rows of this call into them (the previous call's counts were consumed by the GEMM that
    // ran before this kernel).
    if (a.chained)
        for (int64_t mb = blockIdx.x * kThreads + threadIdx.x; mb < (a.m + 255) / 256; mb += kCtas * kThreads)
            *ready(l, l.rank, mb) = 0u;
    // Reduce-scatter by rows: rank c's rows of this rank's partial into rank c's slot[me].
    if (!a.prefilled)
        for (int j = 1; j < l.world; ++j) {  // owners visited from the next rank on: no incast
            const int c = (l.rank + j) % l.world;
            const int64_t r0 = comm_share_row(a.m, l.world, c), r1 = comm_share_row(a.m, l.world, c + 1);
            copy_blocks(slot(l, c, 0, par, l.rank), y + r0 * row_bytes, (r1 - r0) * row_bytes);
        }
    raise_flags(l, 0, par, epoch);
    if (!wait_all_ctas(l, 0, par, epoch, &s_ok)) return;
    const int64_t r0 = comm_share_row(a.m, l.world, l.rank), r1 = comm_share_row(a.m, l.world, l.rank + 1);
    for (int64_t row = r0 + blockIdx.x; row < r1; row += kCtas) {
#pragma unroll
        for (int r = 0; r < NW; ++r) {
            in[r] = r == l.rank && own_y ? ya + row * a.h
                                         : reinterpret_cast<const AT *>(slot(l, l.rank, 0, par, r) + (row - r0) * row_bytes);
            // Destinations from this rank on, so the ranks do not all store into one GPU at once.
            const int d = (l.rank + r) % NW;
            out[r] = reinterpret_cast<uint16_t *>(l.p.base[d] + a.out_offset) + row * a.h;
        }
        boundary_row<V, NW, AT>(in, a.x + row * a.h, true, a.w, a.h, a.eps, out, NW, red);
    }
    if (a.chained) {
        // Count this CTA's rows into every rank's row-block counters, after its stores: the CTA
        // barrier, then a release at system scope by the counting threads (one per rank).
        __syncthreads();
        if (threadIdx.x < NW) {
            const int d = (l.rank + threadIdx.x) % NW;
            int64_t mb = -1;
            unsigned n = 0;
            for (int64_t row = r0 + blockIdx.x; row < r1; row += kCtas) {
                if (row / 256 != mb) {
                    if (n) red_release_sys(ready(l, d, mb), n);
                    mb = row / 256;
                    n = 0;
                }
                ++n;
            }
            if (n) red_release_sys(ready(l, d, mb), n);
        }
        return;
    }
    // The kernel ends only when every rank's rows have arrived in this rank's output region.
    raise_flags(l, 1, par, epoch);
    wait_all_ctas(l, 1, par, epoch, &s_ok);
}

template <int V, typename AT>
cudaError_t launch_boundary_v(int world, cudaStream_t s, const BnArgs &a) {
    const dim3 g(kCtas), b(kThreads);
    switch (world) {
        case 1: return launch_pdl(boundary_kernel<V, 1, AT>, g, b, 0, s, a);
        case 2: return launch_pdl(boundary_kernel<V, 2, AT>, g, b, 0, s, a);
        case 3: return launch_pdl(boundary_kernel<V, 3, AT>, g, b, 0, s, a);
        case 4: return launch_pdl(boundary_kernel<V, 4, AT>, g, b, 0, s, a);
        case 5: return launch_pdl(boundary_kernel<V, 5, AT>, g, b, 0, s, a);
        case 6: return launch_pdl(boundary_kernel<V, 6, AT>, g, b, 0, s, a);
        case 7: return launch_pdl(boundary_kernel<V, 7, AT>, g, b, 0, s, a);
        default: return launch_pdl(boundary_kernel<V, 8, AT>, g, b, 0, s, a);
    }
}

template <typename AT>
cudaError_t launch_boundary_t(int v, int world, cudaStream_t s, const BnArgs &a) {
    if (v == 1) return launch_boundary_v<1, AT>(world, s, a);
    if (v == 2) return launch_boundary_v<2, AT>(world, s, a);
    if (v == 4) return launch_boundary_v<4, AT>(world, s, a);
    return launch_boundary_v<8, AT>(world, s, a);
}

cudaError_t launch_boundary(int v, int world, bool f32, cudaStream_t s, const BnArgs &a) {
    return f32 ? launch_boundary_t<float>(v, world, s, a) : launch_boundary_t<uint16_t>(v, world, s, a);
}

}  // namespace
}  // namespace hmb

using namespace hmb;

struct hmb_comm {
    int rank = 0, world = 1, device = 0;
    size_t max_bytes = 0;   // largest message
    size_t slot_bytes = 0;  // one receive slot
    size_t out_offset = 0;  // output region of the boundary, max_bytes long
    uint8_t *mine = nullptr;
    unsigned *epochs = nullptr;
    Peers peers{};
    bool connected = false;
};

namespace {

Link make_link(const hmb_comm *c, uint64_t spin_limit_ns, int *status) {
    Link l{};
    l.p = c->peers;
    l.rank = c->rank;
    l.world = c->world;
    l.slot_bytes = static_cast<int64_t>(c->slot_bytes);
    l.epochs = c->epochs;
    l.status = status;
    l.limit_ns = spin_limit_ns ? spin_limit_ns : 1000000000ull;
    return l;
}

}  // namespace

namespace hmb {

int comm_world(const hmb_comm *c) { return c ? c->world : 0; }

bool comm_chains(const hmb_comm *c, int64_t m, int64_t h) {
    return c && c->connected && c->world > 1 && m * h * 2 > kOneShotBytes && (m + 255) / 256 <= kReadyBlocks;
}

const unsigned *comm_ready(const hmb_comm *c) { return c ? reinterpret_cast<const unsigned *>(c->mine + kFlagBytes) : nullptr; }

const void *comm_out_region(const hmb_comm *c) { return c ? c->mine + c->out_offset : nullptr; }

int comm_scatter_target(const hmb_comm *c, int64_t m, int64_t h, ScatterTarget *t) {
    if (!c || !t || m <= 0 || h <= 0 || h % 8) return HMB_ERR_ARG;
    if (!c->connected) return HMB_ERR_ARG;
    const int64_t bytes = m * h * 2;
    if (static_cast<size_t>(bytes) > c->max_bytes) return HMB_ERR_WORKSPACE;
    const bool all = bytes <= kOneShotBytes || c->world == 1;
    if (!all && static_cast<size_t>((comm_share_row(m, c->world, 1) + 1) * 2 * h) > c->slot_bytes) return HMB_ERR_WORKSPACE;
    *t = ScatterTarget{};
    for (int r = 0; r < c->world; ++r) t->base[r] = c->peers.base[r];
    t->slot0 = static_cast<int64_t>(kHeadBytes);
    t->slot_bytes = static_cast<int64_t>(c->slot_bytes);
    t->world = c->world;
    t->rank = c->rank;
    t->all = all;
    t->m = m;
    t->h = h;
    t->epochs = c->epochs;
    return HMB_OK;
}

int comm_boundary(hmb_comm *c, const void *y, int y_dtype, void *x, const void *weight, int64_t m, int64_t h, float eps,
                  bool prefilled, cudaStream_t s, uint64_t spin_limit_ns, bool chained) {
    if (!x || !c || m <= 0 || h <= 0 || h % 8 || h > kRowMaxH || !(eps >= 0.0f)) return HMB_ERR_ARG;
    if (!c->connected || (!y && !prefilled)) return HMB_ERR_ARG;
    if (y_dtype != HMB_BF16 && y_dtype != HMB_FP32) return HMB_ERR_ARG;
    if (prefilled && y_dtype != HMB_BF16) return HMB_ERR_ARG;  // the scattering GEMM writes bf16
    if ((y && !aligned(y, 16)) || !aligned(x, 16) || (weight && !aligned(weight, 16))) return HMB_ERR_ALIGN;
    // One-shot or two-shot by the bf16 size of the message, whatever the partials' type, so the rows
    // a rank keeps (hmb_comm_rows) do not depend on it; a one-shot slot holds fp32 partials too.
    const int64_t bytes = m * h * 2, esz = y_dtype == HMB_FP32 ? 4 : 2;
    if (static_cast<size_t>(bytes) > c->max_bytes) return HMB_ERR_WORKSPACE;
    void *out = c->mine + c->out_offset;
    const bool two_shot = bytes > kOneShotBytes && c->world > 1;
    const int64_t slot_need = two_shot ? (comm_share_row(m, c->world, 1) + 1) * esz * h : m * h * esz;
    if (static_cast<size_t>(slot_need) > c->slot_bytes) return HMB_ERR_WORKSPACE;
    if (c->world == 1 && !prefilled && y_dtype == HMB_BF16) return residual_norm_launch(x, h, y, h, nullptr, 0, weight, out, h, m, h, eps, s);
    int *status = device_status_word();
    if (!status) return HMB_ERR_CUDA;
    BnArgs a{};
    a.l = make_link(c, spin_limit_ns, status);
    a.y = y;
    a.x = static_cast<uint16_t *>(x);
    a.w = static_cast<const uint16_t *>(weight);
    a.m = m;
    a.h = static_cast<int>(h);
    a.eps = eps;
    a.two_shot = two_shot;
    a.prefilled = prefilled;
    a.out_offset = static_cast<int64_t>(c->out_offset);
    a.chained = chained && comm_chains(c, m, h);
    const cudaError_t e = launch_boundary(row_vectors(h), c->world, y_dtype == HMB_FP32, s, a);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    return HMB_OK;
}

}  // namespace hmb

extern "C" {

size_t hmb_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int hmb_comm_create(int rank, int world, size_t max_bytes, hmb_comm **out, void *handle) {
    if (!out || !handle || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || max_bytes == 0) return HMB_ERR_ARG;
    hmb_comm *c = new hmb_comm();
    c->rank = rank;
    c->world = world;
    cudaGetDevice(&c->device);
    c->max_bytes = (max_bytes + 255) / 256 * 256;
    // A one-shot slot holds a whole message (<= kOneShotBytes, twice that for the boundary's fp32
    // partials), a two-shot slot one chunk of it (for the boundary, one rank's rows: at most one row
    // more than 1/P of the message).
    c->slot_bytes = std::max<size_t>(2 * kOneShotBytes, ((c->max_bytes + world - 1) / world + kRowSlack + 255) / 256 * 256);
    c->out_offset = kHeadBytes + 2 * 2 * static_cast<size_t>(world) * c->slot_bytes;
    const size_t bytes = c->out_offset + c->max_bytes;
    cudaError_t e = cudaMalloc(&c->mine, bytes);
    if (e == cudaSuccess) e = cudaMemset(c->mine, 0, kHeadBytes);
    if (e == cudaSuccess) e = cudaMalloc(&c->epochs, kCtas * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(c->epochs, 0, kCtas * sizeof(unsigned));
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->mine);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        set_cuda_error(e);
        if (c->mine) cudaFree(c->mine);
        if (c->epochs) cudaFree(c->epochs);
        delete c;
        return HMB_ERR_CUDA;
    }
    std::memcpy(handle, &h, sizeof(h));
    *out = c;
    return HMB_OK;
}

int hmb_comm_connect(hmb_comm *c, const void *handles) {
    if (!c || !handles) return HMB_ERR_ARG;
    const auto *h = static_cast<const cudaIpcMemHandle_t *>(handles);
    for (int r = 0; r < c->world; ++r) {
        if (r == c->rank) {
            c->peers.base[r] = c->mine;
            continue;
        }
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return HMB_ERR_CUDA;
        }
        c->peers.base[r] = static_cast<uint8_t *>(p);
    }
    c->connected = true;
    return HMB_OK;
}

int hmb_allreduce_partials(void *y, int64_t elems, int dtype, hmb_comm *c, hmb_stream_t stream, uint64_t spin_limit_ns) {
    if (!y || !c || elems <= 0) return HMB_ERR_ARG;
    if (!c->connected) return HMB_ERR_ARG;
    if (dtype != HMB_BF16 && dtype != HMB_FP16 && dtype != HMB_FP32) return HMB_ERR_ARG;
    const int esz = dtype == HMB_FP32 ? 4 : 2;
    const int64_t bytes = elems * esz;
    if (bytes % 16 || !aligned(y, 16)) return HMB_ERR_ALIGN;
    if (static_cast<size_t>(bytes) > c->max_bytes) return HMB_ERR_WORKSPACE;
    if (c->world == 1) return HMB_OK;
    int *status = device_status_word();
    if (!status) return HMB_ERR_CUDA;
    ArArgs a{};
    a.l = make_link(c, spin_limit_ns, status);
    a.y = y;
    a.elems = elems;
    a.two_shot = bytes > kOneShotBytes;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == HMB_FP32)
        allreduce_kernel<float><<<kCtas, kThreads, 0, s>>>(a);
    else if (dtype == HMB_BF16)
        allreduce_kernel<__nv_bfloat16><<<kCtas, kThreads, 0, s>>>(a);
    else
        allreduce_kernel<__half><<<kCtas, kThreads, 0, s>>>(a);
    return launch_status();
}

int hmb_comm_out(hmb_comm *c, void **ptr, size_t *bytes) {
    if (!c || !ptr) return HMB_ERR_ARG;
    *ptr = c->mine + c->out_offset;
    if (bytes) *bytes = c->max_bytes;
    return HMB_OK;
}

int hmb_comm_rows(const hmb_comm *c, int64_t m, int64_t h, int64_t *begin, int64_t *end) {
    if (!c || !begin || !end || m <= 0 || h <= 0) return HMB_ERR_ARG;
    if (m * h * 2 <= kOneShotBytes || c->world == 1) {
        *begin = 0;
        *end = m;
    } else {
        *begin = comm_share_row(m, c->world, c->rank);
        *end = comm_share_row(m, c->world, c->rank + 1);
    }
    return HMB_OK;
}

int hmb_allreduce_residual_norm(const void *y, int y_dtype, void *x, const void *weight, int64_t m, int64_t h, float eps, hmb_comm *c,
                                hmb_stream_t stream, uint64_t spin_limit_ns) {
    if (!y) return HMB_ERR_ARG;
    return comm_boundary(c, y, y_dtype, x, weight, m, h, eps, false, static_cast<cudaStream_t>(stream), spin_limit_ns);
}

int hmb_comm_destroy(hmb_comm *c) {
    if (!c) return HMB_ERR_ARG;
    cudaDeviceSynchronize();
    for (int r = 0; r < c->world; ++r)
        if (r != c->rank && c->peers.base[r]) cudaIpcCloseMemHandle(c->peers.base[r]);
    if (c->mine) cudaFree(c->mine);
    if (c->epochs) cudaFree(c->epochs);
    delete c;
    return HMB_OK;
}

}  // extern "C"
