// Tensor-parallel boundary sum over NVLink peer memory: y = sum over the P ranks of each rank's y,
// in place, identical bits on every rank (fp32 sums in rank order, one rounding to the output type).
// It replaces the per-layer NCCL all-reduce of the rank partials and the reference's boundary sum
// residual_add2 / MergedFfn::add_out (kernels/gpu/src/residual_add.cu:55-73,
// src/unified_llm_w4a16_hetero/merged_ffn.cpp:417).
//
// Every rank allocates one symmetric buffer (cudaMalloc) and opens its peers' through CUDA IPC
// handles; the buffer holds receive slots and flag words. Plain stores and loads over NVLink only:
// no multicast, no library kernel on peer memory.
//
// The grid is always kCtas CTAs. Byte block i (4 KB) of a message or slot belongs to CTA i % kCtas
// on every rank and in every call, whatever the message size, so a CTA only ever touches its own
// blocks and synchronizes only with the same CTA of the other ranks, through flag words that carry
// a per-CTA epoch (incremented at every call, the same on all ranks because every rank makes the
// same calls). Receive slots are double-buffered by epoch parity: CTA b cannot be two calls ahead of
// CTA b of a peer, because finishing a call needs every peer's contribution to it.
//   one-shot (small messages): each rank stores its sub-range into every rank's slot[parity][me],
//     raises its flag there, waits for every rank's flag, and sums the P slots in rank order.
//   two-shot (large): the message is cut into P chunks; rank c owns chunk c. Reduce-scatter: each
//     rank stores its part of chunk c into rank c's slot; rank c sums them in rank order. Gather: rank
//     c stores the rounded sum into every rank's gather slot; each rank copies the chunks into y.
// Every wait gives up after spin_limit_ns (default one second) and ORs 1 into the device status word.
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace hmb {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kCtas = 64;
constexpr int kThreads = 256;    // 16 bytes each: one 4 KB block per pass
constexpr int64_t kBlock = 4096;
constexpr size_t kFlagBytes = 2 * 2 * kMaxRanks * kCtas * 4;  // [phase][parity][rank][cta]
constexpr int64_t kOneShotBytes = 512 * 1024;

struct Peers {
    uint8_t *base[kMaxRanks];  // every rank's symmetric buffer (this rank's included)
};

struct ArArgs {
    Peers p;
    void *y;
    int64_t elems;
    int dtype;  // HMB_BF16, HMB_FP16 or HMB_FP32
    int rank, world;
    int two_shot;
    int64_t slot_bytes;  // bytes of one receive slot
    unsigned *epochs;    // this rank's per-CTA call counters (device memory)
    int *status;
    uint64_t limit_ns;
};

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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
__device__ __forceinline__ unsigned *flag(const ArArgs &a, int owner, int phase, int parity, int from, int cta) {
    return reinterpret_cast<unsigned *>(a.p.base[owner]) + ((phase * 2 + parity) * kMaxRanks + from) * kCtas + cta;
}
// Receive slot (phase 0: reduce-scatter / one-shot, phase 1: gather) for data from rank `from`.
__device__ __forceinline__ uint8_t *slot(const ArArgs &a, int owner, int phase, int parity, int from) {
    return a.p.base[owner] + kFlagBytes + ((static_cast<int64_t>(phase) * 2 + parity) * a.world + from) * a.slot_bytes;
}

// Threads of this CTA wait (thread 0 spins, bounded) until rank `from`'s flag reaches `epoch`.
__device__ __forceinline__ bool wait_flag(const ArArgs &a, const unsigned *f, unsigned epoch) {
    const uint64_t start = now_ns();
    for (uint32_t i = 0;; ++i) {
        if (static_cast<int>(ld_acquire_sys(f) - epoch) >= 0) return true;
        if ((i & 15) == 15 && now_ns() - start > a.limit_ns) {
            atomicOr(a.status, 1);
            return false;
        }
        __nanosleep(32);
    }
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

// Raises this CTA's flag `phase` on every rank, then waits (bounded) for every rank's flag here.
__device__ __forceinline__ bool exchange_flags(const ArArgs &a, int phase, int par, unsigned epoch, int *ok) {
    __syncthreads();  // this CTA's stores of the phase are issued
    if (threadIdx.x < a.world) {
        // release at system scope after the CTA barrier: this CTA's stores (to peers too) are visible
        // to whoever acquires the flag
        st_release_sys(flag(a, threadIdx.x, phase, par, a.rank, blockIdx.x), epoch);
        if (!wait_flag(a, flag(a, a.rank, phase, par, threadIdx.x, blockIdx.x), epoch)) *ok = 0;
    }
    __syncthreads();
    return *ok != 0;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) allreduce_kernel(const ArArgs a) {
    __shared__ unsigned s_epoch;
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        s_epoch = ++a.epochs[blockIdx.x];
        s_ok = 1;
    }
    __syncthreads();
    const unsigned epoch = s_epoch;
    const int par = epoch & 1;
    uint8_t *y = static_cast<uint8_t *>(a.y);
    const int64_t bytes = a.elems * static_cast<int64_t>(sizeof(T));
    const uint8_t *in[kMaxRanks];

    if (!a.two_shot) {
        // One-shot: this rank's message into every rank's slot[me]; then sum the P slots here.
        for (int r = 0; r < a.world; ++r) copy_blocks(slot(a, r, 0, par, a.rank), y, bytes);
        if (!exchange_flags(a, 0, par, epoch, &s_ok)) return;
        for (int r = 0; r < a.world; ++r) in[r] = slot(a, a.rank, 0, par, r);
        sum_blocks<T>(a.world, y, in, bytes);
        return;
    }

    // Two-shot. Chunk c = bytes [c * chunk, (c + 1) * chunk) of the message; rank c owns it.
    const int64_t chunk = ((bytes + a.world - 1) / a.world + 15) / 16 * 16;
    auto chunk_bytes = [&](int c) { return std::max<int64_t>(0, std::min<int64_t>(chunk, bytes - c * chunk)); };
    // Reduce-scatter: chunk c of this rank's message into rank c's slot[me].
    for (int c = 0; c < a.world; ++c) copy_blocks(slot(a, c, 0, par, a.rank), y + c * chunk, chunk_bytes(c));
    if (!exchange_flags(a, 0, par, epoch, &s_ok)) return;
    // The sum of this rank's chunk, in rank order, into this rank's gather slot[me], then into every
    // other rank's gather slot[me].
    uint8_t *mine = slot(a, a.rank, 1, par, a.rank);
    for (int r = 0; r < a.world; ++r) in[r] = slot(a, a.rank, 0, par, r);
    sum_blocks<T>(a.world, mine, in, chunk_bytes(a.rank));
    __syncthreads();
    for (int r = 0; r < a.world; ++r)
        if (r != a.rank) copy_blocks(slot(a, r, 1, par, a.rank), mine, chunk_bytes(a.rank));
    if (!exchange_flags(a, 1, par, epoch, &s_ok)) return;
    // Gather: chunk c from gather slot[c] into y.
    for (int c = 0; c < a.world; ++c) copy_blocks(y + c * chunk, slot(a, a.rank, 1, par, c), chunk_bytes(c));
}

}  // namespace
}  // namespace hmb

using namespace hmb;

struct hmb_comm {
    int rank = 0, world = 1, device = 0;
    size_t max_bytes = 0;   // largest message
    size_t slot_bytes = 0;  // one receive slot
    uint8_t *mine = nullptr;
    unsigned *epochs = nullptr;
    Peers peers{};
    bool connected = false;
};

extern "C" {

size_t hmb_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int hmb_comm_create(int rank, int world, size_t max_bytes, hmb_comm **out, void *handle) {
    if (!out || !handle || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || max_bytes == 0) return HMB_ERR_ARG;
    hmb_comm *c = new hmb_comm();
    c->rank = rank;
    c->world = world;
    cudaGetDevice(&c->device);
    c->max_bytes = (max_bytes + 15) / 16 * 16;
    // A one-shot slot holds a whole message (<= kOneShotBytes), a two-shot slot one chunk of it.
    c->slot_bytes = std::max<size_t>(kOneShotBytes, ((c->max_bytes + world - 1) / world + 15) / 16 * 16);
    const size_t bytes = kFlagBytes + 2 * 2 * static_cast<size_t>(world) * c->slot_bytes;
    cudaError_t e = cudaMalloc(&c->mine, bytes);
    if (e == cudaSuccess) e = cudaMemset(c->mine, 0, kFlagBytes);
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
    a.p = c->peers;
    a.y = y;
    a.elems = elems;
    a.dtype = dtype;
    a.rank = c->rank;
    a.world = c->world;
    a.two_shot = bytes > kOneShotBytes;
    a.slot_bytes = static_cast<int64_t>(c->slot_bytes);
    a.epochs = c->epochs;
    a.status = status;
    a.limit_ns = spin_limit_ns ? spin_limit_ns : 1000000000ull;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == HMB_FP32)
        allreduce_kernel<float><<<kCtas, kThreads, 0, s>>>(a);
    else if (dtype == HMB_BF16)
        allreduce_kernel<__nv_bfloat16><<<kCtas, kThreads, 0, s>>>(a);
    else
        allreduce_kernel<__half><<<kCtas, kThreads, 0, s>>>(a);
    return launch_status();
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
