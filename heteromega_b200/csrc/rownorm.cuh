// One row of the layer boundary (residual add + RMSNorm), processed by one CTA of kRowThreads
// threads. The single-GPU boundary (norm.cu) and the tensor-parallel one fused with the rank sum
// (allreduce.cu) share it.
//
// The arithmetic is the reference's residual_norm_kernel (kernels/gpu/src/residual_norm.cu:38-87),
// generalised from two addends to any number:
//   x_new = bf16(((x + in_0) + in_1) + ...)    fp32, left to right, one rounding
//   out   = bf16((x_new * rsqrt(sum(x_new^2) / h + eps)) * w)
// The mean of squares is taken over the rounded values. Without w, out = x_new.
#pragma once
#include "common.cuh"

namespace hmb {

constexpr int kRowThreads = 256;
constexpr int kRowMaxH = 8 * 8 * kRowThreads;  // 8 vectors of 8 values per thread: 16384

// Sum of v over the CTA. Every thread gets the same bits: the warp totals are added in warp order.
// red: kRowThreads / 32 floats of shared memory; all threads of the CTA must call.
__device__ __forceinline__ float cta_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < kRowThreads / 32; ++i) t += red[i];
    __syncthreads();
    return t;
}

__device__ __forceinline__ void unpack8(const uint4 &v, float *f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        f[2 * q] = bf16_to_f32(w[q] & 0xFFFFu);
        f[2 * q + 1] = bf16hi_to_f32(w[q]);
    }
}

__device__ __forceinline__ uint4 pack8(const float *f) {
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) w[q] = f32_to_bf16(f[2 * q]) | (f32_to_bf16(f[2 * q + 1]) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// 8 addend values as loaded: bf16 (one 16-byte word) or fp32 (two).
template <typename AT>
struct Addend8;
template <>
struct Addend8<uint16_t> {
    static constexpr int kWords = 1;
    uint4 w;
    __device__ __forceinline__ void load(const uint16_t *p) { w = *reinterpret_cast<const uint4 *>(p); }
    __device__ __forceinline__ void add_to(float *acc) const {
        float f[8];
        unpack8(w, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += f[e];
    }
};
template <>
struct Addend8<float> {
    static constexpr int kWords = 2;
    float4 a, b;
    __device__ __forceinline__ void load(const float *p) {
        a = *reinterpret_cast<const float4 *>(p);
        b = *reinterpret_cast<const float4 *>(p + 4);
    }
    __device__ __forceinline__ void add_to(float *acc) const {
        acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
};

// Vectors of 8 values per thread for rows of h values: V = 1, 2, 4 or 8 (h <= 2048 V).
__host__ __device__ constexpr int row_vectors(int64_t h) { return h <= 2048 ? 1 : h <= 4096 ? 2 : h <= 8192 ? 4 : 8; }

// in[0..NIN): addend rows (h values of AT: bf16 bits or fp32). x: the residual row, overwritten with
// x_new when NIN > 0 and write_x. out[0..n_out): rows that all receive the result. w: the norm weight
// row or null. h % 8 == 0, h <= V * 2048; every pointer 16-byte aligned. All threads of the CTA must
// call. The loads of x and of every addend are issued before the sums (no load waits for an add), so
// a row costs about one memory latency, not one per addend.
template <int V, int NIN, typename AT = uint16_t>
__device__ __forceinline__ void boundary_row(const AT *const *in, uint16_t *x, bool write_x, const uint16_t *w, int h, float eps,
                                             uint16_t *const *out, int n_out, float *red) {
    const int nv = h >> 3;
    // Vectors in groups of G: every load of a group (x and the addends) is in flight at once, and a
    // group's loads stay within the registers.
    constexpr int kCost = 1 + NIN * Addend8<AT>::kWords;
    constexpr int G = V * kCost <= 40 ? V : (40 / kCost >= 1 ? 40 / kCost : 1);
    uint4 xv[V];
    float ss = 0.0f;
#pragma unroll
    for (int i0 = 0; i0 < V; i0 += G) {
        Addend8<AT> pv[NIN > 0 ? NIN : 1][G];
#pragma unroll
        for (int j = 0; j < G && i0 + j < V; ++j) {
            const int v = (i0 + j) * kRowThreads + threadIdx.x;
            if (v < nv) {
                xv[i0 + j] = *reinterpret_cast<const uint4 *>(x + 8 * v);
#pragma unroll
                for (int r = 0; r < NIN; ++r) pv[r][j].load(in[r] + 8 * v);
            }
        }
#pragma unroll
        for (int j = 0; j < G && i0 + j < V; ++j) {
            const int v = (i0 + j) * kRowThreads + threadIdx.x;
            if (v < nv) {
                if constexpr (NIN > 0) {
                    float acc[8];
                    unpack8(xv[i0 + j], acc);
#pragma unroll
                    for (int r = 0; r < NIN; ++r) pv[r][j].add_to(acc);
                    xv[i0 + j] = pack8(acc);
                    if (write_x) *reinterpret_cast<uint4 *>(x + 8 * v) = xv[i0 + j];
                }
                float f[8];
                unpack8(xv[i0 + j], f);
#pragma unroll
                for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
            }
        }
    }
    float scale = 1.0f;
    if (w != nullptr) scale = rsqrtf(cta_sum(ss, red) / static_cast<float>(h) + eps);
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int v = i * kRowThreads + threadIdx.x;
        if (v < nv) {
            uint4 o = xv[i];
            if (w != nullptr) {
                float f[8], g[8];
                unpack8(o, f);
                unpack8(*reinterpret_cast<const uint4 *>(w + 8 * v), g);
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = f[e] * scale * g[e];
                o = pack8(f);
            }
            for (int d = 0; d < n_out; ++d) *reinterpret_cast<uint4 *>(out[d] + 8 * v) = o;
        }
    }
}

}  // namespace hmb
