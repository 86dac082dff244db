// Small bandwidth-bound kernels around the GEMV/GEMM: exact dequantization, SiLU*up, the boundary
// sum of partial outputs, the device packer and the tile gather of channel slices. Grids are sized
// as a multiple of the SM count and loop (grid-stride) over 16-byte vectors.
#include <algorithm>

#include "common.cuh"

namespace hmb {
namespace {

constexpr int kThreads = 256;

int grid_for(int64_t work) {
    const int64_t blocks = (work + kThreads - 1) / kThreads;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, 8LL * sm_count())));
}

// One thread per weight byte of the leading [k, n] block: 2 outputs.
__global__ void __launch_bounds__(kThreads)
    dequant_kernel(const uint8_t *__restrict__ packed, int tiles_k_total, int tiles_n_total, int k_tiles, int n_tiles,
                   float *__restrict__ out, int64_t ldo) {
    const int64_t total = static_cast<int64_t>(k_tiles) * n_tiles * 4096;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t tile = i >> 12;
        const int o = static_cast<int>(i & 4095);
        const int c = static_cast<int>(tile / k_tiles), r = static_cast<int>(tile % k_tiles);
        const uint8_t *t = packed + tile_index(c, r, tiles_k_total, tiles_n_total) * kTileBytes;
        // Byte o = ((a*8 + cc)*8 + b)*4 + j: row a*8 + b, columns cc*8 + 2j and + 1.
        const int j = o & 3, b = (o >> 2) & 7, cc = (o >> 5) & 7, a = o >> 8;
        const int row = a * 8 + b, col = cc * 8 + 2 * j;
        const uint8_t v = t[o];
        const float s0 = bf16_to_f32(t[4096 + 2 * col] | (t[4096 + 2 * col + 1] << 8));
        const float s1 = bf16_to_f32(t[4096 + 2 * col + 2] | (t[4096 + 2 * col + 3] << 8));
        const float z0 = t[4224 + (col >> 3) * 16 + (col & 7)];
        const float z1 = t[4224 + (col >> 3) * 16 + (col & 7) + 1];
        float *dst = out + (static_cast<int64_t>(r) * kTileK + row) * ldo + static_cast<int64_t>(c) * kTileN + col;
        dst[0] = (static_cast<float>(v & 15) - z0) * s0;
        dst[1] = (static_cast<float>(v >> 4) - z1) * s1;
    }
}

// 8 channels of one row per work item. Interleaved: gate of channel c is column (c/64)*128 + c%64,
// up is 64 columns later. Blocked: gate is column c, up column n + c.
template <bool F16>
__global__ void __launch_bounds__(kThreads)
    silu_mul_kernel(const uint16_t *__restrict__ gu, int64_t ld_in, uint16_t *__restrict__ act, int64_t ld_out, int64_t rows,
                    int64_t n, int interleaved) {
    const int64_t per_row = n / 8, total = rows * per_row;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / per_row, c = (i - r * per_row) * 8;
        const int64_t gc = interleaved ? (c / 64) * 128 + c % 64 : c;
        const int64_t uc = interleaved ? gc + 64 : n + c;
        const uint4 gv = *reinterpret_cast<const uint4 *>(gu + r * ld_in + gc);
        const uint4 uv = *reinterpret_cast<const uint4 *>(gu + r * ld_in + uc);
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
        uint32_t ow[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t o = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float g = from16<F16>((gw[q] >> (16 * h)) & 0xFFFFu);
                const float u = from16<F16>((uw[q] >> (16 * h)) & 0xFFFFu);
                o |= to16<F16>(g / (1.0f + __expf(-g)) * u) << (16 * h);
            }
            ow[q] = o;
        }
        *reinterpret_cast<uint4 *>(act + r * ld_out + c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
}

template <typename T>
__device__ __forceinline__ float load_val(const T *p, int64_t i);
template <>
__device__ __forceinline__ float load_val<uint16_t>(const uint16_t *p, int64_t i) {
    return bf16_to_f32(p[i]);
}
template <>
__device__ __forceinline__ float load_val<float>(const float *p, int64_t i) {
    return p[i];
}

// x += y_g + y_n, partials added first, one rounding. 8 columns per work item.
template <typename G, typename N>
__global__ void __launch_bounds__(kThreads)
    residual_add2_kernel(uint16_t *__restrict__ x, int64_t ldx, const G *__restrict__ yg, int64_t ldg, const N *__restrict__ yn,
                         int64_t ldn, int64_t rows, int64_t cols) {
    const int64_t per_row = cols / 8, total = rows * per_row;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / per_row, c = (i - r * per_row) * 8;
        uint4 xv = *reinterpret_cast<const uint4 *>(x + r * ldx + c);
        uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t o = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t col = c + 2 * q + h;
                const float sum = load_val<G>(yg, r * ldg + col) + load_val<N>(yn, r * ldn + col);
                o |= f32_to_bf16(bf16_to_f32((xw[q] >> (16 * h)) & 0xFFFFu) + sum) << (16 * h);
            }
            xw[q] = o;
        }
        *reinterpret_cast<uint4 *>(x + r * ldx + c) = make_uint4(xw[0], xw[1], xw[2], xw[3]);
    }
}

// One CTA per tile (column c, row r): 256 threads write 16 weight bytes each, then scales and zeros.
__global__ void __launch_bounds__(kThreads)
    pack_kernel(const uint8_t *__restrict__ q, const uint16_t *__restrict__ s, const uint8_t *__restrict__ z, int64_t n,
                int tiles_k, int tiles_n, uint8_t *__restrict__ out, int *bad) {
    const int c = blockIdx.x, r = blockIdx.y;
    uint8_t *t = out + tile_index(c, r, tiles_k, tiles_n) * kTileBytes;
    int flag = 0;
    for (int o = threadIdx.x; o < 4096; o += kThreads) {
        const int j = o & 3, b = (o >> 2) & 7, cc = (o >> 5) & 7, a = o >> 8;
        const uint8_t *src = q + (static_cast<int64_t>(r) * kTileK + a * 8 + b) * n + static_cast<int64_t>(c) * kTileN + cc * 8 + 2 * j;
        flag |= (src[0] | src[1]) > 15;
        t[o] = static_cast<uint8_t>((src[0] & 15) | ((src[1] & 15) << 4));
    }
    if (threadIdx.x < 64) {
        const int64_t i = static_cast<int64_t>(r) * n + static_cast<int64_t>(c) * kTileN + threadIdx.x;
        const uint16_t sv = s[i];
        t[4096 + 2 * threadIdx.x] = static_cast<uint8_t>(sv & 0xFF);
        t[4096 + 2 * threadIdx.x + 1] = static_cast<uint8_t>(sv >> 8);
        const uint8_t zv = z[i];
        flag |= zv > 15;
        const int pos = 4224 + (threadIdx.x >> 3) * 16 + (threadIdx.x & 7);
        t[pos] = zv & 15;
        t[pos + 8] = zv & 15;
    }
    if (flag && bad) atomicOr(bad, 1);
}

// dst tile i <- src tile idx[i]; 16-byte copies, one CTA per tile.
__global__ void __launch_bounds__(kThreads)
    gather_kernel(const uint8_t *__restrict__ src0, int64_t src0_tiles, const uint8_t *__restrict__ src1,
                  const int64_t *__restrict__ idx, int64_t count, uint8_t *__restrict__ dst) {
    for (int64_t i = blockIdx.x; i < count; i += gridDim.x) {
        const int64_t s = idx[i];
        const uint8_t *from = s < src0_tiles ? src0 + s * kTileBytes : src1 + (s - src0_tiles) * kTileBytes;
        const uint4 *f = reinterpret_cast<const uint4 *>(from);
        uint4 *d = reinterpret_cast<uint4 *>(dst + i * kTileBytes);
        for (int v = threadIdx.x; v < kTileBytes / 16; v += kThreads) d[v] = f[v];
    }
}

}  // namespace
}  // namespace hmb

using namespace hmb;

extern "C" {

int hmb_w4a16_dequant(const uint8_t *packed, int64_t packed_k, int64_t packed_n, int64_t k, int64_t n, float *out, int64_t ldo,
                      hmb_stream_t stream) {
    if (!packed || !out || k <= 0 || n <= 0 || k % kTileK || n % kTileN || packed_k % kTileK || packed_n % kTileN ||
        k > packed_k || n > packed_n || ldo < n)
        return HMB_ERR_ARG;
    if (!aligned(out, 8) || ldo % 2) return HMB_ERR_ALIGN;
    const int kt = static_cast<int>(k / kTileK), nt = static_cast<int>(n / kTileN);
    dequant_kernel<<<grid_for(static_cast<int64_t>(kt) * nt * 4096), kThreads, 0, stream>>>(
        packed, static_cast<int>(packed_k / kTileK), static_cast<int>(packed_n / kTileN), kt, nt, out, ldo);
    return launch_status();
}

int hmb_silu_mul(const void *gate_up, int64_t ld_in, void *act, int64_t ld_out, int64_t m, int64_t n, int layout,
                 hmb_stream_t stream) {
    if (!gate_up || !act || m < 0 || n <= 0) return HMB_ERR_ARG;
    if (layout != HMB_GATE_UP_BLOCKED && layout != HMB_GATE_UP_INTERLEAVED) return HMB_ERR_ARG;
    if (n % (layout == HMB_GATE_UP_INTERLEAVED ? 64 : 8) || ld_in < 2 * n || ld_out < n) return HMB_ERR_ARG;
    if (!aligned(gate_up, 16) || !aligned(act, 16) || ld_in % 8 || ld_out % 8) return HMB_ERR_ALIGN;
    if (m == 0) return HMB_OK;
    silu_mul_kernel<false><<<grid_for(m * (n / 8)), kThreads, 0, stream>>>(
        static_cast<const uint16_t *>(gate_up), ld_in, static_cast<uint16_t *>(act), ld_out, m, n, layout);
    return launch_status();
}

int hmb_residual_add2(void *x, int64_t ldx, const void *y_g, int64_t ldg, int g_dtype, const void *y_n, int64_t ldn,
                      int n_dtype, int64_t m, int64_t cols, hmb_stream_t stream) {
    if (!x || !y_g || !y_n || m < 0 || cols <= 0 || cols % 8) return HMB_ERR_ARG;
    if ((g_dtype != HMB_BF16 && g_dtype != HMB_FP32) || (n_dtype != HMB_BF16 && n_dtype != HMB_FP32)) return HMB_ERR_ARG;
    if (ldx < cols || ldg < cols || ldn < cols) return HMB_ERR_ARG;
    if (!aligned(x, 16) || !aligned(y_g, 16) || !aligned(y_n, 16) || ldx % 8 || ldg % 8 || ldn % 8) return HMB_ERR_ALIGN;
    if (m == 0) return HMB_OK;
    auto *xp = static_cast<uint16_t *>(x);
    const int grid = grid_for(m * (cols / 8));
    if (g_dtype == HMB_BF16 && n_dtype == HMB_BF16) {
        residual_add2_kernel<uint16_t, uint16_t><<<grid, kThreads, 0, stream>>>(
            xp, ldx, static_cast<const uint16_t *>(y_g), ldg, static_cast<const uint16_t *>(y_n), ldn, m, cols);
    } else if (g_dtype == HMB_BF16) {
        residual_add2_kernel<uint16_t, float><<<grid, kThreads, 0, stream>>>(
            xp, ldx, static_cast<const uint16_t *>(y_g), ldg, static_cast<const float *>(y_n), ldn, m, cols);
    } else if (n_dtype == HMB_BF16) {
        residual_add2_kernel<float, uint16_t><<<grid, kThreads, 0, stream>>>(
            xp, ldx, static_cast<const float *>(y_g), ldg, static_cast<const uint16_t *>(y_n), ldn, m, cols);
    } else {
        residual_add2_kernel<float, float><<<grid, kThreads, 0, stream>>>(
            xp, ldx, static_cast<const float *>(y_g), ldg, static_cast<const float *>(y_n), ldn, m, cols);
    }
    return launch_status();
}

int hmb_pack_w4a16_device(const uint8_t *q, const uint16_t *scales, const uint8_t *zeros, int64_t k, int64_t n, uint8_t *out,
                          int *bad_flag, hmb_stream_t stream) {
    if (!q || !scales || !zeros || !out || hmb_packed_bytes(k, n) < 0) return HMB_ERR_ARG;
    if (k / kTileK > 65535) return HMB_ERR_UNSUPPORTED;
    const int tk = static_cast<int>(k / kTileK), tn = static_cast<int>(n / kTileN);
    pack_kernel<<<dim3(tn, tk), kThreads, 0, stream>>>(q, scales, zeros, n, tk, tn, out, bad_flag);
    return launch_status();
}

int hmb_gather_tiles(const uint8_t *src0, int64_t src0_tiles, const uint8_t *src1, const int64_t *idx, int64_t count, uint8_t *dst,
                     hmb_stream_t stream) {
    if (!src0 || !idx || !dst || count < 0 || src0_tiles < 0) return HMB_ERR_ARG;
    if (!aligned(src0, 16) || !aligned(dst, 16) || (src1 && !aligned(src1, 16))) return HMB_ERR_ALIGN;
    if (count == 0) return HMB_OK;
    const int grid = static_cast<int>(std::min<int64_t>(count, 16LL * sm_count()));
    gather_kernel<<<grid, kThreads, 0, stream>>>(src0, src0_tiles, src1 ? src1 : src0, idx, count, dst);
    return launch_status();
}

}  // extern "C"
