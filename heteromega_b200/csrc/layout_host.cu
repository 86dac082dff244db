// Host side of the packed W4A16 layout: status strings, the packer, and the tile maps of
// channel slices. The layout itself is the reference's (kernels/gpu/src/pack_w4a16.cpp:30-61),
// restated here; the code is this project's own.
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace hmb {

static thread_local int g_last_cuda_error = 0;

void set_cuda_error(cudaError_t e) { g_last_cuda_error = static_cast<int>(e); }

int sm_count() {
    static std::mutex mu;
    static std::vector<int> counts;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(counts.size()) <= dev) counts.resize(dev + 1, 0);
    if (counts[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        counts[dev] = n;
    }
    return counts[dev];
}

}  // namespace hmb

using namespace hmb;

extern "C" {

const char *hmb_status_string(int status) {
    switch (status) {
    case HMB_OK: return "ok";
    case HMB_ERR_ARG: return "invalid argument (null pointer, size or enum)";
    case HMB_ERR_ALIGN: return "misaligned pointer or stride";
    case HMB_ERR_VALUE: return "weight or zero point outside 0..15";
    case HMB_ERR_WORKSPACE: return "workspace missing or too small";
    case HMB_ERR_UNSUPPORTED: return "shape not supported by this build";
    case HMB_ERR_CUDA: return "CUDA error (see hmb_last_cuda_error)";
    case HMB_ERR_TIMEOUT: return "bounded device wait gave up";
    default: return "unknown status";
    }
}

int hmb_version(void) { return 100; }

int hmb_last_cuda_error(void) { return g_last_cuda_error; }

int64_t hmb_packed_bytes(int64_t k, int64_t n) {
    if (k <= 0 || n <= 0 || k % kTileK || n % kTileN) return -1;
    return (k / kTileK) * (n / kTileN) * kTileBytes;
}

int64_t hmb_packed_tile_index(int64_t c, int64_t r, int64_t tiles_k, int64_t tiles_n) {
    if (c < 0 || r < 0 || c >= tiles_n || r >= tiles_k) return -1;
    return tile_index(c, r, tiles_k, tiles_n);
}

int hmb_pack_w4a16(const uint8_t *q, const uint16_t *scales, const uint8_t *zeros, int64_t k, int64_t n, uint8_t *out) {
    if (!q || !scales || !zeros || !out || hmb_packed_bytes(k, n) < 0) return HMB_ERR_ARG;
    for (int64_t i = 0; i < k * n; ++i) {
        if (q[i] > 15) return HMB_ERR_VALUE;
    }
    for (int64_t i = 0; i < (k / kTileK) * n; ++i) {
        if (zeros[i] > 15) return HMB_ERR_VALUE;
    }
    const int64_t tk = k / kTileK, tn = n / kTileN;
    for (int64_t c = 0; c < tn; ++c) {
        for (int64_t r = 0; r < tk; ++r) {
            uint8_t *t = out + tile_index(c, r, tk, tn) * kTileBytes;
            // 16 row groups x 8 column groups of 32-byte blocks; in a block, 4 bytes per row hold the
            // group's 8 columns, the even column of each pair in the low nibble.
            for (int a = 0; a < 16; ++a) {
                for (int cc = 0; cc < 8; ++cc) {
                    for (int b = 0; b < 8; ++b) {
                        const uint8_t *src = q + (r * kTileK + a * 8 + b) * n + c * kTileN + cc * 8;
                        uint8_t *dst = t + ((a * 8 + cc) * 8 + b) * 4;
                        for (int j = 0; j < 4; ++j) dst[j] = static_cast<uint8_t>(src[2 * j] | (src[2 * j + 1] << 4));
                    }
                }
            }
            std::memcpy(t + 4096, scales + r * n + c * kTileN, 64 * sizeof(uint16_t));
            const uint8_t *zr = zeros + r * n + c * kTileN;
            for (int g = 0; g < 8; ++g) {
                std::memcpy(t + 4224 + g * 16, zr + g * 8, 8);
                std::memcpy(t + 4224 + g * 16 + 8, zr + g * 8, 8);
            }
        }
    }
    return HMB_OK;
}

int hmb_slice_tile_counts(int64_t hidden, int64_t inter, int64_t begin, int64_t end, int64_t *gate_up_tiles,
                          int64_t *down_tiles) {
    if (hidden <= 0 || inter <= 0 || hidden % kTileK || inter % kTileK || begin < 0 || end <= begin || end > inter ||
        begin % kTileK || end % kTileK)
        return HMB_ERR_ARG;
    const int64_t n = end - begin;
    if (gate_up_tiles) *gate_up_tiles = (hidden / kTileK) * (2 * n / kTileN);
    if (down_tiles) *down_tiles = (n / kTileK) * (hidden / kTileN);
    return HMB_OK;
}

int hmb_slice_tile_map(int64_t hidden, int64_t inter, int64_t begin, int64_t end, int layout, int64_t *gate_up_src,
                       int64_t *down_src) {
    int64_t gu_tiles = 0, dn_tiles = 0;
    const int rc = hmb_slice_tile_counts(hidden, inter, begin, end, &gu_tiles, &dn_tiles);
    if (rc != HMB_OK) return rc;
    if (layout != HMB_GATE_UP_BLOCKED && layout != HMB_GATE_UP_INTERLEAVED) return HMB_ERR_ARG;
    const int64_t n = end - begin;
    const int64_t tk = hidden / kTileK, tn = inter / kTileN, matrix_tiles = tk * tn;
    const int64_t out_tn = 2 * n / kTileN, half = n / kTileN;
    if (gate_up_src) {
        // Output tile column oc of gate_up [hidden, 2n] comes from gate or up tile column
        // begin/64 + j: blocked puts the n/64 gate columns first, interleaved alternates them.
        for (int64_t oc = 0; oc < out_tn; ++oc) {
            const bool up = layout == HMB_GATE_UP_BLOCKED ? oc >= half : (oc & 1) != 0;
            const int64_t j = layout == HMB_GATE_UP_BLOCKED ? oc % half : oc / 2;
            for (int64_t r = 0; r < tk; ++r) {
                gate_up_src[tile_index(oc, r, tk, out_tn)] = (up ? matrix_tiles : 0) + tile_index(begin / kTileN + j, r, tk, tn);
            }
        }
    }
    if (down_src) {
        // down [n, hidden]: tile rows begin/128 .. end/128 of each tile column of the full down.
        const int64_t dtk = inter / kTileK, dtn = hidden / kTileN, otk = n / kTileK;
        for (int64_t c = 0; c < dtn; ++c) {
            for (int64_t r = 0; r < otk; ++r) {
                down_src[tile_index(c, r, otk, dtn)] = tile_index(c, begin / kTileK + r, dtk, dtn);
            }
        }
    }
    return HMB_OK;
}

}  // extern "C"
