/*
 * CPU ORACLE -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of HeteroMega's packed W4A16 definition, used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker. The
 * product (heteromega_b200/, libhmb.so) never links, loads or calls this file.
 *
 * Parity is pinned: tests/test_oracle_golden.py checks every routine here
 * against fixtures generated from the reference's own packers, its NumPy
 * oracle and its CPU AVX kernel (tests/golden/make_golden.py), and against the
 * reference AVX kernel compiled unchanged into oracle/_ref/ (oracle/Makefile).
 *
 * Reference definitions restated here (paths inside glassescrab/HeteroMega):
 *   tile layout            kernels/gpu/src/pack_w4a16.cpp:30-61
 *   tile position          kernels/gpu/src/pack_w4a16.cpp:100-107
 *   GEMV arithmetic        src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp:83-289
 *                          (per 128-row tile and column: s * (sum q*x - z * sum x),
 *                          fp32, zero read as uint8, one bf16 rounding at the end)
 *   SiLU * up              kernels/gpu/src/silu_mul.cu:10-30 (fp32, one rounding)
 *   boundary sum           kernels/gpu/src/residual_add.cu:7-28
 *   channel slices         kernels/gpu/src/pack_w4a16.cpp:68-165
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define TILE_K 128
#define TILE_N 64
#define TILE_BYTES 4352

/* fp32 -> bf16 bits, round to nearest even; NaN stays NaN. */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) {
        return (uint16_t)((u >> 16) | ((u & 0x007FFFFFu) ? 0x40u : 0u));
    }
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Tile (column c, row r) of a tiles_k x tiles_n packed matrix. Tiles are ordered by
 * column modulo 8, then column, then row (pack_w4a16.cpp:30-34, 100-107). */
int64_t orc_tile_index(int64_t c, int64_t r, int64_t tiles_k, int64_t tiles_n) {
    int64_t before = c / 8;
    for (int64_t g = 0; g < c % 8; ++g) {
        before += (tiles_n - g + 7) / 8;
    }
    return before * tiles_k + r;
}

/* Byte of the 4096 weight bytes of a tile that holds (row, col); the low nibble holds the
 * even column of a pair. Byte ((a*8 + cc)*8 + b)*4 + j holds row a*8+b, columns cc*8+2j
 * and cc*8+2j+1 (pack_w4a16.cpp:38-49). */
static inline int64_t weight_byte(int row, int col) {
    return (((int64_t)(row >> 3) * 8 + (col >> 3)) * 8 + (row & 7)) * 4 + ((col & 7) >> 1);
}

/* Zero of column c sits at byte 4224 + (c/8)*16 + c%8 and again 8 bytes later. */
static inline int zero_byte(int col) { return 4224 + (col >> 3) * 16 + (col & 7); }

/* q [K,N] (0..15), s [K/128,N] bf16 bits, z [K/128,N] (0..15) -> packed bytes. Returns -1 on
 * a bad shape or value. */
int orc_pack(const uint8_t *q, const uint16_t *s, const uint8_t *z, int64_t K, int64_t N, uint8_t *out) {
    if (K <= 0 || N <= 0 || K % TILE_K || N % TILE_N) return -1;
    const int64_t tk = K / TILE_K, tn = N / TILE_N;
    for (int64_t i = 0; i < K * N; ++i) if (q[i] > 15) return -1;
    for (int64_t i = 0; i < tk * N; ++i) if (z[i] > 15) return -1;
    for (int64_t c = 0; c < tn; ++c) {
        for (int64_t r = 0; r < tk; ++r) {
            uint8_t *t = out + orc_tile_index(c, r, tk, tn) * TILE_BYTES;
            memset(t, 0, 4096);
            for (int row = 0; row < TILE_K; ++row) {
                const uint8_t *src = q + (r * TILE_K + row) * N + c * TILE_N;
                for (int col = 0; col < TILE_N; ++col) {
                    t[weight_byte(row, col)] |= (uint8_t)(src[col] << ((col & 1) * 4));
                }
            }
            for (int col = 0; col < TILE_N; ++col) {
                const uint16_t sv = s[r * N + c * TILE_N + col];
                t[4096 + 2 * col] = (uint8_t)(sv & 0xFF);
                t[4096 + 2 * col + 1] = (uint8_t)(sv >> 8);
                const uint8_t zv = z[r * N + c * TILE_N + col];
                t[zero_byte(col)] = zv;
                t[zero_byte(col) + 8] = zv;
            }
        }
    }
    return 0;
}

/* Decode the leading [k, n] block of a packed [packed_k, packed_n] matrix back to q, s, z.
 * Any of q, s, z may be NULL. */
void orc_unpack(const uint8_t *packed, int64_t packed_k, int64_t packed_n, int64_t k, int64_t n, uint8_t *q, uint16_t *s,
                uint8_t *z) {
    const int64_t tk = packed_k / TILE_K, tn = packed_n / TILE_N;
    for (int64_t c = 0; c < n / TILE_N; ++c) {
        for (int64_t r = 0; r < k / TILE_K; ++r) {
            const uint8_t *t = packed + orc_tile_index(c, r, tk, tn) * TILE_BYTES;
            for (int col = 0; col < TILE_N; ++col) {
                const int64_t gc = c * TILE_N + col;
                if (q) {
                    for (int row = 0; row < TILE_K; ++row) {
                        q[(r * TILE_K + row) * n + gc] = (uint8_t)((t[weight_byte(row, col)] >> ((col & 1) * 4)) & 15);
                    }
                }
                if (s) s[r * n + gc] = (uint16_t)(t[4096 + 2 * col] | (t[4096 + 2 * col + 1] << 8));
                if (z) z[r * n + gc] = t[zero_byte(col)];
            }
        }
    }
}

/* w[k][n] = (q - z) * s in fp32 for the leading [k, n] block. Exact: q - z is a small integer
 * and s has 8 significant bits. */
void orc_dequant(const uint8_t *packed, int64_t packed_k, int64_t packed_n, int64_t k, int64_t n, float *w) {
    const int64_t tk = packed_k / TILE_K, tn = packed_n / TILE_N;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < n / TILE_N; ++c) {
        for (int64_t r = 0; r < k / TILE_K; ++r) {
            const uint8_t *t = packed + orc_tile_index(c, r, tk, tn) * TILE_BYTES;
            for (int col = 0; col < TILE_N; ++col) {
                const float sc = orc_bf16_to_f32((uint16_t)(t[4096 + 2 * col] | (t[4096 + 2 * col + 1] << 8)));
                const float zf = (float)t[zero_byte(col)];
                for (int row = 0; row < TILE_K; ++row) {
                    const float qv = (float)((t[weight_byte(row, col)] >> ((col & 1) * 4)) & 15);
                    w[(r * TILE_K + row) * n + c * TILE_N + col] = (qv - zf) * sc;
                }
            }
        }
    }
}

/* y[m][j] for columns j of [n0, n0 + n) of a packed [packed_k, packed_n] matrix and its first k rows:
 * per tile, s * (sum_r q*x_r - z * sum_r x_r) in fp32, summed over tiles in row order
 * (w4a16_gemv_avx_packed.cpp:90-107, 240-253). x is bf16 [m][ldx]. y32 (fp32, may be NULL) gets the
 * unrounded sums, y16 (bf16 bits, may be NULL) the rounded ones; both [m][ldy]. */
void orc_gemv(const uint8_t *packed, int64_t packed_k, int64_t packed_n, int64_t k, int64_t n0, int64_t n, const uint16_t *x,
              int64_t ldx, int64_t m, float *y32, uint16_t *y16, int64_t ldy) {
    const int64_t tk = packed_k / TILE_K, tn = packed_n / TILE_N;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t row = 0; row < m; ++row) {
        for (int64_t c = 0; c < n / TILE_N; ++c) {
            const uint16_t *xr = x + row * ldx;
            float acc[TILE_N];
            for (int col = 0; col < TILE_N; ++col) acc[col] = 0.0f;
            for (int64_t r = 0; r < k / TILE_K; ++r) {
                const uint8_t *t = packed + orc_tile_index(n0 / TILE_N + c, r, tk, tn) * TILE_BYTES;
                float xs = 0.0f;
                for (int i = 0; i < TILE_K; ++i) xs += orc_bf16_to_f32(xr[r * TILE_K + i]);
                for (int col = 0; col < TILE_N; ++col) {
                    float dot = 0.0f;
                    for (int i = 0; i < TILE_K; ++i) {
                        const float qv = (float)((t[weight_byte(i, col)] >> ((col & 1) * 4)) & 15);
                        dot += qv * orc_bf16_to_f32(xr[r * TILE_K + i]);
                    }
                    const float sc = orc_bf16_to_f32((uint16_t)(t[4096 + 2 * col] | (t[4096 + 2 * col + 1] << 8)));
                    const float zf = (float)t[zero_byte(col)];
                    acc[col] += (dot - zf * xs) * sc;
                }
            }
            for (int col = 0; col < TILE_N; ++col) {
                if (y32) y32[row * ldy + c * TILE_N + col] = acc[col];
                if (y16) y16[row * ldy + c * TILE_N + col] = orc_f32_to_bf16(acc[col]);
            }
        }
    }
}

/* act = bf16(SiLU(g) * u) with fp32 math, g and u bf16 (silu_mul.cu:26). layout 0: gate is column c,
 * up column n + c of gate_up [m][2n]; layout 1 (interleaved): per 64 channels, 64 gate then 64 up columns. */
void orc_silu_mul(const uint16_t *gate_up, int64_t ld_in, uint16_t *act, int64_t ld_out, int64_t m, int64_t n, int layout) {
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < m; ++row) {
        for (int64_t c = 0; c < n; ++c) {
            const int64_t gc = layout ? (c / 64) * 128 + c % 64 : c;
            const int64_t uc = layout ? gc + 64 : n + c;
            const float g = orc_bf16_to_f32(gate_up[row * ld_in + gc]);
            const float u = orc_bf16_to_f32(gate_up[row * ld_in + uc]);
            act[row * ld_out + c] = orc_f32_to_bf16(g / (1.0f + expf(-g)) * u);
        }
    }
}

/* x += y_g + y_n: partials first, fp32 math, one bf16 rounding (residual_add.cu:7-28).
 * y_g and y_n are bf16 (f32 flag 0) or fp32 (flag 1). */
void orc_residual_add2(uint16_t *x, const void *yg, int g32, const void *yn, int n32, int64_t count) {
    for (int64_t i = 0; i < count; ++i) {
        const float a = g32 ? ((const float *)yg)[i] : orc_bf16_to_f32(((const uint16_t *)yg)[i]);
        const float b = n32 ? ((const float *)yn)[i] : orc_bf16_to_f32(((const uint16_t *)yn)[i]);
        x[i] = orc_f32_to_bf16(orc_bf16_to_f32(x[i]) + (a + b));
    }
}

/* The layer boundary of residual_norm_kernel (kernels/gpu/src/residual_norm.cu:38-87) for any number
 * of addends, as its test states the expected values (kernels/gpu/tests/test_gpu_ffn.cpp:266-268):
 *   x      = bf16(((x + a_0) + a_1) + ...)              fp32, left to right, one rounding
 *   normed = bf16((x * 1/sqrt(mean(x^2) + eps)) * w)    the mean over the rounded x
 * addends: n_add bf16 arrays [m][h], one after the other; n_add 0 leaves x as it is. w null: normed = x.
 * normed may be null. The sum of squares is taken in double here; a kernel's order differs, so its
 * normed may differ from this by one bf16 unit in the last place. */
void orc_residual_norm(uint16_t *x, const uint16_t *addends, int n_add, const uint16_t *w, uint16_t *normed, int64_t m, int64_t h,
                       float eps) {
    for (int64_t row = 0; row < m; ++row) {
        uint16_t *xr = x + row * h;
        double ss = 0.0;
        for (int64_t c = 0; c < h; ++c) {
            if (n_add > 0) {
                float acc = orc_bf16_to_f32(xr[c]);
                for (int r = 0; r < n_add; ++r) acc += orc_bf16_to_f32(addends[((int64_t)r * m + row) * h + c]);
                xr[c] = orc_f32_to_bf16(acc);
            }
            const double v = orc_bf16_to_f32(xr[c]);
            ss += v * v;
        }
        if (!normed) continue;
        const float scale = (float)(1.0 / sqrt((double)(float)(ss / (double)h) + (double)eps));
        for (int64_t c = 0; c < h; ++c) {
            const float v = orc_bf16_to_f32(xr[c]);
            normed[row * h + c] = w ? orc_f32_to_bf16(v * scale * orc_bf16_to_f32(w[c])) : xr[c];
        }
    }
}

/* One FFN channel slice as the model runs it on the reference CPU path
 * (unified_llm_w4a16.cpp:2873-2886 with the AVX GEMV): gate and up GEMVs with bf16 outputs,
 * fp32 SiLU*up rounded once, down GEMV. gate_up is packed [h, 2*stored] in `layout` order and
 * down packed [stored, h]; the first n channels are used. scratch: m*(3n) bf16.
 * y16 (bf16) and/or y32 (fp32 down sums before rounding) are [m][h]. */
void orc_ffn(const uint8_t *gate_up, const uint8_t *down, int64_t h, int64_t n, int64_t stored, int layout, const uint16_t *x,
             int64_t m, uint16_t *scratch, uint16_t *y16, float *y32) {
    uint16_t *gu = scratch;          /* [m][2n] */
    uint16_t *act = scratch + m * 2 * n; /* [m][n] */
    if (layout) {
        orc_gemv(gate_up, h, 2 * stored, h, 0, 2 * n, x, h, m, NULL, gu, 2 * n);
    } else {
        orc_gemv(gate_up, h, 2 * stored, h, 0, n, x, h, m, NULL, gu, 2 * n);
        orc_gemv(gate_up, h, 2 * stored, h, stored, n, x, h, m, NULL, gu + n, 2 * n);
    }
    orc_silu_mul(gu, 2 * n, act, n, m, n, layout);
    orc_gemv(down, stored, h, n, 0, h, act, n, m, y32, y16, h);
}
