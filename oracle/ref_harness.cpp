// TEST INFRASTRUCTURE ONLY: a C entry point around the reference's own CPU AVX
// GEMV, w4a16_gemv_cpu_fused_packed (src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp:28-292
// in glassescrab/HeteroMega), which oracle/Makefile compiles unchanged next to
// this file into oracle/_ref/. Used by the tests to pin the C oracle and by
// bench.py as the timed CPU baseline ("kind": "reference").
#include <ATen/ATen.h>
#include <ATen/Parallel.h>
#include <cstdint>

#include "cpu_avx_kernels/w4a16_gemv_avx_packed.hpp"

extern "C" {

// out[n] (bf16 bits) = x[k] (bf16 bits) @ packed [k, n], columns [start_col, end_col).
// threads > 0 sets ATen's intra-op thread count first (the kernel's own argument does
// not limit it). Returns 0, or -1 if ATen threw.
int hmref_gemv(uint16_t *out, const uint16_t *x, const uint8_t *packed, int64_t k, int64_t n, int threads, int64_t start_col,
               int64_t end_col) {
    try {
        if (threads > 0) at::set_num_threads(threads);
        auto o = at::from_blob(out, {1, n}, at::TensorOptions().dtype(at::kBFloat16));
        auto i = at::from_blob(const_cast<uint16_t *>(x), {1, k}, at::TensorOptions().dtype(at::kBFloat16));
        const int64_t bytes = (k / 128) * (n / 64) * 4352;
        auto p = at::from_blob(const_cast<uint8_t *>(packed), {bytes}, at::TensorOptions().dtype(at::kByte));
        w4a16_gemv_cpu_fused_packed(o, i, p, k, n, nullptr, 1, start_col, end_col);
        return 0;
    } catch (...) {
        return -1;
    }
}

int hmref_threads(void) { return at::get_num_threads(); }

#ifdef __AVX512F__
int hmref_avx512(void) { return 1; }
#else
int hmref_avx512(void) { return 0; }
#endif
}
