// The layer boundary on one GPU: x += a + b, then RMSNorm of x (hmb_residual_norm). One CTA per
// row at a time, 16-byte vectors, the row held in registers between the sum of squares and the
// scaling, so x, a, b and w are read once and x and normed written once. HBM-bound.
#include <algorithm>

#include "norm_internal.h"
#include "rownorm.cuh"

namespace hmb {
namespace {

__global__ void __launch_bounds__(kRowThreads, 2)
    residual_norm_kernel(uint16_t *__restrict__ x, int64_t ldx, const uint16_t *__restrict__ a, int64_t lda,
                         const uint16_t *__restrict__ b, int64_t ldb, const uint16_t *__restrict__ w, uint16_t *__restrict__ normed,
                         int64_t ldn, int64_t m, int h, float eps) {
    __shared__ float red[kRowThreads / 32];
    // The next kernel may start its prologue (weight prefetch); it waits for this grid before it
    // reads what this grid writes.
    pdl_launch_dependents();
    pdl_wait();  // a and b come from the previous kernel
    const int n_in = a == nullptr ? 0 : (b == nullptr ? 1 : 2);
    for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
        const uint16_t *in[2] = {a == nullptr ? nullptr : a + row * lda, b == nullptr ? nullptr : b + row * ldb};
        uint16_t *out = normed == nullptr ? nullptr : normed + row * ldn;
        boundary_row(in, n_in, x + row * ldx, true, w, h, eps, &out, normed == nullptr ? 0 : 1, red);
    }
}

}  // namespace

int residual_norm_launch(void *x, int64_t ldx, const void *a, int64_t lda, const void *b, int64_t ldb, const void *weight, void *normed,
                         int64_t ldn, int64_t m, int64_t h, float eps, cudaStream_t stream) {
    if (!x || m <= 0 || h <= 0 || h % 8 || h > kRowMaxH || (b && !a)) return HMB_ERR_ARG;
    if (ldx < h || (a && lda < h) || (b && ldb < h) || (normed && ldn < h)) return HMB_ERR_ARG;
    if (!(eps >= 0.0f)) return HMB_ERR_ARG;
    if (!aligned(x, 16) || (a && !aligned(a, 16)) || (b && !aligned(b, 16)) || (weight && !aligned(weight, 16)) ||
        (normed && !aligned(normed, 16)) || ldx % 8 || (a && lda % 8) || (b && ldb % 8) || (normed && ldn % 8))
        return HMB_ERR_ALIGN;
    if (!a && !normed) return HMB_OK;  // nothing changes and nothing is written
    // Two CTAs per SM keep enough loads in flight; with every CTA resident at once, all of them reach
    // the dependents trigger early.
    const int grid = static_cast<int>(std::min<int64_t>(m, 2LL * sm_count()));
    const cudaError_t e = launch_pdl(residual_norm_kernel, dim3(grid), dim3(kRowThreads), 0, stream, static_cast<uint16_t *>(x), ldx,
                                     static_cast<const uint16_t *>(a), lda, static_cast<const uint16_t *>(b), ldb,
                                     static_cast<const uint16_t *>(weight), static_cast<uint16_t *>(normed), ldn, m, static_cast<int>(h), eps);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return HMB_ERR_CUDA;
    }
    return HMB_OK;
}

}  // namespace hmb

extern "C" int hmb_residual_norm(void *x, int64_t ldx, const void *a, int64_t lda, const void *b, int64_t ldb, const void *weight,
                                 void *normed, int64_t ldn, int64_t m, int64_t h, float eps, hmb_stream_t stream) {
    return hmb::residual_norm_launch(x, ldx, a, lda, b, ldb, weight, normed, ldn, m, h, eps, static_cast<cudaStream_t>(stream));
}
