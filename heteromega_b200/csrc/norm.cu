// The layer boundary on one GPU: x += a + b, then RMSNorm of x (hmb_residual_norm). One CTA per
// row at a time, 16-byte vectors, the row held in registers between the sum of squares and the
// scaling, so x, a, b and w are read once and x and normed written once. HBM-bound.
#include <algorithm>

#include "norm_internal.h"
#include "rownorm.cuh"

namespace hmb {
namespace {

template <int V, int NIN>
__global__ void __launch_bounds__(kRowThreads, 2)
    residual_norm_kernel(uint16_t *__restrict__ x, int64_t ldx, const uint16_t *__restrict__ a, int64_t lda,
                         const uint16_t *__restrict__ b, int64_t ldb, const uint16_t *__restrict__ w, uint16_t *__restrict__ normed,
                         int64_t ldn, int64_t m, int h, float eps) {
    __shared__ float red[kRowThreads / 32];
    // The next kernel may start its prologue (weight prefetch); it waits for this grid before it
    // reads what this grid writes.
    pdl_launch_dependents();
    pdl_wait();  // a and b come from the previous kernel
    for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
        const uint16_t *in[2] = {a == nullptr ? nullptr : a + row * lda, b == nullptr ? nullptr : b + row * ldb};
        uint16_t *out = normed == nullptr ? nullptr : normed + row * ldn;
        boundary_row<V, NIN>(in, x + row * ldx, true, w, h, eps, &out, normed == nullptr ? 0 : 1, red);
    }
}

template <int V>
cudaError_t launch_v(int n_in, int grid, cudaStream_t stream, uint16_t *x, int64_t ldx, const uint16_t *a, int64_t lda, const uint16_t *b,
                     int64_t ldb, const uint16_t *w, uint16_t *normed, int64_t ldn, int64_t m, int h, float eps) {
    const dim3 g(grid), blk(kRowThreads);
    if (n_in == 0) return launch_pdl(residual_norm_kernel<V, 0>, g, blk, 0, stream, x, ldx, a, lda, b, ldb, w, normed, ldn, m, h, eps);
    if (n_in == 1) return launch_pdl(residual_norm_kernel<V, 1>, g, blk, 0, stream, x, ldx, a, lda, b, ldb, w, normed, ldn, m, h, eps);
    return launch_pdl(residual_norm_kernel<V, 2>, g, blk, 0, stream, x, ldx, a, lda, b, ldb, w, normed, ldn, m, h, eps);
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
    const int n_in = a == nullptr ? 0 : (b == nullptr ? 1 : 2);
    auto *xp = static_cast<uint16_t *>(x);
    auto *ap = static_cast<const uint16_t *>(a), *bp = static_cast<const uint16_t *>(b), *wp = static_cast<const uint16_t *>(weight);
    auto *np = static_cast<uint16_t *>(normed);
    const int hi = static_cast<int>(h);
    const int v = row_vectors(h);
    const cudaError_t e = v == 1   ? launch_v<1>(n_in, grid, stream, xp, ldx, ap, lda, bp, ldb, wp, np, ldn, m, hi, eps)
                          : v == 2 ? launch_v<2>(n_in, grid, stream, xp, ldx, ap, lda, bp, ldb, wp, np, ldn, m, hi, eps)
                          : v == 4 ? launch_v<4>(n_in, grid, stream, xp, ldx, ap, lda, bp, ldb, wp, np, ldn, m, hi, eps)
                                   : launch_v<8>(n_in, grid, stream, xp, ldx, ap, lda, bp, ldb, wp, np, ldn, m, hi, eps);
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
