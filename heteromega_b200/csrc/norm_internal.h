// The single-GPU layer boundary, also used by the tensor-parallel boundary for a group of one.
#pragma once
#include "common.cuh"

namespace hmb {

int residual_norm_launch(void *x, int64_t ldx, const void *a, int64_t lda, const void *b, int64_t ldb, const void *weight, void *normed,
                         int64_t ldn, int64_t m, int64_t h, float eps, cudaStream_t stream);

}  // namespace hmb
