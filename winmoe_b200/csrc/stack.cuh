// Layer-stack glue (stack.cu).
#pragma once
#include "gdn_common.cuh"

namespace gdn {

// x <- x + add (add may be NULL), y <- rmsnorm(x) * w (w may be NULL: ones), per row of `hidden`;
// row t of y is stored at y.ptr[b] + y.col0 + t * y.ld for every destination b < y.n.
int launch_add_rmsnorm(float* x, const float* add, const float* w, const RowDest& y, int y_dtype, int64_t T,
                       int64_t hidden, cudaStream_t s);

}  // namespace gdn
