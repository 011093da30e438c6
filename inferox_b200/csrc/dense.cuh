// Dense (f32) matmul weights: the path for GGUF F32 / F16 / Q8_K matrices.
#pragma once
#include "gemv.cuh"
#include "repack.h"

namespace ifx {

// Tensor types that load as dense f32 matrices.
bool dense_type(int type);
// Layout of a dense f32 [rows, cols] matrix (row-major); src_type is the
// GGUF type it was dequantised from.
void make_dense_layout(int64_t rows, int64_t cols, int src_type, QLayout *L);

// Batch-1: y_s += W_s f(x) for the plan's segments (GemvArgs fields: seg
// w / y / rows, K, mode, x, x2, normw, eps, zero_ptr / zero_n).
ifx_status dense_gemv_plan(GemvArgs &a, int *grid, size_t *smem);
ifx_status dense_gemv_launch(const GemvArgs &a, int grid, size_t smem, cudaStream_t st, bool pdl);

// f(X) for M rows of K into `out` (row-major f32; the staging buffers of the
// quantised paths are at least this large).
ifx_status dense_stage(const float *X, const float *X2, const float *normw, float eps, int mode,
                       int64_t M, int64_t K, void *out, cudaStream_t st);
// C[M, rows] (ldc) = or += (accumulate) X W^T, X from dense_stage.
ifx_status dense_gemm(const QMatrix &W, const void *xs, int64_t M, float *C, int64_t ldc,
                      int accumulate, cudaStream_t st);

}  // namespace ifx
