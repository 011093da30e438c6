// Batched (prefill) fused dequant GEMM: C[M, N] = f(X)[M, K] . W[N, K]^T
// (replaces tensor_f32_by_index + matmul_t at m = seq_len,
// src/model/forward.rs:239-241, 308, 321-334, 528).
#pragma once
#include "repack.h"

namespace ifx {

constexpr int kGemmTokens = 64;  // tokens per CTA tile (8 MMA n-tiles)

enum GemmXMode { GX_PLAIN = 0, GX_RMSNORM = 1, GX_SWIGLU = 2 };

// Scratch sized for M tokens and K columns (f16 B fragments of f(X)).
size_t gemm_xfrag_bytes(int64_t M, int64_t K);

// Stage f(X) (row-major f32 [M, K]; for SWIGLU X is gate and X2 is up) as
// f16 fragments in `xfrag`. RMSNORM normalises each row with `normw`.
ifx_status gemm_stage_x(const float *X, const float *X2, const float *normw, float eps, int mode,
                        int64_t M, int64_t K, void *xfrag, cudaStream_t st);

// C[M, rows] (ldc) = or += (accumulate) staged X . W^T.
ifx_status gemm_run(const QMatrix &W, const void *xfrag, int64_t M, float *C, int64_t ldc,
                    int accumulate, int *err, cudaStream_t st);

// Small batches (batched decode, M <= 32 tokens): the exact-integer
// mma.sync kernel with blocks of 16 or 32 tokens and K split over enough
// CTAs to fill the GPU. C += X W^T with atomic adds, so C must hold its
// initial value (zeros, or the residual the result is added to).
constexpr int kGemmSmallMax = 32;
size_t gemm_small_xfrag_bytes(int64_t M, int64_t K);
// Up to two f32 buffers the staging kernel zeroes (after the previous grid
// completes) for the GEMMs that follow it to accumulate into.
struct StageZero {
  float *p[2] = {nullptr, nullptr};
  int64_t n[2] = {0, 0};
};
// pdl: launched with programmatic serialization (the small-batch GEMMs
// are, so their weight fetch overlaps the staging before them).
ifx_status gemm_small_stage_x(const float *X, const float *X2, const float *normw, float eps,
                              int mode, int64_t M, int64_t K, void *xfrag, cudaStream_t st,
                              StageZero zero = StageZero{}, bool pdl = false);
ifx_status gemm_small_run(const QMatrix &W, const void *xfrag, int64_t M, float *C, int64_t ldc,
                          int *err, cudaStream_t st);
// n (<= 3) matrices over one staged input in one launch (Wq/Wk/Wv, W1/W3);
// separate launches when their unit widths differ.
ifx_status gemm_small_run_multi(const QMatrix *const *W, float *const *C, const int64_t *ldc,
                                int n, const void *xfrag, int64_t M, int *err, cudaStream_t st);

// The tensor-memory (tcgen05) GEMM of tcgemm.cu: used by gemm_stage_x and
// gemm_run whenever K is a multiple of 64 (the mma.sync kernel above covers
// the rest).
bool tc_gemm_eligible(int64_t K);
int tc_gemm_ntile(int64_t M);
size_t tc_xtile_bytes(int64_t M, int64_t K);
ifx_status tc_stage_x(const float *X, const float *X2, const float *normw, float eps, int mode,
                      int64_t M, int64_t K, void *xt, cudaStream_t st);
ifx_status tc_gemm_run(const QMatrix &W, const void *xt, int64_t M, float *C, int64_t ldc,
                       int accumulate, int *err, cudaStream_t st);
ifx_status tc_gemm_run_multi(const QMatrix *const *W, float *const *C, const int64_t *ldc, int n,
                             const void *xt, int64_t M, int accumulate, int *err,
                             cudaStream_t st);

// n (<= 3) matrices with the same K over one staged input: a single launch on
// the tensor-memory path (their row tiles side by side), in turn otherwise.
ifx_status gemm_run_multi(const QMatrix *const *W, float *const *C, const int64_t *ldc, int n,
                          const void *xfrag, int64_t M, int accumulate, int *err,
                          cudaStream_t st);

}  // namespace ifx
