// Dense matmul weights: GGUF F32, F16 and Q8_K tensors used as matrices
// (the reference dequantises every matmul weight to f32 and multiplies in
// f32: src/gguf/dequant.rs:10-52, 201-232 and src/ops.rs:33-44; its own
// model fixtures are all-F32, src/model/forward.rs:713). A model with any
// such weight keeps all its matmul weights as row-major f32 on the device,
// dequantised once at load with the reference's formulas, and runs these
// kernels instead of the fused quantised ones:
//   dense_gemv  - batch 1: one warp per output row, f(x) staged once per CTA
//                 in shared memory (plain / RMSNorm / SwiGLU, the same input
//                 transforms as the fused GEMV), y += W f(x);
//   dense_stage - f(X) for M rows into a row-major f32 buffer;
//   dense_gemm  - M >= 2 rows: 64 x 64 output tiles, 16-deep k slices in
//                 shared memory, 4 x 4 outputs per thread, f32 FMA.
// Bound by HBM (4 bytes per weight per pass): this path is for API and
// parity completeness, not a tuned hot path.
#include <algorithm>

#include "dense.cuh"

namespace ifx {

namespace {

constexpr int kDenseThreads = 256;

__device__ __forceinline__ float silu_dense(float v) {
  // ops.rs:199-209: the sigmoid's input clamped to [-80, 80]
  const float c = fminf(fmaxf(v, -80.0f), 80.0f);
  return v * (1.0f / (1.0f + expf(-c)));
}

// 1/rms(x) over K values (ops.rs:155-168: 1/sqrt(sum x^2 / n + eps)); every
// thread of the block gets the value.
__device__ float block_rms_inv(const float *x, int64_t K, float eps) {
  __shared__ float red[kDenseThreads / 32];
  __shared__ float s_inv;
  float ss = 0.f;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) ss += x[k] * x[k];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) s_inv = 1.0f / sqrtf(v / (float)K + eps);
  }
  __syncthreads();
  return s_inv;
}

// f(x)[k]: RMSNorm as (x * s) * w (the reference's order), SwiGLU as
// silu(gate) * up.
__device__ __forceinline__ float fx(int mode, const float *x, const float *x2, const float *w,
                                    float inv, int64_t k) {
  if (mode == GEMV_RMSNORM) return (x[k] * inv) * w[k];
  if (mode == GEMV_SWIGLU) return silu_dense(x[k]) * x2[k];
  return x[k];
}

__global__ void __launch_bounds__(kDenseThreads) dense_gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ float xs[];  // f(x), K floats
  pdl_wait();
  pdl_launch();
  if (a.zero_ptr)
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.zero_n; i += gridDim.x * blockDim.x)
      a.zero_ptr[i] = 0.f;
  const int64_t K = a.K;
  const float inv = a.mode == GEMV_RMSNORM ? block_rms_inv(a.x, K, a.eps) : 1.0f;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) xs[k] = fx(a.mode, a.x, a.x2, a.normw, inv, k);
  __syncthreads();
  int total = 0;
  for (int s = 0; s < a.nseg; ++s) total += a.seg[s].rows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = kDenseThreads / 32;
  for (int r = blockIdx.x * nw + warp; r < total; r += gridDim.x * nw) {
    int s = 0, row = r;
    while (row >= a.seg[s].rows) row -= a.seg[s++].rows;
    const float *w = reinterpret_cast<const float *>(a.seg[s].w) + (size_t)row * K;
    float acc = 0.f;
    for (int64_t k = lane; k < K; k += 32) acc = fmaf(w[k], xs[k], acc);
    acc = warp_sum(acc);
    if (lane == 0) a.seg[s].y[row] += acc;
  }
}

__global__ void __launch_bounds__(kDenseThreads) dense_stage_kernel(const float *X, const float *X2,
                                                                     const float *normw, float eps,
                                                                     int mode, int64_t K, float *out) {
  const int64_t t = blockIdx.x;
  const float *x = X + t * K, *x2 = X2 ? X2 + t * K : nullptr;
  const float inv = mode == GEMV_RMSNORM ? block_rms_inv(x, K, eps) : 1.0f;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) out[t * K + k] = fx(mode, x, x2, normw, inv, k);
}

// C[t, r] (+)= sum_k W[r, k] X[t, k]; a 16 x 16 thread block computes 64
// rows x 64 tokens.
constexpr int kDT = 64, kDK = 16;

__global__ void __launch_bounds__(256) dense_gemm_kernel(const float *W, const float *X, float *C,
                                                         int64_t rows, int64_t M, int64_t K,
                                                         int64_t ldc, int accumulate) {
  __shared__ float Ws[kDK][kDT + 4], Xs[kDK][kDT + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t r0 = (int64_t)blockIdx.x * kDT, t0 = (int64_t)blockIdx.y * kDT;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += kDK) {
    for (int e = threadIdx.x; e < kDT * kDK; e += 256) {
      const int i = e / kDK, kk = e % kDK;  // consecutive threads: consecutive k
      const int64_t k = k0 + kk;
      Ws[kk][i] = (r0 + i < rows && k < K) ? W[(r0 + i) * K + k] : 0.f;
      Xs[kk][i] = (t0 + i < M && k < K) ? X[(t0 + i) * K + k] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kDK; ++kk) {
      float wv[4], xv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        wv[j] = Ws[kk][ty + 16 * j];
        xv[j] = Xs[kk][tx + 16 * j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(wv[i], xv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t r = r0 + ty + 16 * i, t = t0 + tx + 16 * j;
      if (r < rows && t < M) {
        float *p = C + t * ldc + r;
        *p = accumulate ? *p + acc[i][j] : acc[i][j];
      }
    }
}

}  // namespace

bool dense_type(int type) {
  return type == IFX_TYPE_F32 || type == IFX_TYPE_F16 || type == IFX_TYPE_Q8_K;
}

void make_dense_layout(int64_t rows, int64_t cols, int src_type, QLayout *L) {
  *L = QLayout{};
  L->type = src_type;
  L->dense = 1;
  L->rows = rows;
  L->cols = cols;
  L->total_bytes = (uint64_t)rows * (uint64_t)cols * sizeof(float);
}

ifx_status dense_gemv_plan(GemvArgs &a, int *grid, size_t *smem) {
  int total = 0;
  for (int s = 0; s < a.nseg; ++s) total += a.seg[s].rows;
  *grid = std::max(1, std::min((total + 7) / 8, 4 * kNumSMs));
  *smem = (size_t)a.K * sizeof(float);
  if (*smem > 200 * 1024) return fail(IFX_ERR_UNSUPPORTED, "dense gemv: input longer than 51200");
  return IFX_OK;
}

ifx_status dense_gemv_launch(const GemvArgs &a, int grid, size_t smem, cudaStream_t st, bool pdl) {
  static size_t attr = 0;
  if (smem > 48 * 1024 && smem > attr) {
    IFX_CUDA(cudaFuncSetAttribute(dense_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    attr = smem;
  }
  IFX_CUDA(launch(dense_gemv_kernel, dim3(grid), dim3(kDenseThreads), smem, st, pdl, a));
  return IFX_OK;
}

ifx_status dense_stage(const float *X, const float *X2, const float *normw, float eps, int mode,
                       int64_t M, int64_t K, void *out, cudaStream_t st) {
  if (M <= 0 || K <= 0) return fail(IFX_ERR_SHAPE, "dense stage: empty input");
  dense_stage_kernel<<<(unsigned)M, kDenseThreads, 0, st>>>(X, X2, normw, eps, mode, K,
                                                            static_cast<float *>(out));
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status dense_gemm(const QMatrix &W, const void *xs, int64_t M, float *C, int64_t ldc,
                      int accumulate, cudaStream_t st) {
  const dim3 grid((unsigned)((W.L.rows + kDT - 1) / kDT), (unsigned)((M + kDT - 1) / kDT));
  dense_gemm_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const float *>(W.d),
                                          static_cast<const float *>(xs), C, W.L.rows, M, W.L.cols,
                                          ldc, accumulate);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

}  // namespace ifx
