// Device kernels behind the op-level C ABI (mirrors of src/ops.rs) and the
// small fused kernels of the token loop.
#pragma once
#include "common.cuh"

namespace ifx {

ifx_status op_dequantize(int type, const uint8_t *src, size_t nbytes, float *out, size_t n,
                         cudaStream_t st);
ifx_status op_matmul(const float *a, const float *b, float *c, size_t m, size_t n, size_t k,
                     cudaStream_t st);
ifx_status op_matmul_t(const float *a, const float *b, float *c, size_t m, size_t n, size_t k,
                       cudaStream_t st);
ifx_status op_rms_norm_rows(float *x, const float *w, float eps, size_t rows, size_t hidden,
                            cudaStream_t st);
ifx_status op_silu(float *x, size_t n, cudaStream_t st);
ifx_status op_swiglu(const float *g, const float *u, float *o, size_t n, cudaStream_t st);
ifx_status op_add(float *o, const float *b, size_t n, cudaStream_t st);
ifx_status op_softmax_rows(float *x, size_t rows, size_t cols, cudaStream_t st);
ifx_status op_embedding_lookup(const float *emb, size_t emb_len, const uint32_t *ids,
                               size_t n_ids, size_t hidden, float *out, int *err_dev,
                               cudaStream_t st);
ifx_status op_rope(float *x, size_t seq, size_t heads, size_t hd, size_t rope_dim, float base,
                   size_t pos0, cudaStream_t st);
// Argmax with the reference's tie rule (last index). key_dev: 64-bit scratch
// (must start at 0); result written to out_dev.
ifx_status op_argmax(const float *x, size_t n, unsigned long long *key_dev, uint32_t *out_dev,
                     cudaStream_t st);
ifx_status op_sample_u(const float *logits, size_t n, float temperature, uint64_t top_k,
                       float top_p, float u, uint32_t *out_dev, cudaStream_t st);
// Largest logits count op_sample_u_static accepts (its scratch is static).
constexpr size_t kStaticSampleMax = 262144;
// op_sample_u with its scratch in a static device array: allocates nothing,
// writes the token to out_dev on the stream without synchronising. Calls
// that overlap in time on one device share the scratch and race.
ifx_status op_sample_u_static(const float *logits, size_t n, float temperature, uint64_t top_k,
                              float top_p, float u, uint32_t *out_dev, cudaStream_t st);
// Sampler::sample with a Philox uniform (seed, offset) computed on device.
ifx_status op_sample_philox(const float *logits, size_t n, float temperature, uint64_t top_k,
                            float top_p, uint64_t seed, uint64_t offset, uint32_t *out_dev,
                            cudaStream_t st);

// Monotone map float -> uint32 so that unsigned order == float order.
__device__ __forceinline__ uint32_t ordered_bits(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

}  // namespace ifx
