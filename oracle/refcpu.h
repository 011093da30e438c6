/*
 * refcpu — CPU restatement of phraakture/inferox's token loop.
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity oracle: tests, smoke() and
 * bench.py's cpu_baseline / --impl reference legs load it as a checker or as
 * the timed CPU baseline. The product path (inferox_b200) never links, loads
 * or calls it.
 *
 * Parity status: the reference is Rust and no Rust toolchain exists on these
 * machines, so the reference cannot be built or run here. The restatement is
 * pinned against every known-answer test the reference's own sources hold
 * (dequant.rs:247-392, ops.rs:293-416, sampler.rs:89-94, weights.rs:151-183,
 * model/mod.rs:197-238, forward.rs:729-839), ported in tests/test_oracle_kats.py.
 * Forward-pass logits are not pinned by any reference vector (the reference
 * has none); they follow the code line by line, with the file:line cited at
 * each function.
 *
 * Arithmetic follows the Rust semantics exactly: IEEE f32, no FMA contraction
 * except where the reference calls _mm256_fmadd_ps, glibc expf/powf/sinf/cosf
 * (which Rust's f32::exp/powf/sin/cos lower to on linux-gnu), and the AVX2
 * lane and horizontal-sum order of matmul_t_avx2 (ops.rs:106-149).
 */
#ifndef REFCPU_H
#define REFCPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes mirror gguf::Error (src/gguf/error.rs:6-42). */
enum {
  RC_OK = 0,
  RC_ERR_IO = 1,
  RC_ERR_INVALID_MAGIC = 2,
  RC_ERR_UNSUPPORTED_VERSION = 3,
  RC_ERR_UNKNOWN_VALUE_TYPE = 4,
  RC_ERR_UNKNOWN_TENSOR_TYPE = 5,
  RC_ERR_INVALID_UTF8 = 6,
  RC_ERR_INVALID_SHAPE = 7,
  RC_ERR_UNEXPECTED_EOF = 8,
  RC_ERR_TENSOR_NOT_FOUND = 9,
  RC_ERR_INVALID_TENSOR_INDEX = 10,
  RC_ERR_TENSOR_OFFSET_OVERFLOW = 11,
  RC_ERR_UNSUPPORTED_ARCHITECTURE = 12,
};

/* TensorType ids (src/gguf/types.rs:68-99). */
enum {
  RC_F32 = 0, RC_F16 = 1, RC_Q4_0 = 2, RC_Q4_1 = 3, RC_Q5_0 = 5, RC_Q5_1 = 6,
  RC_Q8_0 = 7, RC_Q8_1 = 8, RC_Q2K = 10, RC_Q3K = 11, RC_Q4K = 12, RC_Q5K = 13,
  RC_Q6K = 14, RC_Q8K = 15, RC_I8 = 16, RC_I16 = 17, RC_I32 = 18, RC_I64 = 19,
  RC_F64 = 20, RC_IQ1S = 21, RC_IQ1M = 22, RC_IQ2XXS = 23, RC_IQ2XS = 24,
  RC_IQ2S = 25, RC_IQ3XXS = 26, RC_IQ3S = 27, RC_IQ4XS = 28, RC_IQ4NL = 29,
  RC_IQ4XSS = 30
};

typedef struct {
  uint32_t vocab_size;
  uint64_t hidden_size, n_layers, n_heads, n_kv_heads, head_dim;
  uint64_t intermediate_size;
  float norm_eps, rope_base;
  uint64_t rope_dim, context_length;
  char architecture[64];
} rc_config;

typedef struct rc_model rc_model;
typedef struct rc_kv rc_kv;

/* --- half / dequant (src/gguf/dequant.rs) --- */
float rc_f16_to_f32(uint16_t h);
int64_t rc_type_byte_size(int type, uint64_t n_elements); /* -1 = unknown */
int rc_dequantize(int type, const uint8_t *bytes, size_t nbytes, float *out,
                  size_t n_out);

/* --- ops (src/ops.rs) --- */
void rc_matmul(const float *a, const float *b, float *c, size_t m, size_t n,
               size_t k);
void rc_matmul_t(const float *a, const float *b, float *c, size_t m, size_t n,
                 size_t k);
void rc_matmul_t_scalar_emul(const float *a, const float *b, float *c,
                             size_t m, size_t n, size_t k);
void rc_rms_norm(float *x, const float *w, size_t n, float eps);
void rc_rms_norm_rows(float *x, const float *w, float eps, size_t rows,
                      size_t hidden);
void rc_silu(float *x, size_t n);
void rc_swiglu(const float *gate, const float *up, float *out, size_t n);
void rc_add_in_place(float *out, const float *b, size_t n);
void rc_softmax_rows(float *x, size_t rows, size_t cols);
int rc_embedding_lookup(const float *emb, size_t emb_len, const uint32_t *ids,
                        size_t n_ids, size_t hidden, float *out);
void rc_rope(float *x, size_t seq_len, size_t n_heads, size_t head_dim,
             size_t rope_dim, float base);
uint32_t rc_argmax(const float *x, size_t n);
/* Sampler::sample (src/sampler.rs:28-73) with the RNG draw supplied as a
 * uniform u in [0,1): WeightedIndex picks the first index whose cumulative
 * weight exceeds u * total. */
uint32_t rc_sample(const float *logits, size_t n, float temperature,
                   size_t top_k, float top_p, double u);

/* --- GGUF + model (src/gguf/file.rs, weights.rs, model/{mod,config,cache,forward}.rs) --- */
/* The model keeps a pointer to `bytes`; the caller keeps them alive. */
int rc_model_open_mem(const uint8_t *bytes, size_t len, rc_model **out);
/* GgufFile::read only (file.rs:57-116): no llama config, no layer wiring. */
int rc_gguf_open_mem(const uint8_t *bytes, size_t len, rc_model **out);
/* Weights::tensor (weights.rs:44-51 -> tensor_bytes :97-112). */
int rc_tensor_bytes(const rc_model *m, const char *name, uint64_t *offset_abs,
                    uint64_t *nbytes);
void rc_model_free(rc_model *m);
void rc_model_config(const rc_model *m, rc_config *out);
int rc_model_tensor_info(const rc_model *m, const char *name, int *type,
                         uint64_t *n_elements, uint64_t *offset_abs,
                         uint64_t *nbytes);
int rc_model_has_output(const rc_model *m);
int rc_model_n_tensors(const rc_model *m);

/* Threads for row-parallel matmul/attention (bitwise identical results). */
void rc_set_threads(int n);
/* faithful=1: dequantise the whole tensor into a fresh buffer at every use,
 * as Weights::tensor_f32_by_index does (weights.rs:66-74). faithful=0: fuse
 * the per-row dequant into matmul_t (same bits, far less memory traffic). */
void rc_set_faithful(int on);

rc_kv *rc_kv_new(const rc_model *m, size_t n_layers, size_t max_seq_len);
void rc_kv_free(rc_kv *kv);
void rc_kv_clear(rc_kv *kv);
size_t rc_kv_len(const rc_kv *kv);
/* Read back one layer's K or V cache rows [0, len) (f32 [len, kv_dim]). */
int rc_kv_read(const rc_kv *kv, size_t layer, int which_v, float *out);

/* Model::prefill (forward.rs:496-538). logits: [n, vocab] if last_row_only
 * is 0, else [vocab] for the last row only (the other rows are skipped;
 * rows are independent so the last row's bits are unchanged). */
int rc_prefill(const rc_model *m, rc_kv *kv, const uint32_t *ids, size_t n,
               float *logits, int last_row_only);
/* Model::decode_step (forward.rs:543-586). logits: [vocab]. */
int rc_decode_step(const rc_model *m, rc_kv *kv, uint32_t token,
                   float *logits);
/* Model::forward (forward.rs:448-482): non-causal, no cache. [n, vocab]. */
int rc_forward(const rc_model *m, const uint32_t *ids, size_t n,
               float *logits);
/* Model::generate (forward.rs:592-612): greedy. out: [max_tokens]. */
int rc_generate(const rc_model *m, rc_kv *kv, const uint32_t *prompt,
                size_t n_prompt, size_t max_tokens, uint32_t *out);

/* Synthetic benchmark models (synth_ref.c): the workload definition of the
 * benchmark, independent of the product's generator. */
typedef struct {
  uint32_t vocab, dim, n_layers, n_heads, n_kv_heads, ffn, context;
  float rope_base, norm_eps, sigma;
  int mix, tied;
  uint64_t seed;
  int threads;
} rc_synth_spec;
int rc_synth_gguf(const rc_synth_spec *spec, uint8_t **out, size_t *out_len);
void rc_synth_free(uint8_t *p);

#ifdef __cplusplus
}
#endif
#endif
