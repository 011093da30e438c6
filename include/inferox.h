/*
 * inferox.h — C ABI of libinferox_b200.so, the sm_100a implementation of
 * phraakture/inferox's token loop.
 *
 * The reference is a Rust crate with no FFI; its call surface is the Rust API
 * of `ops`, `model` and `sampler`. Each entry point below names the reference
 * item it replaces (path:line inside the reference crate). A Rust `cuda`
 * module binds these with the `extern "C"` declarations of inferox_ffi.rs
 * (next to this header).
 *
 * Conventions
 *  - Every call returns ifx_status; IFX_OK is 0. ifx_last_error() gives a
 *    thread-local message for the last failure on the calling thread.
 *  - Model-level calls take and return HOST buffers (as the Rust API does);
 *    the library owns all device memory behind ifx_model / ifx_kv.
 *  - Op-level calls (ifx_op_*) take DEVICE pointers and a cudaStream_t passed
 *    as void* (NULL = legacy default stream); they are asynchronous unless
 *    stated otherwise. Shape mismatches that panic in the reference
 *    (assert_eq!, ops.rs:16-18) return IFX_ERR_SHAPE instead.
 *  - No call is re-entrant on the same ifx_model; one model per device.
 */
#ifndef INFEROX_H
#define INFEROX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* gguf::Error (src/gguf/error.rs:6-42) in declaration order, then the codes
 * the GPU build adds. */
typedef enum ifx_status {
  IFX_OK = 0,
  IFX_ERR_IO = 1,
  IFX_ERR_INVALID_MAGIC = 2,
  IFX_ERR_UNSUPPORTED_VERSION = 3,
  IFX_ERR_UNKNOWN_VALUE_TYPE = 4,
  IFX_ERR_UNKNOWN_TENSOR_TYPE = 5,
  IFX_ERR_INVALID_UTF8 = 6,
  IFX_ERR_INVALID_SHAPE = 7,
  IFX_ERR_UNEXPECTED_EOF = 8,
  IFX_ERR_TENSOR_NOT_FOUND = 9,
  IFX_ERR_INVALID_TENSOR_INDEX = 10,
  IFX_ERR_TENSOR_OFFSET_OVERFLOW = 11,
  IFX_ERR_UNSUPPORTED_ARCHITECTURE = 12,
  IFX_ERR_SHAPE = 20,            /* replaces ops.rs assert_eq! panics */
  IFX_ERR_CUDA = 21,             /* CUDA runtime/driver failure */
  IFX_ERR_NCCL = 22,             /* NCCL failure (tensor parallel) */
  IFX_ERR_TIMEOUT = 23,          /* a bounded device wait gave up */
  IFX_ERR_INVALID_ARGUMENT = 24, /* null pointer, zero size, bad enum */
  IFX_ERR_OUT_OF_MEMORY = 25,
  IFX_ERR_UNSUPPORTED = 26,      /* valid input this build does not run */
  IFX_ERR_JSON = 27,             /* TokenizerError::Json (tokenizer/mod.rs:232) */
  IFX_ERR_UNSUPPORTED_MODEL = 28 /* TokenizerError::UnsupportedModel (mod.rs:233) */
} ifx_status;

/* TensorType ids (src/gguf/types.rs:68-99) the kernels accept. */
enum {
  IFX_TYPE_F32 = 0,
  IFX_TYPE_F16 = 1,
  IFX_TYPE_Q4_0 = 2,
  IFX_TYPE_Q8_0 = 7,
  IFX_TYPE_Q4_K = 12,
  IFX_TYPE_Q6_K = 14,
  IFX_TYPE_Q8_K = 15
};

const char *ifx_last_error(void);
const char *ifx_status_name(ifx_status s);
/* Library version, (major << 16) | minor. */
int ifx_version(void);

/* Config (src/model/config.rs:5-30), filled by Config::from_gguf rules
 * (config.rs:34-84). */
typedef struct ifx_config {
  uint32_t vocab_size;
  uint64_t hidden_size, n_layers, n_heads, n_kv_heads, head_dim;
  uint64_t intermediate_size;
  float norm_eps, rope_base;
  uint64_t rope_dim, context_length;
  char architecture[64];
} ifx_config;

/* Load options (no reference counterpart: device placement and the
 * tensor-parallel split are new). */
typedef struct ifx_load_opts {
  int device;      /* CUDA device ordinal */
  int tp_size;     /* tensor-parallel ranks (1, 2, 4, 8) */
  int tp_rank;     /* this process's rank */
  void *nccl_comm; /* ncclComm_t for tp_size > 1, owned by the caller */
  int rope_compat; /* 1 (default): decode applies RoPE at position 0 and
                      prefill at 0..n, exactly as forward.rs:243-244,371-372;
                      0: true positions (cache offset + t) */
  int use_graphs;  /* 1 (default): decode steps replay CUDA graphs */
  int persistent_decode; /* 1 (default): batch-1 decode steps run as one
                            persistent cooperative kernel per token when the
                            head geometry allows it; 0: one kernel per op */
  int kquant_layout; /* IFX_KQUANT_REFERENCE (default): type ids and Q4_K /
                        Q6_K bytes as the reference reads them
                        (types.rs:70-100, dequant.rs:123-199);
                        IFX_KQUANT_GGML: a file written by llama.cpp (ggml
                        ids, ggml block orders, int8 Q6_K scales) */
  int tp_timeout_ms; /* tensor parallel: longest wait for a call's
                        collectives (0: 300000). When a peer rank stops, the
                        call returns IFX_ERR_TIMEOUT (or IFX_ERR_NCCL on an
                        NCCL error) after aborting the communicator, and the
                        model refuses further calls: free it, make a new
                        communicator and load again
                        (ifx_tp_comm_destroy knows the aborted communicator
                        is gone and only forgets it). */
} ifx_load_opts;

enum { IFX_KQUANT_REFERENCE = 0, IFX_KQUANT_GGML = 1 };

void ifx_load_opts_default(ifx_load_opts *o);

typedef struct ifx_model ifx_model;
typedef struct ifx_kv ifx_kv;

/* Model::open (src/model/mod.rs:64-92): parse the GGUF (file.rs:57-116),
 * read the config, wire blk.{i}.* tensors, then upload and repack every
 * weight once (the per-call dequant of weights.rs:66-74 disappears). A file
 * with any F32, F16 or Q8_K matmul weight loads every matmul weight
 * dequantised to f32 and runs the dense kernels (no persistent decode). */
ifx_status ifx_model_load(const char *path, const ifx_load_opts *opts,
                          ifx_model **out);
/* Same, from a GGUF image already in host memory (no file). */
ifx_status ifx_model_load_mem(const void *bytes, size_t len,
                              const ifx_load_opts *opts, ifx_model **out);
void ifx_model_free(ifx_model *m);
/* Model.config (src/model/mod.rs:54). */
ifx_status ifx_model_config(const ifx_model *m, ifx_config *out);
/* Quantised weight bytes one batch-1 decode step reads on this rank
 * (every matmul weight + norms + one embedding row). */
uint64_t ifx_model_decode_weight_bytes(const ifx_model *m);

/* KvCache::new (src/model/cache.rs:16-24): device-resident, f16,
 * [layer][kv_head][max_seq][head_dim]; sharded by kv-head under TP. */
ifx_status ifx_kv_create(ifx_model *m, size_t max_seq_len, ifx_kv **out);
void ifx_kv_free(ifx_kv *kv);
/* KvCache::clear (cache.rs:26-28). */
ifx_status ifx_kv_clear(ifx_kv *kv);
/* KvCache::len (cache.rs:31-33). */
size_t ifx_kv_len(const ifx_kv *kv);
/* Test hook: copy layer `layer`'s K (which_v = 0) or V cache rows [0, len)
 * to host as f32 [len, n_kv_heads_local * head_dim]. */
ifx_status ifx_kv_read(const ifx_kv *kv, size_t layer, int which_v,
                       float *out_host);

/* Model::prefill (src/model/forward.rs:496-538): ids must all be < vocab
 * (else IFX_ERR_INVALID_TENSOR_INDEX, forward.rs:501-503). logits_host is
 * [n, vocab] (last_row_only = 0) or [vocab] (last_row_only = 1), or NULL. */
ifx_status ifx_prefill(ifx_model *m, ifx_kv *kv, const uint32_t *ids, size_t n,
                       float *logits_host, int last_row_only);
/* Model::decode_step (forward.rs:543-586): token >= vocab gives
 * IFX_ERR_INVALID_TENSOR_INDEX (forward.rs:552-554). logits_host: [vocab]
 * or NULL (skip the copy back). */
ifx_status ifx_decode_step(ifx_model *m, ifx_kv *kv, uint32_t token,
                           float *logits_host);
/* Model::forward / Model::forward_last_token_logits (forward.rs:448-495):
 * the layers over the whole prompt with attention over every position (no
 * causal mask), RoPE at positions 0..n, no KV cache. logits_host: [n, vocab]
 * (last_row_only = 0) or [vocab] (1). ids >= vocab give
 * IFX_ERR_INVALID_TENSOR_INDEX (forward.rs:453-455). */
ifx_status ifx_forward(ifx_model *m, const uint32_t *ids, size_t n,
                       float *logits_host, int last_row_only);
/* Model::generate (forward.rs:592-612): kv.clear, prefill, then max_tokens
 * greedy steps; the decode loop runs on the device (argmax feeds the next
 * embedding without a host round trip). out_tokens: [max_tokens]. */
ifx_status ifx_generate(ifx_model *m, ifx_kv *kv, const uint32_t *prompt,
                        size_t n_prompt, size_t max_tokens,
                        uint32_t *out_tokens);

/* Continue greedy decoding from the current cache state: feed `token`, then
 * each step's argmax (last index on ties) to the next step, n_steps times,
 * with no host round trip (the loop of forward.rs:605-609 on the device).
 * out_tokens ([n_steps], nullable) receives the argmax after each step.
 * device_ms (nullable) receives the CUDA-event time of the n_steps steps on
 * the model's stream. */
ifx_status ifx_decode_greedy(ifx_model *m, ifx_kv *kv, uint32_t token,
                             size_t n_steps, uint32_t *out_tokens,
                             float *device_ms);

/* Batched decode: `batch` (1-32) independent sequences sharing every weight
 * read of a step. The reference's KvCache holds one sequence
 * (src/model/cache.rs:7-13); this is that cache times `batch`, each
 * sequence with its own length, prefilled one at a time and decoded
 * together (Model::decode_step, forward.rs:543-586, for every sequence at
 * once). Single GPU only (IFX_ERR_UNSUPPORTED under tensor parallelism). */
typedef struct ifx_kv_batch ifx_kv_batch;
ifx_status ifx_kv_batch_create(ifx_model *m, size_t max_seq_len, int batch,
                               ifx_kv_batch **out);
void ifx_kv_batch_free(ifx_kv_batch *kb);
/* No reference counterpart: a batch whose caches share a pool of n_pages
 * pages of 64 positions (every layer and kv head of those positions). A
 * sequence takes pages as its prefill and decode steps reach them and gives
 * them back on ifx_kv_batch_reset, so batch * max_seq_len may exceed the
 * pool: a step that needs a page when none is free fails with
 * IFX_ERR_OUT_OF_MEMORY and changes no sequence's length. max_seq_len at
 * most 4096. Results are those of ifx_kv_batch_create's batch. */
ifx_status ifx_kv_batch_create_paged(ifx_model *m, size_t max_seq_len, int batch,
                                     size_t n_pages, ifx_kv_batch **out);
/* Pages of a paged batch that no sequence holds, and the pool size (both 0
 * for a batch made by ifx_kv_batch_create). */
ifx_status ifx_kv_batch_pages(const ifx_kv_batch *kb, size_t *free_pages,
                              size_t *total_pages);
/* KvCache::len (cache.rs:31-33) of sequence `seq`. */
ifx_status ifx_kv_batch_len(const ifx_kv_batch *kb, int seq, size_t *len);
/* Model::prefill (forward.rs:496-538) of sequence `seq` of the batch. */
ifx_status ifx_prefill_seq(ifx_model *m, ifx_kv_batch *kb, int seq,
                           const uint32_t *ids, size_t n, float *logits_host,
                           int last_row_only);
/* One decode step of every sequence: tokens [batch]; logits_host
 * [batch, vocab] and argmax_host [batch] (last index on ties) are nullable. */
ifx_status ifx_decode_step_batch(ifx_model *m, ifx_kv_batch *kb,
                                 const uint32_t *tokens, float *logits_host,
                                 uint32_t *argmax_host);
/* No reference counterpart (its KvCache holds one sequence, cache.rs:7-13):
 * one decode step of the n distinct sequences seqs[0..n) only, for a
 * serving loop whose requests come and go (continuous batching); the other
 * sequences keep their caches and lengths. Row i of logits_host [n, vocab]
 * and argmax_host [n] (both nullable) belongs to seqs[i]. After an error
 * from a device wait (IFX_ERR_TIMEOUT) the listed sequences' caches are in
 * an undefined state: reset them (ifx_kv_batch_reset) before reuse. */
ifx_status ifx_decode_step_batch_seqs(ifx_model *m, ifx_kv_batch *kb,
                                      const int *seqs, int n,
                                      const uint32_t *tokens,
                                      float *logits_host,
                                      uint32_t *argmax_host);
/* KvCache::clear (cache.rs:26-28) of sequence `seq` alone, so a new request
 * can take its place in the batch. */
ifx_status ifx_kv_batch_reset(ifx_model *m, ifx_kv_batch *kb, int seq);
/* n_steps greedy steps of every sequence, each step's argmax fed to the next
 * on the device; out_tokens [n_steps, batch] and device_ms are nullable. */
ifx_status ifx_decode_greedy_batch(ifx_model *m, ifx_kv_batch *kb,
                                   const uint32_t *tokens, size_t n_steps,
                                   uint32_t *out_tokens, float *device_ms);

/* Sampler (src/sampler.rs:8-16). */
typedef struct ifx_sampler {
  float temperature; /* 0 = greedy argmax */
  uint64_t top_k;    /* 0 disables */
  float top_p;       /* 1.0 disables */
} ifx_sampler;

/* Sampler::sample (sampler.rs:28-73) on the device over the model's last
 * logits (from the latest prefill/decode_step). The thread_rng draw is a
 * counter-based Philox uniform from (seed, offset). */
ifx_status ifx_sample(ifx_model *m, const ifx_sampler *s, uint64_t seed,
                      uint64_t offset, uint32_t *token_out);

/* ------------------------- op-level entry points ------------------------ */
/* dequantize_f32 (src/gguf/dequant.rs:10-31): bit-exact with the
 * reference's per-type loops (dequant.rs:40-232). */
ifx_status ifx_op_dequantize(int type, const void *bytes_dev, size_t nbytes,
                             float *out_dev, size_t n_out, void *stream);
/* matmul (src/ops.rs:15-26): C[m,n] = A[m,k] B[k,n], f32. */
ifx_status ifx_op_matmul(const float *a, const float *b, float *c, size_t m,
                         size_t n, size_t k, void *stream);
/* matmul_t (src/ops.rs:33-44): C[m,n] = A[m,k] B[n,k]^T, f32. */
ifx_status ifx_op_matmul_t(const float *a, const float *b, float *c, size_t m,
                           size_t n, size_t k, void *stream);

/* A weight matrix [rows, cols] uploaded for the matmul kernels. Replaces
 * tensor_f32_by_index's dequant (weights.rs:66-74). Q4_0, Q8_0, Q4_K and
 * Q6_K are repacked for the fused dequant kernels; F32, F16 and Q8_K are
 * dequantised once to f32 (dequant.rs:10-52, 201-232) for the dense ones. */
typedef struct ifx_qmatrix ifx_qmatrix;
ifx_status ifx_qmatrix_create(int type, const void *gguf_bytes_host,
                              size_t nbytes, size_t rows, size_t cols,
                              int device, ifx_qmatrix **out);
void ifx_qmatrix_free(ifx_qmatrix *w);
/* tensor_f32_by_index + matmul_t fused (forward.rs:366-368 and every other
 * matmul_t site): C[m, rows] = A[m, cols] W^T with dequant in registers. */
ifx_status ifx_op_matmul_t_q(const float *a_dev, const ifx_qmatrix *w,
                             float *c_dev, size_t m, void *stream);

/* rms_norm / rms_norm_rows (src/ops.rs:155-180), in place. */
ifx_status ifx_op_rms_norm_rows(float *x, const float *w, float eps,
                                size_t rows, size_t hidden, void *stream);
/* silu (ops.rs:183-187) in place; swiglu (ops.rs:190-197). */
ifx_status ifx_op_silu(float *x, size_t n, void *stream);
ifx_status ifx_op_swiglu(const float *gate, const float *up, float *out,
                         size_t n, void *stream);
/* add_in_place (ops.rs:212-217). */
ifx_status ifx_op_add_in_place(float *out, const float *b, size_t n,
                               void *stream);
/* softmax_rows (ops.rs:223-239), in place. */
ifx_status ifx_op_softmax_rows(float *x, size_t rows, size_t cols,
                               void *stream);
/* embedding_lookup (ops.rs:246-258). Synchronous: an out-of-range id
 * returns IFX_ERR_INVALID_TENSOR_INDEX (the reference panics). */
ifx_status ifx_op_embedding_lookup(const float *emb, size_t emb_len,
                                   const uint32_t *ids, size_t n_ids,
                                   size_t hidden, float *out, void *stream);
/* rope (ops.rs:265-287) over positions pos0..pos0+seq_len (the reference
 * always uses pos0 = 0). */
ifx_status ifx_op_rope(float *x, size_t seq_len, size_t n_heads,
                       size_t head_dim, size_t rope_dim, float base,
                       size_t pos0, void *stream);
/* argmax (forward.rs:615-622 / sampler.rs:75-82): last index on ties. */
ifx_status ifx_op_argmax(const float *x, size_t n, uint32_t *out_dev,
                         void *stream);
/* Sampler::sample with the uniform draw u in [0,1) supplied per call, so a
 * host oracle can reproduce the pick (sampler.rs:28-73, rand 0.8.6
 * WeightedIndex). Synchronous; token written to *token_host. */
ifx_status ifx_op_sample_u(const float *logits_dev, size_t n,
                           const ifx_sampler *s, float u,
                           uint32_t *token_host, void *stream);
/* No counterpart in the reference (its sampler is host code). The same pick
 * as ifx_op_sample_u, for callers that cannot allocate device memory on this
 * path: a host runtime that reserves its whole device budget up front and
 * forbids later allocation, or a serving loop that must not pay for
 * cudaMalloc/cudaFree (cudaFree synchronises the whole device) on every
 * token. Its scratch is a static device array reserved when the library
 * loads, so n is limited to IFX_SAMPLE_STATIC_MAX logits; larger n returns
 * IFX_ERR_INVALID_ARGUMENT. The token is written to token_dev (device
 * memory) on `stream`; the call does not synchronise. The first call on a
 * device looks up the scratch address with that device current; if that
 * first call could fall inside a stream capture, make one call on the device
 * before the capture begins. Every call on a device uses the same scratch:
 * calls whose work overlaps in time (other streams, other threads) race, so
 * order them on one stream or serialise them. The looked-up address belongs
 * to the device's current context: after cudaDeviceReset on a device, unload
 * and reload this library before calling it again on that device. */
#define IFX_SAMPLE_STATIC_MAX 262144
ifx_status ifx_op_sample_u_static(const float *logits_dev, size_t n,
                                  const ifx_sampler *s, float u,
                                  uint32_t *token_dev, void *stream);

/* ------------------------- tensor parallelism --------------------------- */
/* No reference counterpart (the reference is single-threaded CPU code).
 * Megatron split across tp_size GPUs of one box: Wq/Wk/Wv, W1/W3 and the
 * vocab projection by rows, Wo/W2 by their input dimension, the KV cache by
 * kv head; an NCCL all-reduce after Wo and after W2, an all-gather of the
 * vocab slices. ifx_load_opts.nccl_comm must be a communicator of the NCCL
 * library instance this library uses; these make one: rank 0 calls
 * ifx_tp_unique_id, the caller sends the 128 bytes to every rank, then every
 * rank calls ifx_tp_comm_create (collective: it returns once all joined). */
ifx_status ifx_tp_unique_id(void *id_out /* 128 bytes */);
ifx_status ifx_tp_comm_create(const void *id, int nranks, int rank, int device,
                              void **comm_out);
void ifx_tp_comm_destroy(void *comm);
/* Host only: the shard of a GGUF-layout weight [rows, cols] that `rank` of
 * `tp` holds (split_k = 0: a block of rows; 1: a block of every row's input
 * dimension). out NULL: *out_bytes receives the shard size only. */
ifx_status ifx_tp_shard(int type, const void *gguf_bytes, size_t nbytes,
                        size_t rows, size_t cols, int split_k, int tp, int rank,
                        void *out, size_t *out_bytes);

/* --------------------------- measurement hooks -------------------------- */
/* No reference counterpart. Kernels one decode step on this cache launches:
 * 1 when the step runs as the persistent decode kernel, else the per-op
 * count (3 + 5 * n_layers). Meaningful once the cache has been decoded into
 * (the persistent plan is built by the first decode step); 0 before that. */
int ifx_kv_decode_kernels(const ifx_kv *kv);
/* No reference counterpart (measurement of what replaces
 * tensor_f32_by_index + matmul_t, forward.rs:366-368 / ops.rs:33-44): time
 * the fused dequant matmul the token loop runs at batch m — the batch-1 GEMV
 * for m = 1, the small-batch GEMM for m <= 32, the prefill GEMM above — with
 * its input staging, `reps` launches each timed alone by CUDA events, with a
 * 256 MB buffer written between launches so the weights come from HBM.
 * a_dev [m, cols], c_dev [m, rows] (device). Reports ms per call. */
ifx_status ifx_bench_matmul_t_q(const float *a_dev, const ifx_qmatrix *w,
                                float *c_dev, size_t m, int reps,
                                float *ms_per_call);
/* No reference counterpart. Launch one of the decode step's fused kernels
 * `reps` times in isolation (cycling through the layers so the weights come
 * from HBM, not L2) and report the CUDA-event time per launch and the
 * algorithmic bytes one launch moves. which: "qkv", "attn", "wo", "w13",
 * "w2", "logits". Requires a cache that has been decoded into (for "attn"). */
ifx_status ifx_bench_kernel(ifx_model *m, ifx_kv *kv, const char *which,
                            int reps, float *ms_per_launch,
                            uint64_t *bytes_per_launch);

/* No reference counterpart (the reference reads only its own byte orders).
 * Tensor bytes of ggml type id `ggml_type` in llama.cpp's block order,
 * rewritten into the reference's order (dequant.rs:123-199), as a load with
 * IFX_KQUANT_GGML does: Q4_K and Q6_K blocks are permuted, Q4_0 / Q8_0 /
 * F32 / F16 copied. *type_out receives the reference's type id;
 * *signed_scales_out is 1 for Q6_K, whose scale bytes keep llama.cpp's int8
 * meaning (the reference would read them as u8). Host code; needs no GPU.
 * `dst` holds nbytes and may be `src` itself (converted in place). */
ifx_status ifx_kquant_from_ggml(uint32_t ggml_type, const void *src,
                                size_t nbytes, void *dst, int *type_out,
                                int *signed_scales_out);

/* ------------------------------ tokenizer ------------------------------- */
/* The reference's byte-level BPE tokenizer over a Hugging Face
 * tokenizer.json (BpeTokenizer, src/tokenizer/mod.rs:23-226; GPT-2 byte
 * tables, bytes.rs:10-35). Host code; needs no GPU. Errors: IFX_ERR_IO
 * (TokenizerError::Io, including a file that is not UTF-8), IFX_ERR_JSON
 * (TokenizerError::Json: malformed JSON or a schema mismatch),
 * IFX_ERR_UNSUPPORTED_MODEL (model.type other than "BPE"). */
typedef struct ifx_tokenizer ifx_tokenizer;
/* BpeTokenizer::from_file (mod.rs:61-64). */
ifx_status ifx_tokenizer_load(const char *path, ifx_tokenizer **out);
/* BpeTokenizer::from_json (mod.rs:67-110); `json` is UTF-8, `len` bytes. */
ifx_status ifx_tokenizer_load_json(const char *json, size_t len,
                                   ifx_tokenizer **out);
void ifx_tokenizer_free(ifx_tokenizer *t);
/* Tokenizer::encode (mod.rs:194-204) of `len` bytes of UTF-8 text. Sets
 * *n_ids to the id count; IFX_ERR_SHAPE (nothing written) when it exceeds
 * `cap`, so a caller can size the buffer with a first call of cap 0. */
ifx_status ifx_tokenizer_encode(const ifx_tokenizer *t, const char *text,
                                size_t len, uint32_t *ids, size_t cap,
                                size_t *n_ids);
/* Tokenizer::decode (mod.rs:206-225): UTF-8 bytes (not NUL-terminated)
 * into `text`; *len and IFX_ERR_SHAPE as for encode. */
ifx_status ifx_tokenizer_decode(const ifx_tokenizer *t, const uint32_t *ids,
                                size_t n, char *text, size_t cap,
                                size_t *len);
/* Number of vocabulary entries (model.vocab). */
ifx_status ifx_tokenizer_vocab_size(const ifx_tokenizer *t, size_t *n);

/* ------------------- synthetic workload generator ----------------------- */
/* No reference counterpart: the reference's tests build GGUF fixtures in
 * code (TestGgufBuilder, forward.rs:655-727); these build the benchmark
 * models. Weights are N(0, sigma) from a counter-based generator (splitmix64
 * + Box-Muller) keyed by (seed, tensor index, element index); quantisers
 * emit bytes under the reference's dequant semantics (dequant.rs:62-199). */
typedef struct ifx_synth_spec {
  uint32_t vocab, dim, n_layers, n_heads, n_kv_heads, ffn, context;
  float rope_base, norm_eps, sigma;
  int mix;  /* 0: every matmul weight and token_embd/output Q8_0 (tiny);
               1: Q4_K_M mix (Q6_K for attn_v, even-layer ffn_down and the
                  output/tied embedding, Q4_K elsewhere);
               2: all Q4_0 (for tests) */
  int tied; /* 1: no output.weight (logits use token_embd, forward.rs:573) */
  uint64_t seed;
  int threads; /* host threads for generation (0 = all) */
} ifx_synth_spec;
ifx_status ifx_synth_gguf(const ifx_synth_spec *spec, void **bytes_out,
                          size_t *len_out);
void ifx_synth_free(void *bytes);
/* Quantise n f32 values (n a multiple of the block size) into GGUF bytes. */
ifx_status ifx_quantize(int type, const float *x, size_t n, void *out);
/* The weight generator itself: out[i] = N(0, sigma) sample i of `stream`. */
ifx_status ifx_synth_normal(uint64_t seed, uint64_t stream, float sigma,
                            float *out, size_t n);

#ifdef __cplusplus
}
#endif
#endif /* INFEROX_H */
