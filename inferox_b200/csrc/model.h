// Model / KV cache objects behind ifx_model and ifx_kv.
#pragma once
#include <array>
#include <string>
#include <vector>

#include "common.cuh"
#include "decode_mega.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "repack.h"

namespace ifx {

struct Layer {  // Layer (src/model/mod.rs:18-31), weights resident on the device
  float *attn_norm = nullptr, *ffn_norm = nullptr;
  QMatrix wq, wk, wv, wo, w1, w3, w2;
};

struct Model;

struct KvCache {  // KvCache (src/model/cache.rs:7-14), f16 on the device
  Model *m = nullptr;
  size_t max_seq = 0, len = 0, per_layer = 0;
  __half *k = nullptr, *v = nullptr;  // [layer][kv_head][max_seq][head_dim]
  int *pos = nullptr;                 // device copy of len (read by the kernels)
  uint32_t *tokens = nullptr;         // generated tokens (device)
  cudaGraphExec_t graph = nullptr;    // captured decode step for this cache
  MegaPlan mega;                      // persistent decode plan for this cache
  bool mega_ready = false, mega_tried = false;
  float *part_o = nullptr;            // split-K partials of the persistent kernel
  float2 *part_ml = nullptr;
  unsigned *bar = nullptr;
  bool owner = true;                  // false: a view into a KvBatch's memory
  // a view of one sequence of a paged KvBatch: k / v are the page pool,
  // position t lives in page page_table[t / page_rows] (device array)
  const int *page_table = nullptr;
  int page_rows = 0;
  int64_t page_stride = 0;
  int dev = -1;                       // device of the allocations (the destructor must
                                      // not read the model: it may be freed first)
  ifx_status create(Model *model, size_t max_seq_len);
  ifx_status clear();
  ~KvCache();
};

// B independent sequences decoded together, so one step reads every weight
// once for all of them (the reference's KvCache is single-sequence,
// src/model/cache.rs:7-13). Sequence b's cache has the layout of a KvCache
// at k/v + b * n_layers * per_layer, so a prompt is prefilled through a
// KvCache view of it.
struct KvBatch {
  Model *m = nullptr;
  int batch = 0, ns = 1;
  size_t max_seq = 0, per_layer = 0;
  __half *k = nullptr, *v = nullptr;  // [batch][layer][kv_head][max_seq][head_dim]
  int *pos = nullptr;                 // device [batch]: each sequence's length
  std::vector<size_t> len;            // host mirror of pos
  // step workspace: [batch][...] rows
  float *x = nullptr, *qkv = nullptr, *attn = nullptr, *gate = nullptr, *up = nullptr;
  float *logits = nullptr;
  float *part_o = nullptr;
  float2 *part_ml = nullptr;
  int *counters = nullptr;
  uint8_t *xf = nullptr;
  uint32_t *ids = nullptr, *out = nullptr;  // the step's input tokens and argmax
  int *slots = nullptr;                     // sequences of a subset step
  unsigned long long *keys = nullptr;       // per-sequence argmax keys
  int dev = -1;                             // device of the allocations
  // Paged mode (no reference counterpart): k / v are a pool of n_pages pages
  // of page_rows positions, each holding those rows for every layer and kv
  // head ([layer][kv_head][page_rows][head_dim]); a sequence takes pages
  // from the pool as it grows and returns them on reset, so the pool can be
  // far smaller than batch * max_seq rows. Sequence b's position t is row
  // t % page_rows of page table[b * max_pages + t / page_rows].
  bool paged = false;
  int page_rows = 0, max_pages = 0;
  size_t n_pages = 0;
  int64_t page_stride = 0;                  // elements per page
  int *table_dev = nullptr;                 // [batch][max_pages]
  std::vector<int> table;                   // host mirror
  std::vector<int> free_pages;              // pool pages no sequence holds
  // the full-batch step (kernels + the argmax fed back as the next ids),
  // captured after one eager step has run (first-call attribute setup)
  cudaGraphExec_t graph = nullptr;
  bool warm = false;
  ifx_status create(Model *model, size_t max_seq_len, int nseq, size_t pages = 0);
  // give sequence `seq` pages for positions [0, rows); fails with no change
  // when the pool runs out
  ifx_status reserve(int seq, size_t rows, cudaStream_t st);
  void release(int seq);
  ~KvBatch();
};

struct Model {
  int device = -1;
  ifx_load_opts opts{};
  ifx_config cfg{};  // the checkpoint's (global) config
  // tensor parallelism: this rank's share of the heads, FFN rows and vocab
  int tp = 1, rank = 0;
  void *comm = nullptr;  // ncclComm_t, owned by the caller
  const struct NcclApi *nccl = nullptr;
  uint64_t Hl = 0, Gl = 0, Fl = 0, Vl = 0, v0 = 0;
  float *y = nullptr;               // partial sums of the row-parallel layers
  // the persistent kernel's all-reduce buffers (every rank's, mapped here
  // by CUDA IPC); peers_ok only when every rank mapped every other's
  MegaPeers peers{};
  char *peer_buf = nullptr;
  unsigned *mega_epoch = nullptr;
  bool peers_ok = false;
  ifx_status setup_peers();
  float *logits_local = nullptr;    // this rank's vocab slice (== logits at tp 1)
  unsigned long long *key_global = nullptr;
  float *w_y = nullptr;             // prefill partial sums [n][D]
  float *logits_all_local = nullptr;
  size_t logits_all_local_n = 0;
  cudaStream_t stream = nullptr;
  std::vector<Layer> layers;
  QMatrix out_w;
  float *out_norm = nullptr;
  uint8_t *emb_raw = nullptr;  // token_embd GGUF bytes (exact row dequant)
  int emb_type = 0;
  uint64_t emb_row_bytes = 0;
  // decode state
  float *x = nullptr, *qkv = nullptr, *attn = nullptr, *gu = nullptr, *logits = nullptr;
  int qkv_n = 0;
  float *part_o = nullptr;
  float2 *part_ml = nullptr;
  int *counters = nullptr, ns = 1;
  int *err = nullptr;
  uint32_t *next_token = nullptr;
  unsigned long long *amax_key = nullptr;
  int *amax_count = nullptr, *n_out = nullptr;
  std::vector<GemvPlan> p_qkv, p_wo, p_w13, p_w2;
  // matrices of a fused site whose unit width differs from the first's (a
  // file that mixes Q8_0 with 256-column types in Q/K/V or gate/up): their
  // own plans, run right after the site's plan; empty for usual files
  std::vector<std::vector<GemvPlan>> p_qkv_more, p_w13_more;
  GemvPlan p_logits;
  uint64_t decode_bytes = 0;
  // prefill workspace
  void *ws = nullptr;
  size_t ws_tokens = 0;
  float *w_x = nullptr, *w_q = nullptr, *w_k = nullptr, *w_v = nullptr, *w_attn = nullptr;
  float *w_gate = nullptr, *w_up = nullptr;
  uint8_t *w_xf = nullptr;
  uint32_t *ids_dev = nullptr;
  float *logits_all = nullptr;
  size_t logits_all_n = 0;

  ifx_status load(const uint8_t *bytes, size_t len, const ifx_load_opts &o);
  ifx_status enqueue_decode(KvCache &kv, cudaStream_t st);
  ifx_status build_mega(KvCache &kv);
  // gather_logits: under tensor parallelism, also gather the vocab slices
  // into logits (the persistent kernel leaves each rank's slice only)
  ifx_status run_decode(KvCache &kv, bool gather_logits = true);
  ifx_status step_batch_fed(KvBatch &kb, cudaStream_t st);
  // dense f32 matmul weights (a checkpoint with F32 / F16 / Q8_K matrices):
  // every matrix is kept dequantised and the dense kernels of dense.cu run
  bool dense = false;
  // f(X) staging for the GEMMs: the fused kernels' fragment formats, or the
  // plain f32 rows of the dense path
  ifx_status stage_rows(const float *X, const float *X2, const float *normw, float eps, int mode,
                        int64_t M, int64_t K, void *buf, cudaStream_t st);
  // zero: buffers the following GEMMs accumulate into (zeroed by the
  // staging kernel after the previous grid completes)
  ifx_status stage_small(const float *X, const float *X2, const float *normw, float eps, int mode,
                         int64_t M, int64_t K, void *buf, cudaStream_t st,
                         StageZero zero = StageZero{});
  ifx_status decode_step(KvCache &kv, uint32_t token, float *logits_host);
  ifx_status prefill(KvCache &kv, const uint32_t *ids, size_t n, float *logits_host, int last_row_only);
  ifx_status forward(const uint32_t *ids, size_t n, float *logits_host, int last_row_only);
  ifx_status run_prompt(KvCache *kvp, const uint32_t *ids, size_t n, float *logits_host,
                        int last_row_only);
  ifx_status generate(KvCache &kv, const uint32_t *prompt, size_t n_prompt, size_t max_tokens,
                      uint32_t *out);
  ifx_status kv_read(const KvCache &kv, size_t layer, int which_v, float *out_host);
  ifx_status decode_greedy(KvCache &kv, uint32_t token, size_t n, uint32_t *out, float *device_ms);
  ifx_status bench_kernel(KvCache &kv, const std::string &which, int reps, float *ms,
                          uint64_t *bytes);
  ifx_status prefill_seq(KvBatch &kb, int seq, const uint32_t *ids, size_t n, float *logits_host,
                         int last_row_only);
  // n rows (all kb.batch sequences when n < 0); row i extends sequence
  // slot_dev[i] when slot_dev is set (device array), else sequence i
  ifx_status enqueue_decode_batch(KvBatch &kb, cudaStream_t st, int n = -1,
                                  const int *slot_dev = nullptr);
  ifx_status decode_batch_seqs(KvBatch &kb, const int *seqs, int n, const uint32_t *tokens,
                               float *logits_host, uint32_t *argmax_host);
  ifx_status reset_seq(KvBatch &kb, int seq);
  // the end of a call's device work: a bounded wait that aborts the
  // communicator under tensor parallelism (tp_wait), else a stream sync
  ifx_status step_sync(cudaStream_t st);
  ifx_status tp_usable() const;
  bool comm_aborted = false;
  ifx_status decode_batch(KvBatch &kb, const uint32_t *tokens, float *logits_host,
                          uint32_t *argmax_host);
  ifx_status decode_greedy_batch(KvBatch &kb, const uint32_t *tokens, size_t n, uint32_t *out,
                                 float *device_ms);
  ifx_status ensure_ws(size_t n);
  ifx_status tp_partial_begin(size_t n, cudaStream_t st, float *part = nullptr,
                              const float *resid = nullptr);
  ifx_status tp_partial_end(size_t n, cudaStream_t st, const float *part = nullptr,
                            float *out = nullptr);
  ifx_status check_err();
  ~Model();
};

}  // namespace ifx
