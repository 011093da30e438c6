// extern "C" entry points of include/inferox.h.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <new>
#include <string>

#include "dense.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "model.h"
#include "ops.cuh"
#include "tp.h"

struct ifx_model {
  ifx::Model m;
};
struct ifx_kv {
  ifx::KvCache kv;
};
struct ifx_qmatrix {
  ifx::QMatrix q;
};
struct ifx_kv_batch {
  ifx::KvBatch kb;
};

namespace ifx {

static thread_local std::string g_last_error;

void set_error(const std::string &msg) { g_last_error = msg; }

ifx_status fail(ifx_status s, const std::string &msg) {
  g_last_error = msg;
  return s;
}

ifx_status cuda_fail(cudaError_t e, const char *what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  if (e == cudaErrorMemoryAllocation) return IFX_ERR_OUT_OF_MEMORY;
  return IFX_ERR_CUDA;
}

}  // namespace ifx

using namespace ifx;

#define IFX_GUARD(body)                                                   \
  try {                                                                   \
    body                                                                  \
  } catch (const std::bad_alloc &) {                                      \
    return fail(IFX_ERR_OUT_OF_MEMORY, "host allocation failed");         \
  } catch (const std::exception &ex) {                                    \
    return fail(IFX_ERR_INVALID_ARGUMENT, ex.what());                     \
  }

static cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

const char *ifx_last_error(void) { return g_last_error.c_str(); }

const char *ifx_status_name(ifx_status s) {
  switch (s) {
    case IFX_OK: return "Ok";
    case IFX_ERR_IO: return "Io";
    case IFX_ERR_INVALID_MAGIC: return "InvalidMagic";
    case IFX_ERR_UNSUPPORTED_VERSION: return "UnsupportedVersion";
    case IFX_ERR_UNKNOWN_VALUE_TYPE: return "UnknownValueType";
    case IFX_ERR_UNKNOWN_TENSOR_TYPE: return "UnknownTensorType";
    case IFX_ERR_INVALID_UTF8: return "InvalidUtf8";
    case IFX_ERR_INVALID_SHAPE: return "InvalidShape";
    case IFX_ERR_UNEXPECTED_EOF: return "UnexpectedEof";
    case IFX_ERR_TENSOR_NOT_FOUND: return "TensorNotFound";
    case IFX_ERR_INVALID_TENSOR_INDEX: return "InvalidTensorIndex";
    case IFX_ERR_TENSOR_OFFSET_OVERFLOW: return "TensorOffsetOverflow";
    case IFX_ERR_UNSUPPORTED_ARCHITECTURE: return "UnsupportedArchitecture";
    case IFX_ERR_SHAPE: return "Shape";
    case IFX_ERR_CUDA: return "Cuda";
    case IFX_ERR_NCCL: return "Nccl";
    case IFX_ERR_TIMEOUT: return "Timeout";
    case IFX_ERR_INVALID_ARGUMENT: return "InvalidArgument";
    case IFX_ERR_OUT_OF_MEMORY: return "OutOfMemory";
    case IFX_ERR_UNSUPPORTED: return "Unsupported";
    case IFX_ERR_JSON: return "Json";
    case IFX_ERR_UNSUPPORTED_MODEL: return "UnsupportedModel";
  }
  return "Unknown";
}

int ifx_version(void) { return (0 << 16) | 1; }

void ifx_load_opts_default(ifx_load_opts *o) {
  if (!o) return;
  memset(o, 0, sizeof(*o));
  o->device = 0;
  o->tp_size = 1;
  o->tp_rank = 0;
  o->nccl_comm = nullptr;
  o->rope_compat = 1;
  o->use_graphs = 1;
  o->persistent_decode = 1;
}

ifx_status ifx_model_load_mem(const void *bytes, size_t len, const ifx_load_opts *opts,
                              ifx_model **out) {
  if (!bytes || !out) return fail(IFX_ERR_INVALID_ARGUMENT, "model_load_mem: null argument");
  IFX_GUARD({
    ifx_load_opts o;
    ifx_load_opts_default(&o);
    if (opts) o = *opts;
    ifx_model *m = new ifx_model();
    ifx_status s = m->m.load(static_cast<const uint8_t *>(bytes), len, o);
    if (s != IFX_OK) {
      std::string msg = g_last_error;
      delete m;
      g_last_error = msg;
      *out = nullptr;
      return s;
    }
    *out = m;
    return IFX_OK;
  })
}

ifx_status ifx_model_load(const char *path, const ifx_load_opts *opts, ifx_model **out) {
  if (!path || !out) return fail(IFX_ERR_INVALID_ARGUMENT, "model_load: null argument");
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(IFX_ERR_IO, std::string("io error: cannot open ") + path);
  struct stat sb;
  if (fstat(fd, &sb) != 0) {
    close(fd);
    return fail(IFX_ERR_IO, std::string("io error: cannot stat ") + path);
  }
  const size_t len = (size_t)sb.st_size;
  void *p = len ? mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
  close(fd);
  if (len && p == MAP_FAILED) return fail(IFX_ERR_IO, std::string("io error: mmap ") + path);
  static const uint8_t empty[1] = {0};
  ifx_status s = ifx_model_load_mem(len ? p : empty, len, opts, out);
  if (len) munmap(p, len);
  return s;
}

void ifx_model_free(ifx_model *m) { delete m; }

ifx_status ifx_model_config(const ifx_model *m, ifx_config *out) {
  if (!m || !out) return fail(IFX_ERR_INVALID_ARGUMENT, "model_config: null argument");
  *out = m->m.cfg;
  return IFX_OK;
}

uint64_t ifx_model_decode_weight_bytes(const ifx_model *m) { return m ? m->m.decode_bytes : 0; }

ifx_status ifx_kv_create(ifx_model *m, size_t max_seq_len, ifx_kv **out) {
  if (!m || !out || !max_seq_len) return fail(IFX_ERR_INVALID_ARGUMENT, "kv_create: bad argument");
  IFX_GUARD({
    ifx_kv *kv = new ifx_kv();
    ifx_status s = kv->kv.create(&m->m, max_seq_len);
    if (s != IFX_OK) {
      delete kv;
      return s;
    }
    *out = kv;
    return IFX_OK;
  })
}

void ifx_kv_free(ifx_kv *kv) { delete kv; }

ifx_status ifx_kv_clear(ifx_kv *kv) {
  if (!kv) return fail(IFX_ERR_INVALID_ARGUMENT, "kv_clear: null");
  return kv->kv.clear();
}

size_t ifx_kv_len(const ifx_kv *kv) { return kv ? kv->kv.len : 0; }

int ifx_kv_decode_kernels(const ifx_kv *kv) {
  if (!kv || !kv->kv.m) return 0;
  if (kv->kv.mega_ready) return 1;
  if (!kv->kv.mega_tried && kv->kv.m->opts.persistent_decode) return 0;  // not decided yet
  return 3 + 5 * (int)kv->kv.m->cfg.n_layers;
}

ifx_status ifx_kv_read(const ifx_kv *kv, size_t layer, int which_v, float *out_host) {
  if (!kv || !out_host) return fail(IFX_ERR_INVALID_ARGUMENT, "kv_read: null");
  return kv->kv.m->kv_read(kv->kv, layer, which_v, out_host);
}

ifx_status ifx_prefill(ifx_model *m, ifx_kv *kv, const uint32_t *ids, size_t n, float *logits_host,
                       int last_row_only) {
  if (!m || !kv || (!ids && n)) return fail(IFX_ERR_INVALID_ARGUMENT, "prefill: null argument");
  if (kv->kv.m != &m->m) return fail(IFX_ERR_INVALID_ARGUMENT, "prefill: kv belongs to another model");
  IFX_GUARD({ return m->m.prefill(kv->kv, ids, n, logits_host, last_row_only); })
}

ifx_status ifx_forward(ifx_model *m, const uint32_t *ids, size_t n, float *logits_host,
                       int last_row_only) {
  if (!m || (!ids && n)) return fail(IFX_ERR_INVALID_ARGUMENT, "forward: null argument");
  IFX_GUARD({ return m->m.forward(ids, n, logits_host, last_row_only); })
}

ifx_status ifx_decode_step(ifx_model *m, ifx_kv *kv, uint32_t token, float *logits_host) {
  if (!m || !kv) return fail(IFX_ERR_INVALID_ARGUMENT, "decode_step: null argument");
  if (kv->kv.m != &m->m) return fail(IFX_ERR_INVALID_ARGUMENT, "decode_step: kv belongs to another model");
  IFX_GUARD({ return m->m.decode_step(kv->kv, token, logits_host); })
}

ifx_status ifx_generate(ifx_model *m, ifx_kv *kv, const uint32_t *prompt, size_t n_prompt,
                        size_t max_tokens, uint32_t *out_tokens) {
  if (!m || !kv || !prompt || (!out_tokens && max_tokens))
    return fail(IFX_ERR_INVALID_ARGUMENT, "generate: null argument");
  IFX_GUARD({ return m->m.generate(kv->kv, prompt, n_prompt, max_tokens, out_tokens); })
}

ifx_status ifx_decode_greedy(ifx_model *m, ifx_kv *kv, uint32_t token, size_t n_steps,
                             uint32_t *out_tokens, float *device_ms) {
  if (!m || !kv) return fail(IFX_ERR_INVALID_ARGUMENT, "decode_greedy: null argument");
  if (kv->kv.m != &m->m) return fail(IFX_ERR_INVALID_ARGUMENT, "decode_greedy: kv belongs to another model");
  IFX_GUARD({ return m->m.decode_greedy(kv->kv, token, n_steps, out_tokens, device_ms); })
}

static ifx_status kv_batch_create(ifx_model *m, size_t max_seq_len, int batch, size_t pages,
                                  ifx_kv_batch **out) {
  ifx_kv_batch *kb = new ifx_kv_batch();
  ifx_status s = kb->kb.create(&m->m, max_seq_len, batch, pages);
  if (s != IFX_OK) {
    delete kb;
    return s;
  }
  *out = kb;
  return IFX_OK;
}

ifx_status ifx_kv_batch_create(ifx_model *m, size_t max_seq_len, int batch, ifx_kv_batch **out) {
  if (!m || !out || !max_seq_len) return fail(IFX_ERR_INVALID_ARGUMENT, "kv_batch_create: bad argument");
  IFX_GUARD({ return kv_batch_create(m, max_seq_len, batch, 0, out); })
}

ifx_status ifx_kv_batch_create_paged(ifx_model *m, size_t max_seq_len, int batch, size_t n_pages,
                                     ifx_kv_batch **out) {
  if (!m || !out || !max_seq_len || !n_pages || n_pages > (size_t)INT32_MAX)
    return fail(IFX_ERR_INVALID_ARGUMENT, "kv_batch_create_paged: bad argument");
  IFX_GUARD({ return kv_batch_create(m, max_seq_len, batch, n_pages, out); })
}

ifx_status ifx_kv_batch_pages(const ifx_kv_batch *kb, size_t *free_pages, size_t *total_pages) {
  if (!kb || !free_pages || !total_pages) return fail(IFX_ERR_INVALID_ARGUMENT, "kv_batch_pages: null argument");
  *free_pages = kb->kb.free_pages.size();
  *total_pages = kb->kb.n_pages;
  return IFX_OK;
}

void ifx_kv_batch_free(ifx_kv_batch *kb) { delete kb; }

ifx_status ifx_kv_batch_len(const ifx_kv_batch *kb, int seq, size_t *len) {
  if (!kb || !len || seq < 0 || seq >= kb->kb.batch)
    return fail(IFX_ERR_INVALID_ARGUMENT, "kv_batch_len: bad argument");
  *len = kb->kb.len[(size_t)seq];
  return IFX_OK;
}

ifx_status ifx_prefill_seq(ifx_model *m, ifx_kv_batch *kb, int seq, const uint32_t *ids, size_t n,
                           float *logits_host, int last_row_only) {
  if (!m || !kb || (!ids && n)) return fail(IFX_ERR_INVALID_ARGUMENT, "prefill_seq: null argument");
  if (kb->kb.m != &m->m) return fail(IFX_ERR_INVALID_ARGUMENT, "prefill_seq: batch belongs to another model");
  IFX_GUARD({ return m->m.prefill_seq(kb->kb, seq, ids, n, logits_host, last_row_only); })
}

ifx_status ifx_decode_step_batch(ifx_model *m, ifx_kv_batch *kb, const uint32_t *tokens,
                                 float *logits_host, uint32_t *argmax_host) {
  if (!m || !kb || !tokens) return fail(IFX_ERR_INVALID_ARGUMENT, "decode_step_batch: null argument");
  if (kb->kb.m != &m->m) return fail(IFX_ERR_INVALID_ARGUMENT, "decode_step_batch: batch belongs to another model");
  IFX_GUARD({ return m->m.decode_batch(kb->kb, tokens, logits_host, argmax_host); })
}

ifx_status ifx_decode_step_batch_seqs(ifx_model *m, ifx_kv_batch *kb, const int *seqs, int n,
                                      const uint32_t *tokens, float *logits_host,
                                      uint32_t *argmax_host) {
  if (!m || !kb || !seqs || !tokens)
    return fail(IFX_ERR_INVALID_ARGUMENT, "decode_step_batch_seqs: null argument");
  if (kb->kb.m != &m->m) return fail(IFX_ERR_INVALID_ARGUMENT, "decode_step_batch_seqs: batch belongs to another model");
  IFX_GUARD({ return m->m.decode_batch_seqs(kb->kb, seqs, n, tokens, logits_host, argmax_host); })
}

ifx_status ifx_kv_batch_reset(ifx_model *m, ifx_kv_batch *kb, int seq) {
  if (!m || !kb) return fail(IFX_ERR_INVALID_ARGUMENT, "kv_batch_reset: null argument");
  if (kb->kb.m != &m->m) return fail(IFX_ERR_INVALID_ARGUMENT, "kv_batch_reset: batch belongs to another model");
  IFX_GUARD({ return m->m.reset_seq(kb->kb, seq); })
}

ifx_status ifx_decode_greedy_batch(ifx_model *m, ifx_kv_batch *kb, const uint32_t *tokens,
                                   size_t n_steps, uint32_t *out_tokens, float *device_ms) {
  if (!m || !kb || !tokens) return fail(IFX_ERR_INVALID_ARGUMENT, "decode_greedy_batch: null argument");
  if (kb->kb.m != &m->m) return fail(IFX_ERR_INVALID_ARGUMENT, "decode_greedy_batch: batch belongs to another model");
  IFX_GUARD({ return m->m.decode_greedy_batch(kb->kb, tokens, n_steps, out_tokens, device_ms); })
}

ifx_status ifx_bench_kernel(ifx_model *m, ifx_kv *kv, const char *which, int reps,
                            float *ms_per_launch, uint64_t *bytes_per_launch) {
  if (!m || !kv || !which || !ms_per_launch || !bytes_per_launch)
    return fail(IFX_ERR_INVALID_ARGUMENT, "bench_kernel: null argument");
  IFX_GUARD({ return m->m.bench_kernel(kv->kv, which, reps, ms_per_launch, bytes_per_launch); })
}

ifx_status ifx_sample(ifx_model *m, const ifx_sampler *s, uint64_t seed, uint64_t offset,
                      uint32_t *token_out) {
  if (!m || !s || !token_out) return fail(IFX_ERR_INVALID_ARGUMENT, "sample: null argument");
  Model &M = m->m;
  IFX_CUDA(cudaSetDevice(M.device));
  uint32_t *d = nullptr;
  IFX_CUDA(cudaMalloc(&d, sizeof(uint32_t)));
  ifx_status st;
  if (s->temperature == 0.0f) {
    unsigned long long *key = nullptr;
    IFX_CUDA(cudaMalloc(&key, sizeof(unsigned long long)));
    cudaMemsetAsync(key, 0, sizeof(unsigned long long), M.stream);
    st = op_argmax(M.logits, M.cfg.vocab_size, key, d, M.stream);
    cudaStreamSynchronize(M.stream);
    cudaFree(key);
  } else {
    st = op_sample_philox(M.logits, M.cfg.vocab_size, s->temperature, s->top_k, s->top_p, seed,
                          offset, d, M.stream);
  }
  if (st == IFX_OK) {
    cudaError_t e = cudaMemcpyAsync(token_out, d, sizeof(uint32_t), cudaMemcpyDeviceToHost, M.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(M.stream);
    if (e != cudaSuccess) st = cuda_fail(e, "sample");
  }
  cudaFree(d);
  return st;
}

// ----------------------------------------------------------------- ops ----
ifx_status ifx_op_dequantize(int type, const void *bytes_dev, size_t nbytes, float *out_dev,
                             size_t n_out, void *stream) {
  if ((!bytes_dev && nbytes) || (!out_dev && n_out))
    return fail(IFX_ERR_INVALID_ARGUMENT, "dequantize: null pointer");
  return op_dequantize(type, static_cast<const uint8_t *>(bytes_dev), nbytes, out_dev, n_out, S(stream));
}

ifx_status ifx_op_matmul(const float *a, const float *b, float *c, size_t m, size_t n, size_t k,
                         void *stream) {
  if (!a || !b || !c) return fail(IFX_ERR_INVALID_ARGUMENT, "matmul: null pointer");
  return op_matmul(a, b, c, m, n, k, S(stream));
}

ifx_status ifx_op_matmul_t(const float *a, const float *b, float *c, size_t m, size_t n, size_t k,
                           void *stream) {
  if (!a || !b || !c) return fail(IFX_ERR_INVALID_ARGUMENT, "matmul_t: null pointer");
  return op_matmul_t(a, b, c, m, n, k, S(stream));
}

ifx_status ifx_qmatrix_create(int type, const void *gguf_bytes_host, size_t nbytes, size_t rows,
                              size_t cols, int device, ifx_qmatrix **out) {
  if (!gguf_bytes_host || !out) return fail(IFX_ERR_INVALID_ARGUMENT, "qmatrix_create: null");
  IFX_GUARD({
    ifx_qmatrix *w = new ifx_qmatrix();
    w->q.device = device;
    const bool dense = dense_type(type);  // F32 / F16 / Q8_K: dequantised f32 rows
    if (dense) make_dense_layout((int64_t)rows, (int64_t)cols, type, &w->q.L);
    if (!dense && !make_layout(type, (int64_t)rows, (int64_t)cols, &w->q.L)) {
      delete w;
      return fail(IFX_ERR_UNSUPPORTED, "qmatrix_create: unsupported type or shape");
    }
    BlockInfo b = block_info(type);
    if ((uint64_t)rows * cols / b.elems * b.bytes != nbytes) {
      delete w;
      return fail(IFX_ERR_UNEXPECTED_EOF, "qmatrix_create: byte count does not match the shape");
    }
    cudaSetDevice(device);
    uint8_t *staging = nullptr;
    cudaError_t e = cudaMalloc(&staging, nbytes);
    if (e == cudaSuccess) e = cudaMemcpy(staging, gguf_bytes_host, nbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&w->q.d, w->q.L.total_bytes);
    ifx_status s = e != cudaSuccess ? cuda_fail(e, "qmatrix_create")
                   : dense ? op_dequantize(type, staging, nbytes, reinterpret_cast<float *>(w->q.d),
                                           rows * cols, 0)
                           : repack_to_device(w->q.L, staging, w->q.d, 0);
    if (s == IFX_OK) {
      e = cudaDeviceSynchronize();
      if (e != cudaSuccess) s = cuda_fail(e, "qmatrix repack");
    }
    if (staging) cudaFree(staging);
    if (s != IFX_OK) {
      if (w->q.d) cudaFree(w->q.d);
      delete w;
      return s;
    }
    *out = w;
    return IFX_OK;
  })
}

void ifx_qmatrix_free(ifx_qmatrix *w) {
  if (!w) return;
  if (w->q.d) cudaFree(w->q.d);
  delete w;
}

ifx_status ifx_op_matmul_t_q(const float *a_dev, const ifx_qmatrix *w, float *c_dev, size_t m,
                             void *stream) {
  if (!a_dev || !w || !c_dev) return fail(IFX_ERR_INVALID_ARGUMENT, "matmul_t_q: null");
  if (m == 0) return IFX_OK;
  cudaStream_t st = S(stream);
  const QMatrix &W = w->q;
  int *err = nullptr;
  IFX_CUDA(cudaMalloc(&err, sizeof(int)));
  IFX_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st));
  ifx_status s = IFX_OK;
  if (m == 1) {
    IFX_CUDA(cudaMemsetAsync(c_dev, 0, W.L.rows * sizeof(float), st));
    GemvPlan p;
    const QMatrix *mats[1] = {&W};
    float *ys[1] = {c_dev};
    s = gemv_plan(mats, ys, 1, GEMV_PLAIN, a_dev, nullptr, nullptr, 0.f, err, &p);
    if (s == IFX_OK) s = gemv_launch(p, st, false);
    cudaStreamSynchronize(st);
    gemv_plan_free(&p);
  } else {
    void *xf = nullptr;
    IFX_CUDA(cudaMalloc(&xf, std::max(gemm_xfrag_bytes((int64_t)m, W.L.cols),
                                      (size_t)m * W.L.cols * sizeof(float))));
    s = W.L.dense ? dense_stage(a_dev, nullptr, nullptr, 0.f, GX_PLAIN, (int64_t)m, W.L.cols, xf, st)
                  : gemm_stage_x(a_dev, nullptr, nullptr, 0.f, GX_PLAIN, (int64_t)m, W.L.cols, xf, st);
    if (s == IFX_OK) s = gemm_run(W, xf, (int64_t)m, c_dev, W.L.rows, 0, err, st);
    cudaStreamSynchronize(st);
    cudaFree(xf);
  }
  int h = 0;
  cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(err);
  if (s == IFX_OK && h) s = fail(IFX_ERR_TIMEOUT, "matmul_t_q: a bounded device wait gave up");
  if (s == IFX_OK) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) s = cuda_fail(e, "matmul_t_q");
  }
  return s;
}

// Times the fused dequant matmul the token loop runs at batch m: the batch-1
// GEMV (x staged inside the kernel), the small-batch GEMM for m <= 32 (decode
// of several sequences) or the prefill GEMM above that, each with its input
// staging launch. Every timed launch is bracketed by its own events; between
// launches a 256 MB buffer is written so the weights come from HBM.
static ifx_status bench_matmul_t_q(const float *a_dev, const QMatrix &W, float *c_dev, size_t m,
                                 int reps, float *ms_per_call) {
  IFX_CUDA(cudaSetDevice(W.device));
  cudaStream_t st = nullptr;
  IFX_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  constexpr size_t kFlush = 256ull << 20;
  int *err = nullptr;
  void *flush = nullptr, *xf = nullptr;
  GemvPlan p;
  bool planned = false;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float total = 0.f;
  ifx_status s = IFX_OK;
  auto cuda_ok = [&](cudaError_t e, const char *what) {
    if (e != cudaSuccess && s == IFX_OK) s = cuda_fail(e, what);
    return s == IFX_OK;
  };
  if (cuda_ok(cudaMalloc(&err, sizeof(int)), "cudaMalloc") &&
      cuda_ok(cudaMemsetAsync(err, 0, sizeof(int), st), "cudaMemset") &&
      cuda_ok(cudaMalloc(&flush, kFlush), "cudaMalloc") && cuda_ok(cudaEventCreate(&e0), "event") &&
      cuda_ok(cudaEventCreate(&e1), "event")) {
    const int64_t M = (int64_t)m, K = W.L.cols, R = W.L.rows;
    const bool small = m > 1 && M <= kGemmSmallMax;
    if (m == 1) {
      const QMatrix *mats[1] = {&W};
      float *ys[1] = {c_dev};
      s = gemv_plan(mats, ys, 1, GEMV_PLAIN, a_dev, nullptr, nullptr, 0.f, err, &p);
      planned = s == IFX_OK;
    } else {
      cuda_ok(cudaMalloc(&xf, small ? gemm_small_xfrag_bytes(M, K) : gemm_xfrag_bytes(M, K)), "cudaMalloc");
    }
    for (int r = -1; r < reps && s == IFX_OK; ++r) {  // r = -1: untimed first launch
      // outputs the kernels accumulate into start at zero (outside the timing)
      if (m == 1 || small) cuda_ok(cudaMemsetAsync(c_dev, 0, sizeof(float) * (size_t)(M * R), st), "cudaMemset");
      cuda_ok(cudaMemsetAsync(flush, r & 0xff, kFlush, st), "cudaMemset");
      if (s != IFX_OK) break;
      cuda_ok(cudaEventRecord(e0, st), "event");
      if (m == 1) {
        s = gemv_launch(p, st, false);
      } else if (small) {
        s = gemm_small_stage_x(a_dev, nullptr, nullptr, 0.f, GX_PLAIN, M, K, xf, st);
        if (s == IFX_OK) s = gemm_small_run(W, xf, M, c_dev, R, err, st);
      } else {
        s = gemm_stage_x(a_dev, nullptr, nullptr, 0.f, GX_PLAIN, M, K, xf, st);
        if (s == IFX_OK) s = gemm_run(W, xf, M, c_dev, R, 0, err, st);
      }
      if (s != IFX_OK || !cuda_ok(cudaEventRecord(e1, st), "event") ||
          !cuda_ok(cudaEventSynchronize(e1), "event"))
        break;
      float t = 0.f;
      cuda_ok(cudaEventElapsedTime(&t, e0, e1), "event");
      if (r >= 0) total += t;
    }
    cudaStreamSynchronize(st);
    int h = 0;
    cuda_ok(cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost), "cudaMemcpy");
    if (s == IFX_OK && h) s = fail(IFX_ERR_TIMEOUT, "bench_matmul_t_q: a bounded device wait gave up");
  }
  if (planned) gemv_plan_free(&p);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaFree(xf);
  cudaFree(flush);
  cudaFree(err);
  cudaStreamDestroy(st);
  if (s == IFX_OK) *ms_per_call = total / (float)reps;
  return s;
}

ifx_status ifx_bench_matmul_t_q(const float *a_dev, const ifx_qmatrix *w, float *c_dev, size_t m,
                                int reps, float *ms_per_call) {
  if (!a_dev || !w || !c_dev || !ms_per_call) return fail(IFX_ERR_INVALID_ARGUMENT, "bench_matmul_t_q: null");
  if (m == 0 || reps < 1) return fail(IFX_ERR_INVALID_ARGUMENT, "bench_matmul_t_q: m and reps must be >= 1");
  if (w->q.L.dense) return fail(IFX_ERR_UNSUPPORTED, "bench_matmul_t_q: times the fused quantised kernels only");
  IFX_GUARD({ return bench_matmul_t_q(a_dev, w->q, c_dev, m, reps, ms_per_call); })
}

ifx_status ifx_op_rms_norm_rows(float *x, const float *w, float eps, size_t rows, size_t hidden,
                                void *stream) {
  if (!x || !w) return fail(IFX_ERR_INVALID_ARGUMENT, "rms_norm_rows: null");
  return op_rms_norm_rows(x, w, eps, rows, hidden, S(stream));
}

ifx_status ifx_op_silu(float *x, size_t n, void *stream) {
  if (!x && n) return fail(IFX_ERR_INVALID_ARGUMENT, "silu: null");
  return op_silu(x, n, S(stream));
}

ifx_status ifx_op_swiglu(const float *gate, const float *up, float *out, size_t n, void *stream) {
  if ((!gate || !up || !out) && n) return fail(IFX_ERR_INVALID_ARGUMENT, "swiglu: null");
  return op_swiglu(gate, up, out, n, S(stream));
}

ifx_status ifx_op_add_in_place(float *out, const float *b, size_t n, void *stream) {
  if ((!out || !b) && n) return fail(IFX_ERR_INVALID_ARGUMENT, "add_in_place: null");
  return op_add(out, b, n, S(stream));
}

ifx_status ifx_op_softmax_rows(float *x, size_t rows, size_t cols, void *stream) {
  if (!x && rows * cols) return fail(IFX_ERR_INVALID_ARGUMENT, "softmax_rows: null");
  return op_softmax_rows(x, rows, cols, S(stream));
}

ifx_status ifx_op_embedding_lookup(const float *emb, size_t emb_len, const uint32_t *ids,
                                   size_t n_ids, size_t hidden, float *out, void *stream) {
  if ((!emb || !ids || !out) && n_ids) return fail(IFX_ERR_INVALID_ARGUMENT, "embedding_lookup: null");
  int *err = nullptr;
  IFX_CUDA(cudaMalloc(&err, sizeof(int)));
  IFX_CUDA(cudaMemsetAsync(err, 0, sizeof(int), S(stream)));
  ifx_status s = op_embedding_lookup(emb, emb_len, ids, n_ids, hidden, out, err, S(stream));
  int h = 0;
  cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, S(stream));
  cudaStreamSynchronize(S(stream));
  cudaFree(err);
  if (s == IFX_OK && h)
    return fail(IFX_ERR_INVALID_TENSOR_INDEX, "embedding_lookup: token id out of vocabulary bounds");
  return s;
}

ifx_status ifx_op_rope(float *x, size_t seq_len, size_t n_heads, size_t head_dim, size_t rope_dim,
                       float base, size_t pos0, void *stream) {
  if (!x && seq_len) return fail(IFX_ERR_INVALID_ARGUMENT, "rope: null");
  return op_rope(x, seq_len, n_heads, head_dim, rope_dim, base, pos0, S(stream));
}

ifx_status ifx_op_argmax(const float *x, size_t n, uint32_t *out_dev, void *stream) {
  if (!x || !out_dev) return fail(IFX_ERR_INVALID_ARGUMENT, "argmax: null");
  unsigned long long *key = nullptr;
  IFX_CUDA(cudaMallocAsync(&key, sizeof(unsigned long long), S(stream)));
  IFX_CUDA(cudaMemsetAsync(key, 0, sizeof(unsigned long long), S(stream)));
  ifx_status s = op_argmax(x, n, key, out_dev, S(stream));
  cudaFreeAsync(key, S(stream));
  return s;
}

ifx_status ifx_op_sample_u(const float *logits_dev, size_t n, const ifx_sampler *s, float u,
                           uint32_t *token_host, void *stream) {
  if (!logits_dev || !s || !token_host) return fail(IFX_ERR_INVALID_ARGUMENT, "sample_u: null");
  uint32_t *d = nullptr;
  IFX_CUDA(cudaMalloc(&d, sizeof(uint32_t)));
  ifx_status st;
  if (s->temperature == 0.0f) {
    unsigned long long *key = nullptr;
    IFX_CUDA(cudaMalloc(&key, sizeof(unsigned long long)));
    cudaMemsetAsync(key, 0, sizeof(unsigned long long), S(stream));
    st = op_argmax(logits_dev, n, key, d, S(stream));
    cudaStreamSynchronize(S(stream));
    cudaFree(key);
  } else {
    st = op_sample_u(logits_dev, n, s->temperature, s->top_k, s->top_p, u, d, S(stream));
  }
  if (st == IFX_OK) {
    cudaError_t e = cudaMemcpyAsync(token_host, d, sizeof(uint32_t), cudaMemcpyDeviceToHost, S(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(S(stream));
    if (e != cudaSuccess) st = cuda_fail(e, "sample_u");
  }
  cudaFree(d);
  return st;
}

ifx_status ifx_op_sample_u_static(const float *logits_dev, size_t n, const ifx_sampler *s,
                                  float u, uint32_t *token_dev, void *stream) {
  if (!logits_dev || !s || !token_dev) return fail(IFX_ERR_INVALID_ARGUMENT, "sample_u_static: null");
  return op_sample_u_static(logits_dev, n, s->temperature, s->top_k, s->top_p, u, token_dev,
                            S(stream));
}

ifx_status ifx_tp_unique_id(void *id_out) {
  if (!id_out) return fail(IFX_ERR_INVALID_ARGUMENT, "tp_unique_id: null");
  const NcclApi *api = nullptr;
  IFX_TRY(nccl_api(&api));
  ncclUniqueId id;
  IFX_NCCL(api, api->GetUniqueId(&id));
  memcpy(id_out, &id, sizeof(id));
  return IFX_OK;
}

ifx_status ifx_tp_comm_create(const void *id, int nranks, int rank, int device, void **comm_out) {
  if (!id || !comm_out || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(IFX_ERR_INVALID_ARGUMENT, "tp_comm_create: bad argument");
  const NcclApi *api = nullptr;
  IFX_TRY(nccl_api(&api));
  IFX_CUDA(cudaSetDevice(device));
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  IFX_NCCL(api, api->CommInitRank(&c, nranks, uid, rank));
  *comm_out = c;
  return IFX_OK;
}

void ifx_tp_comm_destroy(void *comm) {
  const NcclApi *api = nullptr;
  if (!comm || tp_take_aborted(comm)) return;  // an aborted communicator is already freed
  if (nccl_api(&api) == IFX_OK) api->CommDestroy((ncclComm_t)comm);
}

ifx_status ifx_tp_shard(int type, const void *gguf_bytes, size_t nbytes, size_t rows, size_t cols,
                        int split_k, int tp, int rank, void *out, size_t *out_bytes) {
  if (!gguf_bytes || !out_bytes) return fail(IFX_ERR_INVALID_ARGUMENT, "tp_shard: null");
  IFX_GUARD({
    std::vector<uint8_t> sh;
    IFX_TRY(tp_shard(type, static_cast<const uint8_t *>(gguf_bytes), nbytes, rows, cols, split_k,
                     tp, rank, &sh));
    *out_bytes = sh.size();
    if (out) memcpy(out, sh.data(), sh.size());
    return IFX_OK;
  })
}

}  // extern "C"
