// The token loop on the device: Model::open / prefill / decode_step /
// generate (src/model/forward.rs:496-612, src/model/mod.rs:64-92) behind the
// C ABI of include/inferox.h.
//
// Decode step (batch 1), one CUDA graph per KV cache, every kernel launched
// with programmatic dependent launch so each GEMV's weight stream starts
// while its predecessor drains:
//   embed   : dequant one row of token_embd (bit-exact) -> x; zero logits/qkv
//   per layer l:
//     QKV   : qkv  += [Wq;Wk;Wv] . rms_norm(x) * attn_norm          (GEMV)
//     ATT   : append k,v (f16) at pos; split-K flash-decoding -> attn; zero gu
//     WO    : x    += Wo . attn            (residual add fused, GEMV)
//     W13   : gu   += [W1;W3] . rms_norm(x) * ffn_norm; zero qkv     (GEMV)
//     W2    : x    += W2 . (silu(gate) * up)  (SwiGLU fused into staging)
//   LOGITS  : logits += Wout . rms_norm(x) * output_norm            (GEMV)
//   ARGMAX  : last-index argmax -> next token (feeds the next embed); pos++
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "attention.cuh"
#include "dense.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "kquant.h"
#include "nvtx3/nvToolsExt.h"
#include "gguf.h"
#include "model.h"
#include "tp.h"
#include "ops.cuh"
#include "quant.cuh"

namespace ifx {

namespace {

__global__ void embed_kernel(const uint8_t *emb, int type, int D, const uint32_t *token,
                             float *x, float *zero_a, int na, float *zero_b, int nb) {
  pdl_wait();
  pdl_launch();
  const uint64_t base = (uint64_t)(*token) * (uint64_t)D;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x)
    x[i] = dequant_elem(type, emb, base + i);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < na; i += gridDim.x * blockDim.x)
    zero_a[i] = 0.f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nb; i += gridDim.x * blockDim.x)
    zero_b[i] = 0.f;
}

__global__ void embed_rows_kernel(const uint8_t *emb, int type, int D, const uint32_t *ids,
                                  float *x) {
  const uint64_t base = (uint64_t)ids[blockIdx.x] * (uint64_t)D;
  for (int i = threadIdx.x; i < D; i += blockDim.x)
    x[(size_t)blockIdx.x * D + i] = dequant_elem(type, emb, base + i);
}

// Argmax over logits (last index on ties, forward.rs:615-622); the last CTA
// publishes the token, optionally records it and advances the position.
// With publish = 0 (a vocab shard under tensor parallelism) the key of the
// shard's maximum is left in *key (indices offset by v0) for the all-reduce.
__global__ void argmax_step_kernel(const float *logits, int n, unsigned long long *key,
                                   int *count, uint32_t *next_token, uint32_t *tokens,
                                   int *n_out, int *pos, int record, int inc_pos, int v0,
                                   int publish) {
  pdl_wait();
  pdl_launch();
  unsigned long long best = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float v = logits[i];
    if (v != v) continue;
    const unsigned long long k = ((unsigned long long)ordered_bits(v) << 32) | (unsigned)(i + v0);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0 && best) atomicMax(key, best);
  __threadfence();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = (atomicAdd(count, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  if (!publish) {
    *count = 0;
    return;
  }
  const unsigned long long k = atomicAdd(key, 0ull);
  const uint32_t tok = (uint32_t)(k & 0xffffffffull);
  *next_token = tok;
  if (record) {
    tokens[*n_out] = tok;
    *n_out = *n_out + 1;
  }
  if (inc_pos) *pos = *pos + 1;
  *key = 0;
  *count = 0;
}

// K/V rows of a prefill chunk into the f16 cache at positions start + t
// (forward.rs:246-253). k/v: [n][G*hd] f32; cache: [G][max_seq][hd].
__global__ void kv_write_kernel(const float *k, const float *v, __half *kc, __half *vc, int n,
                                int G, int hd, int max_seq, int start) {
  const int t = blockIdx.x;
  for (int e = threadIdx.x; e < G * hd; e += blockDim.x) {
    const int g = e / hd, d = e % hd;
    const size_t dst = ((size_t)g * max_seq + start + t) * hd + kv_col(start + t, d, hd);
    kc[dst] = __float2half_rn(k[(size_t)t * G * hd + e]);
    vc[dst] = __float2half_rn(v[(size_t)t * G * hd + e]);
  }
}

// The same rows into a paged cache: position p = start + t is row p % P of
// page table[p / P]; kc / vc point at this layer's rows in page 0.
__global__ void kv_write_paged_kernel(const float *k, const float *v, __half *kc, __half *vc, int n,
                                      int G, int hd, int P, int64_t page_stride, const int *table,
                                      int start) {
  const int t = blockIdx.x, p = start + t;
  const size_t page = (size_t)table[p / P] * (size_t)page_stride;
  for (int e = threadIdx.x; e < G * hd; e += blockDim.x) {
    const int g = e / hd, d = e % hd;
    const size_t dst = page + ((size_t)g * P + p % P) * hd + kv_col(p, d, hd);
    kc[dst] = __float2half_rn(k[(size_t)t * G * hd + e]);
    vc[dst] = __float2half_rn(v[(size_t)t * G * hd + e]);
  }
}

__global__ void add_int_kernel(int *p, int v) { *p += v; }

// Row-wise argmax of x [rows][n] (last index on ties, NaN skipped:
// forward.rs:615-622): CTA (row, part) reduces a contiguous part of the row
// to a 64-bit key (ordered value bits << 32 | index) and takes the maximum
// with keys[row] (zeroed before); argmax_keys_kernel extracts the indices.
constexpr int kArgmaxParts = 32;

__global__ void argmax_rows_kernel(const float *x, int n, unsigned long long *keys) {
  const float *r = x + (size_t)blockIdx.x * n;
  const int per = (n + kArgmaxParts - 1) / kArgmaxParts;
  const int i0 = blockIdx.y * per, i1 = min(n, i0 + per);
  unsigned long long best = 0;
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const float v = r[i];
    if (v != v) continue;
    const unsigned long long k = ((unsigned long long)ordered_bits(v) << 32) | (unsigned)i;
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  __shared__ unsigned long long w[32];
  if ((threadIdx.x & 31) == 0) w[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) best = w[i] > best ? w[i] : best;
    best = w[0] > best ? w[0] : best;
    if (best) atomicMax(&keys[blockIdx.x], best);
  }
}

// The step's tokens from the row keys; every sequence's position advances.
__global__ void argmax_keys_kernel(const unsigned long long *keys, int rows, uint32_t *out,
                                   int *pos, const int *slot) {
  const int i = threadIdx.x;
  if (i < rows) {
    out[i] = (uint32_t)(keys[i] & 0xffffffffull);
    pos[slot ? slot[i] : i] += 1;
  }
}

// in: [tp][n][vl] (rank-major, as gathered); out: [n][tp * vl].
__global__ void shard_interleave_kernel(const float *in, float *out, int n, int vl, int tp) {
  const int t = blockIdx.x;
  for (int e = threadIdx.x; e < tp * vl; e += blockDim.x) {
    const int r = e / vl, j = e - r * vl;
    out[(size_t)t * tp * vl + e] = in[((size_t)r * n + t) * vl + j];
  }
}

// After the all-reduce of the shards' keys: publish the global argmax and
// clear this rank's shard key for the next step.
__global__ void token_publish_kernel(const unsigned long long *key_global,
                                     unsigned long long *key_local, uint32_t *next_token,
                                     uint32_t *tokens, int *n_out, int *pos, int record,
                                     int inc_pos) {
  const uint32_t tok = (uint32_t)(*key_global & 0xffffffffull);
  *next_token = tok;
  if (record) {
    tokens[*n_out] = tok;
    *n_out = *n_out + 1;
  }
  if (inc_pos) *pos = *pos + 1;
  *key_local = 0;
}

__global__ void kv_read_kernel(const __half *c, float *out, int len, int G, int hd, int max_seq) {
  const int t = blockIdx.x;
  for (int e = threadIdx.x; e < G * hd; e += blockDim.x) {
    const int g = e / hd, d = e % hd;
    out[(size_t)t * G * hd + e] = __half2float(c[((size_t)g * max_seq + t) * hd + kv_col(t, d, hd)]);
  }
}

template <typename T>
ifx_status dalloc(T **p, size_t n) {
  IFX_CUDA(cudaMalloc(reinterpret_cast<void **>(p), std::max<size_t>(n, 1) * sizeof(T)));
  IFX_CUDA(cudaMemset(*p, 0, std::max<size_t>(n, 1) * sizeof(T)));
  return IFX_OK;
}

}  // namespace

// An NVTX range over a host entry point (named "ifx:<what>"), so a timeline
// tool shows prefill, decode steps and loops; free when no tool listens.
struct NvtxRange {
  explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange &) = delete;
  NvtxRange &operator=(const NvtxRange &) = delete;
};

// ------------------------------------------------------------------ load --
// A tensor's bytes in the reference's block order: llama.cpp-ordered Q4_K /
// Q6_K blocks (ggml = true) are permuted into `conv` and *type becomes the
// converted type (kTypeQ6KS8 for Q6_K); anything else is used in place.
static ifx_status reference_order(bool ggml, const uint8_t **src, uint64_t size, int *type,
                                  std::vector<uint8_t> *conv) {
  if (!ggml || (*type != IFX_TYPE_Q4_K && *type != IFX_TYPE_Q6_K)) return IFX_OK;
  conv->resize(size);
  IFX_TRY(ggml_to_reference(*type, *src, size, conv->data(), type));
  *src = conv->data();
  return IFX_OK;
}

// A weight [rows, cols] uploaded and repacked; under tensor parallelism only
// this rank's shard (split_k = 0: a block of rows; 1: a block of the input
// dimension of every row) is kept.
static ifx_status upload_matrix(const GgufFile &f, const uint8_t *bytes, size_t len, int idx,
                                uint64_t rows, uint64_t cols, uint8_t *staging, cudaStream_t st,
                                QMatrix *out, int tp = 1, int rank = 0, int split_k = 0,
                                bool ggml = false, bool dense = false) {
  uint64_t start, size;
  IFX_TRY(gguf_tensor_range(f, len, idx, &start, &size));
  const GgufTensor &t = f.tensors[idx];
  if (t.n_elements() != rows * cols)
    return fail(IFX_ERR_SHAPE, "tensor " + t.name + ": element count does not match the config");
  const uint8_t *src = bytes + start;
  int type = (int)t.type;
  std::vector<uint8_t> conv;
  IFX_TRY(reference_order(ggml, &src, size, &type, &conv));
  std::vector<uint8_t> shard;
  if (tp > 1) {
    IFX_TRY(tp_shard(type, src, size, rows, cols, split_k, tp, rank, &shard));
    if (split_k) cols /= tp;
    else rows /= tp;
    src = shard.data();
    size = shard.size();
  }
  if (dense) {  // row-major f32 with the reference's dequantisation (weights.rs:66-74)
    make_dense_layout((int64_t)rows, (int64_t)cols, type, &out->L);
    IFX_CUDA(cudaMemcpyAsync(staging, src, size, cudaMemcpyHostToDevice, st));
    IFX_CUDA(cudaMalloc(&out->d, out->L.total_bytes));
    IFX_TRY(op_dequantize(type, staging, size, reinterpret_cast<float *>(out->d), rows * cols, st));
    IFX_CUDA(cudaStreamSynchronize(st));
    return IFX_OK;
  }
  if (!make_layout(type, (int64_t)rows, (int64_t)cols, &out->L))
    return fail(IFX_ERR_UNSUPPORTED,
                "tensor " + t.name + ": weight type " + std::to_string(t.type) +
                    " is not supported by the fused kernels (Q4_0, Q8_0, Q4_K, Q6_K)");
  IFX_CUDA(cudaMemcpyAsync(staging, src, size, cudaMemcpyHostToDevice, st));
  IFX_CUDA(cudaMalloc(&out->d, out->L.total_bytes));
  IFX_TRY(repack_to_device(out->L, staging, out->d, st));
  IFX_CUDA(cudaStreamSynchronize(st));
  return IFX_OK;
}

static ifx_status upload_norm(const GgufFile &f, const uint8_t *bytes, size_t len, int idx,
                              uint64_t n, uint8_t *staging, cudaStream_t st, float **out) {
  uint64_t start, size;
  IFX_TRY(gguf_tensor_range(f, len, idx, &start, &size));
  const GgufTensor &t = f.tensors[idx];
  if (t.n_elements() != n) return fail(IFX_ERR_SHAPE, "tensor " + t.name + ": length mismatch");
  IFX_TRY(dalloc(out, n));
  IFX_CUDA(cudaMemcpyAsync(staging, bytes + start, size, cudaMemcpyHostToDevice, st));
  IFX_TRY(op_dequantize((int)t.type, staging, size, *out, n, st));  // weights.rs:66-74 exactly
  IFX_CUDA(cudaStreamSynchronize(st));
  return IFX_OK;
}

ifx_status Model::load(const uint8_t *bytes, size_t len, const ifx_load_opts &o) {
  NvtxRange nvtx_("ifx:load");
  opts = o;
  tp = opts.tp_size;
  rank = opts.tp_rank;
  if (tp < 1 || tp > 8 || rank < 0 || rank >= tp)
    return fail(IFX_ERR_INVALID_ARGUMENT, "tp_size must be 1..8 and 0 <= tp_rank < tp_size");
  if (tp > 1 && !opts.nccl_comm)
    return fail(IFX_ERR_INVALID_ARGUMENT, "tensor parallel loading needs nccl_comm");
  if (opts.kquant_layout != IFX_KQUANT_REFERENCE && opts.kquant_layout != IFX_KQUANT_GGML)
    return fail(IFX_ERR_INVALID_ARGUMENT, "kquant_layout must be IFX_KQUANT_REFERENCE or IFX_KQUANT_GGML");
  const bool ggml = opts.kquant_layout == IFX_KQUANT_GGML;
  GgufFile f;
  IFX_TRY(gguf_parse(bytes, len, &f));  // host-only checks first: no GPU needed to reject a file
  if (ggml) {
    // llama.cpp's type ids (Q8_0 = 8, ...) onto the reference's; a type with
    // no counterpart gets an id no size is known for, so any use of it fails
    // as an unknown tensor type
    for (GgufTensor &t : f.tensors) {
      const int r = ggml_type_to_reference(t.type);
      t.type = r < 0 ? 0xFFFFu : (uint32_t)r;
    }
  }
  IFX_TRY(gguf_config(f, &cfg));
  if (cfg.vocab_size == 0) return fail(IFX_ERR_SHAPE, "llama.vocab_size is missing or zero");
  const uint64_t D = cfg.hidden_size, H = cfg.n_heads, G = cfg.n_kv_heads, hd = cfg.head_dim;
  const uint64_t F = cfg.intermediate_size, V = cfg.vocab_size;
  // G == 0 first: the remainder below (and every later H / G) would divide
  // by zero (the reference's integer division panics there)
  if (G == 0) return fail(IFX_ERR_SHAPE, "llama.attention.head_count_kv is 0");
  if (H * hd != D || H % G || hd % 2 || cfg.rope_dim > hd || cfg.rope_dim % 2)
    return fail(IFX_ERR_SHAPE, "unsupported head geometry");
  // Megatron split: q/k/v by heads, W1/W3 and the vocab by rows, Wo/W2 by
  // their input dimension; a rank's q heads map onto its own kv heads
  if (G % tp || F % tp || V % tp)
    return fail(IFX_ERR_SHAPE, "tensor parallel: kv heads, ffn rows and vocab must divide by tp_size");
  Hl = H / tp;
  Gl = G / tp;
  Fl = F / tp;
  Vl = V / tp;
  v0 = Vl * (uint64_t)rank;
  if (tp > 1) {
    comm = opts.nccl_comm;
    IFX_TRY(nccl_api(&nccl));
  }
  static const char *suffix[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                  "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
  std::vector<std::array<int, 9>> idx(cfg.n_layers);
  for (uint64_t l = 0; l < cfg.n_layers; ++l)
    for (int s = 0; s < 9; ++s) {
      const std::string nm = "blk." + std::to_string(l) + "." + suffix[s] + ".weight";
      idx[l][s] = f.tensor_index(nm);
      if (idx[l][s] < 0)  // model/mod.rs:72-74
        return fail(IFX_ERR_TENSOR_NOT_FOUND, "tensor not found: blk." + std::to_string(l) + ".*");
    }
  const int i_emb = f.tensor_index("token_embd.weight");
  if (i_emb < 0) return fail(IFX_ERR_TENSOR_NOT_FOUND, "tensor not found: token_embd.weight");
  const int i_onorm = f.tensor_index("output_norm.weight");
  if (i_onorm < 0) return fail(IFX_ERR_TENSOR_NOT_FOUND, "tensor not found: output_norm.weight");
  const int i_out = f.tensor_index("output.weight");  // optional, forward.rs:573
  device = opts.device;
  IFX_CUDA(cudaSetDevice(device));
  IFX_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));

  // staging buffer: the largest tensor
  uint64_t max_bytes = 0;
  for (size_t i = 0; i < f.tensors.size(); ++i) {
    int64_t b = gguf_type_bytes(f.tensors[i].type, f.tensors[i].n_elements());
    if (b > 0) max_bytes = std::max<uint64_t>(max_bytes, (uint64_t)b);
  }
  uint8_t *staging = nullptr;
  IFX_CUDA(cudaMalloc(&staging, max_bytes + 256));
  ifx_status st = IFX_OK;
  auto guard = [&](ifx_status s) {
    if (s != IFX_OK && st == IFX_OK) st = s;
    return s == IFX_OK;
  };
  // a checkpoint with any dense (F32 / F16 / Q8_K) matrix runs every matrix
  // dense: dequantised once to f32, as the reference does per call
  dense = dense_type((int)f.tensors[i_out >= 0 ? i_out : i_emb].type);
  for (uint64_t l = 0; l < cfg.n_layers; ++l)
    for (int s = 1; s < 9; ++s)
      if (s != 5 && dense_type((int)f.tensors[idx[l][s]].type)) dense = true;
  const bool dn = dense;
  layers.resize(cfg.n_layers);
  for (uint64_t l = 0; l < cfg.n_layers && st == IFX_OK; ++l) {
    Layer &L = layers[l];
    guard(upload_norm(f, bytes, len, idx[l][0], D, staging, stream, &L.attn_norm)) &&
        guard(upload_matrix(f, bytes, len, idx[l][1], D, D, staging, stream, &L.wq, tp, rank, 0, ggml, dn)) &&
        guard(upload_matrix(f, bytes, len, idx[l][2], G * hd, D, staging, stream, &L.wk, tp, rank, 0, ggml, dn)) &&
        guard(upload_matrix(f, bytes, len, idx[l][3], G * hd, D, staging, stream, &L.wv, tp, rank, 0, ggml, dn)) &&
        guard(upload_matrix(f, bytes, len, idx[l][4], D, D, staging, stream, &L.wo, tp, rank, 1, ggml, dn)) &&
        guard(upload_norm(f, bytes, len, idx[l][5], D, staging, stream, &L.ffn_norm)) &&
        guard(upload_matrix(f, bytes, len, idx[l][6], F, D, staging, stream, &L.w1, tp, rank, 0, ggml, dn)) &&
        guard(upload_matrix(f, bytes, len, idx[l][7], F, D, staging, stream, &L.w3, tp, rank, 0, ggml, dn)) &&
        guard(upload_matrix(f, bytes, len, idx[l][8], D, F, staging, stream, &L.w2, tp, rank, 1, ggml, dn));
  }
  if (st == IFX_OK) guard(upload_norm(f, bytes, len, i_onorm, D, staging, stream, &out_norm));
  if (st == IFX_OK)
    guard(upload_matrix(f, bytes, len, i_out >= 0 ? i_out : i_emb, V, D, staging, stream, &out_w,
                        tp, rank, 0, ggml, dn));
  if (st == IFX_OK) {
    uint64_t s0, sz;
    if (guard(gguf_tensor_range(f, len, i_emb, &s0, &sz))) {
      const GgufTensor &t = f.tensors[i_emb];
      emb_type = (int)t.type;
      const uint8_t *esrc = bytes + s0;
      std::vector<uint8_t> conv;
      if (t.n_elements() != V * D) guard(fail(IFX_ERR_SHAPE, "token_embd.weight: element count"));
      else if (!block_info(emb_type).elems)
        guard(fail(IFX_ERR_UNSUPPORTED, "token_embd.weight: type not supported"));
      else if (guard(reference_order(ggml, &esrc, sz, &emb_type, &conv)) &&
               (cudaMalloc(&emb_raw, sz) != cudaSuccess ||
                cudaMemcpy(emb_raw, esrc, sz, cudaMemcpyHostToDevice) != cudaSuccess))
        guard(fail(IFX_ERR_CUDA, "token_embd upload"));
      emb_row_bytes = (V ? sz / V : 0);
    }
  }
  cudaFree(staging);
  if (st != IFX_OK) return st;

  // decode buffers (this rank's heads / rows; x and the gathered logits whole)
  qkv_n = (int)((Hl + 2 * Gl) * hd);
  IFX_TRY(dalloc(&x, D));
  IFX_TRY(dalloc(&qkv, qkv_n));
  IFX_TRY(dalloc(&attn, Hl * hd));
  IFX_TRY(dalloc(&gu, 2 * Fl));
  IFX_TRY(dalloc(&logits, V));
  if (tp > 1) {
    IFX_TRY(dalloc(&y, D));
    IFX_TRY(dalloc(&logits_local, Vl));
    IFX_TRY(dalloc(&key_global, 1));
    if (opts.persistent_decode) IFX_TRY(setup_peers());
  } else {
    logits_local = logits;
  }
  IFX_TRY(dalloc(&err, 1));
  IFX_TRY(dalloc(&next_token, 1));
  IFX_TRY(dalloc(&amax_key, 1));
  IFX_TRY(dalloc(&amax_count, 1));
  IFX_TRY(dalloc(&n_out, 1));
  // split-K factor of the decode attention: about two CTAs per SM in total
  ns = (int)std::max<uint64_t>(1, std::min<uint64_t>(64, 2 * kNumSMs / Gl));
  IFX_TRY(dalloc(&part_o, Hl * ns * hd));
  IFX_TRY(dalloc(&part_ml, Hl * ns));
  IFX_TRY(dalloc(&counters, Gl));

  // one GEMV plan (pointers + byte-balanced schedule) per call site
  const float eps = cfg.norm_eps;
  p_qkv.resize(cfg.n_layers);
  p_wo.resize(cfg.n_layers);
  p_w13.resize(cfg.n_layers);
  p_w2.resize(cfg.n_layers);
  p_qkv_more.resize(cfg.n_layers);
  p_w13_more.resize(cfg.n_layers);
  // the matrices of one fused site grouped by unit width: the group of the
  // first matrix in `first`, any other group in its own plan in `more`
  auto plan_site = [&](const QMatrix *const *mats, float *const *ys, int n, int mode,
                       const float *xin, const float *normw, GemvPlan *first,
                       std::vector<GemvPlan> *more) -> ifx_status {
    std::vector<int> kcs;
    for (int i = 0; i < n; ++i)
      if (std::find(kcs.begin(), kcs.end(), mats[i]->L.kc) == kcs.end()) kcs.push_back(mats[i]->L.kc);
    more->resize(kcs.size() - 1);
    for (size_t g = 0; g < kcs.size(); ++g) {
      const QMatrix *gm[kGemvMaxSegs];
      float *gy[kGemvMaxSegs];
      int gn = 0;
      for (int i = 0; i < n; ++i)
        if (mats[i]->L.kc == kcs[g]) {
          gm[gn] = mats[i];
          gy[gn++] = ys[i];
        }
      IFX_TRY(gemv_plan(gm, gy, gn, mode, xin, nullptr, normw, eps, err,
                        g == 0 ? first : &(*more)[g - 1]));
    }
    return IFX_OK;
  };
  for (uint64_t l = 0; l < cfg.n_layers; ++l) {
    Layer &L = layers[l];
    const QMatrix *mq[3] = {&L.wq, &L.wk, &L.wv};
    float *yq[3] = {qkv, qkv + Hl * hd, qkv + (Hl + Gl) * hd};
    // the row-parallel layers accumulate into a partial buffer under tensor
    // parallelism (all-reduced into x), into x itself otherwise
    float *acc = tp > 1 ? y : x;
    const QMatrix *mo[1] = {&L.wo};
    float *yo[1] = {acc};
    const QMatrix *m13[2] = {&L.w1, &L.w3};
    float *y13[2] = {gu, gu + Fl};
    const QMatrix *m2[1] = {&L.w2};
    float *y2[1] = {acc};
    IFX_TRY(plan_site(mq, yq, 3, GEMV_RMSNORM, x, L.attn_norm, &p_qkv[l], &p_qkv_more[l]));
    IFX_TRY(gemv_plan(mo, yo, 1, GEMV_PLAIN, attn, nullptr, nullptr, eps, err, &p_wo[l]));
    IFX_TRY(plan_site(m13, y13, 2, GEMV_RMSNORM, x, L.ffn_norm, &p_w13[l], &p_w13_more[l]));
    IFX_TRY(gemv_plan(m2, y2, 1, GEMV_SWIGLU, gu, gu + Fl, nullptr, eps, err, &p_w2[l]));
    p_w13[l].args.zero_ptr = qkv;  // qkv was consumed by ATT; the next QKV refills it
    p_w13[l].args.zero_n = qkv_n;
  }
  const QMatrix *mout[1] = {&out_w};
  float *yout[1] = {logits_local};
  IFX_TRY(gemv_plan(mout, yout, 1, GEMV_RMSNORM, x, nullptr, out_norm, eps, err, &p_logits));

  decode_bytes = 0;
  for (auto &L : layers)
    decode_bytes += L.wq.gguf_bytes() + L.wk.gguf_bytes() + L.wv.gguf_bytes() + L.wo.gguf_bytes() +
                    L.w1.gguf_bytes() + L.w3.gguf_bytes() + L.w2.gguf_bytes() + 2 * D * 4;
  decode_bytes += out_w.gguf_bytes() + D * 4 + emb_row_bytes;
  IFX_CUDA(cudaStreamSynchronize(stream));
  return IFX_OK;
}

Model::~Model() {
  if (device >= 0) cudaSetDevice(device);
  auto F = [](void *p) {
    if (p) cudaFree(p);
  };
  for (auto &L : layers) {
    F(L.attn_norm);
    F(L.ffn_norm);
    for (QMatrix *q : {&L.wq, &L.wk, &L.wv, &L.wo, &L.w1, &L.w3, &L.w2}) F(q->d);
  }
  F(out_w.d);
  F(out_norm);
  F(emb_raw);
  for (auto *v : std::vector<void *>{x, qkv, attn, gu, logits, err, next_token, amax_key, amax_count,
                                     n_out, part_o, part_ml, counters, ws, logits_all, ids_dev,
                                     y, key_global, logits_all_local})
    F(v);
  if (logits_local != logits) F(logits_local);
  for (int r = 0; r < kMaxRanks; ++r)
    if (r != rank && peers.buf[r]) cudaIpcCloseMemHandle(peers.buf[r]);
  F(peer_buf);
  F(mega_epoch);
  for (size_t l = 0; l < p_qkv.size(); ++l) {
    gemv_plan_free(&p_qkv[l]);
    for (auto &p : p_qkv_more[l]) gemv_plan_free(&p);
    for (auto &p : p_w13_more[l]) gemv_plan_free(&p);
    gemv_plan_free(&p_wo[l]);
    gemv_plan_free(&p_w13[l]);
    gemv_plan_free(&p_w2[l]);
  }
  gemv_plan_free(&p_logits);
  if (stream) cudaStreamDestroy(stream);
}

// --------------------------------------------------------------- KV cache --
ifx_status KvCache::create(Model *model, size_t max_seq_len) {
  m = model;
  max_seq = max_seq_len;
  const ifx_config &c = m->cfg;
  per_layer = (size_t)m->Gl * max_seq * c.head_dim;  // this rank's kv heads
  dev = m->device;
  IFX_CUDA(cudaSetDevice(m->device));
  IFX_TRY(dalloc(&k, per_layer * c.n_layers));
  IFX_TRY(dalloc(&v, per_layer * c.n_layers));
  IFX_TRY(dalloc(&pos, 1));
  IFX_TRY(dalloc(&tokens, max_seq + 1));
  return IFX_OK;
}

KvCache::~KvCache() {
  if (!owner) return;
  if (dev >= 0) cudaSetDevice(dev);
  if (graph) cudaGraphExecDestroy(graph);
  for (void *p : {(void *)k, (void *)v, (void *)pos, (void *)tokens, (void *)part_o,
                  (void *)part_ml, (void *)bar})
    if (p) cudaFree(p);
  mega_free(&mega);
}

constexpr int kPageRows = 64;   // positions per page of a paged batch
constexpr int kMaxPages = 64;   // pages per sequence (the attention splits)

ifx_status KvBatch::create(Model *model, size_t max_seq_len, int nseq, size_t pages) {
  m = model;
  batch = nseq;
  max_seq = max_seq_len;
  const ifx_config &c = m->cfg;
  if (m->tp > 1) return fail(IFX_ERR_UNSUPPORTED, "batched decode: tensor parallelism not supported");
  if (nseq < 1 || nseq > kGemmSmallMax)
    return fail(IFX_ERR_INVALID_ARGUMENT, "batched decode: 1 to 32 sequences");
  const int G = (int)m->Gl, H = (int)m->Hl, hd = (int)c.head_dim, grp = H / G;
  paged = pages > 0;
  if (paged) {
    // one attention split per page
    page_rows = kPageRows;
    max_pages = (int)((max_seq + kPageRows - 1) / kPageRows);
    if (max_pages > kMaxPages)
      return fail(IFX_ERR_INVALID_ARGUMENT, "paged batch: max_seq_len above " +
                                                std::to_string(kPageRows * kMaxPages));
    n_pages = pages;
    page_stride = (int64_t)c.n_layers * G * kPageRows * hd;
    per_layer = (size_t)G * kPageRows * hd;  // a layer's rows within one page
    ns = max_pages;
  } else {
    per_layer = (size_t)G * max_seq * hd;
    // split-K factor: at least two CTAs per SM, and chunks of at most 64 cache
    // rows (small shared-memory footprint, several CTAs per SM)
    ns = std::max(1, (2 * kNumSMs + nseq * G - 1) / (nseq * G));
    ns = std::max(ns, (int)((max_seq + 63) / 64));
    ns = std::min(ns, 64);
    while (ns < 64 && decode_attention_smem(grp, hd, (int)max_seq, ns) > 160 * 1024) ++ns;
  }
  const size_t D = c.hidden_size, F = m->Fl, V = c.vocab_size;
  const size_t qkvw = (size_t)(H + 2 * G) * hd;
  dev = m->device;
  IFX_CUDA(cudaSetDevice(m->device));
  const size_t cache = paged ? (size_t)page_stride * n_pages : per_layer * c.n_layers * nseq;
  IFX_TRY(dalloc(&k, cache));
  IFX_TRY(dalloc(&v, cache));
  if (paged) {
    IFX_TRY(dalloc(&table_dev, (size_t)nseq * max_pages));
    table.assign((size_t)nseq * max_pages, -1);
    free_pages.clear();
    for (size_t i = n_pages; i-- > 0;) free_pages.push_back((int)i);  // page 0 handed out first
  }
  IFX_TRY(dalloc(&pos, (size_t)nseq));
  IFX_TRY(dalloc(&x, nseq * D));
  IFX_TRY(dalloc(&qkv, nseq * qkvw));
  IFX_TRY(dalloc(&attn, (size_t)nseq * H * hd));
  IFX_TRY(dalloc(&gate, nseq * F));
  IFX_TRY(dalloc(&up, nseq * F));
  IFX_TRY(dalloc(&logits, nseq * V));
  IFX_TRY(dalloc(&part_o, (size_t)nseq * H * ns * hd));
  IFX_TRY(dalloc(&part_ml, (size_t)nseq * H * ns));
  IFX_TRY(dalloc(&counters, (size_t)nseq * G));
  IFX_TRY(dalloc(&ids, (size_t)nseq));
  IFX_TRY(dalloc(&out, (size_t)nseq));
  IFX_TRY(dalloc(&keys, (size_t)nseq));
  IFX_TRY(dalloc(&slots, (size_t)nseq));
  const size_t kmax = std::max<size_t>(std::max<size_t>(D, F), (size_t)H * hd);
  IFX_CUDA(cudaMalloc(&xf, std::max(gemm_small_xfrag_bytes(nseq, (int64_t)kmax),
                                    (size_t)nseq * kmax * sizeof(float))));
  len.assign((size_t)nseq, 0);
  return IFX_OK;
}

KvBatch::~KvBatch() {
  if (dev >= 0) cudaSetDevice(dev);
  if (graph) cudaGraphExecDestroy(graph);
  for (void *p : {(void *)k, (void *)v, (void *)pos, (void *)x, (void *)qkv, (void *)attn,
                  (void *)gate, (void *)up, (void *)logits, (void *)part_o, (void *)part_ml,
                  (void *)counters, (void *)xf, (void *)ids, (void *)out, (void *)keys,
                  (void *)slots, (void *)table_dev})
    if (p) cudaFree(p);
}

ifx_status KvBatch::reserve(int seq, size_t rows, cudaStream_t st) {
  if (!paged) return IFX_OK;
  if (rows > max_seq) return fail(IFX_ERR_INVALID_TENSOR_INDEX, "KV cache is full");
  int *row = table.data() + (size_t)seq * max_pages;
  const int need = (int)((rows + page_rows - 1) / page_rows);
  int have = 0;
  while (have < max_pages && row[have] >= 0) ++have;
  if (need <= have) return IFX_OK;
  if ((size_t)(need - have) > free_pages.size())
    return fail(IFX_ERR_OUT_OF_MEMORY, "paged batch: the page pool is exhausted (" +
                                           std::to_string(n_pages) + " pages)");
  for (int i = have; i < need; ++i) {
    row[i] = free_pages.back();
    free_pages.pop_back();
  }
  IFX_CUDA(cudaMemcpyAsync(table_dev + (size_t)seq * max_pages + have, row + have,
                           sizeof(int) * (size_t)(need - have), cudaMemcpyHostToDevice, st));
  return IFX_OK;
}

void KvBatch::release(int seq) {
  if (!paged) return;
  int *row = table.data() + (size_t)seq * max_pages;
  for (int i = 0; i < max_pages; ++i)
    if (row[i] >= 0) {
      free_pages.push_back(row[i]);
      row[i] = -1;
    }
}

ifx_status KvCache::clear() {
  len = 0;
  IFX_CUDA(cudaMemsetAsync(pos, 0, sizeof(int), m->stream));
  IFX_CUDA(cudaStreamSynchronize(m->stream));
  return IFX_OK;
}

// ---------------------------------------------------------- decode step ---
ifx_status Model::enqueue_decode(KvCache &kv, cudaStream_t st) {
  const ifx_config &c = cfg;
  const bool pdl = tp == 1;  // NCCL work sits between the kernels under tensor parallelism
  const int D = (int)c.hidden_size, H = (int)Hl, G = (int)Gl, hd = (int)c.head_dim;
  IFX_CUDA(launch(embed_kernel, dim3(8), dim3(256), 0, st, pdl, (const uint8_t *)emb_raw, emb_type,
                  D, (const uint32_t *)next_token, x, logits_local, (int)Vl, qkv, qkv_n));
  for (uint64_t l = 0; l < c.n_layers; ++l) {
    IFX_TRY(gemv_launch(p_qkv[l], st, pdl));
    for (const GemvPlan &p : p_qkv_more[l]) IFX_TRY(gemv_launch(p, st, pdl));
    DecodeAttnArgs a{};
    a.qkv = qkv;
    a.kc = kv.k + l * kv.per_layer;
    a.vc = kv.v + l * kv.per_layer;
    a.pos = kv.pos;
    a.part_o = part_o;
    a.part_ml = part_ml;
    a.counters = counters;
    a.attn_out = attn;
    a.zero_ptr = gu;
    a.zero_n = (int)(2 * Fl);
    a.H = H;
    a.G = G;
    a.hd = hd;
    a.max_seq = (int)kv.max_seq;
    a.ns = ns;
    a.rope_compat = opts.rope_compat;
    a.rope_dim = (int)c.rope_dim;
    a.rope_base = c.rope_base;
    a.err = err;
    IFX_TRY(decode_attention(a, st, pdl));
    if (tp > 1) {
      IFX_TRY(tp_partial_begin(D, st));
      IFX_TRY(gemv_launch(p_wo[l], st, pdl));
      IFX_TRY(tp_partial_end(D, st));
      IFX_TRY(gemv_launch(p_w13[l], st, pdl));
      for (const GemvPlan &p : p_w13_more[l]) IFX_TRY(gemv_launch(p, st, pdl));
      IFX_TRY(tp_partial_begin(D, st));
      IFX_TRY(gemv_launch(p_w2[l], st, pdl));
      IFX_TRY(tp_partial_end(D, st));
    } else {
      IFX_TRY(gemv_launch(p_wo[l], st, pdl));
      IFX_TRY(gemv_launch(p_w13[l], st, pdl));
      for (const GemvPlan &p : p_w13_more[l]) IFX_TRY(gemv_launch(p, st, pdl));
      IFX_TRY(gemv_launch(p_w2[l], st, pdl));
    }
  }
  IFX_TRY(gemv_launch(p_logits, st, pdl));
  if (tp > 1) {
    // the argmax of this rank's vocab slice as a 64-bit key, the maximum
    // over ranks (ties go to the highest global index), then the token
    const NcclApi *N = nccl;
    IFX_CUDA(launch(argmax_step_kernel, dim3(kNumSMs), dim3(256), 0, st, false,
                    (const float *)logits_local, (int)Vl, amax_key, amax_count, next_token,
                    kv.tokens, n_out, kv.pos, 0, 0, (int)v0, 0));
    IFX_NCCL(N, N->AllReduce(amax_key, key_global, 1, ncclUint64, ncclMax, (ncclComm_t)comm, st));
    token_publish_kernel<<<1, 1, 0, st>>>(key_global, amax_key, next_token, kv.tokens, n_out,
                                          kv.pos, 1, 1);
    IFX_CUDA(cudaGetLastError());
    IFX_NCCL(N, N->AllGather(logits_local, logits, Vl, ncclFloat32, (ncclComm_t)comm, st));
  } else {
    IFX_CUDA(launch(argmax_step_kernel, dim3(kNumSMs), dim3(256), 0, st, pdl, (const float *)logits,
                    (int)c.vocab_size, amax_key, amax_count, next_token, kv.tokens, n_out, kv.pos, 1,
                    1, 0, 1));
  }
  (void)D;
  return IFX_OK;
}

// Row-parallel layers under tensor parallelism: the partial buffer starts as
// the residual on rank 0 and as zeros elsewhere, the layer accumulates its
// slice into it, and the all-reduce leaves the full sum (residual + layer
// output) in x on every rank.
ifx_status Model::tp_partial_begin(size_t n, cudaStream_t st, float *part, const float *resid) {
  if (!part) part = y;
  if (!resid) resid = x;
  if (rank == 0)
    IFX_CUDA(cudaMemcpyAsync(part, resid, n * sizeof(float), cudaMemcpyDeviceToDevice, st));
  else
    IFX_CUDA(cudaMemsetAsync(part, 0, n * sizeof(float), st));
  return IFX_OK;
}

ifx_status Model::tp_partial_end(size_t n, cudaStream_t st, const float *part, float *out) {
  if (!part) part = y;
  if (!out) out = x;
  IFX_NCCL(nccl, nccl->AllReduce(part, out, n, ncclFloat32, ncclSum, (ncclComm_t)comm, st));
  return IFX_OK;
}

// The persistent kernel's all-reduce buffers under tensor parallelism: each
// rank allocates one, zeroes it, and maps every other rank's through CUDA
// IPC (handles exchanged with an NCCL all-gather, which also orders every
// rank's zeroing before any rank's first push). The persistent path is used
// only when every rank mapped every buffer (an all-reduce of the outcome),
// so all ranks take the same path; otherwise the per-op kernels run with
// NCCL between them.
ifx_status Model::setup_peers() {
  const size_t bytes = mega_peer_bytes((int)cfg.hidden_size, kNumSMs, &peers);
  IFX_CUDA(cudaMalloc(&peer_buf, bytes));
  IFX_CUDA(cudaMemsetAsync(peer_buf, 0, bytes, stream));
  IFX_TRY(dalloc(&mega_epoch, 2));
  cudaIpcMemHandle_t h{};
  int ok = cudaIpcGetMemHandle(&h, peer_buf) == cudaSuccess ? 1 : 0;
  cudaGetLastError();
  constexpr size_t hb = sizeof(cudaIpcMemHandle_t);
  char *dh = nullptr;
  IFX_CUDA(cudaMalloc(&dh, hb * (size_t)tp + sizeof(int)));
  int *dok = reinterpret_cast<int *>(dh + hb * (size_t)tp);
  IFX_CUDA(cudaMemcpyAsync(dh + hb * (size_t)rank, &h, hb, cudaMemcpyHostToDevice, stream));
  IFX_NCCL(nccl, nccl->AllGather(dh + hb * (size_t)rank, dh, hb, ncclUint8, (ncclComm_t)comm, stream));
  std::vector<cudaIpcMemHandle_t> all((size_t)tp);
  IFX_CUDA(cudaMemcpyAsync(all.data(), dh, hb * (size_t)tp, cudaMemcpyDeviceToHost, stream));
  IFX_CUDA(cudaStreamSynchronize(stream));
  for (int r = 0; r < kMaxRanks; ++r) peers.buf[r] = nullptr;
  peers.buf[rank] = peer_buf;
  for (int r = 0; r < tp && ok; ++r) {
    if (r == rank) continue;
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, all[(size_t)r], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess)
      peers.buf[r] = static_cast<char *>(p);
    else
      ok = 0;
    cudaGetLastError();
  }
  IFX_CUDA(cudaMemcpyAsync(dok, &ok, sizeof(int), cudaMemcpyHostToDevice, stream));
  IFX_NCCL(nccl, nccl->AllReduce(dok, dok, 1, ncclInt32, ncclMin, (ncclComm_t)comm, stream));
  IFX_CUDA(cudaMemcpyAsync(&ok, dok, sizeof(int), cudaMemcpyDeviceToHost, stream));
  IFX_CUDA(cudaStreamSynchronize(stream));
  cudaFree(dh);
  peers.epoch = mega_epoch;
  // the host-side bound of the collectives, 20 s unless set
  peers.wait_ns = (uint64_t)(opts.tp_timeout_ms > 0 ? opts.tp_timeout_ms : 20000) * 1000000ull;
  peers_ok = ok != 0;
  return IFX_OK;
}

// The persistent decode plan of a cache: the token step as a phase list.
ifx_status Model::build_mega(KvCache &kv) {
  kv.mega_tried = true;
  const ifx_config &c = cfg;
  // this rank's heads (all of them at tp 1)
  const int H = (int)Hl, G = (int)Gl, hd = (int)c.head_dim;
  if (tp > 1 && !peers_ok) return IFX_OK;  // the all-reduces run between the per-op kernels
  if (dense) return IFX_OK;                 // the dense kernels run per op
  if (hd % 8 || hd > 256 || H % G || H / G > 8) return IFX_OK;  // separate kernels instead
  int dev_sms = 0;
  IFX_CUDA(cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, device));
  if (dev_sms != kNumSMs) return IFX_OK;
  MegaArgs &A = kv.mega.args;
  A.nsa = mega_attn_splits(G, (int)kv.max_seq, kNumSMs);
  A.nsa_base = std::min(A.nsa, mega_attn_splits_base(G, kNumSMs));
  A.attn_tc = (hd % 64 == 0 && hd <= 256 && H / G <= 8) ? (H / G <= 4 ? 4 : 8) : 0;
  IFX_TRY(dalloc(&kv.part_o, (size_t)H * A.nsa * hd));
  IFX_TRY(dalloc(&kv.part_ml, (size_t)H * A.nsa));
  IFX_TRY(dalloc(&kv.bar, 1 + (size_t)G));  // barrier counter + per-kv-head split counters
  A.bar = kv.bar;
  A.err = err;
  A.emb = emb_raw;
  A.emb_type = emb_type;
  A.D = (int)c.hidden_size;
  A.V = (int)Vl;  // this rank's vocab slice
  A.v0 = (int)v0;
  A.rank = rank;
  A.nranks = tp;
  A.peers = peers;
  A.n_ar = tp > 1 ? 2 * (int)c.n_layers : 0;
  A.next_token = next_token;
  A.x = x;
  A.attn = attn;
  A.logits = logits_local;
  A.part_o = kv.part_o;
  A.part_ml = kv.part_ml;
  A.H = H;
  A.G = G;
  A.hd = hd;
  A.max_seq = (int)kv.max_seq;
  A.rope_compat = opts.rope_compat;
  A.rope_dim = (int)c.rope_dim;
  A.rope_base = c.rope_base;
  A.qkv = qkv;
  A.kc0 = kv.k;
  A.vc0 = kv.v;
  A.kv_layer_elems = kv.per_layer;
  A.pos = kv.pos;
  A.amax_key = amax_key;
  A.amax_count = amax_count;
  A.tokens = kv.tokens;
  A.n_out = n_out;
  std::vector<MegaPhase> ph;
  auto gemv = [&](const GemvPlan &p, float *zero, int zn) {
    MegaPhase m{};
    m.kind = PH_GEMV;
    m.g = p.args;
    m.g.zero_ptr = nullptr;  // zeroing is a phase duty here
    m.zero_ptr = zero;
    m.zero_n = zn;
    ph.push_back(m);
  };
  auto simple = [&](int kind, float *zero, int zn) {
    MegaPhase m{};
    m.kind = kind;
    m.zero_ptr = zero;
    m.zero_n = zn;
    ph.push_back(m);
  };
  // tensor parallelism: Wo and W2 accumulate this rank's partial sums into
  // y, and an all-reduce phase adds every rank's into x (and zeroes y)
  int n_ar = 0;
  auto allreduce = [&]() {
    MegaPhase m{};
    m.kind = PH_ALLREDUCE;
    m.ar_src = y;
    m.ar_dst = x;
    m.ar_n = (int)c.hidden_size;
    m.ar_index = ++n_ar;
    ph.push_back(m);
  };
  if (tp > 1 && c.hidden_size % 4) return IFX_OK;  // the all-reduce moves float4s
  simple(PH_EMBED, logits_local, (int)Vl);
  for (uint64_t l = 0; l < c.n_layers; ++l) {
    if (l == 0 && tp > 1) gemv(p_qkv[l], y, (int)c.hidden_size);  // the all-reduces re-zero it
    else gemv(p_qkv[l], nullptr, 0);
    ph.back().attn_prefetch = (int)l + 1;  // this layer's K/V rows land during QKV
    for (const GemvPlan &p : p_qkv_more[l]) gemv(p, nullptr, 0);
    MegaPhase at{};
    at.kind = PH_ATTN;
    at.at.kc = kv.k + l * kv.per_layer;
    at.at.vc = kv.v + l * kv.per_layer;
    at.at.layer = (int)l;
    at.zero_ptr = gu;  // consumed by the previous layer's W2, refilled by W13
    at.zero_n = (int)(2 * Fl);  // this rank's W1 / W3 rows
    ph.push_back(at);
    gemv(p_wo[l], nullptr, 0);  // the attention phase leaves the combined heads in attn
    if (tp > 1) allreduce();
    gemv(p_w13[l], qkv, qkv_n);  // qkv was consumed by ATTN; the next QKV refills it
    for (const GemvPlan &p : p_w13_more[l]) gemv(p, nullptr, 0);
    gemv(p_w2[l], nullptr, 0);
    if (tp > 1) allreduce();
  }
  gemv(p_logits, nullptr, 0);
  simple(PH_ARGMAX, nullptr, 0);
  ifx_status s = mega_finalize(&kv.mega, ph, kNumSMs);
  if (s != IFX_OK) {
    mega_free(&kv.mega);
    return IFX_OK;  // too large for the persistent kernel: separate kernels
  }
  kv.mega_ready = true;
  return IFX_OK;
}

ifx_status Model::stage_rows(const float *X, const float *X2, const float *normw, float eps,
                             int mode, int64_t M, int64_t K, void *buf, cudaStream_t st) {
  if (dense) return dense_stage(X, X2, normw, eps, mode, M, K, buf, st);
  return gemm_stage_x(X, X2, normw, eps, mode, M, K, buf, st);
}

ifx_status Model::stage_small(const float *X, const float *X2, const float *normw, float eps,
                              int mode, int64_t M, int64_t K, void *buf, cudaStream_t st,
                              StageZero zero) {
  if (dense) {
    for (int i = 0; i < 2; ++i)
      if (zero.p[i]) IFX_CUDA(cudaMemsetAsync(zero.p[i], 0, sizeof(float) * (size_t)zero.n[i], st));
    return dense_stage(X, X2, normw, eps, mode, M, K, buf, st);
  }
  return gemm_small_stage_x(X, X2, normw, eps, mode, M, K, buf, st, zero, true);
}

ifx_status Model::run_decode(KvCache &kv, bool gather_logits) {
  if (opts.persistent_decode && !kv.mega_tried) IFX_TRY(build_mega(kv));
  if (kv.mega_ready) {
    IFX_TRY(mega_launch(kv.mega, stream));
    if (tp > 1 && gather_logits)
      IFX_NCCL(nccl, nccl->AllGather(logits_local, logits, Vl, ncclFloat32, (ncclComm_t)comm, stream));
    return IFX_OK;
  }
  if (!opts.use_graphs) return enqueue_decode(kv, stream);
  if (!kv.graph) {
    cudaGraph_t g;
    IFX_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    ifx_status s = enqueue_decode(kv, stream);
    cudaError_t e = cudaStreamEndCapture(stream, &g);
    if (s != IFX_OK) return s;
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    IFX_CUDA(cudaGraphInstantiate(&kv.graph, g, 0));
    cudaGraphDestroy(g);
  }
  IFX_CUDA(cudaGraphLaunch(kv.graph, stream));
  return IFX_OK;
}

ifx_status Model::check_err() {
  int h = 0;
  IFX_CUDA(cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h) {
    cudaMemset(err, 0, sizeof(int));
    // under tensor parallelism the ranks may now disagree on where the step
    // stopped (the persistent kernel's all-reduce epochs, the collectives):
    // refuse further calls, as after an aborted communicator
    if (tp > 1) comm_aborted = true;
    return fail(IFX_ERR_TIMEOUT, "a bounded device wait gave up (code " + std::to_string(h) + ")");
  }
  return IFX_OK;
}

ifx_status Model::decode_step(KvCache &kv, uint32_t token, float *logits_host) {
  NvtxRange nvtx_("ifx:decode_step");
  IFX_TRY(tp_usable());
  if (token >= cfg.vocab_size)
    return fail(IFX_ERR_INVALID_TENSOR_INDEX, "tensor index out of bounds: " + std::to_string(token));
  if (kv.len >= kv.max_seq) return fail(IFX_ERR_INVALID_TENSOR_INDEX, "KV cache is full");
  IFX_CUDA(cudaSetDevice(device));
  IFX_CUDA(cudaMemcpyAsync(next_token, &token, sizeof(uint32_t), cudaMemcpyHostToDevice, stream));
  IFX_CUDA(cudaMemsetAsync(n_out, 0, sizeof(int), stream));
  IFX_TRY(run_decode(kv));
  if (logits_host)
    IFX_CUDA(cudaMemcpyAsync(logits_host, logits, cfg.vocab_size * sizeof(float),
                             cudaMemcpyDeviceToHost, stream));
  IFX_TRY(step_sync(stream));
  kv.len += 1;
  return check_err();
}

// --------------------------------------------------------------- prefill --
ifx_status Model::ensure_ws(size_t n) {
  if (n <= ws_tokens) return IFX_OK;
  if (ws) cudaFree(ws);
  if (ids_dev) cudaFree(ids_dev);
  ws = nullptr;
  ids_dev = nullptr;
  const ifx_config &c = cfg;
  const size_t D = c.hidden_size, Hh = Hl * c.head_dim, kvd = Gl * c.head_dim;
  const size_t F = Fl;
  // staged inputs: the fused kernels' fragments, or plain f32 rows (dense)
  const size_t xf = std::max(gemm_xfrag_bytes((int64_t)n, (int64_t)std::max(D, F)),
                             n * std::max(std::max(D, F), Hh) * sizeof(float));
  const size_t floats = n * (D + Hh + 2 * kvd + Hh + 2 * F + (tp > 1 ? D : 0));
  IFX_CUDA(cudaMalloc(&ws, floats * sizeof(float) + xf + 1024));
  IFX_CUDA(cudaMalloc(&ids_dev, n * sizeof(uint32_t)));
  float *p = reinterpret_cast<float *>(ws);
  w_x = p; p += n * D;
  w_q = p; p += n * Hh;
  w_k = p; p += n * kvd;
  w_v = p; p += n * kvd;
  w_attn = p; p += n * Hh;
  w_gate = p; p += n * F;
  w_up = p; p += n * F;
  if (tp > 1) {
    w_y = p;
    p += n * D;
  }
  w_xf = reinterpret_cast<uint8_t *>(reinterpret_cast<uintptr_t>(p + 64) & ~(uintptr_t)255);
  ws_tokens = n;
  return IFX_OK;
}

ifx_status Model::prefill(KvCache &kv, const uint32_t *ids, size_t n, float *logits_host,
                          int last_row_only) {
  return run_prompt(&kv, ids, n, logits_host, last_row_only);
}

// Model::forward (forward.rs:448-482): the layers over the whole prompt with
// attention over every position (no mask), RoPE at positions 0..n, no cache.
ifx_status Model::forward(const uint32_t *ids, size_t n, float *logits_host, int last_row_only) {
  return run_prompt(nullptr, ids, n, logits_host, last_row_only);
}

// ------------------------------------------------------ batched decode --
static ifx_status cuda_ok(cudaError_t e) {
  return e == cudaSuccess ? IFX_OK : cuda_fail(e, "batched greedy decode");
}

// Prefill of sequence `seq` of a batch: Model::prefill on a KvCache view of
// that sequence's cache slice.
ifx_status Model::prefill_seq(KvBatch &kb, int seq, const uint32_t *ids, size_t n,
                              float *logits_host, int last_row_only) {
  if (seq < 0 || seq >= kb.batch) return fail(IFX_ERR_INVALID_ARGUMENT, "batch: no such sequence");
  KvCache view;
  view.owner = false;
  view.m = this;
  view.max_seq = kb.max_seq;
  view.per_layer = kb.per_layer;
  if (kb.paged) {
    if (kb.len[(size_t)seq] + n > kb.max_seq)
      return fail(IFX_ERR_INVALID_TENSOR_INDEX, "KV cache is full");
    IFX_CUDA(cudaSetDevice(device));
    IFX_TRY(kb.reserve(seq, kb.len[(size_t)seq] + n, stream));
    view.k = kb.k;
    view.v = kb.v;
    view.page_table = kb.table_dev + (size_t)seq * kb.max_pages;
    view.page_rows = kb.page_rows;
    view.page_stride = kb.page_stride;
  } else {
    view.k = kb.k + (size_t)seq * cfg.n_layers * kb.per_layer;
    view.v = kb.v + (size_t)seq * cfg.n_layers * kb.per_layer;
  }
  view.pos = kb.pos + seq;
  view.len = kb.len[(size_t)seq];
  view.mega_tried = true;  // never planned for the persistent kernel
  const ifx_status s = run_prompt(&view, ids, n, logits_host, last_row_only);
  kb.len[(size_t)seq] = view.len;
  return s;
}

// One decode step of every sequence of the batch (Model::decode_step,
// forward.rs:543-586, for B tokens at once): each weight matrix is read once
// by the small-batch GEMM (exact integer weights, K split over the GPU,
// results added atomically, so outputs start zeroed and the residual
// projections add straight into x), attention runs per (sequence, kv head,
// split) at each sequence's own position, then the logits and their argmax.
ifx_status Model::enqueue_decode_batch(KvBatch &kb, cudaStream_t st, int n, const int *slot_dev) {
  const ifx_config &c = cfg;
  const int B = n < 0 ? kb.batch : n, D = (int)c.hidden_size, H = (int)Hl, G = (int)Gl, hd = (int)c.head_dim;
  const int F = (int)Fl, V = (int)c.vocab_size, Hh = H * hd;
  const int64_t qkvw = (int64_t)(H + 2 * G) * hd;
  const float eps = c.norm_eps;
  embed_rows_kernel<<<(unsigned)B, 256, 0, st>>>(emb_raw, emb_type, D, kb.ids, kb.x);
  IFX_CUDA(cudaGetLastError());
  for (uint64_t l = 0; l < c.n_layers; ++l) {
    Layer &L = layers[l];
    StageZero zq;  // the QKV GEMMs accumulate into qkv
    zq.p[0] = kb.qkv;
    zq.n[0] = (int64_t)B * qkvw;
    IFX_TRY(stage_small(kb.x, nullptr, L.attn_norm, eps, GX_RMSNORM, B, D, kb.xf, st, zq));
    {  // Wq, Wk, Wv in one launch
      const QMatrix *ws[3] = {&L.wq, &L.wk, &L.wv};
      float *cs[3] = {kb.qkv, kb.qkv + Hh, kb.qkv + Hh + G * hd};
      const int64_t ls[3] = {qkvw, qkvw, qkvw};
      IFX_TRY(gemm_small_run_multi(ws, cs, ls, 3, kb.xf, B, err, st));
    }
    DecodeAttnArgs a{};
    a.qkv = kb.qkv;
    a.qkv_stride = qkvw;
    a.kc = kb.k + l * kb.per_layer;
    a.vc = kb.v + l * kb.per_layer;
    a.kv_seq_stride = kb.paged ? 0 : (int64_t)(c.n_layers * kb.per_layer);
    if (kb.paged) {
      a.page_table = kb.table_dev;
      a.page_rows = kb.page_rows;
      a.max_pages = kb.max_pages;
      a.page_stride = kb.page_stride;
    }
    a.pos = kb.pos;
    a.part_o = kb.part_o;
    a.part_ml = kb.part_ml;
    a.counters = kb.counters;
    a.attn_out = kb.attn;
    a.H = H;
    a.G = G;
    a.hd = hd;
    a.max_seq = (int)kb.max_seq;
    a.ns = kb.ns;
    a.rope_compat = opts.rope_compat;
    a.rope_dim = (int)c.rope_dim;
    a.rope_base = c.rope_base;
    a.err = err;
    a.batch = B;
    a.slot = slot_dev;
    IFX_TRY(decode_attention(a, st, true));
    IFX_TRY(stage_small(kb.attn, nullptr, nullptr, 0.f, GX_PLAIN, B, Hh, kb.xf, st));
    IFX_TRY(gemm_small_run(L.wo, kb.xf, B, kb.x, D, err, st));  // x += attn Wo^T
    StageZero zf;  // W1 / W3 accumulate into gate / up
    zf.p[0] = kb.gate;
    zf.p[1] = kb.up;
    zf.n[0] = zf.n[1] = (int64_t)B * F;
    IFX_TRY(stage_small(kb.x, nullptr, L.ffn_norm, eps, GX_RMSNORM, B, D, kb.xf, st, zf));
    {  // W1, W3 in one launch
      const QMatrix *ws[2] = {&L.w1, &L.w3};
      float *cs[2] = {kb.gate, kb.up};
      const int64_t ls[2] = {F, F};
      IFX_TRY(gemm_small_run_multi(ws, cs, ls, 2, kb.xf, B, err, st));
    }
    IFX_TRY(stage_small(kb.gate, kb.up, nullptr, 0.f, GX_SWIGLU, B, F, kb.xf, st));
    IFX_TRY(gemm_small_run(L.w2, kb.xf, B, kb.x, D, err, st));  // x += swiglu W2^T
  }
  StageZero zl;  // the logits GEMM accumulates into logits
  zl.p[0] = kb.logits;
  zl.n[0] = (int64_t)B * V;
  IFX_TRY(stage_small(kb.x, nullptr, out_norm, eps, GX_RMSNORM, B, D, kb.xf, st, zl));
  IFX_TRY(gemm_small_run(out_w, kb.xf, B, kb.logits, V, err, st));
  IFX_CUDA(cudaMemsetAsync(kb.keys, 0, sizeof(unsigned long long) * (size_t)B, st));
  argmax_rows_kernel<<<dim3((unsigned)B, kArgmaxParts), 256, 0, st>>>(kb.logits, V, kb.keys);
  argmax_keys_kernel<<<1, 32, 0, st>>>(kb.keys, B, kb.out, kb.pos, slot_dev);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status Model::decode_batch(KvBatch &kb, const uint32_t *tokens, float *logits_host,
                               uint32_t *argmax_host) {
  NvtxRange nvtx_("ifx:decode_step_batch");
  for (int b = 0; b < kb.batch; ++b) {
    if (tokens[b] >= cfg.vocab_size)
      return fail(IFX_ERR_INVALID_TENSOR_INDEX,
                  "tensor index out of bounds: " + std::to_string(tokens[b]));
    if (kb.len[(size_t)b] >= kb.max_seq) return fail(IFX_ERR_INVALID_TENSOR_INDEX, "KV cache is full");
  }
  IFX_CUDA(cudaSetDevice(device));
  cudaStream_t st = stream;
  for (int b = 0; b < kb.batch; ++b) IFX_TRY(kb.reserve(b, kb.len[(size_t)b] + 1, st));
  IFX_CUDA(cudaMemcpyAsync(kb.ids, tokens, sizeof(uint32_t) * kb.batch, cudaMemcpyHostToDevice, st));
  IFX_TRY(enqueue_decode_batch(kb, st));
  if (logits_host)
    IFX_CUDA(cudaMemcpyAsync(logits_host, kb.logits, sizeof(float) * kb.batch * cfg.vocab_size,
                             cudaMemcpyDeviceToHost, st));
  if (argmax_host)
    IFX_CUDA(cudaMemcpyAsync(argmax_host, kb.out, sizeof(uint32_t) * kb.batch,
                             cudaMemcpyDeviceToHost, st));
  IFX_CUDA(cudaStreamSynchronize(st));
  for (auto &n : kb.len) n += 1;
  return check_err();
}

// One decode step of the n distinct sequences seqs[0..n) of the batch (a
// serving loop whose requests come and go: the others keep their caches and
// positions). Row i of logits_host [n, vocab] / argmax_host [n] is seqs[i].
ifx_status Model::decode_batch_seqs(KvBatch &kb, const int *seqs, int n, const uint32_t *tokens,
                                    float *logits_host, uint32_t *argmax_host) {
  NvtxRange nvtx_("ifx:decode_step_batch_seqs");
  if (n < 1 || n > kb.batch)
    return fail(IFX_ERR_INVALID_ARGUMENT, "batch step: 1 to batch sequences");
  std::vector<char> seen((size_t)kb.batch, 0);
  for (int i = 0; i < n; ++i) {
    if (seqs[i] < 0 || seqs[i] >= kb.batch) return fail(IFX_ERR_INVALID_ARGUMENT, "batch: no such sequence");
    if (seen[(size_t)seqs[i]]++) return fail(IFX_ERR_INVALID_ARGUMENT, "batch step: a sequence listed twice");
    if (tokens[i] >= cfg.vocab_size)
      return fail(IFX_ERR_INVALID_TENSOR_INDEX,
                  "tensor index out of bounds: " + std::to_string(tokens[i]));
    if (kb.len[(size_t)seqs[i]] >= kb.max_seq) return fail(IFX_ERR_INVALID_TENSOR_INDEX, "KV cache is full");
  }
  IFX_CUDA(cudaSetDevice(device));
  cudaStream_t st = stream;
  for (int i = 0; i < n; ++i) IFX_TRY(kb.reserve(seqs[i], kb.len[(size_t)seqs[i]] + 1, st));
  IFX_CUDA(cudaMemcpyAsync(kb.ids, tokens, sizeof(uint32_t) * n, cudaMemcpyHostToDevice, st));
  IFX_CUDA(cudaMemcpyAsync(kb.slots, seqs, sizeof(int) * n, cudaMemcpyHostToDevice, st));
  IFX_TRY(enqueue_decode_batch(kb, st, n, kb.slots));
  if (logits_host)
    IFX_CUDA(cudaMemcpyAsync(logits_host, kb.logits, sizeof(float) * n * cfg.vocab_size,
                             cudaMemcpyDeviceToHost, st));
  if (argmax_host)
    IFX_CUDA(cudaMemcpyAsync(argmax_host, kb.out, sizeof(uint32_t) * n, cudaMemcpyDeviceToHost, st));
  IFX_CUDA(cudaStreamSynchronize(st));
  for (int i = 0; i < n; ++i) kb.len[(size_t)seqs[i]] += 1;
  return check_err();
}

ifx_status Model::step_sync(cudaStream_t st) {
  if (tp <= 1) {
    IFX_CUDA(cudaStreamSynchronize(st));
    return IFX_OK;
  }
  const double ms = opts.tp_timeout_ms > 0 ? (double)opts.tp_timeout_ms : 300000.0;
  const ifx_status s = tp_wait(st, (ncclComm_t)comm, nccl, ms);
  if (s == IFX_ERR_NCCL || s == IFX_ERR_TIMEOUT) comm_aborted = true;
  return s;
}

ifx_status Model::tp_usable() const {
  if (!comm_aborted) return IFX_OK;
  return fail(IFX_ERR_NCCL,
              "tensor parallel: the communicator was aborted after a failed call; free the model, "
              "make a new communicator and load again");
}

// KvCache::clear (cache.rs:26-28) for one sequence of the batch.
ifx_status Model::reset_seq(KvBatch &kb, int seq) {
  if (seq < 0 || seq >= kb.batch) return fail(IFX_ERR_INVALID_ARGUMENT, "batch: no such sequence");
  IFX_CUDA(cudaSetDevice(device));
  IFX_CUDA(cudaMemsetAsync(kb.pos + seq, 0, sizeof(int), stream));
  IFX_CUDA(cudaStreamSynchronize(stream));
  kb.len[(size_t)seq] = 0;
  kb.release(seq);
  return IFX_OK;
}

// n greedy steps of every sequence, each step's argmax fed to the next on
// the device; out[i * batch + b] is sequence b's token of step i.
// One full-batch step with its argmax fed back as the next step's ids: a
// CUDA graph replay once a first step has run eagerly (the launch sequence
// does not change between steps: positions and page tables live on the
// device, pages are reserved before the loop).
ifx_status Model::step_batch_fed(KvBatch &kb, cudaStream_t st) {
  auto enqueue = [&]() -> ifx_status {
    IFX_TRY(enqueue_decode_batch(kb, st));
    IFX_CUDA(cudaMemcpyAsync(kb.ids, kb.out, sizeof(uint32_t) * kb.batch, cudaMemcpyDeviceToDevice, st));
    return IFX_OK;
  };
  if (!opts.use_graphs || !kb.warm) {
    kb.warm = true;
    return enqueue();
  }
  if (!kb.graph) {
    cudaGraph_t g;
    IFX_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    ifx_status s = enqueue();
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (s != IFX_OK) return s;
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&kb.graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      kb.graph = nullptr;
      return cuda_fail(e, "cudaGraphInstantiate");
    }
  }
  IFX_CUDA(cudaGraphLaunch(kb.graph, st));
  return IFX_OK;
}

ifx_status Model::decode_greedy_batch(KvBatch &kb, const uint32_t *tokens, size_t n,
                                      uint32_t *out, float *device_ms) {
  NvtxRange nvtx_("ifx:decode_greedy_batch");
  for (int b = 0; b < kb.batch; ++b) {
    if (tokens[b] >= cfg.vocab_size)
      return fail(IFX_ERR_INVALID_TENSOR_INDEX,
                  "tensor index out of bounds: " + std::to_string(tokens[b]));
    if (kb.len[(size_t)b] + n > kb.max_seq) return fail(IFX_ERR_INVALID_TENSOR_INDEX, "KV cache is full");
  }
  IFX_CUDA(cudaSetDevice(device));
  cudaStream_t st = stream;
  for (int b = 0; b < kb.batch; ++b) IFX_TRY(kb.reserve(b, kb.len[(size_t)b] + n, st));
  uint32_t *toks = nullptr;  // every step's tokens, copied out once at the end
  IFX_TRY(dalloc(&toks, std::max<size_t>(1, n) * kb.batch));
  IFX_CUDA(cudaMemcpyAsync(kb.ids, tokens, sizeof(uint32_t) * kb.batch, cudaMemcpyHostToDevice, st));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (device_ms) {
    IFX_CUDA(cudaEventCreate(&e0));
    IFX_CUDA(cudaEventCreate(&e1));
    IFX_CUDA(cudaEventRecord(e0, st));
  }
  ifx_status s = IFX_OK;
  for (size_t i = 0; i < n && s == IFX_OK; ++i) {
    s = step_batch_fed(kb, st);
    if (s == IFX_OK)
      s = cuda_ok(cudaMemcpyAsync(toks + i * kb.batch, kb.out, sizeof(uint32_t) * kb.batch,
                                  cudaMemcpyDeviceToDevice, st));
  }
  if (device_ms && s == IFX_OK) s = cuda_ok(cudaEventRecord(e1, st));
  if (s == IFX_OK && out && n)
    s = cuda_ok(cudaMemcpyAsync(out, toks, sizeof(uint32_t) * n * kb.batch, cudaMemcpyDeviceToHost, st));
  cudaStreamSynchronize(st);
  cudaFree(toks);
  if (device_ms) {
    if (s == IFX_OK) s = cuda_ok(cudaEventElapsedTime(device_ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }
  IFX_TRY(s);
  for (auto &l : kb.len) l += n;
  return check_err();
}

// Shared body of prefill (kvp set: causal attention, K/V appended to the
// cache) and forward (kvp null: full attention, no cache).
ifx_status Model::run_prompt(KvCache *kvp, const uint32_t *ids, size_t n, float *logits_host,
                             int last_row_only) {
  NvtxRange nvtx_("ifx:prompt");
  IFX_TRY(tp_usable());
  const ifx_config &c = cfg;
  for (size_t i = 0; i < n; ++i)
    if (ids[i] >= c.vocab_size)  // forward.rs:453-455, 501-503
      return fail(IFX_ERR_INVALID_TENSOR_INDEX, "tensor index out of bounds: 0");
  if (n == 0) return IFX_OK;
  if (kvp && kvp->len + n > kvp->max_seq)
    return fail(IFX_ERR_INVALID_TENSOR_INDEX, "prompt exceeds the KV cache");
  IFX_CUDA(cudaSetDevice(device));
  IFX_TRY(ensure_ws(n));
  cudaStream_t st = stream;
  const int64_t N = (int64_t)n;
  const int D = (int)c.hidden_size, H = (int)Hl, G = (int)Gl, hd = (int)c.head_dim;
  const int F = (int)Fl;
  const int Hh = H * hd, kvd = G * hd;
  const int start = kvp ? (int)kvp->len : 0;
  IFX_CUDA(cudaMemcpyAsync(ids_dev, ids, n * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
  embed_rows_kernel<<<(unsigned)n, 256, 0, st>>>(emb_raw, emb_type, D, ids_dev, w_x);
  IFX_CUDA(cudaGetLastError());
  const int pos0 = opts.rope_compat ? 0 : start;  // forward.rs:243-244 ignores cache_start
  for (uint64_t l = 0; l < c.n_layers; ++l) {
    Layer &L = layers[l];
    IFX_TRY(stage_rows(w_x, nullptr, L.attn_norm, c.norm_eps, GX_RMSNORM, N, D, w_xf, st));
    {  // Wq, Wk, Wv over one staged input
      const QMatrix *ws[3] = {&L.wq, &L.wk, &L.wv};
      float *cs[3] = {w_q, w_k, w_v};
      const int64_t ls[3] = {Hh, kvd, kvd};
      IFX_TRY(gemm_run_multi(ws, cs, ls, 3, w_xf, N, 0, err, st));
    }
    IFX_TRY(op_rope(w_q, n, H, hd, c.rope_dim, c.rope_base, pos0, st));
    IFX_TRY(op_rope(w_k, n, G, hd, c.rope_dim, c.rope_base, pos0, st));
    if (kvp) {
      KvCache &kv = *kvp;
      if (kv.page_table)
        kv_write_paged_kernel<<<(unsigned)n, 256, 0, st>>>(w_k, w_v, kv.k + l * kv.per_layer,
                                                           kv.v + l * kv.per_layer, (int)n, G, hd,
                                                           kv.page_rows, kv.page_stride,
                                                           kv.page_table, start);
      else
        kv_write_kernel<<<(unsigned)n, 256, 0, st>>>(w_k, w_v, kv.k + l * kv.per_layer,
                                                     kv.v + l * kv.per_layer, (int)n, G, hd,
                                                     (int)kv.max_seq, start);
      IFX_CUDA(cudaGetLastError());
    }
    PrefillAttnArgs pa{w_q, w_k, w_v, w_attn, (int)n, H, G, hd, kvp ? 1 : 0};
    if (kvp) {  // the chunk's K/V rows were just written to the cache: stream them from there
      const KvCache &kv = *kvp;
      pa.kc = kv.k + l * kv.per_layer;
      pa.vc = kv.v + l * kv.per_layer;
      pa.start = start;
      pa.max_seq = (int)kv.max_seq;
      pa.page_table = kv.page_table;
      pa.page_rows = kv.page_rows;
      pa.page_stride = kv.page_stride;
      pa.err = err;
    }
    IFX_TRY(prefill_attention(pa, st));
    IFX_TRY(stage_rows(w_attn, nullptr, nullptr, 0.f, GX_PLAIN, N, Hh, w_xf, st));
    if (tp > 1) {
      IFX_TRY(tp_partial_begin((size_t)N * D, st, w_y, w_x));
      IFX_TRY(gemm_run(L.wo, w_xf, N, w_y, D, 1, err, st));
      IFX_TRY(tp_partial_end((size_t)N * D, st, w_y, w_x));
    } else {
      IFX_TRY(gemm_run(L.wo, w_xf, N, w_x, D, 1, err, st));
    }
    IFX_TRY(stage_rows(w_x, nullptr, L.ffn_norm, c.norm_eps, GX_RMSNORM, N, D, w_xf, st));
    {  // W1, W3 over one staged input
      const QMatrix *ws[2] = {&L.w1, &L.w3};
      float *cs[2] = {w_gate, w_up};
      const int64_t ls[2] = {F, F};
      IFX_TRY(gemm_run_multi(ws, cs, ls, 2, w_xf, N, 0, err, st));
    }
    IFX_TRY(stage_rows(w_gate, w_up, nullptr, 0.f, GX_SWIGLU, N, F, w_xf, st));
    if (tp > 1) {
      IFX_TRY(tp_partial_begin((size_t)N * D, st, w_y, w_x));
      IFX_TRY(gemm_run(L.w2, w_xf, N, w_y, D, 1, err, st));
      IFX_TRY(tp_partial_end((size_t)N * D, st, w_y, w_x));
    } else {
      IFX_TRY(gemm_run(L.w2, w_xf, N, w_x, D, 1, err, st));
    }
  }
  if (kvp) {
    add_int_kernel<<<1, 1, 0, st>>>(kvp->pos, (int)n);  // forward.rs:520
    IFX_CUDA(cudaGetLastError());
  }
  if (last_row_only || !logits_host) {
    // logits of the last row into the decode logits buffer (GEMV; under
    // tensor parallelism this rank's vocab slice, then gathered)
    IFX_CUDA(cudaMemsetAsync(logits_local, 0, Vl * sizeof(float), st));
    GemvPlan p = p_logits;
    const QMatrix *mo[1] = {&out_w};
    float *yo[1] = {logits_local};
    gemv_plan_rebind(&p, mo, yo, w_x + (size_t)(n - 1) * D, nullptr, out_norm);
    IFX_TRY(gemv_launch(p, st, false));
    if (tp > 1)
      IFX_NCCL(nccl, nccl->AllGather(logits_local, logits, Vl, ncclFloat32, (ncclComm_t)comm, st));
    if (logits_host)
      IFX_CUDA(cudaMemcpyAsync(logits_host, logits, c.vocab_size * sizeof(float),
                               cudaMemcpyDeviceToHost, st));
  } else {
    const size_t need = n * c.vocab_size;
    if (need > logits_all_n) {
      if (logits_all) cudaFree(logits_all);
      logits_all = nullptr;
      IFX_CUDA(cudaMalloc(&logits_all, need * sizeof(float)));
      logits_all_n = need;
    }
    IFX_TRY(stage_rows(w_x, nullptr, out_norm, c.norm_eps, GX_RMSNORM, N, D, w_xf, st));
    if (tp > 1) {
      // [n][Vl] per rank, gathered rank-major, then interleaved to [n][V]
      const size_t loc = n * Vl;
      if (2 * loc * tp > logits_all_local_n) {
        if (logits_all_local) cudaFree(logits_all_local);
        logits_all_local = nullptr;
        IFX_CUDA(cudaMalloc(&logits_all_local, 2 * loc * tp * sizeof(float)));
        logits_all_local_n = 2 * loc * tp;
      }
      float *mine = logits_all_local, *gathered = logits_all_local + loc * tp;
      IFX_TRY(gemm_run(out_w, w_xf, N, mine, (int)Vl, 0, err, st));
      IFX_NCCL(nccl, nccl->AllGather(mine, gathered, loc, ncclFloat32, (ncclComm_t)comm, st));
      shard_interleave_kernel<<<(unsigned)n, 256, 0, st>>>(gathered, logits_all, (int)n, (int)Vl, tp);
      IFX_CUDA(cudaGetLastError());
    } else {
      IFX_TRY(gemm_run(out_w, w_xf, N, logits_all, c.vocab_size, 0, err, st));
    }
    IFX_CUDA(cudaMemcpyAsync(logits_host, logits_all, need * sizeof(float), cudaMemcpyDeviceToHost, st));
    // keep the last row as "the model's last logits" for ifx_sample
    IFX_CUDA(cudaMemcpyAsync(logits, logits_all + (n - 1) * c.vocab_size,
                             c.vocab_size * sizeof(float), cudaMemcpyDeviceToDevice, st));
  }
  IFX_TRY(step_sync(st));
  if (kvp) kvp->len += n;
  return check_err();
}

ifx_status Model::generate(KvCache &kv, const uint32_t *prompt, size_t n_prompt,
                           size_t max_tokens, uint32_t *out) {
  if (n_prompt == 0) return fail(IFX_ERR_SHAPE, "generate: empty prompt");
  IFX_TRY(kv.clear());  // forward.rs:600
  if (n_prompt + max_tokens > kv.max_seq)
    return fail(IFX_ERR_INVALID_TENSOR_INDEX, "prompt + max_tokens exceeds the KV cache");
  IFX_TRY(prefill(kv, prompt, n_prompt, nullptr, 1));
  cudaStream_t st = stream;
  IFX_CUDA(cudaMemsetAsync(n_out, 0, sizeof(int), st));
  IFX_CUDA(launch(argmax_step_kernel, dim3(kNumSMs), dim3(256), 0, st, false, (const float *)logits,
                  (int)cfg.vocab_size, amax_key, amax_count, next_token, kv.tokens, n_out, kv.pos, 1, 0,
                  0, 1));
  for (size_t i = 0; i < max_tokens; ++i) IFX_TRY(run_decode(kv, i + 1 == max_tokens));
  if (max_tokens)
    IFX_CUDA(cudaMemcpyAsync(out, kv.tokens, max_tokens * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  IFX_TRY(step_sync(st));
  kv.len += max_tokens;
  return check_err();
}

ifx_status Model::decode_greedy(KvCache &kv, uint32_t token, size_t n, uint32_t *out,
                                float *device_ms) {
  NvtxRange nvtx_("ifx:decode_greedy");
  IFX_TRY(tp_usable());
  if (token >= cfg.vocab_size)
    return fail(IFX_ERR_INVALID_TENSOR_INDEX, "tensor index out of bounds: " + std::to_string(token));
  if (kv.len + n > kv.max_seq) return fail(IFX_ERR_INVALID_TENSOR_INDEX, "KV cache is full");
  IFX_CUDA(cudaSetDevice(device));
  cudaStream_t st = stream;
  IFX_CUDA(cudaMemcpyAsync(next_token, &token, sizeof(uint32_t), cudaMemcpyHostToDevice, st));
  IFX_CUDA(cudaMemsetAsync(n_out, 0, sizeof(int), st));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (device_ms) {
    IFX_CUDA(cudaEventCreate(&e0));
    IFX_CUDA(cudaEventCreate(&e1));
    IFX_CUDA(cudaEventRecord(e0, st));
  }
  for (size_t i = 0; i < n; ++i) IFX_TRY(run_decode(kv, i + 1 == n));
  if (device_ms) IFX_CUDA(cudaEventRecord(e1, st));
  if (out && n)
    IFX_CUDA(cudaMemcpyAsync(out, kv.tokens, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  IFX_TRY(step_sync(st));
  if (device_ms) {
    IFX_CUDA(cudaEventElapsedTime(device_ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }
  kv.len += n;
  return check_err();
}

ifx_status Model::bench_kernel(KvCache &kv, const std::string &which, int reps, float *ms,
                               uint64_t *bytes) {
  if (reps < 1) return fail(IFX_ERR_INVALID_ARGUMENT, "bench_kernel: reps < 1");
  IFX_CUDA(cudaSetDevice(device));
  cudaStream_t st = stream;
  const int L = (int)cfg.n_layers;
  std::vector<GemvPlan> *plans = nullptr;
  if (which == "qkv") plans = &p_qkv;
  else if (which == "wo") plans = &p_wo;
  else if (which == "w13") plans = &p_w13;
  else if (which == "w2") plans = &p_w2;
  else if (which != "logits" && which != "attn")
    return fail(IFX_ERR_INVALID_ARGUMENT, "bench_kernel: unknown kernel " + which);
  cudaEvent_t e0, e1;
  IFX_CUDA(cudaEventCreate(&e0));
  IFX_CUDA(cudaEventCreate(&e1));
  uint64_t b = 0;
  // one untimed pass so first-launch costs stay out of the timing
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) IFX_CUDA(cudaEventRecord(e0, st));
    b = 0;
    for (int r = 0; r < reps; ++r) {
      const int l = r % L;
      if (plans) {
        IFX_TRY(gemv_launch((*plans)[l], st, false));
        b += (*plans)[l].weight_bytes;
      } else if (which == "logits") {
        IFX_TRY(gemv_launch(p_logits, st, false));
        b += p_logits.weight_bytes;
      } else {
        DecodeAttnArgs a{};
        a.qkv = qkv;
        a.kc = kv.k + l * kv.per_layer;
        a.vc = kv.v + l * kv.per_layer;
        a.pos = kv.pos;
        a.part_o = part_o;
        a.part_ml = part_ml;
        a.counters = counters;
        a.attn_out = attn;
        a.H = (int)Hl;
        a.G = (int)Gl;
        a.hd = (int)cfg.head_dim;
        a.max_seq = (int)kv.max_seq;
        a.ns = ns;
        a.rope_compat = opts.rope_compat;
        a.rope_dim = (int)cfg.rope_dim;
        a.rope_base = cfg.rope_base;
        a.err = err;
        IFX_TRY(decode_attention(a, st, false));
        b += 2ull * Gl * (kv.len + 1) * cfg.head_dim * sizeof(__half);
      }
    }
  }
  IFX_CUDA(cudaEventRecord(e1, st));
  IFX_CUDA(cudaEventSynchronize(e1));
  float t = 0.f;
  IFX_CUDA(cudaEventElapsedTime(&t, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *ms = t / reps;
  *bytes = b / (uint64_t)reps;
  return check_err();
}

ifx_status Model::kv_read(const KvCache &kv, size_t layer, int which_v, float *out_host) {
  if (layer >= cfg.n_layers) return fail(IFX_ERR_INVALID_TENSOR_INDEX, "layer out of range");
  const int G = (int)Gl, hd = (int)cfg.head_dim;
  if (kv.len == 0) return IFX_OK;
  float *tmp = nullptr;
  IFX_CUDA(cudaMalloc(&tmp, kv.len * G * hd * sizeof(float)));
  const __half *src = (which_v ? kv.v : kv.k) + layer * kv.per_layer;
  kv_read_kernel<<<(unsigned)kv.len, 256, 0, stream>>>(src, tmp, (int)kv.len, G, hd, (int)kv.max_seq);
  cudaMemcpyAsync(out_host, tmp, kv.len * G * hd * sizeof(float), cudaMemcpyDeviceToHost, stream);
  cudaStreamSynchronize(stream);
  cudaFree(tmp);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

}  // namespace ifx
