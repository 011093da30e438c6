/*
 * refcpu.c — CPU restatement of phraakture/inferox's token loop (TEST
 * INFRASTRUCTURE ONLY; see refcpu.h for the parity status and rules).
 *
 * Build: oracle/Makefile (gcc -O2 -mavx2 -mfma -ffp-contract=off
 * -fno-fast-math). Every function cites the reference file:line it follows;
 * paths are relative to the reference crate root.
 */
#define _GNU_SOURCE
#include "refcpu.h"

#include <math.h>
#include <stdio.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define RC_HAVE_AVX2 1
#else
#define RC_HAVE_AVX2 0
#endif

static int g_threads = 1;
static int g_faithful = 0;

void rc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
void rc_set_faithful(int on) { g_faithful = on ? 1 : 0; }

/* ------------------------------------------------------------------------ */
/* half -> f32 (the `half` 2.7.1 crate's to_f32 is the exact IEEE widening). */
float rc_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while ((man & 0x400u) == 0);
      man &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    /* half 2.x f16_to_f32: infinities kept, NaNs keep their payload and get
     * the quiet bit (0x7FC0_0000), in both its F16C and software paths */
    bits = sign | (man ? 0x7fc00000u : 0x7f800000u) | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline float ld_f16(const uint8_t *p) {
  return rc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
}

/* TensorType::element_size / block_layout (src/gguf/types.rs:181-229). */
static int elem_size(int t) {
  switch (t) {
  case RC_F32: return 4;
  case RC_F16: return 2;
  case RC_I8: return 1;
  case RC_I16: return 2;
  case RC_I32: return 4;
  case RC_I64: return 8;
  case RC_F64: return 8;
  default: return 0;
  }
}
static int block_layout(int t, int *elems, int *bytes) {
  int e = 0, b = 0;
  switch (t) {
  case RC_Q4_0: e = 32; b = 18; break;
  case RC_Q4_1: e = 32; b = 20; break;
  case RC_Q5_0: e = 32; b = 22; break;
  case RC_Q5_1: e = 32; b = 24; break;
  case RC_Q8_0: e = 32; b = 34; break;
  case RC_Q8_1: e = 32; b = 36; break;
  case RC_IQ4NL: e = 32; b = 18; break;
  case RC_Q2K: e = 256; b = 96; break;
  case RC_Q3K: e = 256; b = 110; break;
  case RC_Q4K: e = 256; b = 144; break;
  case RC_Q5K: e = 256; b = 176; break;
  case RC_Q6K: e = 256; b = 210; break;
  case RC_Q8K: e = 256; b = 292; break;
  case RC_IQ1S: e = 256; b = 166; break;
  case RC_IQ1M: e = 256; b = 184; break;
  case RC_IQ2XXS: e = 256; b = 66; break;
  case RC_IQ2XS: e = 256; b = 104; break;
  case RC_IQ2S: e = 256; b = 176; break;
  case RC_IQ3XXS: e = 256; b = 98; break;
  case RC_IQ3S: e = 256; b = 166; break;
  case RC_IQ4XS: e = 256; b = 136; break;
  case RC_IQ4XSS: e = 256; b = 116; break;
  default: return 0;
  }
  *elems = e;
  *bytes = b;
  return 1;
}

static int valid_type_id(uint32_t v) {
  /* TensorType::from_u32 (types.rs:110-142): 0..30 except 4 and 9. */
  return v <= 30 && v != 4 && v != 9;
}

/* TensorInfo::byte_size (src/gguf/tensor.rs:30-40). */
int64_t rc_type_byte_size(int type, uint64_t n) {
  int es = elem_size(type);
  if (es) return (int64_t)(n * (uint64_t)es);
  int be, bb;
  if (block_layout(type, &be, &bb)) {
    uint64_t blocks = (n + (uint64_t)be - 1) / (uint64_t)be;
    return (int64_t)(blocks * (uint64_t)bb);
  }
  return -1;
}

/* ---------------------------- dequantisers ------------------------------ */
/* Each writes out[0..n_out); blocks past n_out are ignored (the reference
 * would index out of bounds there). */

/* dequantize_f32_f32 (dequant.rs:40-45) */
static void dq_f32(const uint8_t *b, size_t nb, float *o, size_t n) {
  size_t cnt = nb / 4;
  for (size_t i = 0; i < cnt && i < n; i++) memcpy(&o[i], b + 4 * i, 4);
}
/* dequantize_f16_f32 (dequant.rs:47-52) */
static void dq_f16(const uint8_t *b, size_t nb, float *o, size_t n) {
  size_t cnt = nb / 2;
  for (size_t i = 0; i < cnt && i < n; i++) o[i] = ld_f16(b + 2 * i);
}
/* dequantize_q4_0 (dequant.rs:62-84): (nib-8)*delta, low nibble -> j,
 * high nibble -> j+16. */
static void dq_q4_0(const uint8_t *b, size_t nb, float *o, size_t n) {
  for (size_t blk = 0; blk < nb / 18; blk++) {
    const uint8_t *c = b + blk * 18;
    float delta = ld_f16(c);
    size_t base = blk * 32;
    for (int j = 0; j < 16; j++) {
      int q0 = (c[2 + j] & 0x0f) - 8, q1 = (c[2 + j] >> 4) - 8;
      if (base + j < n) o[base + j] = (float)q0 * delta;
      if (base + j + 16 < n) o[base + j + 16] = (float)q1 * delta;
    }
  }
}
/* dequantize_q8_0 (dequant.rs:93-111): i8 * delta */
static void dq_q8_0(const uint8_t *b, size_t nb, float *o, size_t n) {
  for (size_t blk = 0; blk < nb / 34; blk++) {
    const uint8_t *c = b + blk * 34;
    float delta = ld_f16(c);
    size_t base = blk * 32;
    for (int j = 0; j < 32 && base + j < n; j++)
      o[base + j] = (float)(int8_t)c[2 + j] * delta;
  }
}
/* dequantize_q4_k (dequant.rs:123-163): 6-bit scale/min unpack (:141-149),
 * dall = d*sc, dm = dmin*mn, y = dall*q - dm (:151-158); nibble l of group
 * g at qs[g*16 + l/2], even l -> low nibble (:155-157). */
static void q4k_scale_min(const uint8_t *s, int g, float *sc, float *mn) {
  if (g < 4) {
    *sc = (float)(s[g] & 0x3f);
    *mn = (float)(s[g + 4] & 0x3f);
  } else {
    *sc = (float)((uint32_t)(s[g + 4] & 0x0f) | (((uint32_t)s[g - 4] >> 6) << 4));
    *mn = (float)(((uint32_t)s[g + 4] >> 4) | (((uint32_t)s[g] >> 6) << 4));
  }
}
static void dq_q4_k(const uint8_t *b, size_t nb, float *o, size_t n) {
  for (size_t blk = 0; blk < nb / 144; blk++) {
    const uint8_t *c = b + blk * 144;
    float d = ld_f16(c), dmin = ld_f16(c + 2);
    const uint8_t *scales = c + 4, *qs = c + 16;
    size_t base = blk * 256;
    for (int g = 0; g < 8; g++) {
      float sc, mn;
      q4k_scale_min(scales, g, &sc, &mn);
      float dall = d * sc;
      float dmv = dmin * mn;
      for (int l = 0; l < 32; l++) {
        uint8_t byte = qs[g * 16 + l / 2];
        uint8_t q = (l % 2 == 0) ? (byte & 0x0f) : (byte >> 4);
        size_t idx = base + (size_t)g * 32 + (size_t)l;
        if (idx < n) o[idx] = dall * (float)q - dmv;
      }
    }
  }
}
/* dequantize_q6_k (dequant.rs:174-199): d@0, u8 scales@2..18, ql@18..146,
 * qh@146..210; q = nib(ql[j/2], j%2) | ((qh[j/4] >> 2(j%4)) & 3) << 4;
 * y = d * scales[j/16] as f32 * (q - 32) — the scale byte is read as u8. */
static void dq_q6_k(const uint8_t *b, size_t nb, float *o, size_t n) {
  for (size_t blk = 0; blk < nb / 210; blk++) {
    const uint8_t *c = b + blk * 210;
    float d = ld_f16(c);
    const uint8_t *sc = c + 2, *ql = c + 18, *qh = c + 146;
    size_t base = blk * 256;
    for (int j = 0; j < 256 && base + j < n; j++) {
      uint8_t qlb = ql[j / 2];
      uint8_t nib = (j % 2 == 0) ? (qlb & 0x0f) : (qlb >> 4);
      uint8_t hb = (qh[j / 4] >> (2 * (j % 4))) & 3;
      int q = nib | (hb << 4);
      o[base + j] = d * (float)sc[j / 16] * (float)(q - 32);
    }
  }
}
/* dequantize_q8_k (dequant.rs:210-232): y = d * scales[j/8] * qs[j] - dmin */
static void dq_q8_k(const uint8_t *b, size_t nb, float *o, size_t n) {
  for (size_t blk = 0; blk < nb / 292; blk++) {
    const uint8_t *c = b + blk * 292;
    float d = ld_f16(c), dmin = ld_f16(c + 2);
    const uint8_t *sc = c + 4, *qs = c + 36;
    size_t base = blk * 256;
    for (int j = 0; j < 256 && base + j < n; j++)
      o[base + j] = d * (float)sc[j / 8] * (float)(int8_t)qs[j] - dmin;
  }
}

/* dequantize_f32 (dequant.rs:10-31): size checks, then per-type dispatch;
 * each per-type routine also rejects a byte count that is not a whole number
 * of blocks (e.g. dequant.rs:66-68). */
int rc_dequantize(int type, const uint8_t *bytes, size_t nbytes, float *out,
                  size_t n_out) {
  int64_t expected = rc_type_byte_size(type, n_out);
  if (expected < 0) return RC_ERR_UNKNOWN_TENSOR_TYPE;
  if ((int64_t)nbytes != expected) return RC_ERR_UNEXPECTED_EOF;
  switch (type) {
  case RC_F32: dq_f32(bytes, nbytes, out, n_out); return RC_OK;
  case RC_F16: dq_f16(bytes, nbytes, out, n_out); return RC_OK;
  case RC_Q4_0:
    if (nbytes % 18) return RC_ERR_UNEXPECTED_EOF;
    dq_q4_0(bytes, nbytes, out, n_out); return RC_OK;
  case RC_Q8_0:
    if (nbytes % 34) return RC_ERR_UNEXPECTED_EOF;
    dq_q8_0(bytes, nbytes, out, n_out); return RC_OK;
  case RC_Q4K:
    if (nbytes % 144) return RC_ERR_UNEXPECTED_EOF;
    dq_q4_k(bytes, nbytes, out, n_out); return RC_OK;
  case RC_Q6K:
    if (nbytes % 210) return RC_ERR_UNEXPECTED_EOF;
    dq_q6_k(bytes, nbytes, out, n_out); return RC_OK;
  case RC_Q8K:
    if (nbytes % 292) return RC_ERR_UNEXPECTED_EOF;
    dq_q8_k(bytes, nbytes, out, n_out); return RC_OK;
  default: return RC_ERR_UNKNOWN_TENSOR_TYPE;
  }
}

/* Dequantise elements [e0, e0+cnt) of a tensor (same bits as a whole-tensor
 * dequant followed by a slice). */
static void dequant_range(int type, const uint8_t *bytes, uint64_t e0,
                          size_t cnt, float *out, float *tmp) {
  int es = elem_size(type);
  if (type == RC_F32) { memcpy(out, bytes + e0 * 4, cnt * 4); return; }
  if (type == RC_F16) { dq_f16(bytes + e0 * 2, cnt * 2, out, cnt); return; }
  (void)es;
  int be, bb;
  block_layout(type, &be, &bb);
  uint64_t b0 = e0 / (uint64_t)be, b1 = (e0 + cnt + (uint64_t)be - 1) / (uint64_t)be;
  size_t off = (size_t)(e0 - b0 * (uint64_t)be);
  size_t nel = (size_t)((b1 - b0) * (uint64_t)be);
  const uint8_t *p = bytes + b0 * (uint64_t)bb;
  size_t nb = (size_t)((b1 - b0) * (uint64_t)bb);
  float *dst = (off == 0 && nel == cnt) ? out : tmp;
  switch (type) {
  case RC_Q4_0: dq_q4_0(p, nb, dst, nel); break;
  case RC_Q8_0: dq_q8_0(p, nb, dst, nel); break;
  case RC_Q4K: dq_q4_k(p, nb, dst, nel); break;
  case RC_Q6K: dq_q6_k(p, nb, dst, nel); break;
  case RC_Q8K: dq_q8_k(p, nb, dst, nel); break;
  default: memset(dst, 0, nel * 4); break;
  }
  if (dst == tmp) memcpy(out, tmp + off, cnt * 4);
}

/* ------------------------------- ops ------------------------------------ */
/* hsum256_ps (ops.rs:137-149) lane order:
 * ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)). */
static inline float dot_avx2_order(const float *a, const float *b, size_t k) {
#if RC_HAVE_AVX2
  __m256 acc = _mm256_setzero_ps();
  size_t l = 0;
  for (; l + 8 <= k; l += 8)
    acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + l), _mm256_loadu_ps(b + l), acc);
  __m128 lo = _mm256_castps256_ps128(acc);
  __m128 hi = _mm256_extractf128_ps(acc, 1);
  __m128 s128 = _mm_add_ps(lo, hi);
  __m128 shuf = _mm_movehdup_ps(s128);
  __m128 sums = _mm_add_ps(s128, shuf);
  __m128 shuf2 = _mm_movehl_ps(shuf, sums);
  __m128 sums2 = _mm_add_ss(sums, shuf2);
  float sum = _mm_cvtss_f32(sums2);
  for (; l < k; l++) sum += a[l] * b[l];
  return sum;
#else
  float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t l = 0;
  for (; l + 8 <= k; l += 8)
    for (int i = 0; i < 8; i++) lane[i] = fmaf(a[l + i], b[l + i], lane[i]);
  float s0 = lane[0] + lane[4], s1 = lane[1] + lane[5];
  float s2 = lane[2] + lane[6], s3 = lane[3] + lane[7];
  float sum = (s0 + s1) + (s2 + s3);
  for (; l < k; l++) sum += a[l] * b[l];
  return sum;
#endif
}

/* Portable restatement of the same lane order with fmaf (used by tests to
 * show the intrinsic path and the scalar emulation agree bit for bit). */
void rc_matmul_t_scalar_emul(const float *a, const float *b, float *c,
                             size_t m, size_t n, size_t k) {
  for (size_t i = 0; i < m; i++)
    for (size_t j = 0; j < n; j++) {
      const float *ar = a + i * k, *br = b + j * k;
      float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      size_t l = 0;
      for (; l + 8 <= k; l += 8)
        for (int t = 0; t < 8; t++) lane[t] = fmaf(ar[l + t], br[l + t], lane[t]);
      float s0 = lane[0] + lane[4], s1 = lane[1] + lane[5];
      float s2 = lane[2] + lane[6], s3 = lane[3] + lane[7];
      float sum = (s0 + s1) + (s2 + s3);
      for (; l < k; l++) sum += ar[l] * br[l];
      c[i * n + j] = sum;
    }
}

/* ---- a tiny fork/join helper: fn(ctx, t, nthreads) on g_threads threads */
typedef void (*par_fn)(void *ctx, int t, int nt);
typedef struct { par_fn fn; void *ctx; int t, nt; } par_arg;
static void *par_tramp(void *p) {
  par_arg *a = (par_arg *)p;
  a->fn(a->ctx, a->t, a->nt);
  return NULL;
}
static void par_run(par_fn fn, void *ctx, size_t work) {
  int nt = g_threads;
  if ((size_t)nt > work) nt = (int)(work ? work : 1);
  if (nt <= 1) { fn(ctx, 0, 1); return; }
  pthread_t th[256];
  par_arg args[256];
  if (nt > 256) nt = 256;
  for (int t = 1; t < nt; t++) {
    args[t] = (par_arg){fn, ctx, t, nt};
    pthread_create(&th[t], NULL, par_tramp, &args[t]);
  }
  fn(ctx, 0, nt);
  for (int t = 1; t < nt; t++) pthread_join(th[t], NULL);
}

/* matmul_t (ops.rs:33-44) -> matmul_t_avx2 (ops.rs:106-134): parallel over
 * output columns j; each c[i,j] uses the identical per-element arithmetic. */
typedef struct { const float *a, *b; float *c; size_t m, n, k; } mmt_ctx;
static void mmt_worker(void *p, int t, int nt) {
  mmt_ctx *x = (mmt_ctx *)p;
  size_t j0 = x->n * (size_t)t / (size_t)nt, j1 = x->n * (size_t)(t + 1) / (size_t)nt;
  for (size_t i = 0; i < x->m; i++)
    for (size_t j = j0; j < j1; j++)
      x->c[i * x->n + j] = dot_avx2_order(x->a + i * x->k, x->b + j * x->k, x->k);
}
void rc_matmul_t(const float *a, const float *b, float *c, size_t m, size_t n,
                 size_t k) {
  mmt_ctx x = {a, b, c, m, n, k};
  par_run(mmt_worker, &x, n);
}

/* matmul (ops.rs:15-26) -> matmul_avx2 (ops.rs:75-102): c.fill(0); for each
 * (i, l): c_row[j] = fma(a[i,l], b[l,j], c_row[j]) for the 8-wide body,
 * c_row[j] += a*b for the tail. */
void rc_matmul(const float *a, const float *b, float *c, size_t m, size_t n,
               size_t k) {
  memset(c, 0, m * n * sizeof(float));
  for (size_t i = 0; i < m; i++)
    for (size_t l = 0; l < k; l++) {
      float av = a[i * k + l];
      const float *br = b + l * n;
      float *cr = c + i * n;
      size_t j = 0;
      for (; j + 8 <= n; j += 8)
        for (int t = 0; t < 8; t++) cr[j + t] = fmaf(av, br[j + t], cr[j + t]);
      for (; j < n; j++) cr[j] += a[i * k + l] * br[j];
    }
}

/* rms_norm (ops.rs:155-168): sequential sum of v*v, / len, 1/sqrt(ms+eps),
 * x = x*scale*w. */
void rc_rms_norm(float *x, const float *w, size_t n, float eps) {
  if (n == 0) return;
  float ms = 0.0f;
  for (size_t i = 0; i < n; i++) ms += x[i] * x[i];
  ms = ms / (float)n;
  float scale = 1.0f / sqrtf(ms + eps);
  for (size_t i = 0; i < n; i++) x[i] = x[i] * scale * w[i];
}
/* rms_norm_rows (ops.rs:173-180) */
void rc_rms_norm_rows(float *x, const float *w, float eps, size_t rows,
                      size_t hidden) {
  for (size_t r = 0; r < rows; r++) rc_rms_norm(x + r * hidden, w, hidden, eps);
}
/* sigmoid / silu (ops.rs:199-209): clamp to [-80, 80], 1/(1+exp(-x)). */
static inline float sigmoidf_ref(float x) {
  if (x < -80.0f) x = -80.0f;
  if (x > 80.0f) x = 80.0f;
  return 1.0f / (1.0f + expf(-x));
}
static inline float silu_ref(float x) { return x * sigmoidf_ref(x); }
void rc_silu(float *x, size_t n) {
  for (size_t i = 0; i < n; i++) x[i] = silu_ref(x[i]);
}
/* swiglu (ops.rs:190-197) */
void rc_swiglu(const float *g, const float *u, float *o, size_t n) {
  for (size_t i = 0; i < n; i++) o[i] = silu_ref(g[i]) * u[i];
}
/* add_in_place (ops.rs:212-217) */
void rc_add_in_place(float *o, const float *b, size_t n) {
  for (size_t i = 0; i < n; i++) o[i] += b[i];
}
/* softmax_rows (ops.rs:223-239): f32::max fold from -inf (NaN-ignoring),
 * exp(v - max), sequential sum, divide. */
void rc_softmax_rows(float *x, size_t rows, size_t cols) {
  for (size_t i = 0; i < rows; i++) {
    float *r = x + i * cols;
    float mx = -INFINITY;
    for (size_t j = 0; j < cols; j++) mx = fmaxf(mx, r[j]);
    float sum = 0.0f;
    for (size_t j = 0; j < cols; j++) {
      r[j] = expf(r[j] - mx);
      sum += r[j];
    }
    for (size_t j = 0; j < cols; j++) r[j] /= sum;
  }
}
/* embedding_lookup (ops.rs:246-258): out-of-range id is an error. */
int rc_embedding_lookup(const float *emb, size_t emb_len, const uint32_t *ids,
                        size_t n_ids, size_t hidden, float *out) {
  for (size_t p = 0; p < n_ids; p++) {
    size_t src = (size_t)ids[p] * hidden;
    if (src + hidden > emb_len) return RC_ERR_INVALID_TENSOR_INDEX;
    memcpy(out + p * hidden, emb + src, hidden * sizeof(float));
  }
  return RC_OK;
}
/* rope (ops.rs:265-287): interleaved pairs, inv = 1/base.powf(i/rope_dim),
 * angle = pos*inv, x0 = a*cos - b*sin, x1 = a*sin + b*cos, positions
 * 0..seq_len. */
void rc_rope(float *x, size_t seq_len, size_t n_heads, size_t head_dim,
             size_t rope_dim, float base) {
  for (size_t pos = 0; pos < seq_len; pos++)
    for (size_t h = 0; h < n_heads; h++) {
      size_t ho = (pos * n_heads + h) * head_dim;
      for (size_t i = 0; i < rope_dim; i += 2) {
        size_t idx = ho + i;
        float a = x[idx], b = x[idx + 1];
        float inv = 1.0f / powf(base, (float)i / (float)rope_dim);
        float ang = (float)pos * inv;
        float s = sinf(ang), c = cosf(ang);
        x[idx] = a * c - b * s;
        x[idx + 1] = a * s + b * c;
      }
    }
}
/* argmax (forward.rs:615-622, sampler.rs:75-82): Iterator::max_by keeps the
 * LAST maximum on ties. */
uint32_t rc_argmax(const float *x, size_t n) {
  if (n == 0) return 0;
  size_t best = 0;
  for (size_t i = 1; i < n; i++)
    if (!(x[i] < x[best])) best = i;
  return (uint32_t)best;
}

/* Sampler::sample (sampler.rs:28-73). The thread_rng draw is replaced by the
 * supplied uniform u; rand 0.8.6's WeightedIndex builds cumulative weights
 * [w0, w0+w1, ...] (n-1 entries), samples chosen = u * scale from
 * Uniform(0, total) (UniformFloat<f32>, whose scale is stepped down until
 * the largest draw stays below total) and returns the first index whose
 * cumulative weight is greater than `chosen` (partition_point(w <= chosen)).
 */
typedef struct { uint32_t i; float p; } ip_t;
static void stable_sort_desc(ip_t *v, size_t n) {
  /* insertion-merge: a plain stable merge sort */
  if (n < 2) return;
  ip_t *tmp = (ip_t *)malloc(n * sizeof(ip_t));
  for (size_t w = 1; w < n; w *= 2) {
    for (size_t lo = 0; lo < n; lo += 2 * w) {
      size_t mid = lo + w < n ? lo + w : n, hi = lo + 2 * w < n ? lo + 2 * w : n;
      size_t a = lo, b = mid, o = lo;
      while (a < mid && b < hi) {
        /* b goes first only if strictly greater (descending, stable) */
        if (v[b].p > v[a].p) tmp[o++] = v[b++];
        else tmp[o++] = v[a++];
      }
      while (a < mid) tmp[o++] = v[a++];
      while (b < hi) tmp[o++] = v[b++];
    }
    memcpy(v, tmp, n * sizeof(ip_t));
  }
  free(tmp);
}
uint32_t rc_sample(const float *logits, size_t n, float temperature,
                   size_t top_k, float top_p, double u) {
  if (temperature == 0.0f || n == 0) return rc_argmax(logits, n);
  ip_t *pr = (ip_t *)malloc(n * sizeof(ip_t));
  for (size_t i = 0; i < n; i++) { pr[i].i = (uint32_t)i; pr[i].p = expf(logits[i] / temperature); }
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) sum += pr[i].p;
  for (size_t i = 0; i < n; i++) pr[i].p /= sum;
  size_t len = n;
  if (top_k > 0) {
    stable_sort_desc(pr, len);
    if (top_k < len) len = top_k;
  }
  if (top_p < 1.0f) {
    stable_sort_desc(pr, len);
    float cs = 0.0f;
    size_t cut = len;
    for (size_t i = 0; i < len; i++) {
      cs += pr[i].p;
      if (cs >= top_p) { cut = i + 1; break; }
    }
    len = cut;
  }
  float s2 = 0.0f;
  for (size_t i = 0; i < len; i++) s2 += pr[i].p;
  float *w = (float *)malloc(len * sizeof(float));
  for (size_t i = 0; i < len; i++) w[i] = pr[i].p / s2;
  /* WeightedIndex::new */
  float total = w[0];
  float *cum = (float *)malloc((len ? len : 1) * sizeof(float));
  for (size_t i = 1; i < len; i++) { cum[i - 1] = total; total += w[i]; }
  /* UniformFloat<f32>::new(0, total): scale stepped down while
   * max_rand*scale + 0 >= total, max_rand = 1 - 2^-23. */
  float scale = total;
  const float max_rand = 1.0f - 1.1920929e-7f;
  while (scale * max_rand >= total) {
    uint32_t bits;
    memcpy(&bits, &scale, 4);
    bits -= 1;
    memcpy(&scale, &bits, 4);
  }
  float uf = (float)u;
  float chosen = uf * scale + 0.0f;
  size_t idx = 0;
  while (idx < len - 1 && cum[idx] <= chosen) idx++;
  uint32_t tok = pr[idx].i;
  free(pr); free(w); free(cum);
  return tok;
}

/* ------------------------------- GGUF ----------------------------------- */
typedef struct {
  const uint8_t *p;
  size_t len, pos;
  int err;
} rd_t;
static int rd(rd_t *r, void *dst, size_t n) {
  if (r->err) return 0;
  if (r->pos + n > r->len || r->pos + n < r->pos) { r->err = RC_ERR_IO; return 0; }
  memcpy(dst, r->p + r->pos, n);
  r->pos += n;
  return 1;
}
static uint32_t rd_u32(rd_t *r) { uint32_t v = 0; rd(r, &v, 4); return v; }
static uint64_t rd_u64(rd_t *r) { uint64_t v = 0; rd(r, &v, 8); return v; }

static int utf8_ok(const uint8_t *s, size_t n) {
  size_t i = 0;
  while (i < n) {
    uint8_t c = s[i];
    size_t k;
    uint32_t cp;
    if (c < 0x80) { i++; continue; }
    else if ((c & 0xe0) == 0xc0) { k = 1; cp = c & 0x1f; }
    else if ((c & 0xf0) == 0xe0) { k = 2; cp = c & 0x0f; }
    else if ((c & 0xf8) == 0xf0) { k = 3; cp = c & 0x07; }
    else return 0;
    for (size_t t = 1; t <= k; t++) {
      if (i + t >= n || (s[i + t] & 0xc0) != 0x80) return 0;
      cp = (cp << 6) | (s[i + t] & 0x3f);
    }
    if ((k == 1 && cp < 0x80) || (k == 2 && cp < 0x800) || (k == 3 && cp < 0x10000) ||
        cp > 0x10ffff || (cp >= 0xd800 && cp <= 0xdfff))
      return 0;
    i += k + 1;
  }
  return 1;
}

/* read_string (src/gguf/value.rs:108-113) */
static char *rd_string(rd_t *r, size_t *out_len) {
  uint64_t n = rd_u64(r);
  if (r->err) return NULL;
  if (n > r->len - r->pos) { r->err = RC_ERR_IO; return NULL; }
  char *s = (char *)malloc((size_t)n + 1);
  rd(r, s, (size_t)n);
  s[n] = 0;
  if (!utf8_ok((const uint8_t *)s, (size_t)n)) { r->err = RC_ERR_INVALID_UTF8; free(s); return NULL; }
  if (out_len) *out_len = (size_t)n;
  return s;
}

typedef struct {
  char *key;
  uint32_t vt; /* ValueType */
  union { uint64_t u; int64_t i; double f; } v;
  char *str;
} kv_t;

typedef struct {
  char *name;
  uint32_t n_dims;
  uint64_t shape[4];
  int type;
  uint64_t offset;
} tinfo_t;

struct rc_model {
  const uint8_t *bytes;
  size_t len;
  uint32_t version;
  uint64_t n_tensors, n_kv;
  kv_t *kv;
  tinfo_t *ti;
  uint64_t data_off;
  rc_config cfg;
  /* layer tensor indices: attn_norm, q, k, v, o, ffn_norm, gate, up, down */
  int (*layer)[9];
  int tok_emb, out_norm, output; /* output: -1 if absent */
};

/* Value::read (value.rs:45-71); scalars are kept, arrays are skipped. */
static int skip_or_read_value(rd_t *r, uint32_t vt, kv_t *kv, int depth) {
  switch (vt) {
  case 0: { uint8_t v = 0; rd(r, &v, 1); if (kv) kv->v.u = v; break; }
  case 1: { int8_t v = 0; rd(r, &v, 1); if (kv) kv->v.i = v; break; }
  case 2: { uint16_t v = 0; rd(r, &v, 2); if (kv) kv->v.u = v; break; }
  case 3: { int16_t v = 0; rd(r, &v, 2); if (kv) kv->v.i = v; break; }
  case 4: { uint32_t v = 0; rd(r, &v, 4); if (kv) kv->v.u = v; break; }
  case 5: { int32_t v = 0; rd(r, &v, 4); if (kv) kv->v.i = v; break; }
  case 6: { float v = 0; rd(r, &v, 4); if (kv) kv->v.f = v; break; }
  case 7: { uint8_t v = 0; rd(r, &v, 1); if (kv) kv->v.u = v != 0; break; }
  case 8: {
    char *s = rd_string(r, NULL);
    if (kv) kv->str = s; else free(s);
    break;
  }
  case 9: {
    uint32_t it = rd_u32(r);
    if (r->err) return r->err;
    if (it > 12) { r->err = RC_ERR_UNKNOWN_VALUE_TYPE; return r->err; }
    uint64_t n = rd_u64(r);
    for (uint64_t i = 0; i < n && !r->err; i++) skip_or_read_value(r, it, NULL, depth + 1);
    break;
  }
  case 10: { uint64_t v = 0; rd(r, &v, 8); if (kv) kv->v.u = v; break; }
  case 11: { int64_t v = 0; rd(r, &v, 8); if (kv) kv->v.i = v; break; }
  case 12: { double v = 0; rd(r, &v, 8); if (kv) kv->v.f = v; break; }
  default: r->err = RC_ERR_UNKNOWN_VALUE_TYPE;
  }
  return r->err;
}

/* GgufFile::get: first entry with that key (file.rs:119-121). */
static const kv_t *get_kv(const rc_model *m, const char *key) {
  for (uint64_t i = 0; i < m->n_kv; i++)
    if (strcmp(m->kv[i].key, key) == 0) return &m->kv[i];
  return NULL;
}
/* get_u32 / get_u64 / get_f32 / get_string (file.rs:141-194). */
static int get_uint(const rc_model *m, const char *key, uint64_t *out, int as32) {
  const kv_t *kv = get_kv(m, key);
  if (!kv) return 0;
  uint64_t v;
  switch (kv->vt) {
  case 0: case 2: case 4: case 10: v = kv->v.u; break;
  case 1: case 3: case 5: case 11: v = (uint64_t)kv->v.i; break;
  default: return 0;
  }
  *out = as32 ? (uint64_t)(uint32_t)v : v;
  return 1;
}
static int get_f32(const rc_model *m, const char *key, float *out) {
  const kv_t *kv = get_kv(m, key);
  if (!kv) return 0;
  switch (kv->vt) {
  case 6: case 12: *out = (float)kv->v.f; return 1;
  case 0: case 2: case 4: case 10: *out = (float)kv->v.u; return 1;
  case 1: case 3: case 5: case 11: *out = (float)kv->v.i; return 1;
  default: return 0;
  }
}
static const char *get_str(const rc_model *m, const char *key) {
  const kv_t *kv = get_kv(m, key);
  return (kv && kv->vt == 8) ? kv->str : NULL;
}
/* GgufFile::tensor_index: first tensor with that name (file.rs:129-131). */
static int tensor_index(const rc_model *m, const char *name) {
  for (uint64_t i = 0; i < m->n_tensors; i++)
    if (strcmp(m->ti[i].name, name) == 0) return (int)i;
  return -1;
}

void rc_model_free(rc_model *m) {
  if (!m) return;
  if (m->kv) {
    for (uint64_t i = 0; i < m->n_kv; i++) { free(m->kv[i].key); free(m->kv[i].str); }
    free(m->kv);
  }
  if (m->ti) {
    for (uint64_t i = 0; i < m->n_tensors; i++) free(m->ti[i].name);
    free(m->ti);
  }
  free(m->layer);
  free(m);
}

/* GgufFile::read (file.rs:57-116) + Config::from_gguf (config.rs:34-84) +
 * Model::open (model/mod.rs:64-92). */
static int open_mem(const uint8_t *bytes, size_t len, rc_model **out, int parse_only) {
  *out = NULL;
  rc_model *m = (rc_model *)calloc(1, sizeof(rc_model));
  m->bytes = bytes;
  m->len = len;
  rd_t r = {bytes, len, 0, 0};
  uint8_t magic[4];
  if (!rd(&r, magic, 4)) { rc_model_free(m); return RC_ERR_IO; }
  if (memcmp(magic, "GGUF", 4) != 0) { rc_model_free(m); return RC_ERR_INVALID_MAGIC; }
  m->version = rd_u32(&r);
  if (r.err) { rc_model_free(m); return r.err; }
  if (m->version != 2 && m->version != 3) { rc_model_free(m); return RC_ERR_UNSUPPORTED_VERSION; }
  m->n_tensors = rd_u64(&r);
  m->n_kv = rd_u64(&r);
  if (r.err) { rc_model_free(m); return r.err; }
  if (m->n_kv > len || m->n_tensors > len) { rc_model_free(m); return RC_ERR_IO; }
  m->kv = (kv_t *)calloc(m->n_kv ? m->n_kv : 1, sizeof(kv_t));
  for (uint64_t i = 0; i < m->n_kv; i++) {
    m->kv[i].key = rd_string(&r, NULL);
    if (r.err) { m->n_kv = i + 1; rc_model_free(m); return r.err; }
    uint32_t vt = rd_u32(&r);
    if (!r.err && vt > 12) r.err = RC_ERR_UNKNOWN_VALUE_TYPE;
    if (r.err) { m->n_kv = i + 1; rc_model_free(m); return r.err; }
    m->kv[i].vt = vt;
    skip_or_read_value(&r, vt, &m->kv[i], 0);
    if (r.err) { m->n_kv = i + 1; rc_model_free(m); return r.err; }
  }
  m->ti = (tinfo_t *)calloc(m->n_tensors ? m->n_tensors : 1, sizeof(tinfo_t));
  for (uint64_t i = 0; i < m->n_tensors; i++) {
    tinfo_t *t = &m->ti[i];
    t->name = rd_string(&r, NULL);
    if (r.err) { m->n_tensors = i + 1; rc_model_free(m); return r.err; }
    t->n_dims = rd_u32(&r);
    if (r.err) { m->n_tensors = i + 1; rc_model_free(m); return r.err; }
    if (t->n_dims > 4) { m->n_tensors = i + 1; rc_model_free(m); return RC_ERR_INVALID_SHAPE; }
    for (uint32_t d = 0; d < t->n_dims; d++) t->shape[d] = rd_u64(&r);
    uint32_t ty = rd_u32(&r);
    if (!r.err && !valid_type_id(ty)) r.err = RC_ERR_UNKNOWN_TENSOR_TYPE;
    t->type = (int)ty;
    t->offset = rd_u64(&r);
    if (r.err) { m->n_tensors = i + 1; rc_model_free(m); return r.err; }
  }
  m->data_off = (r.pos + 31) / 32 * 32;
  if (parse_only) { *out = m; return RC_OK; }

  /* Config::from_gguf */
  rc_config *c = &m->cfg;
  const char *arch = get_str(m, "general.architecture");
  if (!arch) { rc_model_free(m); return RC_ERR_TENSOR_NOT_FOUND; }
  strncpy(c->architecture, arch, sizeof(c->architecture) - 1);
  if (strcmp(arch, "llama") != 0) { rc_model_free(m); return RC_ERR_UNSUPPORTED_ARCHITECTURE; }
  uint64_t v;
  if (!get_uint(m, "llama.embedding_length", &c->hidden_size, 0) ||
      !get_uint(m, "llama.block_count", &c->n_layers, 0) ||
      !get_uint(m, "llama.attention.head_count", &c->n_heads, 0)) {
    rc_model_free(m);
    return RC_ERR_TENSOR_NOT_FOUND;
  }
  c->n_kv_heads = get_uint(m, "llama.attention.head_count_kv", &v, 1) ? v : c->n_heads;
  if (c->n_heads == 0) { rc_model_free(m); return RC_ERR_INVALID_SHAPE; }
  c->head_dim = get_uint(m, "llama.attention.key_length", &v, 1) ? v : c->hidden_size / c->n_heads;
  if (!get_uint(m, "llama.feed_forward_length", &c->intermediate_size, 0)) {
    rc_model_free(m);
    return RC_ERR_TENSOR_NOT_FOUND;
  }
  if (!get_f32(m, "llama.attention.layer_norm_rms_epsilon", &c->norm_eps)) c->norm_eps = 1e-5f;
  if (!get_f32(m, "llama.rope.freq_base", &c->rope_base)) c->rope_base = 10000.0f;
  c->rope_dim = get_uint(m, "llama.rope.dimension_count", &v, 1) ? v : c->head_dim;
  c->context_length = get_uint(m, "llama.context_length", &v, 1) ? v : 4096;
  c->vocab_size = get_uint(m, "llama.vocab_size", &v, 1) ? (uint32_t)v : 0;

  /* Layer::from_weights (model/mod.rs:34-48) */
  static const char *suffix[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                  "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
  m->layer = (int(*)[9])calloc(c->n_layers ? c->n_layers : 1, sizeof(int[9]));
  char nm[128];
  for (uint64_t l = 0; l < c->n_layers; l++)
    for (int s = 0; s < 9; s++) {
      snprintf(nm, sizeof nm, "blk.%llu.%s.weight", (unsigned long long)l, suffix[s]);
      m->layer[l][s] = tensor_index(m, nm);
      if (m->layer[l][s] < 0) { rc_model_free(m); return RC_ERR_TENSOR_NOT_FOUND; }
    }
  m->tok_emb = tensor_index(m, "token_embd.weight");
  if (m->tok_emb < 0) { rc_model_free(m); return RC_ERR_TENSOR_NOT_FOUND; }
  m->out_norm = tensor_index(m, "output_norm.weight");
  if (m->out_norm < 0) { rc_model_free(m); return RC_ERR_TENSOR_NOT_FOUND; }
  m->output = tensor_index(m, "output.weight");
  *out = m;
  return RC_OK;
}

int rc_model_open_mem(const uint8_t *bytes, size_t len, rc_model **out) {
  return open_mem(bytes, len, out, 0);
}
int rc_gguf_open_mem(const uint8_t *bytes, size_t len, rc_model **out) {
  return open_mem(bytes, len, out, 1);
}

void rc_model_config(const rc_model *m, rc_config *out) { *out = m->cfg; }
int rc_model_has_output(const rc_model *m) { return m->output >= 0; }
int rc_model_n_tensors(const rc_model *m) { return (int)m->n_tensors; }

static uint64_t n_elem(const tinfo_t *t) {
  uint64_t n = 1;
  for (uint32_t d = 0; d < t->n_dims; d++) n *= t->shape[d];
  return n;
}

/* Weights::tensor_bytes (weights.rs:97-112). */
static int tensor_bytes(const rc_model *m, int idx, const uint8_t **p, size_t *nb) {
  if (idx < 0 || (uint64_t)idx >= m->n_tensors) return RC_ERR_INVALID_TENSOR_INDEX;
  const tinfo_t *t = &m->ti[idx];
  int64_t size = rc_type_byte_size(t->type, n_elem(t));
  if (size < 0) return RC_ERR_UNKNOWN_TENSOR_TYPE;
  uint64_t start = m->data_off + t->offset;
  if (start < m->data_off) return RC_ERR_TENSOR_OFFSET_OVERFLOW;
  uint64_t end = start + (uint64_t)size;
  if (end < start) return RC_ERR_TENSOR_OFFSET_OVERFLOW;
  if (end > m->len) return RC_ERR_UNEXPECTED_EOF;
  *p = m->bytes + start;
  *nb = (size_t)size;
  return RC_OK;
}

/* Weights::tensor (weights.rs:44-51): name lookup + bounds-checked slice. */
int rc_tensor_bytes(const rc_model *m, const char *name, uint64_t *offset_abs,
                    uint64_t *nbytes) {
  int i = tensor_index(m, name);
  if (i < 0) return RC_ERR_TENSOR_NOT_FOUND;
  const uint8_t *p;
  size_t nb;
  int st = tensor_bytes(m, i, &p, &nb);
  if (st) return st;
  *offset_abs = (uint64_t)(p - m->bytes);
  *nbytes = nb;
  return RC_OK;
}

int rc_model_tensor_info(const rc_model *m, const char *name, int *type,
                         uint64_t *n_elements, uint64_t *offset_abs,
                         uint64_t *nbytes) {
  int i = tensor_index(m, name);
  if (i < 0) return RC_ERR_TENSOR_NOT_FOUND;
  const tinfo_t *t = &m->ti[i];
  *type = t->type;
  *n_elements = n_elem(t);
  *offset_abs = m->data_off + t->offset;
  int64_t s = rc_type_byte_size(t->type, n_elem(t));
  *nbytes = s < 0 ? 0 : (uint64_t)s;
  return RC_OK;
}

/* Weights::tensor_f32_by_index (weights.rs:66-74): whole-tensor dequant into
 * a fresh buffer (caller frees). */
/* The whole-tensor dequantisation of tensor_f32 split over g_threads threads
 * at block boundaries (each element still goes through the same formula). */
typedef struct {
  int type;
  const uint8_t *p;
  float *out;
  uint64_t nblocks, blk_elems, blk_bytes;
  int st;
} dq_ctx;
static void dq_worker(void *vp, int t, int nt) {
  dq_ctx *x = (dq_ctx *)vp;
  uint64_t b0 = x->nblocks * (uint64_t)t / (uint64_t)nt, b1 = x->nblocks * (uint64_t)(t + 1) / (uint64_t)nt;
  if (b1 <= b0) return;
  int st = rc_dequantize(x->type, x->p + b0 * x->blk_bytes, (size_t)((b1 - b0) * x->blk_bytes),
                         x->out + b0 * x->blk_elems, (size_t)((b1 - b0) * x->blk_elems));
  if (st) x->st = st;
}

/* Weights::tensor_f32_by_index (weights.rs:66-74): a fresh zeroed buffer of
 * the whole tensor, dequantised (dequant.rs:34-38). */
static int tensor_f32(const rc_model *m, int idx, float **out) {
  const uint8_t *p;
  size_t nb;
  int st = tensor_bytes(m, idx, &p, &nb);
  if (st) return st;
  uint64_t n = n_elem(&m->ti[idx]);
  float *buf = (float *)calloc(n ? n : 1, sizeof(float));
  const int type = m->ti[idx].type;
  const uint64_t be = (type == RC_Q4_0 || type == RC_Q8_0) ? 32
                      : (type == RC_Q4K || type == RC_Q6K || type == RC_Q8K) ? 256 : 1;
  const int64_t bb = rc_type_byte_size(type, be);
  if (g_threads > 1 && bb > 0 && n % be == 0 && (uint64_t)nb == n / be * (uint64_t)bb) {
    dq_ctx x = {type, p, buf, n / be, be, (uint64_t)bb, 0};
    par_run(dq_worker, &x, (size_t)(n / be));
    st = x.st;
  } else {
    st = rc_dequantize(type, p, nb, buf, (size_t)n);
  }
  if (st) { free(buf); return st; }
  *out = buf;
  return RC_OK;
}

/* matmul_t against a weight tensor (a is [mrows, k], W is [n, k]).
 * faithful: whole-tensor dequant + matmul_t; otherwise per-row dequant fused
 * into the dot (identical bits: every element goes through the same
 * dequant formula and the same dot order). */
typedef struct {
  const rc_model *m;
  int idx;
  const uint8_t *p;
  const float *a;
  float *c;
  size_t mrows, n, k;
} mtq_ctx;
static void mtq_worker(void *vp, int t, int nt) {
  mtq_ctx *x = (mtq_ctx *)vp;
  size_t j0 = x->n * (size_t)t / (size_t)nt, j1 = x->n * (size_t)(t + 1) / (size_t)nt;
  float *row = (float *)malloc((x->k + 512) * sizeof(float));
  float *tmp = (float *)malloc((x->k + 512) * sizeof(float));
  int type = x->m->ti[x->idx].type;
  for (size_t j = j0; j < j1; j++) {
    dequant_range(type, x->p, (uint64_t)j * x->k, x->k, row, tmp);
    for (size_t i = 0; i < x->mrows; i++)
      x->c[i * x->n + j] = dot_avx2_order(x->a + i * x->k, row, x->k);
  }
  free(row);
  free(tmp);
}
static int matmul_t_w(const rc_model *m, int idx, const float *a, float *c,
                      size_t mrows, size_t n, size_t k) {
  const uint8_t *p;
  size_t nb;
  int st = tensor_bytes(m, idx, &p, &nb);
  if (st) return st;
  uint64_t ne = n_elem(&m->ti[idx]);
  if (ne != (uint64_t)n * k) return RC_ERR_INVALID_SHAPE; /* assert in ops.rs:35 */
  if (g_faithful) {
    float *w;
    st = tensor_f32(m, idx, &w);
    if (st) return st;
    rc_matmul_t(a, w, c, mrows, n, k);
    free(w);
    return RC_OK;
  }
  int t = m->ti[idx].type;
  if (t != RC_F32 && t != RC_F16 && t != RC_Q4_0 && t != RC_Q8_0 && t != RC_Q4K &&
      t != RC_Q6K && t != RC_Q8K)
    return RC_ERR_UNKNOWN_TENSOR_TYPE;
  mtq_ctx x = {m, idx, p, a, c, mrows, n, k};
  par_run(mtq_worker, &x, n);
  return RC_OK;
}

/* A norm weight (F32 [D] in practice). */
static int norm_weight(const rc_model *m, int idx, float **out) {
  return tensor_f32(m, idx, out);
}

/* --------------------------- KV cache ----------------------------------- */
struct rc_kv {
  size_t n_layers, max_seq, kv_dim, len;
  float **k, **v;
};
/* KvCache::new (model/cache.rs:16-24) */
rc_kv *rc_kv_new(const rc_model *m, size_t n_layers, size_t max_seq) {
  rc_kv *kv = (rc_kv *)calloc(1, sizeof(rc_kv));
  kv->n_layers = n_layers;
  kv->max_seq = max_seq;
  kv->kv_dim = (size_t)(m->cfg.n_kv_heads * m->cfg.head_dim);
  kv->k = (float **)calloc(n_layers ? n_layers : 1, sizeof(float *));
  kv->v = (float **)calloc(n_layers ? n_layers : 1, sizeof(float *));
  for (size_t l = 0; l < n_layers; l++) {
    kv->k[l] = (float *)calloc(max_seq * kv->kv_dim + 1, sizeof(float));
    kv->v[l] = (float *)calloc(max_seq * kv->kv_dim + 1, sizeof(float));
  }
  return kv;
}
void rc_kv_free(rc_kv *kv) {
  if (!kv) return;
  for (size_t l = 0; l < kv->n_layers; l++) { free(kv->k[l]); free(kv->v[l]); }
  free(kv->k);
  free(kv->v);
  free(kv);
}
void rc_kv_clear(rc_kv *kv) { kv->len = 0; }
size_t rc_kv_len(const rc_kv *kv) { return kv->len; }
int rc_kv_read(const rc_kv *kv, size_t layer, int which_v, float *out) {
  if (layer >= kv->n_layers) return RC_ERR_INVALID_TENSOR_INDEX;
  memcpy(out, which_v ? kv->v[layer] : kv->k[layer], kv->len * kv->kv_dim * sizeof(float));
  return RC_OK;
}

/* ---------------------------- attention --------------------------------- */
/* Per-query-head attention bodies, parallel over heads. Each head writes its
 * own [hd] slice of attn_out, so threading does not change any bits. */
typedef struct {
  const rc_config *c;
  const float *q;     /* [seq, H*hd] */
  const float *k, *v; /* rows of kv_dim, row t at k + t*kv_dim */
  float *attn_out;    /* [seq, D] */
  size_t seq;         /* query rows */
  size_t nkeys;       /* decode: key rows */
  int mode;           /* 0 = non-causal full, 1 = causal chunk, 2 = decode */
} att_ctx;

static void att_worker(void *vp, int t, int nt) {
  att_ctx *x = (att_ctx *)vp;
  const rc_config *c = x->c;
  size_t H = c->n_heads, hd = c->head_dim, G = c->n_kv_heads, D = c->hidden_size;
  size_t kv_dim = G * hd, group = H / G;
  size_t h0 = H * (size_t)t / (size_t)nt, h1 = H * (size_t)(t + 1) / (size_t)nt;
  float sq = sqrtf((float)hd);
  if (x->mode == 2) {
    size_t n = x->nkeys;
    float *scores = (float *)malloc((n ? n : 1) * sizeof(float));
    float *ho = (float *)malloc(hd * sizeof(float));
    for (size_t hq = h0; hq < h1; hq++) {
      size_t hkv = hq / group;
      const float *qh = x->q + hq * hd;
      /* forward.rs:388-397 */
      for (size_t tt = 0; tt < n; tt++) {
        const float *kh = x->k + tt * kv_dim + hkv * hd;
        float s = 0.0f;
        for (size_t d = 0; d < hd; d++) s += qh[d] * kh[d];
        scores[tt] = s / sq;
      }
      rc_softmax_rows(scores, 1, n); /* forward.rs:399 */
      for (size_t d = 0; d < hd; d++) ho[d] = 0.0f;
      for (size_t tt = 0; tt < n; tt++) { /* forward.rs:401-409 */
        float s = scores[tt];
        const float *vh = x->v + tt * kv_dim + hkv * hd;
        for (size_t d = 0; d < hd; d++) ho[d] += s * vh[d];
      }
      memcpy(x->attn_out + hq * hd, ho, hd * sizeof(float));
    }
    free(scores);
    free(ho);
    return;
  }
  size_t S = x->seq;
  float *scores = (float *)malloc(((S * S) > 0 ? S * S : 1) * sizeof(float));
  float *ho = (float *)malloc((S ? S : 1) * hd * sizeof(float));
  for (size_t hq = h0; hq < h1; hq++) {
    size_t hkv = hq / group;
    for (size_t pos = 0; pos < S; pos++) {
      const float *qh = x->q + (pos * H + hq) * hd;
      for (size_t tt = 0; tt < S; tt++) {
        if (x->mode == 1 && tt > pos) { /* forward.rs:266-271 */
          scores[pos * S + tt] = -INFINITY;
          continue;
        }
        const float *kh = x->k + (tt * G + hkv) * hd;
        float s = 0.0f;
        for (size_t d = 0; d < hd; d++) s += qh[d] * kh[d];
        scores[pos * S + tt] = s / sq;
      }
    }
    rc_softmax_rows(scores, S, S);
    for (size_t pos = 0; pos < S; pos++) {
      float *o = ho + pos * hd;
      for (size_t d = 0; d < hd; d++) o[d] = 0.0f;
      size_t tend = x->mode == 1 ? pos + 1 : S; /* forward.rs:290 vs :138 */
      for (size_t tt = 0; tt < tend; tt++) {
        float s = scores[pos * S + tt];
        const float *vh = x->v + (tt * G + hkv) * hd;
        for (size_t d = 0; d < hd; d++) o[d] += s * vh[d];
      }
      memcpy(x->attn_out + pos * D + hq * hd, o, hd * sizeof(float));
    }
  }
  free(scores);
  free(ho);
}

/* ---------------------------- layer bodies ------------------------------ */
typedef struct {
  float *q, *k, *v, *attn_out, *gate, *up, *mid, *down, *residual;
} lbuf_t;
static void lbuf_alloc(lbuf_t *b, const rc_config *c, size_t S) {
  size_t D = c->hidden_size, kvd = c->n_kv_heads * c->head_dim, F = c->intermediate_size;
  b->q = (float *)calloc(S * D + 1, 4);
  b->k = (float *)calloc(S * kvd + 1, 4);
  b->v = (float *)calloc(S * kvd + 1, 4);
  b->attn_out = (float *)calloc(S * D + 1, 4);
  b->gate = (float *)calloc(S * F + 1, 4);
  b->up = (float *)calloc(S * F + 1, 4);
  b->mid = (float *)calloc(S * F + 1, 4);
  b->down = (float *)calloc(S * D + 1, 4);
  b->residual = (float *)calloc(S * D + 1, 4);
}
static void lbuf_free(lbuf_t *b) {
  free(b->q); free(b->k); free(b->v); free(b->attn_out); free(b->gate);
  free(b->up); free(b->mid); free(b->down); free(b->residual);
}

#define CHK(e) do { int _s = (e); if (_s) { st = _s; goto done; } } while (0)

/* The FFN half shared by forward/prefill/decode (forward.rs:167-204,
 * 311-334, 421-437). */
static int ffn_block(const rc_model *m, const int *L, float *x, size_t S, lbuf_t *b) {
  const rc_config *c = &m->cfg;
  size_t D = c->hidden_size, F = c->intermediate_size;
  int st = RC_OK;
  float *wn = NULL;
  memcpy(b->residual, x, S * D * 4);
  CHK(norm_weight(m, L[5], &wn));
  rc_rms_norm_rows(x, wn, c->norm_eps, S, D);
  CHK(matmul_t_w(m, L[6], x, b->gate, S, F, D));
  CHK(matmul_t_w(m, L[7], x, b->up, S, F, D));
  rc_swiglu(b->gate, b->up, b->mid, S * F);
  CHK(matmul_t_w(m, L[8], b->mid, b->down, S, D, F));
  memcpy(x, b->down, S * D * 4);
  rc_add_in_place(x, b->residual, S * D);
done:
  free(wn);
  return st;
}

/* Layer::forward (mode 0, forward.rs:62-207) and Layer::prefill (mode 1,
 * forward.rs:215-337). */
static int layer_seq(const rc_model *m, const int *L, float *x, size_t S, lbuf_t *b,
                     rc_kv *kv, size_t layer, size_t cache_start, int mode) {
  const rc_config *c = &m->cfg;
  size_t D = c->hidden_size, H = c->n_heads, G = c->n_kv_heads, hd = c->head_dim;
  size_t kvd = G * hd;
  int st = RC_OK;
  float *wn = NULL;
  memcpy(b->residual, x, S * D * 4);
  CHK(norm_weight(m, L[0], &wn));
  rc_rms_norm_rows(x, wn, c->norm_eps, S, D);
  CHK(matmul_t_w(m, L[1], x, b->q, S, D, D));
  CHK(matmul_t_w(m, L[2], x, b->k, S, kvd, D));
  CHK(matmul_t_w(m, L[3], x, b->v, S, kvd, D));
  rc_rope(b->q, S, H, hd, c->rope_dim, c->rope_base);
  rc_rope(b->k, S, G, hd, c->rope_dim, c->rope_base);
  if (mode == 1) { /* forward.rs:246-253 */
    if (cache_start + S > kv->max_seq) { st = RC_ERR_INVALID_TENSOR_INDEX; goto done; }
    for (size_t t = 0; t < S; t++) {
      memcpy(kv->k[layer] + (cache_start + t) * kvd, b->k + t * kvd, kvd * 4);
      memcpy(kv->v[layer] + (cache_start + t) * kvd, b->v + t * kvd, kvd * 4);
    }
  }
  memset(b->attn_out, 0, S * D * 4);
  {
    att_ctx a = {c, b->q, b->k, b->v, b->attn_out, S, S, mode};
    par_run(att_worker, &a, H);
  }
  CHK(matmul_t_w(m, L[4], b->attn_out, x, S, D, D));
  rc_add_in_place(x, b->residual, S * D);
  CHK(ffn_block(m, L, x, S, b));
done:
  free(wn);
  return st;
}

/* Embedding rows for ids (forward.rs:505-507 / 556-558). */
static int embed(const rc_model *m, const uint32_t *ids, size_t n, float *out) {
  const rc_config *c = &m->cfg;
  size_t D = c->hidden_size;
  if (g_faithful) {
    float *e;
    int st = tensor_f32(m, m->tok_emb, &e);
    if (st) return st;
    st = rc_embedding_lookup(e, (size_t)n_elem(&m->ti[m->tok_emb]), ids, n, D, out);
    free(e);
    return st;
  }
  const uint8_t *p;
  size_t nb;
  int st = tensor_bytes(m, m->tok_emb, &p, &nb);
  if (st) return st;
  uint64_t ne = n_elem(&m->ti[m->tok_emb]);
  float *tmp = (float *)malloc((D + 512) * 4);
  for (size_t i = 0; i < n; i++) {
    uint64_t src = (uint64_t)ids[i] * D;
    if (src + D > ne) { free(tmp); return RC_ERR_INVALID_TENSOR_INDEX; }
    dequant_range(m->ti[m->tok_emb].type, p, src, D, out + i * D, tmp);
  }
  free(tmp);
  return RC_OK;
}

/* Output norm + logits for rows [r0, S) of hidden (forward.rs:522-536). */
static int logits_rows(const rc_model *m, float *hidden, size_t S, size_t r0,
                       float *logits) {
  const rc_config *c = &m->cfg;
  size_t D = c->hidden_size, V = c->vocab_size;
  float *wn = NULL;
  int st = norm_weight(m, m->out_norm, &wn);
  if (st) return st;
  rc_rms_norm_rows(hidden + r0 * D, wn, c->norm_eps, S - r0, D);
  free(wn);
  int oi = m->output >= 0 ? m->output : m->tok_emb; /* forward.rs:526 */
  return matmul_t_w(m, oi, hidden + r0 * D, logits, S - r0, V, D);
}

static int seq_forward(const rc_model *m, rc_kv *kv, const uint32_t *ids, size_t n,
                       float *logits, int last_row_only, int mode) {
  const rc_config *c = &m->cfg;
  size_t D = c->hidden_size, V = c->vocab_size;
  for (size_t i = 0; i < n; i++)
    if (ids[i] >= V) return RC_ERR_INVALID_TENSOR_INDEX; /* forward.rs:501-503 */
  if (n == 0) return RC_OK;
  float *hidden = (float *)calloc(n * D, 4);
  lbuf_t b;
  lbuf_alloc(&b, c, n);
  int st = embed(m, ids, n, hidden);
  size_t cache_start = kv ? kv->len : 0;
  for (size_t l = 0; l < c->n_layers && !st; l++)
    st = layer_seq(m, m->layer[l], hidden, n, &b, kv, l, cache_start, mode);
  if (!st && mode == 1) kv->len += n; /* forward.rs:520 */
  if (!st && logits) st = logits_rows(m, hidden, n, last_row_only ? n - 1 : 0, logits);
  lbuf_free(&b);
  free(hidden);
  return st;
}

int rc_prefill(const rc_model *m, rc_kv *kv, const uint32_t *ids, size_t n,
               float *logits, int last_row_only) {
  return seq_forward(m, kv, ids, n, logits, last_row_only, 1);
}
int rc_forward(const rc_model *m, const uint32_t *ids, size_t n, float *logits) {
  return seq_forward(m, NULL, ids, n, logits, 0, 0);
}

/* Model::decode_step (forward.rs:543-586) -> Layer::decode_step
 * (forward.rs:344-440). */
int rc_decode_step(const rc_model *m, rc_kv *kv, uint32_t token, float *logits) {
  const rc_config *c = &m->cfg;
  size_t D = c->hidden_size, H = c->n_heads, G = c->n_kv_heads, hd = c->head_dim;
  size_t kvd = G * hd, V = c->vocab_size;
  if (token >= V) return RC_ERR_INVALID_TENSOR_INDEX; /* forward.rs:552-554 */
  if (kv->len >= kv->max_seq) return RC_ERR_INVALID_TENSOR_INDEX;
  float *h = (float *)calloc(D, 4);
  lbuf_t b;
  lbuf_alloc(&b, c, 1);
  float *wn = NULL;
  int st = embed(m, &token, 1, h);
  for (size_t l = 0; l < c->n_layers && !st; l++) {
    const int *L = m->layer[l];
    size_t cl = kv->len;
    memcpy(b.residual, h, D * 4);
    CHK(norm_weight(m, L[0], &wn));
    rc_rms_norm(h, wn, D, c->norm_eps);
    free(wn);
    wn = NULL;
    CHK(matmul_t_w(m, L[1], h, b.q, 1, D, D));
    CHK(matmul_t_w(m, L[2], h, b.k, 1, kvd, D));
    CHK(matmul_t_w(m, L[3], h, b.v, 1, kvd, D));
    rc_rope(b.q, 1, H, hd, c->rope_dim, c->rope_base); /* position 0: forward.rs:371-372 */
    rc_rope(b.k, 1, G, hd, c->rope_dim, c->rope_base);
    memcpy(kv->k[l] + cl * kvd, b.k, kvd * 4);
    memcpy(kv->v[l] + cl * kvd, b.v, kvd * 4);
    memset(b.attn_out, 0, D * 4);
    {
      att_ctx a = {c, b.q, kv->k[l], kv->v[l], b.attn_out, 1, cl + 1, 2};
      par_run(att_worker, &a, H);
    }
    CHK(matmul_t_w(m, L[4], b.attn_out, h, 1, D, D));
    rc_add_in_place(h, b.residual, D);
    CHK(ffn_block(m, L, h, 1, &b));
  }
  if (!st) st = logits_rows(m, h, 1, 0, logits);
  if (!st) kv->len += 1; /* forward.rs:584 */
done:
  free(wn);
  lbuf_free(&b);
  free(h);
  return st;
}

/* Model::generate (forward.rs:592-612). */
int rc_generate(const rc_model *m, rc_kv *kv, const uint32_t *prompt, size_t n_prompt,
                size_t max_tokens, uint32_t *out) {
  size_t V = m->cfg.vocab_size;
  rc_kv_clear(kv);
  float *logits = (float *)malloc((V ? V : 1) * 4);
  int st = rc_prefill(m, kv, prompt, n_prompt, logits, 1);
  for (size_t i = 0; i < max_tokens && !st; i++) {
    uint32_t nt = rc_argmax(logits, V);
    out[i] = nt;
    st = rc_decode_step(m, kv, nt, logits);
  }
  free(logits);
  return st;
}
