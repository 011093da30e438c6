/* Oracle-side generator of the benchmark's synthetic models (TEST
 * INFRASTRUCTURE ONLY: the reference arm of bench.py builds its input model
 * with this, so timing the reference's CPU path never loads the product
 * library).
 *
 * The reference has no quantiser and no model generator (its fixtures are
 * built in test code, src/model/forward.rs:655-727). This file states the
 * workload definition the benchmark uses, independently of the product's
 * generator, and a CPU test checks that both produce the same bytes:
 *  - weights N(0, sigma): splitmix64 counter stream per tensor, Box-Muller
 *    over pairs (cos, sin) with two 24-bit uniforms per draw, in f32;
 *  - Q8_0 / Q4_0 blocks as ggml lays them (identical in the reference);
 *  - Q4_K and Q6_K blocks in the reference's element order
 *    (src/gguf/dequant.rs:123-199), scales fitted per group, d / dmin in f16;
 *  - the Q4_K_M mix: Q6_K for attn_v, even-layer ffn_down and the output
 *    (or a tied token_embd), Q4_K elsewhere; mix 0 = all Q8_0, 2 = Q4_0;
 *  - norm weights F32 ones; GGUF v3 with 32-byte aligned tensor data
 *    (src/gguf/file.rs:112-116). */
#define _GNU_SOURCE /* sincosf */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include "refcpu.h"

static uint64_t sm64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static void gauss_pair(uint64_t key, uint64_t pair, float *a, float *b) {
  const uint64_t r = sm64(key ^ pair);
  const float u1 = ((float)(r >> 40) + 1.0f) * (1.0f / 16777216.0f);
  const float u2 = (float)((r >> 8) & 0xffffffu) * (1.0f / 16777216.0f);
  const float rad = sqrtf(-2.0f * logf(u1));
  float s, c;
  sincosf(6.2831853f * u2, &s, &c);
  *a = rad * c;
  *b = rad * s;
}

static uint64_t tensor_key(uint64_t seed, uint64_t stream) {
  return sm64(seed * 0x100000001B3ull + stream * 0x9E3779B97F4A7C15ull);
}

/* elements [start, start + n) of the stream (element 2p is the cos half of
 * pair p, element 2p + 1 the sin half) */
static void fill_normal(uint64_t key, uint64_t start, size_t n, float sigma, float *out) {
  size_t i = 0;
  while (i < n) {
    const uint64_t e = start + i;
    float a, b;
    gauss_pair(key, e / 2, &a, &b);
    if (e % 2) {
      out[i++] = b * sigma;
    } else {
      out[i++] = a * sigma;
      if (i < n) out[i++] = b * sigma;
    }
  }
}

static uint16_t to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const float a = fabsf(f);
  if (isnan(f)) return (uint16_t)(sign | 0x7e00u);
  if (a >= 65520.0f) return (uint16_t)(sign | 0x7c00u);
  if (a < 6.103515625e-05f) return (uint16_t)(sign | (uint16_t)nearbyintf(a * 16777216.0f));
  const uint32_t ax = x & 0x7fffffffu;
  uint32_t v = (ax - 0x38000000u) >> 13;
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (v & 1u))) ++v;
  return (uint16_t)(sign | v);
}

static int clamp_int(long v, int lo, int hi) { return (int)(v < lo ? lo : (v > hi ? hi : v)); }

static void wr16(uint8_t *p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xff);
  p[1] = (uint8_t)(v >> 8);
}

static void blk_q8_0(const float *x, uint8_t *o) {
  float amax = 0.f;
  for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
  const uint16_t dh = to_f16(amax / 127.0f);
  const float d = rc_f16_to_f32(dh);
  wr16(o, dh);
  for (int j = 0; j < 32; j++)
    o[2 + j] = (uint8_t)(int8_t)(d > 0 ? clamp_int(lroundf(x[j] / d), -127, 127) : 0);
}

static void blk_q4_0(const float *x, uint8_t *o) {
  float amax = 0.f, mx = 0.f;
  for (int j = 0; j < 32; j++)
    if (fabsf(x[j]) > amax) { amax = fabsf(x[j]); mx = x[j]; }
  const uint16_t dh = to_f16(mx / -8.0f);
  const float d = rc_f16_to_f32(dh);
  const float id = d != 0.f ? 1.0f / d : 0.f;
  wr16(o, dh);
  for (int j = 0; j < 16; j++) {
    const int q0 = clamp_int((long)(x[j] * id + 8.5f), 0, 15);
    const int q1 = clamp_int((long)(x[j + 16] * id + 8.5f), 0, 15);
    o[2 + j] = (uint8_t)(q0 | (q1 << 4));
  }
}

/* reference order: nibble l of group g at qs[g*16 + l/2], even l low
 * (dequant.rs:151-158); 6-bit scale/min packing undone by dequant.rs:141-149 */
static void blk_q4_k(const float *x, uint8_t *o) {
  float sc_f[8], mn_f[8], smax = 0.f, mmax = 0.f;
  for (int g = 0; g < 8; g++) {
    float lo = 0.f, hi = x[g * 32];
    for (int l = 0; l < 32; l++) {
      lo = fminf(lo, x[g * 32 + l]);
      hi = fmaxf(hi, x[g * 32 + l]);
    }
    sc_f[g] = (hi - lo) / 15.0f;
    mn_f[g] = -lo;
    smax = fmaxf(smax, sc_f[g]);
    mmax = fmaxf(mmax, mn_f[g]);
  }
  const uint16_t dh = to_f16(smax / 63.0f), mh = to_f16(mmax / 63.0f);
  const float d = rc_f16_to_f32(dh), dmin = rc_f16_to_f32(mh);
  int sc[8], mn[8];
  for (int g = 0; g < 8; g++) {
    sc[g] = d > 0 ? clamp_int(lroundf(sc_f[g] / d), 0, 63) : 0;
    mn[g] = dmin > 0 ? clamp_int(lroundf(mn_f[g] / dmin), 0, 63) : 0;
  }
  wr16(o, dh);
  wr16(o + 2, mh);
  uint8_t *s = o + 4;
  for (int g = 0; g < 4; g++) {
    s[g] = (uint8_t)(sc[g] | ((sc[g + 4] >> 4) << 6));
    s[g + 4] = (uint8_t)(mn[g] | ((mn[g + 4] >> 4) << 6));
    s[g + 8] = (uint8_t)((sc[g + 4] & 15) | ((mn[g + 4] & 15) << 4));
  }
  uint8_t *qs = o + 16;
  memset(qs, 0, 128);
  for (int g = 0; g < 8; g++) {
    const float dall = d * (float)sc[g], dm = dmin * (float)mn[g];
    for (int l = 0; l < 32; l++) {
      const int q = dall > 0 ? clamp_int(lroundf((x[g * 32 + l] + dm) / dall), 0, 15) : 0;
      qs[g * 16 + l / 2] |= (uint8_t)(l % 2 == 0 ? q : q << 4);
    }
  }
}

/* reference order: d@0, u8 scales@2..18, ql@18..146, qh@146..210
 * (dequant.rs:182-196); scales in 0..127 */
static void blk_q6_k(const float *x, uint8_t *o) {
  float sc_f[16], smax = 0.f;
  for (int g = 0; g < 16; g++) {
    float amax = 0.f;
    for (int l = 0; l < 16; l++) amax = fmaxf(amax, fabsf(x[g * 16 + l]));
    sc_f[g] = amax / 31.0f;
    smax = fmaxf(smax, sc_f[g]);
  }
  const uint16_t dh = to_f16(smax / 127.0f);
  const float d = rc_f16_to_f32(dh);
  wr16(o, dh);
  uint8_t *sc = o + 2, *ql = o + 18, *qh = o + 146;
  memset(ql, 0, 128);
  memset(qh, 0, 64);
  for (int g = 0; g < 16; g++) sc[g] = (uint8_t)(d > 0 ? clamp_int(lroundf(sc_f[g] / d), 0, 127) : 0);
  for (int j = 0; j < 256; j++) {
    const float ds = d * (float)sc[j / 16];
    const int q = ds > 0 ? clamp_int(lroundf(x[j] / ds) + 32, 0, 63) : 32;
    ql[j / 2] |= (uint8_t)(j % 2 == 0 ? (q & 15) : (q & 15) << 4);
    qh[j / 4] |= (uint8_t)(((q >> 4) & 3) << (2 * (j % 4)));
  }
}

typedef struct {
  int elems, bytes;
  void (*fn)(const float *, uint8_t *);
} blk_fmt;

static int blk_format(int type, blk_fmt *f) {
  switch (type) {
    case RC_Q8_0: f->elems = 32; f->bytes = 34; f->fn = blk_q8_0; return 1;
    case RC_Q4_0: f->elems = 32; f->bytes = 18; f->fn = blk_q4_0; return 1;
    case RC_Q4K: f->elems = 256; f->bytes = 144; f->fn = blk_q4_k; return 1;
    case RC_Q6K: f->elems = 256; f->bytes = 210; f->fn = blk_q6_k; return 1;
    default: return 0;
  }
}

typedef struct {
  char name[64];
  uint64_t rows, cols;
  int type; /* -1: F32 ones */
  uint64_t off, bytes;
} tspec;

typedef struct {
  uint8_t *p;
  size_t n, cap;
} wbuf;

static void wput(wbuf *b, const void *src, size_t n) {
  if (b->n + n > b->cap) {
    b->cap = (b->n + n) * 2 + 1024;
    b->p = (uint8_t *)realloc(b->p, b->cap);
  }
  memcpy(b->p + b->n, src, n);
  b->n += n;
}
static void wput_str(wbuf *b, const char *s) {
  const uint64_t n = strlen(s);
  wput(b, &n, 8);
  wput(b, s, n);
}
static void wput_u32(wbuf *b, uint32_t v) { wput(b, &v, 4); }
static void wput_u64(wbuf *b, uint64_t v) { wput(b, &v, 8); }
static void kv_u32(wbuf *b, const char *k, uint32_t v) {
  wput_str(b, k);
  wput_u32(b, 4);
  wput_u32(b, v);
}
static void kv_f32(wbuf *b, const char *k, float v) {
  wput_str(b, k);
  wput_u32(b, 6);
  wput(b, &v, 4);
}

typedef struct {
  const tspec *t;
  blk_fmt f;
  uint8_t *dst;
  uint64_t key, b0, b1;
  float sigma;
} qjob;

static void *qjob_run(void *arg) {
  const qjob *j = (const qjob *)arg;
  float tmp[256];
  for (uint64_t b = j->b0; b < j->b1; b++) {
    fill_normal(j->key, b * (uint64_t)j->f.elems, (size_t)j->f.elems, j->sigma, tmp);
    j->f.fn(tmp, j->dst + b * (uint64_t)j->f.bytes);
  }
  return NULL;
}

static int pick_type(const rc_synth_spec *sp, const char *role, uint64_t layer) {
  if (sp->mix == 0) return RC_Q8_0;
  if (sp->mix == 2) return RC_Q4_0;
  if (!strcmp(role, "attn_v") || !strcmp(role, "output")) return RC_Q6K;
  if (!strcmp(role, "ffn_down") && layer % 2 == 0) return RC_Q6K;
  if (!strcmp(role, "token_embd")) return sp->tied ? RC_Q6K : RC_Q4K;
  return RC_Q4K;
}

int rc_synth_gguf(const rc_synth_spec *sp, uint8_t **out, size_t *out_len) {
  if (!sp || !out || !out_len) return RC_ERR_IO;
  const uint64_t V = sp->vocab, D = sp->dim, L = sp->n_layers, H = sp->n_heads,
                 G = sp->n_kv_heads, F = sp->ffn;
  if (!V || !D || !H || !G || !F || D % H || H % G) return RC_ERR_INVALID_SHAPE;
  const uint64_t kvd = G * (D / H);
  const size_t nt = 2 + (sp->tied ? 0 : 1) + 9 * (size_t)L;
  tspec *ts = (tspec *)calloc(nt, sizeof(tspec));
  size_t k = 0;
#define ADD(NM, R, C, T)                                   \
  do {                                                     \
    snprintf(ts[k].name, sizeof ts[k].name, "%s", NM);     \
    ts[k].rows = (R); ts[k].cols = (C); ts[k].type = (T);  \
    k++;                                                   \
  } while (0)
  ADD("token_embd.weight", V, D, pick_type(sp, "token_embd", 0));
  ADD("output_norm.weight", 1, D, -1);
  if (!sp->tied) ADD("output.weight", V, D, pick_type(sp, "output", 0));
  for (uint64_t l = 0; l < L; l++) {
    char nm[64];
#define LAYER(SUFFIX, R, C, ROLE)                                             \
    snprintf(nm, sizeof nm, "blk.%llu." SUFFIX, (unsigned long long)l);       \
    ADD(nm, R, C, ROLE ? pick_type(sp, ROLE, l) : -1);
    LAYER("attn_norm.weight", 1, D, NULL)
    LAYER("attn_q.weight", D, D, "attn_q")
    LAYER("attn_k.weight", kvd, D, "attn_k")
    LAYER("attn_v.weight", kvd, D, "attn_v")
    LAYER("attn_output.weight", D, D, "attn_output")
    LAYER("ffn_norm.weight", 1, D, NULL)
    LAYER("ffn_gate.weight", F, D, "ffn_gate")
    LAYER("ffn_up.weight", F, D, "ffn_up")
    LAYER("ffn_down.weight", D, F, "ffn_down")
#undef LAYER
  }
#undef ADD
  uint64_t off = 0;
  for (size_t i = 0; i < nt; i++) {
    if (ts[i].type < 0) {
      ts[i].bytes = ts[i].rows * ts[i].cols * 4;
    } else {
      blk_fmt f = {0, 0, NULL};
      if (!blk_format(ts[i].type, &f)) { free(ts); return RC_ERR_UNKNOWN_TENSOR_TYPE; }
      if (ts[i].cols % (uint64_t)f.elems) { free(ts); return RC_ERR_INVALID_SHAPE; }
      ts[i].bytes = ts[i].rows * (ts[i].cols / (uint64_t)f.elems) * (uint64_t)f.bytes;
    }
    ts[i].off = off;
    off = (off + ts[i].bytes + 31) / 32 * 32;
  }
  wbuf h = {0};
  wput(&h, "GGUF", 4);
  wput_u32(&h, 3);
  wput_u64(&h, nt);
  wput_u64(&h, 10);
  wput_str(&h, "general.architecture");
  wput_u32(&h, 8);
  wput_str(&h, "llama");
  kv_u32(&h, "llama.vocab_size", (uint32_t)V);
  kv_u32(&h, "llama.embedding_length", (uint32_t)D);
  kv_u32(&h, "llama.block_count", (uint32_t)L);
  kv_u32(&h, "llama.attention.head_count", (uint32_t)H);
  kv_u32(&h, "llama.attention.head_count_kv", (uint32_t)G);
  kv_u32(&h, "llama.feed_forward_length", (uint32_t)F);
  kv_f32(&h, "llama.attention.layer_norm_rms_epsilon", sp->norm_eps);
  kv_u32(&h, "llama.context_length", sp->context);
  kv_f32(&h, "llama.rope.freq_base", sp->rope_base);
  for (size_t i = 0; i < nt; i++) {
    wput_str(&h, ts[i].name);
    const int vec = ts[i].rows == 1;
    wput_u32(&h, vec ? 1 : 2);
    wput_u64(&h, ts[i].cols);
    if (!vec) wput_u64(&h, ts[i].rows);
    wput_u32(&h, (uint32_t)(ts[i].type < 0 ? 0 : ts[i].type));
    wput_u64(&h, ts[i].off);
  }
  const uint8_t zero = 0;
  while (h.n % 32) wput(&h, &zero, 1);
  const size_t total = h.n + off;
  uint8_t *buf = (uint8_t *)malloc(total);
  if (!buf) { free(h.p); free(ts); return RC_ERR_IO; }
  memcpy(buf, h.p, h.n);
  uint8_t *data = buf + h.n;
  memset(data, 0, off);
  int nthr = sp->threads > 0 ? sp->threads : 1;
  if (nthr > 256) nthr = 256;
  for (size_t i = 0; i < nt; i++) {
    uint8_t *dst = data + ts[i].off;
    if (ts[i].type < 0) {
      const float one = 1.0f;
      for (uint64_t e = 0; e < ts[i].cols; e++) memcpy(dst + 4 * e, &one, 4);
      continue;
    }
    blk_fmt f = {0, 0, NULL};
    blk_format(ts[i].type, &f);
    const uint64_t nb = ts[i].rows * ts[i].cols / (uint64_t)f.elems;
    const uint64_t key = tensor_key(sp->seed, (uint64_t)i);
    int w = (int)((nb + 1023) / 1024);
    if (w > nthr) w = nthr;
    if (w < 1) w = 1;
    qjob jobs[256];
    pthread_t th[256];
    for (int t = 0; t < w; t++) {
      jobs[t] = (qjob){&ts[i], f, dst, key, nb * (uint64_t)t / (uint64_t)w,
                       nb * (uint64_t)(t + 1) / (uint64_t)w, sp->sigma};
      if (w > 1) pthread_create(&th[t], NULL, qjob_run, &jobs[t]);
      else qjob_run(&jobs[t]);
    }
    if (w > 1)
      for (int t = 0; t < w; t++) pthread_join(th[t], NULL);
  }
  free(h.p);
  free(ts);
  *out = buf;
  *out_len = total;
  return RC_OK;
}

void rc_synth_free(uint8_t *p) { free(p); }
