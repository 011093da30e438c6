// Synthetic benchmark models. No reference counterpart: the reference builds
// its GGUF fixtures in test code (TestGgufBuilder, src/model/forward.rs:655-727)
// and has no quantiser. Weights are N(0, sigma) from a counter-based
// generator; the quantisers emit bytes whose dequantisation under the
// reference's semantics (src/gguf/dequant.rs:62-199) approximates them.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "status.h"

namespace ifx {

namespace {

inline uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Elements 2p and 2p+1 of stream `key`: Box-Muller over pair p (cos, sin),
// uniforms from one splitmix64 draw split into two 24-bit halves, in f32.
inline void normal_pair(uint64_t key, uint64_t pair, float *z0, float *z1) {
  const uint64_t a = splitmix64(key ^ pair);
  const float u1 = ((float)(a >> 40) + 1.0f) * (1.0f / 16777216.0f);         // (0, 1]
  const float u2 = (float)((a >> 8) & 0xffffffu) * (1.0f / 16777216.0f);     // [0, 1)
  const float r = std::sqrt(-2.0f * std::log(u1));
  float s, c;
  sincosf(6.2831853f * u2, &s, &c);
  *z0 = r * c;
  *z1 = r * s;
}

inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return splitmix64(seed * 0x100000001B3ull + stream * 0x9E3779B97F4A7C15ull);
}

void gen_normal(uint64_t key, uint64_t start, size_t n, float sigma, float *out) {
  size_t i = 0;
  if (start % 2 == 1 && n) {
    float z0, z1;
    normal_pair(key, start / 2, &z0, &z1);
    out[i++] = z1 * sigma;
  }
  for (; i + 1 < n; i += 2) {
    float z0, z1;
    normal_pair(key, (start + i) / 2, &z0, &z1);
    out[i] = z0 * sigma;
    out[i + 1] = z1 * sigma;
  }
  if (i < n) {
    float z0, z1;
    normal_pair(key, (start + i) / 2, &z0, &z1);
    out[i] = z0 * sigma;
  }
}

// f32 -> f16 bits, round to nearest even.
uint16_t f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const float a = std::fabs(f);
  if (std::isnan(f)) return (uint16_t)(sign | 0x7e00u);
  if (a >= 65520.0f) return (uint16_t)(sign | 0x7c00u);
  if (a < 6.103515625e-05f) {  // below 2^-14: subnormal, in units of 2^-24
    return (uint16_t)(sign | (uint16_t)std::nearbyint(a * 16777216.0f));
  }
  const uint32_t ax = x & 0x7fffffffu;
  uint32_t v = (ax - 0x38000000u) >> 13;
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (v & 1u))) ++v;
  return (uint16_t)(sign | v);
}

float h2f_host(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while (!(man & 0x400u));
      bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

inline void put16(uint8_t *p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xff);
  p[1] = (uint8_t)(v >> 8);
}

int clampi(long v, int lo, int hi) { return (int)(v < lo ? lo : (v > hi ? hi : v)); }

void quant_q8_0(const float *x, uint8_t *o) {  // 32 -> 34 bytes (ggml layout)
  float amax = 0.f;
  for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(x[j]));
  const uint16_t dh = f2h(amax / 127.0f);
  const float d = h2f_host(dh);
  put16(o, dh);
  for (int j = 0; j < 32; ++j)
    o[2 + j] = (uint8_t)(int8_t)(d > 0 ? clampi(std::lround(x[j] / d), -127, 127) : 0);
}

void quant_q4_0(const float *x, uint8_t *o) {  // 32 -> 18 bytes (ggml layout)
  float amax = 0.f, mx = 0.f;
  for (int j = 0; j < 32; ++j)
    if (std::fabs(x[j]) > amax) {
      amax = std::fabs(x[j]);
      mx = x[j];
    }
  const uint16_t dh = f2h(mx / -8.0f);
  const float d = h2f_host(dh);
  const float id = d != 0.f ? 1.0f / d : 0.f;
  put16(o, dh);
  for (int j = 0; j < 16; ++j) {
    const int q0 = clampi((long)(x[j] * id + 8.5f), 0, 15);
    const int q1 = clampi((long)(x[j + 16] * id + 8.5f), 0, 15);
    o[2 + j] = (uint8_t)(q0 | (q1 << 4));
  }
}

// Q4_K under the reference's layout: nibble l of group g at qs[g*16 + l/2],
// even l in the low nibble (dequant.rs:151-158); 6-bit sc/mn packed so that
// the unpack of dequant.rs:141-149 returns them.
void quant_q4_k(const float *x, uint8_t *o) {  // 256 -> 144 bytes
  float scale[8], minv[8];
  for (int g = 0; g < 8; ++g) {
    float mn = 0.f, mx = x[g * 32];
    for (int l = 0; l < 32; ++l) {
      mn = std::fmin(mn, x[g * 32 + l]);
      mx = std::fmax(mx, x[g * 32 + l]);
    }
    scale[g] = (mx - mn) / 15.0f;
    minv[g] = -mn;
  }
  float smax = 0.f, mmax = 0.f;
  for (int g = 0; g < 8; ++g) {
    smax = std::fmax(smax, scale[g]);
    mmax = std::fmax(mmax, minv[g]);
  }
  const uint16_t dh = f2h(smax / 63.0f), mh = f2h(mmax / 63.0f);
  const float d = h2f_host(dh), dmin = h2f_host(mh);
  int sc[8], mn[8];
  for (int g = 0; g < 8; ++g) {
    sc[g] = d > 0 ? clampi(std::lround(scale[g] / d), 0, 63) : 0;
    mn[g] = dmin > 0 ? clampi(std::lround(minv[g] / dmin), 0, 63) : 0;
  }
  put16(o, dh);
  put16(o + 2, mh);
  uint8_t *s = o + 4;
  for (int g = 0; g < 4; ++g) {
    s[g] = (uint8_t)(sc[g] | ((sc[g + 4] >> 4) << 6));
    s[g + 4] = (uint8_t)(mn[g] | ((mn[g + 4] >> 4) << 6));
    s[g + 8] = (uint8_t)((sc[g + 4] & 15) | ((mn[g + 4] & 15) << 4));
  }
  uint8_t *qs = o + 16;
  memset(qs, 0, 128);
  for (int g = 0; g < 8; ++g) {
    const float dall = d * (float)sc[g], dm = dmin * (float)mn[g];
    for (int l = 0; l < 32; ++l) {
      const int q = dall > 0 ? clampi(std::lround((x[g * 32 + l] + dm) / dall), 0, 15) : 0;
      qs[g * 16 + l / 2] |= (uint8_t)(l % 2 == 0 ? q : q << 4);
    }
  }
}

// Q6_K under the reference's layout: d@0, u8 scales@2..18, ql@18..146,
// qh@146..210, element j in ql[j/2] (nibble j%2) and qh[j/4] (bits 2(j%4))
// (dequant.rs:182-196). Scales stay in 0..127 so u8 and i8 readings agree.
void quant_q6_k(const float *x, uint8_t *o) {  // 256 -> 210 bytes
  float scale[16];
  float smax = 0.f;
  for (int g = 0; g < 16; ++g) {
    float amax = 0.f;
    for (int l = 0; l < 16; ++l) amax = std::fmax(amax, std::fabs(x[g * 16 + l]));
    scale[g] = amax / 31.0f;
    smax = std::fmax(smax, scale[g]);
  }
  const uint16_t dh = f2h(smax / 127.0f);
  const float d = h2f_host(dh);
  put16(o, dh);
  uint8_t *sc = o + 2, *ql = o + 18, *qh = o + 146;
  memset(ql, 0, 128);
  memset(qh, 0, 64);
  for (int g = 0; g < 16; ++g) sc[g] = (uint8_t)(d > 0 ? clampi(std::lround(scale[g] / d), 0, 127) : 0);
  for (int j = 0; j < 256; ++j) {
    const float ds = d * (float)sc[j / 16];
    const int q = ds > 0 ? clampi(std::lround(x[j] / ds) + 32, 0, 63) : 32;
    ql[j / 2] |= (uint8_t)(j % 2 == 0 ? (q & 15) : (q & 15) << 4);
    qh[j / 4] |= (uint8_t)(((q >> 4) & 3) << (2 * (j % 4)));
  }
}

struct TypeInfo {
  int elems, bytes;
  void (*quant)(const float *, uint8_t *);
};

bool type_info(int type, TypeInfo *t) {
  switch (type) {
    case IFX_TYPE_Q8_0: *t = {32, 34, quant_q8_0}; return true;
    case IFX_TYPE_Q4_0: *t = {32, 18, quant_q4_0}; return true;
    case IFX_TYPE_Q4_K: *t = {256, 144, quant_q4_k}; return true;
    case IFX_TYPE_Q6_K: *t = {256, 210, quant_q6_k}; return true;
    default: return false;
  }
}

struct TensorSpec {
  std::string name;
  uint64_t rows, cols;  // logical [rows, cols]; GGUF dims are [cols, rows]
  int type;             // 0 = F32 ones (norms)
  uint64_t offset = 0, bytes = 0;
};

void wstr(std::vector<uint8_t> &b, const std::string &s) {
  uint64_t n = s.size();
  b.insert(b.end(), reinterpret_cast<uint8_t *>(&n), reinterpret_cast<uint8_t *>(&n) + 8);
  b.insert(b.end(), s.begin(), s.end());
}
template <typename T>
void wpod(std::vector<uint8_t> &b, T v) {
  b.insert(b.end(), reinterpret_cast<uint8_t *>(&v), reinterpret_cast<uint8_t *>(&v) + sizeof(T));
}

}  // namespace

}  // namespace ifx

using namespace ifx;

extern "C" {

ifx_status ifx_synth_normal(uint64_t seed, uint64_t stream, float sigma, float *out, size_t n) {
  if (!out && n) return fail(IFX_ERR_INVALID_ARGUMENT, "synth_normal: null output");
  gen_normal(stream_key(seed, stream), 0, n, sigma, out);
  return IFX_OK;
}

ifx_status ifx_quantize(int type, const float *x, size_t n, void *out) {
  TypeInfo t;
  if (!type_info(type, &t)) return fail(IFX_ERR_UNKNOWN_TENSOR_TYPE, "quantize: unsupported type");
  if (n % t.elems) return fail(IFX_ERR_SHAPE, "quantize: n not a multiple of the block size");
  for (size_t b = 0; b < n / t.elems; ++b)
    t.quant(x + b * t.elems, static_cast<uint8_t *>(out) + b * t.bytes);
  return IFX_OK;
}

void ifx_synth_free(void *bytes) { free(bytes); }

ifx_status ifx_synth_gguf(const ifx_synth_spec *sp, void **bytes_out, size_t *len_out) {
  if (!sp || !bytes_out || !len_out) return fail(IFX_ERR_INVALID_ARGUMENT, "synth: null argument");
  const uint64_t V = sp->vocab, D = sp->dim, L = sp->n_layers, H = sp->n_heads, G = sp->n_kv_heads,
                 F = sp->ffn;
  if (!V || !D || !H || !G || !F || D % H || H % G)
    return fail(IFX_ERR_SHAPE, "synth: inconsistent shape");
  const uint64_t hd = D / H, kvd = G * hd;
  auto pick = [&](const std::string &role, uint64_t layer) -> int {
    if (sp->mix == 0) return IFX_TYPE_Q8_0;
    if (sp->mix == 2) return IFX_TYPE_Q4_0;
    // Q4_K_M: Q6_K for attn_v, every other ffn_down, and output/tied embedding
    if (role == "attn_v" || role == "output") return IFX_TYPE_Q6_K;
    if (role == "ffn_down" && layer % 2 == 0) return IFX_TYPE_Q6_K;
    if (role == "token_embd") return sp->tied ? IFX_TYPE_Q6_K : IFX_TYPE_Q4_K;
    return IFX_TYPE_Q4_K;
  };
  std::vector<TensorSpec> ts;
  ts.push_back({"token_embd.weight", V, D, pick("token_embd", 0)});
  ts.push_back({"output_norm.weight", 1, D, 0});
  if (!sp->tied) ts.push_back({"output.weight", V, D, pick("output", 0)});
  for (uint64_t l = 0; l < L; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    ts.push_back({p + "attn_norm.weight", 1, D, 0});
    ts.push_back({p + "attn_q.weight", D, D, pick("attn_q", l)});
    ts.push_back({p + "attn_k.weight", kvd, D, pick("attn_k", l)});
    ts.push_back({p + "attn_v.weight", kvd, D, pick("attn_v", l)});
    ts.push_back({p + "attn_output.weight", D, D, pick("attn_output", l)});
    ts.push_back({p + "ffn_norm.weight", 1, D, 0});
    ts.push_back({p + "ffn_gate.weight", F, D, pick("ffn_gate", l)});
    ts.push_back({p + "ffn_up.weight", F, D, pick("ffn_up", l)});
    ts.push_back({p + "ffn_down.weight", D, F, pick("ffn_down", l)});
  }
  uint64_t off = 0;
  for (auto &t : ts) {
    if (t.type == 0) {
      t.bytes = t.rows * t.cols * 4;
    } else {
      TypeInfo ti;
      type_info(t.type, &ti);
      if (t.cols % ti.elems) return fail(IFX_ERR_SHAPE, "synth: " + t.name + " columns not a multiple of the block");
      t.bytes = t.rows * (t.cols / ti.elems) * ti.bytes;
    }
    t.offset = off;
    off = (off + t.bytes + 31) / 32 * 32;
  }
  std::vector<uint8_t> hdr;
  hdr.insert(hdr.end(), {'G', 'G', 'U', 'F'});
  wpod<uint32_t>(hdr, 3);
  wpod<uint64_t>(hdr, ts.size());
  wpod<uint64_t>(hdr, 10);
  auto kv_u32 = [&](const char *k, uint32_t v) {
    wstr(hdr, k);
    wpod<uint32_t>(hdr, 4);
    wpod<uint32_t>(hdr, v);
  };
  auto kv_f32 = [&](const char *k, float v) {
    wstr(hdr, k);
    wpod<uint32_t>(hdr, 6);
    wpod<float>(hdr, v);
  };
  wstr(hdr, "general.architecture");
  wpod<uint32_t>(hdr, 8);
  wstr(hdr, "llama");
  kv_u32("llama.vocab_size", (uint32_t)V);
  kv_u32("llama.embedding_length", (uint32_t)D);
  kv_u32("llama.block_count", (uint32_t)L);
  kv_u32("llama.attention.head_count", (uint32_t)H);
  kv_u32("llama.attention.head_count_kv", (uint32_t)G);
  kv_u32("llama.feed_forward_length", (uint32_t)F);
  kv_f32("llama.attention.layer_norm_rms_epsilon", sp->norm_eps);
  kv_u32("llama.context_length", sp->context);
  kv_f32("llama.rope.freq_base", sp->rope_base);
  for (auto &t : ts) {
    wstr(hdr, t.name);
    const bool vec = t.rows == 1;
    wpod<uint32_t>(hdr, vec ? 1 : 2);
    wpod<uint64_t>(hdr, t.cols);
    if (!vec) wpod<uint64_t>(hdr, t.rows);
    wpod<uint32_t>(hdr, (uint32_t)t.type);
    wpod<uint64_t>(hdr, t.offset);
  }
  while (hdr.size() % 32) hdr.push_back(0);
  const size_t total = hdr.size() + off;
  uint8_t *buf = static_cast<uint8_t *>(malloc(total));
  if (!buf) return fail(IFX_ERR_OUT_OF_MEMORY, "synth: host allocation");
  memcpy(buf, hdr.data(), hdr.size());
  uint8_t *data = buf + hdr.size();
  memset(data, 0, off);
  int nthr = sp->threads > 0 ? sp->threads : (int)std::thread::hardware_concurrency();
  if (nthr < 1) nthr = 1;
  for (size_t ti_ = 0; ti_ < ts.size(); ++ti_) {
    const TensorSpec &t = ts[ti_];
    uint8_t *dst = data + t.offset;
    if (t.type == 0) {
      float one = 1.0f;
      for (uint64_t i = 0; i < t.cols; ++i) memcpy(dst + 4 * i, &one, 4);
      continue;
    }
    TypeInfo ti;
    type_info(t.type, &ti);
    const uint64_t key = stream_key(sp->seed, ti_);
    const uint64_t nblocks = t.rows * t.cols / ti.elems;
    const int nt = (int)std::min<uint64_t>((uint64_t)nthr, (nblocks + 1023) / 1024);
    std::vector<std::thread> th;
    auto work = [&, dst, key, nblocks](int w, int nw) {
      std::vector<float> tmp(ti.elems);
      const uint64_t b0 = nblocks * w / nw, b1 = nblocks * (w + 1) / nw;
      for (uint64_t b = b0; b < b1; ++b) {
        gen_normal(key, b * ti.elems, ti.elems, sp->sigma, tmp.data());
        ti.quant(tmp.data(), dst + b * ti.bytes);
      }
    };
    if (nt <= 1) {
      work(0, 1);
    } else {
      for (int w = 0; w < nt; ++w) th.emplace_back(work, w, nt);
      for (auto &x : th) x.join();
    }
  }
  *bytes_out = buf;
  *len_out = total;
  return IFX_OK;
}

}  // extern "C"
