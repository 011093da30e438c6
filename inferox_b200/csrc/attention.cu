// Decode: split-K flash-decoding over the f16 KV cache (replaces the decode
// attention loop of Layer::decode_step, src/model/forward.rs:375-414).
// Prefill: causal attention within the prompt chunk (forward.rs:246-305).
#include <algorithm>

#include "attention.cuh"

namespace ifx {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kMaxGroup = 8;    // q heads per kv head handled per CTA
constexpr int kMaxSplits = 64;  // split-K factor ceiling (model.cu picks <= 64)

__device__ __forceinline__ void rope_pair(float &a, float &b, int i, int rope_dim, float base,
                                          int pos) {
  float inv = 1.0f / powf(base, (float)i / (float)rope_dim);
  float ang = __fmul_rn((float)pos, inv);
  float s, c;
  sincosf(ang, &s, &c);
  float x0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  float x1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  a = x0;
  b = x1;
}

// Cache rows one split can hold (its chunk plus this token's row), rounded
// up to whole 16-row MMA tiles.
__host__ __device__ __forceinline__ int attn_rows(int max_seq, int ns) {
  return ((max_seq + ns - 1) / ns + 1 + 15) & ~15;
}

// Combine the NS partial softmaxes of kv head h (run by the CTA that
// finished the head's last split): weights exp(m_s - M) / L per split and
// head, then the weighted sum of the partial outputs. All loads of a phase
// are issued together (one L2 round trip each) instead of a serial walk.
__device__ __noinline__ void attn_combine(const float *part_o, const float2 *part_ml,
                                          float *attn_out, int *counters, int h, int NS,
                                          int grp, int hd, int tid, int nthr) {
  __shared__ float c_m[kMaxSplits * kMaxGroup], c_w[kMaxSplits * kMaxGroup], c_M[kMaxGroup],
      c_L[kMaxGroup];
  for (int e = tid; e < NS * grp; e += nthr) {
    const float2 ml = __ldcg(&part_ml[h * NS * grp + e]);
    c_m[e] = ml.x;
    c_w[e] = ml.y;
  }
  __syncthreads();
  if (tid < grp) {
    float M = -INFINITY;
    for (int t = 0; t < NS; ++t)
      if (c_w[t * grp + tid] > 0.f) M = fmaxf(M, c_m[t * grp + tid]);
    float L = 0.f;
    for (int t = 0; t < NS; ++t)
      if (c_w[t * grp + tid] > 0.f) L = fmaf(c_w[t * grp + tid], expf(c_m[t * grp + tid] - M), L);
    c_M[tid] = M;
    c_L[tid] = L;
  }
  __syncthreads();
  for (int e = tid; e < NS * grp; e += nthr) {
    const int j = e % grp;
    c_w[e] = (c_w[e] > 0.f) ? expf(c_m[e] - c_M[j]) / c_L[j] : 0.f;
  }
  __syncthreads();
  const float4 *po4 = reinterpret_cast<const float4 *>(part_o + (size_t)h * NS * grp * hd);
  float4 *out4 = reinterpret_cast<float4 *>(attn_out + (size_t)h * grp * hd);
  const int n4 = grp * hd / 4;
  for (int e4 = tid; e4 < n4; e4 += nthr) {
    const int j = (e4 * 4) / hd;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int t = 0; t < NS; ++t) {
      const float w = c_w[t * grp + j];
      const float4 p = __ldcg(&po4[(size_t)t * n4 + e4]);
      o.x = fmaf(w, p.x, o.x);
      o.y = fmaf(w, p.y, o.y);
      o.z = fmaf(w, p.z, o.z);
      o.w = fmaf(w, p.w, o.w);
    }
    out4[e4] = o;
  }
  if (tid == 0) counters[h] = 0;
}

// W = 4 or 8: scores and P V on tensor cores (head size a multiple of 64, at
// most W query heads per kv head): S = K Q^T with the chunk-swizzled cache
// rows as ldmatrix A fragments and the query heads as B columns carrying
// each head's hi and lo f16 planes, O^T = V^T P the same way with
// ldmatrix.trans. W = 4: one 8-column tile (column j the hi plane of head j,
// column 4 + j its lo plane, added across lanes); W = 8: two tiles (hi
// planes, lo planes). W = 0: FMA loops.
template <int W>
__global__ void __launch_bounds__(kAttnThreads) decode_attn_kernel(const __grid_constant__ DecodeAttnArgs a) {
  extern __shared__ __align__(128) uint8_t smraw[];
  const int h = blockIdx.x, s = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  const int grp = a.H / a.G, hd = a.hd, NS = a.ns;
  // this sequence's slices of the inputs, caches, partials and output
  const float *qkv = a.qkv + (size_t)b * a.qkv_stride;
  const int sq = a.slot ? a.slot[b] : b;  // the sequence whose cache this row extends
  __half *kcb = a.kc + (size_t)sq * a.kv_seq_stride, *vcb = a.vc + (size_t)sq * a.kv_seq_stride;
  float *part_o = a.part_o + (size_t)b * a.G * NS * grp * hd;
  float2 *part_ml = a.part_ml + (size_t)b * a.G * NS * grp;
  int *counters = a.counters + (size_t)b * a.G;
  float *attn_out = a.attn_out + (size_t)b * a.H * hd;
  const int cap = attn_rows(a.max_seq, NS);
  __half *Ks = reinterpret_cast<__half *>(smraw);  // [cap][hd]
  __half *Vs = Ks + (size_t)cap * hd;               // [cap][hd]
  // FMA path: q [grp][hd] f32, scores [grp][cap]; tensor-core path: q hi/lo
  // [2][W][hd + 8] halves, scores [W][cap], p hi/lo [2][W][cap + 8] halves
  constexpr bool TC = W > 0;
  constexpr int NT = W / 4;  // 8-column B tiles per MMA step
  const int qs_ = hd + 8, ps_ = cap + 8;
  float *qs = reinterpret_cast<float *>(Vs + (size_t)cap * hd);
  __half *qh = Vs + (size_t)cap * hd;
  float *sc = TC ? reinterpret_cast<float *>(qh + 2 * W * qs_) : qs + grp * hd;
  __half *ph = reinterpret_cast<__half *>(sc + W * cap);
  __shared__ float s_m[kMaxGroup], s_l[kMaxGroup];
  __shared__ int s_last;
  __shared__ __align__(8) uint64_t bar;

  // Pre-wait: the cache rows [0, pos) of this layer and `pos` itself were
  // written by kernels that completed before the previous kernel in the
  // stream started its main phase, so this CTA's chunk can be fetched while
  // the QKV GEMV is still draining.
  const int pos = a.pos[sq];
  const int len = pos + 1;
  const int chunk = a.page_table ? a.page_rows : (len + NS - 1) / NS;
  const int t0 = s * chunk, t1 = min(len, t0 + chunk);
  const int nk = max(0, t1 - t0);
  const int nold = max(0, min(t1, pos) - t0);  // rows already in the cache
  // kc / vc address rows by position t (kc + t * hd); a page is indexed from
  // its first position t0
  __half *kc, *vc;
  if (a.page_table) {
    const int pg = nk > 0 ? a.page_table[(size_t)sq * a.max_pages + s] : 0;
    const size_t off = (size_t)pg * a.page_stride + (size_t)h * a.page_rows * hd;
    kc = a.kc + off - (size_t)t0 * hd;
    vc = a.vc + off - (size_t)t0 * hd;
  } else {
    kc = kcb + (size_t)h * a.max_seq * hd;
    vc = vcb + (size_t)h * a.max_seq * hd;
  }
  const uint32_t row_bytes = (uint32_t)hd * 2u;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    if (nold > 0) {
      mbar_arrive_expect_tx(&bar, 2u * nold * row_bytes);
      bulk_g2s(Ks, kc + (size_t)t0 * hd, nold * row_bytes, &bar);
      bulk_g2s(Vs, vc + (size_t)t0 * hd, nold * row_bytes, &bar);
    }
  }
  __syncthreads();  // the barrier is initialised before any thread waits on it

  pdl_wait();
  pdl_launch();

  if (a.zero_ptr && b == 0) {
    const int nb = a.G * NS, b = h * NS + s;
    for (int i = b * kAttnThreads + tid; i < a.zero_n; i += nb * kAttnThreads) a.zero_ptr[i] = 0.f;
  }

  const float *q = qkv + (size_t)h * grp * hd;
  const int rpos = a.rope_compat ? 0 : pos;
  for (int e = tid; e < (TC ? W : grp) * hd / 2; e += kAttnThreads) {
    const int j = e / (hd / 2), i = 2 * (e % (hd / 2));
    float x0 = 0.f, x1 = 0.f;
    if (j < grp) {
      x0 = q[j * hd + i];
      x1 = q[j * hd + i + 1];
      if (i < a.rope_dim) rope_pair(x0, x1, i, a.rope_dim, a.rope_base, rpos);
    }
    if (TC) {
      const __half2 hi = __floats2half2_rn(x0, x1);
      *reinterpret_cast<__half2 *>(qh + j * qs_ + i) = hi;
      *reinterpret_cast<__half2 *>(qh + (W + j) * qs_ + i) =
          __floats2half2_rn(x0 - __low2float(hi), x1 - __high2float(hi));
    } else {
      qs[j * hd + i] = x0;
      qs[j * hd + i + 1] = x1;
    }
  }
  if (t0 <= pos && pos < t1) {
    // append this token's K/V (forward.rs:375-378), K rotated like q
    const float *kn = qkv + (size_t)a.H * hd + (size_t)h * hd;
    const float *vn = qkv + (size_t)(a.H + a.G) * hd + (size_t)h * hd;
    const int r = pos - t0;
    for (int e = tid; e < hd / 2; e += kAttnThreads) {
      const int i = 2 * e;
      float x0 = kn[i], x1 = kn[i + 1];
      if (i < a.rope_dim) rope_pair(x0, x1, i, a.rope_dim, a.rope_base, rpos);
      const __half2 kh = __floats2half2_rn(x0, x1), vh = __floats2half2_rn(vn[i], vn[i + 1]);
      const int ip = kv_col(pos, i, hd);
      *reinterpret_cast<__half2 *>(kc + (size_t)pos * hd + ip) = kh;
      *reinterpret_cast<__half2 *>(vc + (size_t)pos * hd + ip) = vh;
      *reinterpret_cast<__half2 *>(Ks + (size_t)r * hd + ip) = kh;
      *reinterpret_cast<__half2 *>(Vs + (size_t)r * hd + ip) = vh;
    }
  }
  if (nold > 0) mbar_wait(&bar, 0, a.err, 301);
  __syncthreads();

  float *po = part_o + (size_t)(h * NS + s) * grp * hd;
  if constexpr (TC) {
    const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
    const int nk16 = (nk + 15) & ~15;
    // V rows [nk, nk16) enter P V with p = 0: they must be finite
    for (int e = tid; e < (nk16 - nk) * hd / 2; e += kAttnThreads)
      *reinterpret_cast<__half2 *>(Vs + (size_t)nk * hd + 2 * e) = __floats2half2_rn(0.f, 0.f);
    const float isq = 1.0f / sqrtf((float)hd);
    for (int mt = warp; mt < nk16 / 16; mt += kAttnThreads / 32) {
      float D[NT][4] = {};
      const int row = 16 * mt + (lane & 7) + 8 * ((lane >> 3) & 1);
      const int key = kv_col(t0 + row, 0, hd) >> 3;
      for (int ks = 0; ks < hd / 16; ++ks) {
        uint32_t av[4];
        ldsm_x4(av, smem_u32(Ks + (size_t)row * hd + (((2 * ks + (lane >> 4)) ^ key) << 3)));
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          // tile t, column g: row 8 t + g of qh (W = 4: plane g / 4, head g % 4)
          const __half *qp = qh + (8 * t + g) * qs_ + 2 * c + 16 * ks;
          mma_16816(D[t], av[0], av[1], av[2], av[3], *reinterpret_cast<const uint32_t *>(qp),
                    *reinterpret_cast<const uint32_t *>(qp + 8), D[t]);
        }
      }
      float S[4];
#pragma unroll
      for (int i2 = 0; i2 < 4; ++i2)  // hi + lo
        S[i2] = NT == 2 ? D[0][i2] + D[NT - 1][i2]
                        : D[0][i2] + __shfl_xor_sync(0xffffffffu, D[0][i2], 2);
      if (NT == 2 || c < 2) {
        const int ra = 16 * mt + g, rb = ra + 8;
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j2 = 2 * c + jj;
          if (j2 < grp) {
            sc[j2 * cap + ra] = ra < nk ? S[jj] * isq : -INFINITY;  // forward.rs:396
            sc[j2 * cap + rb] = rb < nk ? S[2 + jj] * isq : -INFINITY;
          }
        }
      }
    }
    __syncthreads();
    for (int j2 = warp; j2 < W; j2 += kAttnThreads / 32) {
      // softmax statistics of this split (head j2); p as hi/lo planes
      float m = -INFINITY;
      if (j2 < grp)
        for (int t = lane; t < nk; t += 32) m = fmaxf(m, sc[j2 * cap + t]);
      m = warp_max(m);
      float l = 0.f;
      for (int t = lane; t < nk16; t += 32) {
        const float p = (j2 < grp && t < nk) ? expf(sc[j2 * cap + t] - m) : 0.f;
        const __half hp = __float2half_rn(p);
        ph[j2 * ps_ + t] = hp;
        ph[(W + j2) * ps_ + t] = __float2half_rn(p - __half2float(hp));
        l += p;
      }
      l = warp_sum(l);
      if (lane == 0 && j2 < grp) {
        s_m[j2] = m;
        s_l[j2] = l;
      }
    }
    __syncthreads();
    for (int mt = warp; mt < hd / 16; mt += kAttnThreads / 32) {
      float D[NT][4] = {};
      for (int ks = 0; ks < nk16 / 16; ++ks) {
        const int t = 16 * ks + (lane & 7) + 8 * (lane >> 4);
        const int ch = (2 * mt + ((lane >> 3) & 1)) ^ (kv_col(t0 + t, 0, hd) >> 3);
        uint32_t av[4];
        ldsm_x4_t(av, smem_u32(Vs + (size_t)t * hd + (ch << 3)));
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
          const __half *pp = ph + (8 * tt + g) * ps_ + 2 * c + 16 * ks;
          mma_16816(D[tt], av[0], av[1], av[2], av[3], *reinterpret_cast<const uint32_t *>(pp),
                    *reinterpret_cast<const uint32_t *>(pp + 8), D[tt]);
        }
      }
      float O[4];
#pragma unroll
      for (int i2 = 0; i2 < 4; ++i2)
        O[i2] = NT == 2 ? D[0][i2] + D[NT - 1][i2]
                        : D[0][i2] + __shfl_xor_sync(0xffffffffu, D[0][i2], 2);
      if (NT == 2 || c < 2) {
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j2 = 2 * c + jj;
          if (j2 < grp) {
            po[j2 * hd + 16 * mt + g] = O[jj];
            po[j2 * hd + 16 * mt + g + 8] = O[2 + jj];
          }
        }
      }
    }
  } else {
  // scores: one thread per (head j, position t); the 16-byte K chunks are
  // visited in a rotated order so neighbouring threads hit different banks
  const float sq = sqrtf((float)hd);
  const int nch = hd / 8;
  for (int e = tid; e < grp * nk; e += kAttnThreads) {
    const int j = e / nk, t = e % nk;
    const uint4 *kr = reinterpret_cast<const uint4 *>(Ks + (size_t)t * hd);
    const float *qj = qs + j * hd;
    float acc = 0.f;
    const int key = kv_col(t0 + t, 0, hd) >> 3;  // chunk permutation of this cache row
    for (int cc = 0; cc < nch; ++cc) {
      const int c8 = (cc + t) % nch;
      const uint4 kv = kr[c8 ^ key];
      const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(&kw[u]));
        acc = fmaf(qj[c8 * 8 + 2 * u], kf.x, acc);
        acc = fmaf(qj[c8 * 8 + 2 * u + 1], kf.y, acc);
      }
    }
    sc[j * cap + t] = acc / sq;  // forward.rs:396
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  // per-head softmax statistics over this chunk
  for (int j = warp; j < grp; j += kAttnThreads / 32) {
    float m = -INFINITY;
    for (int t = lane; t < nk; t += 32) m = fmaxf(m, sc[j * cap + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < nk; t += 32) {
      const float p = (nk > 0) ? expf(sc[j * cap + t] - m) : 0.f;
      sc[j * cap + t] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      s_m[j] = m;
      s_l[j] = l;
    }
  }
  __syncthreads();
  for (int e = tid; e < grp * hd; e += kAttnThreads) {
    const int j = e / hd, d = e % hd;
    float o = 0.f;
    for (int t = 0; t < nk; ++t)
      o = fmaf(sc[j * cap + t], __half2float(Vs[(size_t)t * hd + kv_col(t0 + t, d, hd)]), o);
    po[e] = o;
  }
  }
  if (tid < grp) part_ml[(h * NS + s) * grp + tid] = make_float2(s_m[tid], s_l[tid]);
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&counters[h], 1);
    s_last = (prev == NS - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  attn_combine(part_o, part_ml, attn_out, counters, h, NS, grp, hd, tid, kAttnThreads);
}

// ------------------------------------------------------ decode, small heads --
// Head sizes that are not a multiple of 8 (the reference's own test fixtures
// use 4-wide heads): one CTA per (kv head, sequence) with plain loads of
// every cached row and an exact softmax over the whole context, in the
// reference's order (forward.rs:379-414): scores q.k / sqrt(d), max, exp,
// sum, then the weighted sum of V divided by the sum.
__global__ void __launch_bounds__(128) decode_attn_small_kernel(const __grid_constant__ DecodeAttnArgs a) {
  extern __shared__ float sml[];  // q [grp][hd] | scores [max_seq]
  __shared__ float red[4], s_val;
  const int h = blockIdx.x, b = blockIdx.z, tid = threadIdx.x;
  const int grp = a.H / a.G, hd = a.hd;
  const float *qkv = a.qkv + (size_t)b * a.qkv_stride;
  const int sq = a.slot ? a.slot[b] : b;
  float *attn_out = a.attn_out + (size_t)b * a.H * hd;
  auto row_off = [&](int t) -> size_t {
    if (a.page_table) {
      const int pg = a.page_table[(size_t)sq * a.max_pages + t / a.page_rows];
      return (size_t)pg * a.page_stride + ((size_t)h * a.page_rows + t % a.page_rows) * hd;
    }
    return (size_t)sq * a.kv_seq_stride + ((size_t)h * a.max_seq + t) * hd;
  };
  pdl_wait();
  pdl_launch();
  if (a.zero_ptr && b == 0)
    for (int i = h * 128 + tid; i < a.zero_n; i += a.G * 128) a.zero_ptr[i] = 0.f;
  const int pos = a.pos[sq], len = pos + 1;
  const int rpos = a.rope_compat ? 0 : pos;
  float *qs = sml, *sc = sml + grp * hd;
  const float *q = qkv + (size_t)h * grp * hd;
  for (int e = tid; e < grp * hd / 2; e += 128) {
    const int j = e / (hd / 2), i = 2 * (e % (hd / 2));
    float x0 = q[j * hd + i], x1 = q[j * hd + i + 1];
    if (i < a.rope_dim) rope_pair(x0, x1, i, a.rope_dim, a.rope_base, rpos);
    qs[j * hd + i] = x0;
    qs[j * hd + i + 1] = x1;
  }
  {  // append this token's K/V (forward.rs:375-378), K rotated like q
    const float *kn = qkv + (size_t)a.H * hd + (size_t)h * hd;
    const float *vn = qkv + (size_t)(a.H + a.G) * hd + (size_t)h * hd;
    const size_t off = row_off(pos);
    for (int e = tid; e < hd / 2; e += 128) {
      const int i = 2 * e;
      float x0 = kn[i], x1 = kn[i + 1];
      if (i < a.rope_dim) rope_pair(x0, x1, i, a.rope_dim, a.rope_base, rpos);
      const int ip = kv_col(pos, i, hd);
      a.kc[off + ip] = __float2half_rn(x0);
      a.kc[off + ip + 1] = __float2half_rn(x1);
      a.vc[off + ip] = __float2half_rn(vn[i]);
      a.vc[off + ip + 1] = __float2half_rn(vn[i + 1]);
    }
  }
  __syncthreads();
  const float sqd = sqrtf((float)hd);
  auto block_reduce = [&](float v, bool is_max) -> float {
    for (int o = 16; o; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, w) : v + w;
    }
    if ((tid & 31) == 0) red[tid >> 5] = v;
    __syncthreads();
    if (tid == 0) {
      float r = red[0];
      for (int i = 1; i < 4; ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
      s_val = r;
    }
    __syncthreads();
    const float r = s_val;
    __syncthreads();
    return r;
  };
  for (int j = 0; j < grp; ++j) {
    float mx = -INFINITY;
    for (int t = tid; t < len; t += 128) {
      const __half *kr = a.kc + row_off(t);
      float acc = 0.f;
      for (int d = 0; d < hd; ++d) acc = fmaf(qs[j * hd + d], __half2float(kr[kv_col(t, d, hd)]), acc);
      sc[t] = acc / sqd;  // forward.rs:396
      mx = fmaxf(mx, sc[t]);
    }
    mx = block_reduce(mx, true);
    float sum = 0.f;
    for (int t = tid; t < len; t += 128) {
      const float p = expf(sc[t] - mx);
      sc[t] = p;
      sum += p;
    }
    sum = block_reduce(sum, false);  // also orders the score writes before the reads below
    for (int d = tid; d < hd; d += 128) {
      float o = 0.f;
      for (int t = 0; t < len; ++t) o = fmaf(sc[t], __half2float(a.vc[row_off(t) + kv_col(t, d, hd)]), o);
      attn_out[(size_t)(h * grp + j) * hd + d] = o / sum;
    }
    __syncthreads();  // sc is reused by the next head
  }
}

// ------------------------------------------------------ decode, streamed --
// Split-K decode attention for head sizes 64 and 128 with at most eight
// query heads per kv head, written for many cached rows per CTA (the batched
// step, long contexts). A split covers consecutive 16-row tiles of one
// sequence's kv head; warp w of the CTA takes tiles w, w + 4, ... and keeps
// its own online softmax (flash decoding), so no CTA-wide barrier sits in
// the loop. Each warp double-buffers its tiles: lane 0 bulk-copies tile
// i + 2 while the warp computes tile i.
//
// Per tile, on tensor cores (mma.m16n8k16, f16 in, f32 accumulate):
//   S^T = Q K^T  with Q as the A operand, rows 0-7 the hi f16 planes of the
//                query heads and rows 8-15 their lo planes (about 22 bits;
//                rows beyond the group are zero), K^T from ldmatrix on the
//                chunk-swizzled cache rows; lane (g, c) ends with head g's
//                hi and lo scores of positions 8 nt + 2c (+1), added in-lane;
//   O += P V     with P re-used from the score registers as the A operand
//                (rows 0-7 hi planes, 8-15 lo planes of the probabilities)
//                and V from ldmatrix.trans; the hi and lo halves of O are
//                added at the end.
// The four warps' (m, l, O) are merged through shared memory into the
// split's partial, and the CTA that finishes a kv head's last split combines
// the partials (the same format and combine as decode_attn_kernel).
constexpr int kFlashWarps = 4;
constexpr int kFlashRows = 16;  // cache rows per tile

template <int HD, int WARPS>
__host__ __device__ constexpr int flash_smem_bytes() {
  // stages [warp][2][K tile | V tile] halves, Q [16][HD + 8] halves, 2 mbarriers per warp
  return WARPS * 2 * 2 * kFlashRows * HD * 2 + 16 * (HD + 8) * 2 + WARPS * 2 * 8;
}

template <int HD, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, WARPS == 4 ? 3 : 1)
    decode_attn_flash_kernel(const __grid_constant__ DecodeAttnArgs a) {
  constexpr int KSTEPS = HD / 16, NDT = HD / 8, TH = kFlashRows * HD, QS = HD + 8;
  extern __shared__ __align__(128) uint8_t smraw[];
  __half *stage = reinterpret_cast<__half *>(smraw);  // [warp][2][2][TH]
  __half *qsm = stage + WARPS * 2 * 2 * TH;      // [16][QS]
  uint64_t *bars = reinterpret_cast<uint64_t *>(qsm + 16 * QS);  // [warp][2]
  __shared__ float s_m[WARPS][kMaxGroup], s_l[WARPS][kMaxGroup];
  __shared__ int s_last;
  const int h = blockIdx.x, s = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int grp = a.H / a.G, NS = a.ns;
  const float *qkv = a.qkv + (size_t)b * a.qkv_stride;
  const int sq = a.slot ? a.slot[b] : b;
  float *part_o = a.part_o + (size_t)b * a.G * NS * grp * HD;
  float2 *part_ml = a.part_ml + (size_t)b * a.G * NS * grp;
  int *counters = a.counters + (size_t)b * a.G;
  float *attn_out = a.attn_out + (size_t)b * a.H * HD;

  // cache row t of this sequence's kv head h (paged: a page holds page_rows
  // rows of every layer and kv head; a 16-row tile never straddles pages)
  auto row_off = [&](int t) -> size_t {
    if (a.page_table) {
      const int pg = a.page_table[(size_t)sq * a.max_pages + t / a.page_rows];
      return (size_t)pg * a.page_stride + ((size_t)h * a.page_rows + t % a.page_rows) * HD;
    }
    return (size_t)sq * a.kv_seq_stride + ((size_t)h * a.max_seq + t) * HD;
  };

  // tiles of this split (the sequence's rows 0..pos, pos the new token)
  const int pos = a.pos[sq];
  const int ntile = (pos + 1 + kFlashRows - 1) / kFlashRows;
  const int per = (ntile + NS - 1) / NS;
  const int tb = min(ntile, s * per), te = min(ntile, tb + per);
  __half *myst = stage + (size_t)warp * 2 * 2 * TH;
  uint64_t *mybar = bars + warp * 2;
  // rows of tile T that come from the cache (those before pos)
  uint32_t iss[2] = {0u, 0u}, done[2] = {0u, 0u};  // lane 0: copies issued / waited per stage
  // off: row_off of the tile's first row (read ahead: a paged cache costs a
  // page-table load)
  auto issue = [&](int T, int st, size_t off) {
    ++iss[st];
    const int t0 = T * kFlashRows;
    const int nold = max(0, min(t0 + kFlashRows, pos) - t0);
    __half *dk = myst + (size_t)st * 2 * TH;
    if (nold > 0) {
      mbar_arrive_expect_tx(&mybar[st], 2u * (uint32_t)nold * HD * 2u);
      bulk_g2s(dk, a.kc + off, (uint32_t)nold * HD * 2u, &mybar[st]);
      bulk_g2s(dk + TH, a.vc + off, (uint32_t)nold * HD * 2u, &mybar[st]);
    } else {
      mbar_arrive(&mybar[st]);
    }
  };
  if (lane == 0) {
    mbar_init(&mybar[0], 1);
    mbar_init(&mybar[1], 1);
    fence_mbar_init();
    // the cached rows were written by kernels that completed before the
    // previous kernel in the stream began its main phase
    if (tb + warp < te) issue(tb + warp, 0, row_off((tb + warp) * kFlashRows));
    if (tb + warp + WARPS < te)
      issue(tb + warp + WARPS, 1, row_off((tb + warp + WARPS) * kFlashRows));
  }

  pdl_wait();
  pdl_launch();

  if (a.zero_ptr && b == 0) {
    const int nb = a.G * NS, bi = h * NS + s;
    for (int i = bi * blockDim.x + tid; i < a.zero_n; i += nb * blockDim.x) a.zero_ptr[i] = 0.f;
  }
  // the query heads of this kv head, rotated, as hi / lo f16 rows of Q
  const int rpos = a.rope_compat ? 0 : pos;
  {
    const float *q = qkv + (size_t)h * grp * HD;
    for (int e = tid; e < 8 * HD / 2; e += WARPS * 32) {
      const int j = e / (HD / 2), i = 2 * (e % (HD / 2));
      float x0 = 0.f, x1 = 0.f;
      if (j < grp) {
        x0 = q[j * HD + i];
        x1 = q[j * HD + i + 1];
        if (i < a.rope_dim) rope_pair(x0, x1, i, a.rope_dim, a.rope_base, rpos);
      }
      const __half2 hi = __floats2half2_rn(x0, x1);
      *reinterpret_cast<__half2 *>(qsm + j * QS + i) = hi;
      *reinterpret_cast<__half2 *>(qsm + (8 + j) * QS + i) =
          __floats2half2_rn(x0 - __low2float(hi), x1 - __high2float(hi));
    }
  }
  __syncthreads();
  uint32_t qa[KSTEPS][4];
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks)
    ldsm_x4(qa[ks], smem_u32(qsm + (lane & 15) * QS + ks * 16 + (lane >> 4) * 8));

  float o[NDT][4];
#pragma unroll
  for (int i = 0; i < NDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const float isq = 1.0f / sqrtf((float)HD);
  // ldmatrix row addresses of this lane: K (non-trans) and V (trans)
  const int krow = (lane & 7) + 8 * (lane >> 4), kch = (lane >> 3) & 1;
  const int vrow = (lane & 7) + 8 * ((lane >> 3) & 1), vch = lane >> 4;
  bool ok = true;
  for (int i = 0;; ++i) {
    const int T = tb + warp + WARPS * i;
    if (T >= te) break;
    const int st = i & 1;
    // the cache offset of the tile this stage takes next, loaded before the wait
    const bool more = T + 2 * WARPS < te;
    const size_t next_off = (lane == 0 && more) ? row_off((T + 2 * WARPS) * kFlashRows) : 0;
    ok = __all_sync(0xffffffffu, mbar_wait(&mybar[st], (uint32_t)(i >> 1) & 1u, a.err, 306));
    if (!ok) break;  // the error flag is set; the host reports a timeout
    ++done[st];
    __half *Ks = myst + (size_t)st * 2 * TH, *Vs = Ks + TH;
    const int t0 = T * kFlashRows;
    if (pos < t0 + kFlashRows) {
      // the last tile: append this token's K/V (forward.rs:375-378), K
      // rotated like q, into the cache and this tile; rows beyond it zero
      const int r = pos - t0;
      const float *kn = qkv + (size_t)a.H * HD + (size_t)h * HD;
      const float *vn = qkv + (size_t)(a.H + a.G) * HD + (size_t)h * HD;
      const size_t off = row_off(pos);
      for (int e = lane; e < HD / 2; e += 32) {
        const int ii = 2 * e;
        float x0 = kn[ii], x1 = kn[ii + 1];
        if (ii < a.rope_dim) rope_pair(x0, x1, ii, a.rope_dim, a.rope_base, rpos);
        const __half2 kh = __floats2half2_rn(x0, x1), vh = __floats2half2_rn(vn[ii], vn[ii + 1]);
        const int ip = kv_col(pos, ii, HD);
        *reinterpret_cast<__half2 *>(a.kc + off + ip) = kh;
        *reinterpret_cast<__half2 *>(a.vc + off + ip) = vh;
        *reinterpret_cast<__half2 *>(Ks + r * HD + ip) = kh;
        *reinterpret_cast<__half2 *>(Vs + r * HD + ip) = vh;
      }
      for (int e = lane; e < (kFlashRows - 1 - r) * HD / 2; e += 32) {
        reinterpret_cast<__half2 *>(Ks + (r + 1) * HD)[e] = __floats2half2_rn(0.f, 0.f);
        reinterpret_cast<__half2 *>(Vs + (r + 1) * HD)[e] = __floats2half2_rn(0.f, 0.f);
      }
      __syncwarp();
    }
    // S^T = Q K^T over the tile's 16 rows (two 8-position n-tiles)
    float sacc[2][4] = {};
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      uint32_t kb[4];
      ldsm_x4(kb, smem_u32(Ks + krow * HD + (((2 * ks + kch) ^ (krow & 7)) << 3)));
      mma_16816(sacc[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[0], kb[1], sacc[0]);
      mma_16816(sacc[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[2], kb[3], sacc[1]);
    }
    float sv[2][2];
    float mt = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int t = t0 + 8 * nt + 2 * c + j;
        sv[nt][j] = t <= pos ? (sacc[nt][j] + sacc[nt][2 + j]) * isq : -INFINITY;  // forward.rs:396
        mt = fmaxf(mt, sv[nt][j]);
      }
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float m_new = fmaxf(m_run, mt);  // finite: row t0 <= pos is in every tile
    const float alpha = expf(m_run - m_new);
    m_run = m_new;
    uint32_t pa[4];
    float psum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const float p0 = expf(sv[nt][0] - m_new), p1 = expf(sv[nt][1] - m_new);
      psum += p0 + p1;
      const __half2 hp = __floats2half2_rn(p0, p1);
      const __half2 lp = __floats2half2_rn(p0 - __low2float(hp), p1 - __high2float(hp));
      pa[2 * nt] = *reinterpret_cast<const uint32_t *>(&hp);
      pa[2 * nt + 1] = *reinterpret_cast<const uint32_t *>(&lp);
    }
    l_run = l_run * alpha + psum;
#pragma unroll
    for (int nd = 0; nd < NDT; ++nd) {
      o[nd][0] *= alpha;
      o[nd][1] *= alpha;
      o[nd][2] *= alpha;
      o[nd][3] *= alpha;
    }
    // O += P V: B = V (k = position, n = dimension) from ldmatrix.trans
#pragma unroll
    for (int nd = 0; nd < NDT; nd += 2) {
      uint32_t vb[4];
      ldsm_x4_t(vb, smem_u32(Vs + vrow * HD + (((nd + vch) ^ (vrow & 7)) << 3)));
      mma_16816(o[nd], pa[0], pa[1], pa[2], pa[3], vb[0], vb[1], o[nd]);
      mma_16816(o[nd + 1], pa[0], pa[1], pa[2], pa[3], vb[2], vb[3], o[nd + 1]);
    }
    __syncwarp();  // every lane has read this stage
    if (lane == 0 && more) issue(T + 2 * WARPS, st, next_off);
  }
  // leave no copy in flight after an early exit: wait (bounded) for the
  // stages this warp issued but did not consume
  if (lane == 0)
    for (int i = 0; i < 2; ++i)
      if (iss[i] > done[i]) mbar_wait(&mybar[i], (iss[i] - 1u) & 1u, nullptr, 0);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  __syncthreads();  // every warp is done with its stages: reuse them
  float *mo = reinterpret_cast<float *>(stage);  // [warp][8][HD]
  if (g < grp) {
#pragma unroll
    for (int nd = 0; nd < NDT; ++nd) {
      float *dst = mo + ((size_t)warp * 8 + g) * HD + 8 * nd + 2 * c;
      dst[0] = o[nd][0] + o[nd][2];
      dst[1] = o[nd][1] + o[nd][3];
    }
    if (c == 0) {
      s_m[warp][g] = m_run;
      s_l[warp][g] = l_run;
    }
  }
  __syncthreads();
  if (NS == 1) {  // one split: the merged warps are the whole softmax
    for (int e = tid; e < grp * HD; e += WARPS * 32) {
      const int j = e / HD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_m[w][j]);
      float O = 0.f, Lw = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w)
        if (s_m[w][j] != -INFINITY) {
          const float f = expf(s_m[w][j] - M);
          O = fmaf(f, mo[((size_t)w * 8 + j) * HD + (e % HD)], O);
          Lw = fmaf(s_l[w][j], f, Lw);
        }
      attn_out[(size_t)h * grp * HD + e] = O / Lw;
    }
    return;
  }
  float *po = part_o + (size_t)(h * NS + s) * grp * HD;
  for (int e = tid; e < grp * HD; e += WARPS * 32) {
    const int j = e / HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_m[w][j]);
    float O = 0.f;
    if (M != -INFINITY)
#pragma unroll
      for (int w = 0; w < WARPS; ++w)
        if (s_m[w][j] != -INFINITY) O = fmaf(expf(s_m[w][j] - M), mo[((size_t)w * 8 + j) * HD + (e % HD)], O);
    po[e] = O;
  }
  if (tid < grp) {
    float M = -INFINITY, L = 0.f;
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_m[w][tid]);
    if (M != -INFINITY)
      for (int w = 0; w < WARPS; ++w)
        if (s_m[w][tid] != -INFINITY) L = fmaf(s_l[w][tid], expf(s_m[w][tid] - M), L);
    part_ml[(h * NS + s) * grp + tid] = make_float2(M, L);  // l = 0 marks an empty split
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&counters[h], 1) == NS - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  attn_combine(part_o, part_ml, attn_out, counters, h, NS, grp, HD, tid, WARPS * 32);
}

// ------------------------------------------------------------ prefill ----
constexpr int kPQ = 32;  // query rows per CTA
constexpr int kPK = 32;  // keys per tile

__global__ void __launch_bounds__(128) prefill_attn_kernel(PrefillAttnArgs a) {
  extern __shared__ float sm[];
  const int hq = blockIdx.x, qb = blockIdx.y, tid = threadIdx.x;
  const int hd = a.hd, grp = a.H / a.G, hk = hq / grp;
  const int r0 = qb * kPQ;
  const int nq = min(kPQ, a.n - r0);
  float *Qs = sm;                    // [kPQ][hd]
  float *Ks = Qs + kPQ * hd;         // [kPK][hd+1]
  float *Vs = Ks + kPK * (hd + 1);   // [kPK][hd]
  float *S = Vs + kPK * hd;          // [kPQ][kPK]
  float *mrow = S + kPQ * kPK;       // [kPQ]
  float *lrow = mrow + kPQ;          // [kPQ]
  float *alpha = lrow + kPQ;         // [kPQ]
  const int qstride = a.H * hd, kstride = a.G * hd;
  for (int e = tid; e < kPQ * hd; e += 128) {
    const int r = e / hd, d = e % hd;
    Qs[e] = (r < nq) ? a.q[(size_t)(r0 + r) * qstride + hq * hd + d] : 0.f;
  }
  if (tid < kPQ) {
    mrow[tid] = -INFINITY;
    lrow[tid] = 0.f;
  }
  // each thread owns output elements e = tid + 128*i of [kPQ][hd]
  constexpr int kMaxOut = kPQ * 128 / 128;
  float acc[kMaxOut];
  const int nout = kPQ * hd / 128;
#pragma unroll
  for (int i = 0; i < kMaxOut; ++i) acc[i] = 0.f;
  const float sq = sqrtf((float)hd);
  const int kend = a.causal ? r0 + nq : a.n;  // causal: keys 0..r0+nq-1
  __syncthreads();
  for (int k0 = 0; k0 < kend; k0 += kPK) {
    const int nk = min(kPK, kend - k0);
    for (int e = tid; e < kPK * hd; e += 128) {
      const int t = e / hd, d = e % hd;
      const bool ok = t < nk;
      Ks[t * (hd + 1) + d] = ok ? a.k[(size_t)(k0 + t) * kstride + hk * hd + d] : 0.f;
      Vs[t * hd + d] = ok ? a.v[(size_t)(k0 + t) * kstride + hk * hd + d] : 0.f;
    }
    __syncthreads();
    for (int e = tid; e < kPQ * kPK; e += 128) {
      const int r = e / kPK, t = e % kPK;
      float sc = -INFINITY;
      if (t < nk && r < nq && (!a.causal || k0 + t <= r0 + r)) {  // causal mask, forward.rs:266-271
        float s = 0.f;
        for (int d = 0; d < hd; ++d) s = fmaf(Qs[r * hd + d], Ks[t * (hd + 1) + d], s);
        sc = s / sq;
      }
      S[e] = sc;
    }
    __syncthreads();
    if (tid < kPQ) {
      const int r = tid;
      float m = mrow[r];
      float mt = -INFINITY;
      for (int t = 0; t < kPK; ++t) mt = fmaxf(mt, S[r * kPK + t]);
      const float mn = fmaxf(m, mt);
      const float al = (mn == -INFINITY) ? 1.f : expf(m - mn);
      float l = lrow[r] * al;
      for (int t = 0; t < kPK; ++t) {
        const float p = (S[r * kPK + t] == -INFINITY) ? 0.f : expf(S[r * kPK + t] - mn);
        S[r * kPK + t] = p;
        l += p;
      }
      mrow[r] = mn;
      lrow[r] = l;
      alpha[r] = al;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxOut; ++i) {
      if (i < nout) {
        const int e = tid + 128 * i, r = e / hd, d = e % hd;
        float o = acc[i] * alpha[r];
        for (int t = 0; t < nk; ++t) o = fmaf(S[r * kPK + t], Vs[t * hd + d], o);
        acc[i] = o;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < kMaxOut; ++i) {
    if (i < nout) {
      const int e = tid + 128 * i, r = e / hd, d = e % hd;
      if (r < nq) a.out[(size_t)(r0 + r) * qstride + hq * hd + d] = acc[i] / lrow[r];
    }
  }
}

}  // namespace

// head slots per plane of the tensor-core items (4 or 8), 0 for the FMA loops
static int attn_tc_slots(int grp, int hd) {
  if (hd % 64 || hd > 256 || grp > 8) return 0;
  return grp <= 4 ? 4 : 8;
}

int decode_attention_smem(int grp, int hd, int max_seq, int ns) {
  const int cap = attn_rows(max_seq, ns), W = attn_tc_slots(grp, hd);
  if (W) return 2 * cap * hd * 2 + 2 * W * (hd + 8) * 2 + W * cap * 4 + 2 * W * (cap + 8) * 2;
  return 2 * cap * hd * 2 + (grp * hd + grp * cap) * (int)sizeof(float);
}

template <int HD, int WARPS>
static ifx_status launch_flash_w(const DecodeAttnArgs &f, cudaStream_t st, bool pdl) {
  constexpr int smem = flash_smem_bytes<HD, WARPS>();
  static bool attr = false;
  if (!attr) {
    IFX_CUDA(cudaFuncSetAttribute(decode_attn_flash_kernel<HD, WARPS>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr = true;
  }
  IFX_CUDA(launch(decode_attn_flash_kernel<HD, WARPS>, dim3(f.G, f.ns, f.batch), dim3(WARPS * 32),
                  (size_t)smem, st, pdl, f));
  return IFX_OK;
}

template <int HD>
static ifx_status launch_flash(const DecodeAttnArgs &a, cudaStream_t st, bool pdl) {
  // Many (sequence, kv head) pairs (a batch): one 8-warp CTA per pair and
  // SM, each streaming the whole context (no split combine). Few pairs:
  // 4-warp CTAs, about three per SM, the context split among them (at
  // least two tiles per warp) and no more splits than the caller's
  // partial buffers hold.
  DecodeAttnArgs f = a;
  const int tiles = (a.max_seq + kFlashRows - 1) / kFlashRows;
  const int pairs = std::max(1, a.G * a.batch);
  if (pairs >= kNumSMs / 2 && tiles >= 32) {
    f.ns = std::max(1, std::min({a.ns, kNumSMs / pairs, tiles / 32}));
    return launch_flash_w<HD, 8>(f, st, pdl);
  }
  const int want = std::max(1, 3 * kNumSMs / pairs);
  f.ns = std::max(1, std::min({a.ns, want, kMaxSplits, (tiles + 2 * kFlashWarps - 1) / (2 * kFlashWarps)}));
  return launch_flash_w<HD, kFlashWarps>(f, st, pdl);
}

ifx_status decode_attention(const DecodeAttnArgs &a, cudaStream_t st, bool pdl) {
  const int grp = a.H / a.G;
  if (a.G < 1 || a.H % a.G || grp > kMaxGroup || a.ns < 1)
    return fail(IFX_ERR_UNSUPPORTED, "attention shape");
  // the streamed kernel for the tensor-core head sizes (any number of
  // pages: its splits are its own, at most the caller's)
  if (a.hd == 128) return launch_flash<128>(a, st, pdl);
  if (a.hd == 64) return launch_flash<64>(a, st, pdl);
  if (a.hd % 8 && a.hd % 2 == 0) {  // narrow heads: one CTA per kv head and sequence
    const size_t smem = (size_t)(grp * a.hd + a.max_seq) * sizeof(float);
    if (smem > 200 * 1024) return fail(IFX_ERR_UNSUPPORTED, "attention: context too long for small heads");
    static size_t attr = 0;
    if (smem > 48 * 1024 && smem > attr) {
      IFX_CUDA(cudaFuncSetAttribute(decode_attn_small_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      attr = smem;
    }
    IFX_CUDA(launch(decode_attn_small_kernel, dim3(a.G, 1, a.batch), dim3(128), smem, st, pdl, a));
    return IFX_OK;
  }
  if (a.hd > 256 || a.hd % 8 || a.ns > kMaxSplits) return fail(IFX_ERR_UNSUPPORTED, "attention shape");
  const size_t smem = (size_t)decode_attention_smem(grp, a.hd, a.max_seq, a.ns);
  if (smem > 200 * 1024) return fail(IFX_ERR_UNSUPPORTED, "attention: KV chunk too large for shared memory");
  const int W = attn_tc_slots(grp, a.hd), k = W / 4;
  void (*const kern[3])(DecodeAttnArgs) = {decode_attn_kernel<0>, decode_attn_kernel<4>,
                                           decode_attn_kernel<8>};
  static size_t attr[3] = {0, 0, 0};
  if (smem > attr[k]) {  // the static arrays count against the 48 KB default too
    IFX_CUDA(cudaFuncSetAttribute(kern[k], cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr[k] = smem;
  }
  IFX_CUDA(launch(kern[k], dim3(a.G, a.ns, a.batch), dim3(kAttnThreads), smem, st, pdl, a));
  return IFX_OK;
}

// Prefill attention on tensor cores (flash-attention style): a CTA takes one
// query head and 64 query rows (4 warps x 16), streams 64-key blocks of K
// and V (f32 from the prefill workspace, converted to f16 into shared
// memory, both row-major with padded rows), computes S = Q K^T with
// mma.m16n8k16 (f16 in, f32 accumulate), applies the causal chunk mask (key
// <= query row, keys of this chunk only: forward.rs:266-274), keeps an online
// softmax per row in registers and accumulates O += P V with P re-used from
// the S fragments and V's B fragments taken with ldmatrix.trans.
constexpr int kTQ = 64;  // query rows per CTA
constexpr int kTK = 64;  // keys per block

__device__ __forceinline__ uint32_t pack_h2(float x, float y) {
  __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t *>(&h);
}

template <int HD>
__global__ void __launch_bounds__(128) prefill_attn_tc_kernel(PrefillAttnArgs a) {
  constexpr int KS = HD + 8;   // K / V row stride (halves): the 8 rows a fragment load
                               // touches fall on distinct banks
  extern __shared__ __align__(16) __half smh[];
  __half *Ks = smh;             // [kTK][KS]
  __half *Vs = smh + kTK * KS;  // [kTK][KS]
  const int hq = blockIdx.x, qb = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int grp = a.H / a.G, hk = hq / grp;
  const int qstride = a.H * HD, kstride = a.G * HD;
  const int r0 = qb * kTQ;
  const int row_a = r0 + warp * 16 + g, row_b = row_a + 8;
  const bool va = row_a < a.n, vb = row_b < a.n;
  // this warp's 16 query rows as A fragments (row-major 16 x HD)
  uint32_t qa[HD / 16][4];
  {
    const float *qra = a.q + (size_t)(va ? row_a : 0) * qstride + hq * HD;
    const float *qrb = a.q + (size_t)(vb ? row_b : 0) * qstride + hq * HD;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      const int d0 = ks * 16 + 2 * c;
      const float2 x0 = va ? *reinterpret_cast<const float2 *>(qra + d0) : make_float2(0.f, 0.f);
      const float2 x1 = vb ? *reinterpret_cast<const float2 *>(qrb + d0) : make_float2(0.f, 0.f);
      const float2 x2 = va ? *reinterpret_cast<const float2 *>(qra + d0 + 8) : make_float2(0.f, 0.f);
      const float2 x3 = vb ? *reinterpret_cast<const float2 *>(qrb + d0 + 8) : make_float2(0.f, 0.f);
      qa[ks][0] = pack_h2(x0.x, x0.y);
      qa[ks][1] = pack_h2(x1.x, x1.y);
      qa[ks][2] = pack_h2(x2.x, x2.y);
      qa[ks][3] = pack_h2(x3.x, x3.y);
    }
  }
  float o[HD / 8][4];
#pragma unroll
  for (int nt = 0; nt < HD / 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  const float scale = 1.0f / sqrtf((float)HD);
  const int kend = a.causal ? min(a.n, r0 + kTQ) : a.n;  // causal: no key beyond the block's last row
  // causal: kb <= r0, so every row has a key in every block; otherwise every
  // block holds keys for every row
  for (int kb = 0; kb < kend; kb += kTK) {
    __syncthreads();  // the previous block's K/V are no longer read
    for (int e = tid; e < kTK * HD / 4; e += 128) {
      const int t = e / (HD / 4), d = (e % (HD / 4)) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (kb + t < a.n) {
        kv = *reinterpret_cast<const float4 *>(a.k + (size_t)(kb + t) * kstride + hk * HD + d);
        vv = *reinterpret_cast<const float4 *>(a.v + (size_t)(kb + t) * kstride + hk * HD + d);
      }
      *reinterpret_cast<uint2 *>(Ks + t * KS + d) = make_uint2(pack_h2(kv.x, kv.y), pack_h2(kv.z, kv.w));
      *reinterpret_cast<uint2 *>(Vs + t * KS + d) = make_uint2(pack_h2(vv.x, vv.y), pack_h2(vv.z, vv.w));
    }
    __syncthreads();
    float sv[kTK / 8][4];
#pragma unroll
    for (int nt = 0; nt < kTK / 8; ++nt) {
      sv[nt][0] = sv[nt][1] = sv[nt][2] = sv[nt][3] = 0.f;
      const __half *kr = Ks + (nt * 8 + g) * KS + 2 * c;
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(kr + ks * 16);
        const uint32_t b1 = *reinterpret_cast<const uint32_t *>(kr + ks * 16 + 8);
        mma_16816(sv[nt], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1, sv[nt]);
      }
    }
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < kTK / 8; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int key = kb + nt * 8 + 2 * c + j;
        const bool kin = key < a.n;
        sv[nt][j] = (kin && (!a.causal || key <= row_a)) ? sv[nt][j] * scale : -INFINITY;
        sv[nt][2 + j] = (kin && (!a.causal || key <= row_b)) ? sv[nt][2 + j] * scale : -INFINITY;
        mx_a = fmaxf(mx_a, sv[nt][j]);
        mx_b = fmaxf(mx_b, sv[nt][2 + j]);
      }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float al_a = mn_a == -INFINITY ? 1.f : expf(m_a - mn_a);
    const float al_b = mn_b == -INFINITY ? 1.f : expf(m_b - mn_b);
    m_a = mn_a;
    m_b = mn_b;
    l_a *= al_a;
    l_b *= al_b;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt) {
      o[nt][0] *= al_a;
      o[nt][1] *= al_a;
      o[nt][2] *= al_b;
      o[nt][3] *= al_b;
    }
#pragma unroll
    for (int nt = 0; nt < kTK / 8; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float pa = sv[nt][j] == -INFINITY ? 0.f : expf(sv[nt][j] - mn_a);
        const float pb = sv[nt][2 + j] == -INFINITY ? 0.f : expf(sv[nt][2 + j] - mn_b);
        sv[nt][j] = pa;
        sv[nt][2 + j] = pb;
        l_a += pa;
        l_b += pb;
      }
#pragma unroll
    for (int k2 = 0; k2 < kTK / 16; ++k2) {
      const uint32_t p0 = pack_h2(sv[2 * k2][0], sv[2 * k2][1]);
      const uint32_t p1 = pack_h2(sv[2 * k2][2], sv[2 * k2][3]);
      const uint32_t p2 = pack_h2(sv[2 * k2 + 1][0], sv[2 * k2 + 1][1]);
      const uint32_t p3 = pack_h2(sv[2 * k2 + 1][2], sv[2 * k2 + 1][3]);
      // B = V[keys 16 k2 .. + 15][dims]: ldmatrix.trans of (keys 0-7 | 8-15) x
      // (dims of n-tiles nt | nt + 1) gives b0, b1 of both n-tiles
      const int vkey = k2 * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
      for (int nt = 0; nt < HD / 8; nt += 2) {
        uint32_t b[4];
        ldsm_x4_t(b, smem_u32(Vs + vkey * KS + (nt + (lane >> 4)) * 8));
        mma_16816(o[nt], p0, p1, p2, p3, b[0], b[1], o[nt]);
        mma_16816(o[nt + 1], p0, p1, p2, p3, b[2], b[3], o[nt + 1]);
      }
    }
  }
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float ia = 1.0f / l_a, ib = 1.0f / l_b;
#pragma unroll
  for (int nt = 0; nt < HD / 8; ++nt) {
    const int d = nt * 8 + 2 * c;
    if (va)
      *reinterpret_cast<float2 *>(a.out + (size_t)row_a * qstride + hq * HD + d) =
          make_float2(o[nt][0] * ia, o[nt][1] * ia);
    if (vb)
      *reinterpret_cast<float2 *>(a.out + (size_t)row_b * qstride + hq * HD + d) =
          make_float2(o[nt][2] * ib, o[nt][3] * ib);
  }
}

// Causal prefill attention streamed from the KV cache: a CTA takes one kv
// head and 16 RT query rows of every one of its query heads (8 warps: warp
// w = head w / RT, row tile w % RT), so each 64-key tile of K and V is
// fetched once for all of them, as f16 rows bulk-copied from the cache the
// chunk was just written to (double-buffered; thread 0 refills a stage
// once all eight warps have released it). Per tile and warp: S = Q K^T
// (mma.m16n8k16, K from ldmatrix on the position-swizzled rows), the causal
// chunk mask (key <= row, forward.rs:266-274), an online softmax in
// registers, O += P V with P re-used from the S fragments and V from
// ldmatrix.trans. Q and P are single f16 planes and accumulation is f32, as
// in prefill_attn_tc_kernel.
constexpr int kPFK = 64;  // keys per tile

template <int HD>
__host__ __device__ constexpr int pflash_smem_bytes() {
  return 2 * 2 * kPFK * HD * 2 + 4 * 8;
}

template <int HD, int RT>
__global__ void __launch_bounds__(256, 1) prefill_attn_flash_kernel(const __grid_constant__ PrefillAttnArgs a) {
  constexpr int KSTEPS = HD / 16, NDT = HD / 8, TH = kPFK * HD;
  extern __shared__ __align__(128) uint8_t smraw[];
  __half *stage = reinterpret_cast<__half *>(smraw);                // [2][K | V][64][HD]
  uint64_t *full = reinterpret_cast<uint64_t *>(stage + 2 * 2 * TH);  // [2]
  uint64_t *empty = full + 2;                                       // [2]
  const int h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int grp = a.H / a.G;
  const int j = warp / RT, rt = warp % RT;   // query head (within the group), row tile
  const bool active = j < grp;
  const int hq = h * grp + (active ? j : 0);
  const int r0 = blockIdx.y * 16 * RT;        // the CTA's first query row
  const int row_a = r0 + rt * 16 + g, row_b = row_a + 8;
  const int qstride = a.H * HD;
  const int kend = min(a.n, r0 + 16 * RT);    // keys this CTA needs (causal)
  const int ntile = (kend + kPFK - 1) / kPFK;
  auto row_off = [&](int p) -> size_t {       // absolute position p of this kv head
    if (a.page_table)
      return (size_t)a.page_table[p / a.page_rows] * a.page_stride +
             ((size_t)h * a.page_rows + p % a.page_rows) * HD;
    return ((size_t)h * a.max_seq + p) * HD;
  };
  // tile i: keys [64 i, min(64 i + 64, kend)), positions start + key; a
  // paged tile splits where a page ends
  auto issue = [&](int i) {
    const int st = i & 1, k0 = i * kPFK, nk = min(kPFK, kend - k0);
    __half *dk = stage + (size_t)st * 2 * TH;
    mbar_arrive_expect_tx(&full[st], 2u * (uint32_t)nk * HD * 2u);
    int r = 0;
    while (r < nk) {
      const int p = a.start + k0 + r;
      int run = nk - r;
      if (a.page_table) run = min(run, a.page_rows - p % a.page_rows);
      const size_t off = row_off(p);
      bulk_g2s(dk + (size_t)r * HD, a.kc + off, (uint32_t)run * HD * 2u, &full[st]);
      bulk_g2s(dk + TH + (size_t)r * HD, a.vc + off, (uint32_t)run * HD * 2u, &full[st]);
      r += run;
    }
  };
  // Rows of a short last tile are never copied: start every stage at zero so
  // such a row holds zeros or an earlier tile's finite values (its P is 0,
  // and 0 times a NaN pattern would not be). The bulk copies write after the
  // proxy fence.
  for (int e = tid; e < 2 * 2 * TH / 8; e += 256) reinterpret_cast<uint4 *>(stage)[e] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  int issued = 0;  // thread 0: tiles issued
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    fence_mbar_init();
    issue(0);
    issued = 1;
    if (ntile > 1) {
      issue(1);
      issued = 2;
    }
  }
  // this warp's 16 query rows as A fragments (single f16 plane)
  uint32_t qa[KSTEPS][4];
  {
    const bool va = active && row_a < a.n, vb = active && row_b < a.n;
    const float *qra = a.q + (size_t)(va ? row_a : 0) * qstride + hq * HD;
    const float *qrb = a.q + (size_t)(vb ? row_b : 0) * qstride + hq * HD;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      const int d0 = ks * 16 + 2 * c;
      const float2 x0 = va ? *reinterpret_cast<const float2 *>(qra + d0) : make_float2(0.f, 0.f);
      const float2 x1 = vb ? *reinterpret_cast<const float2 *>(qrb + d0) : make_float2(0.f, 0.f);
      const float2 x2 = va ? *reinterpret_cast<const float2 *>(qra + d0 + 8) : make_float2(0.f, 0.f);
      const float2 x3 = vb ? *reinterpret_cast<const float2 *>(qrb + d0 + 8) : make_float2(0.f, 0.f);
      qa[ks][0] = pack_h2(x0.x, x0.y);
      qa[ks][1] = pack_h2(x1.x, x1.y);
      qa[ks][2] = pack_h2(x2.x, x2.y);
      qa[ks][3] = pack_h2(x3.x, x3.y);
    }
  }
  __syncthreads();  // the barriers are initialised
  float o[NDT][4];
#pragma unroll
  for (int nt = 0; nt < NDT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  const float scale = 1.0f / sqrtf((float)HD);
  const int krow = (lane & 7) + 8 * (lane >> 4), kch = (lane >> 3) & 1;
  const int vrow = (lane & 7) + 8 * ((lane >> 3) & 1), vch = lane >> 4;
  bool ok = true;
  int waited = 0;
  for (int i = 0; i < ntile; ++i) {
    const int st = i & 1, k0 = i * kPFK;
    ok = __all_sync(0xffffffffu, mbar_wait(&full[st], (uint32_t)(i >> 1) & 1u, a.err, 307));
    if (!ok) break;
    waited = i + 1;
    const __half *Ks = stage + (size_t)st * 2 * TH, *Vs = Ks + TH;
    const int sw = a.start + k0;  // swizzle key of smem row r: (sw + r) & 7
    float sv[kPFK / 8][4];
#pragma unroll
    for (int nt2 = 0; nt2 < kPFK / 16; ++nt2) {  // key n-tiles 2 nt2, 2 nt2 + 1
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
      const int r = 16 * nt2 + krow;
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        uint32_t kb[4];
        ldsm_x4(kb, smem_u32(Ks + r * HD + (((2 * ks + kch) ^ ((sw + r) & 7)) << 3)));
        mma_16816(s0, qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[0], kb[1], s0);
        mma_16816(s1, qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[2], kb[3], s1);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        sv[2 * nt2][e] = s0[e];
        sv[2 * nt2 + 1][e] = s1[e];
      }
    }
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < kPFK / 8; ++nt)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int key = k0 + nt * 8 + 2 * c + jj;
        const bool kin = key < kend;
        sv[nt][jj] = (kin && key <= row_a) ? sv[nt][jj] * scale : -INFINITY;
        sv[nt][2 + jj] = (kin && key <= row_b) ? sv[nt][2 + jj] * scale : -INFINITY;
        mx_a = fmaxf(mx_a, sv[nt][jj]);
        mx_b = fmaxf(mx_b, sv[nt][2 + jj]);
      }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float al_a = mn_a == -INFINITY ? 1.f : expf(m_a - mn_a);
    const float al_b = mn_b == -INFINITY ? 1.f : expf(m_b - mn_b);
    m_a = mn_a;
    m_b = mn_b;
    l_a *= al_a;
    l_b *= al_b;
#pragma unroll
    for (int nt = 0; nt < NDT; ++nt) {
      o[nt][0] *= al_a;
      o[nt][1] *= al_a;
      o[nt][2] *= al_b;
      o[nt][3] *= al_b;
    }
#pragma unroll
    for (int nt = 0; nt < kPFK / 8; ++nt)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const float pa = sv[nt][jj] == -INFINITY ? 0.f : expf(sv[nt][jj] - mn_a);
        const float pb = sv[nt][2 + jj] == -INFINITY ? 0.f : expf(sv[nt][2 + jj] - mn_b);
        sv[nt][jj] = pa;
        sv[nt][2 + jj] = pb;
        l_a += pa;
        l_b += pb;
      }
#pragma unroll
    for (int k2 = 0; k2 < kPFK / 16; ++k2) {
      const uint32_t p0 = pack_h2(sv[2 * k2][0], sv[2 * k2][1]);
      const uint32_t p1 = pack_h2(sv[2 * k2][2], sv[2 * k2][3]);
      const uint32_t p2 = pack_h2(sv[2 * k2 + 1][0], sv[2 * k2 + 1][1]);
      const uint32_t p3 = pack_h2(sv[2 * k2 + 1][2], sv[2 * k2 + 1][3]);
      const int r = 16 * k2 + vrow;
#pragma unroll
      for (int nd = 0; nd < NDT; nd += 2) {
        uint32_t vb[4];
        ldsm_x4_t(vb, smem_u32(Vs + r * HD + (((nd + vch) ^ ((sw + r) & 7)) << 3)));
        mma_16816(o[nd], p0, p1, p2, p3, vb[0], vb[1], o[nd]);
        mma_16816(o[nd + 1], p0, p1, p2, p3, vb[2], vb[3], o[nd + 1]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (tid == 0 && i + 2 < ntile) {  // refill this stage once every warp released it
      if (!mbar_wait(&empty[st], (uint32_t)(i >> 1) & 1u, a.err, 308)) {
        ok = false;
      } else {
        issue(i + 2);
        issued = i + 3;
      }
    }
  }
  // no copy may outlive the CTA: thread 0 waits (bounded) for every issued
  // tile that no warp waited for
  if (tid == 0)
    for (int i = waited; i < issued; ++i) mbar_wait(&full[i & 1], (uint32_t)(i >> 1) & 1u, nullptr, 0);
  if (!active) return;
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float ia = 1.0f / l_a, ib = 1.0f / l_b;
#pragma unroll
  for (int nt = 0; nt < NDT; ++nt) {
    const int d = nt * 8 + 2 * c;
    if (row_a < a.n)
      *reinterpret_cast<float2 *>(a.out + (size_t)row_a * qstride + hq * HD + d) =
          make_float2(o[nt][0] * ia, o[nt][1] * ia);
    if (row_b < a.n)
      *reinterpret_cast<float2 *>(a.out + (size_t)row_b * qstride + hq * HD + d) =
          make_float2(o[nt][2] * ib, o[nt][3] * ib);
  }
}

template <int HD, int RT>
static ifx_status launch_prefill_flash(const PrefillAttnArgs &a, cudaStream_t st) {
  constexpr int smem = pflash_smem_bytes<HD>();
  static bool attr = false;
  if (!attr) {
    IFX_CUDA(cudaFuncSetAttribute(prefill_attn_flash_kernel<HD, RT>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr = true;
  }
  const dim3 grid((unsigned)a.G, (unsigned)((a.n + 16 * RT - 1) / (16 * RT)));
  prefill_attn_flash_kernel<HD, RT><<<grid, 256, smem, st>>>(a);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

template <int HD>
static ifx_status launch_prefill_tc(const PrefillAttnArgs &a, cudaStream_t st) {
  const size_t smem = (size_t)(2 * kTK * (HD + 8)) * sizeof(__half);
  dim3 grid(a.H, (a.n + kTQ - 1) / kTQ);
  prefill_attn_tc_kernel<HD><<<grid, 128, smem, st>>>(a);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status prefill_attention(const PrefillAttnArgs &a, cudaStream_t st) {
  // causal prefill into a cache: the streamed kernel (8 warps = the kv
  // head's query heads x row tiles)
  const int grp = a.G > 0 ? a.H / a.G : 0;
  if (a.kc && a.causal && a.err && (a.hd == 64 || a.hd == 128) && grp > 0 && 8 % grp == 0) {
    const int rt = 8 / grp;
    if (a.hd == 128) {
      if (rt == 1) return launch_prefill_flash<128, 1>(a, st);
      if (rt == 2) return launch_prefill_flash<128, 2>(a, st);
      if (rt == 4) return launch_prefill_flash<128, 4>(a, st);
      return launch_prefill_flash<128, 8>(a, st);
    }
    if (rt == 1) return launch_prefill_flash<64, 1>(a, st);
    if (rt == 2) return launch_prefill_flash<64, 2>(a, st);
    if (rt == 4) return launch_prefill_flash<64, 4>(a, st);
    return launch_prefill_flash<64, 8>(a, st);
  }
  switch (a.hd) {  // tensor-core path for the common head sizes
    case 48: return launch_prefill_tc<48>(a, st);
    case 64: return launch_prefill_tc<64>(a, st);
    case 96: return launch_prefill_tc<96>(a, st);
    case 128: return launch_prefill_tc<128>(a, st);
    default: break;
  }
  if (a.hd > 128 || (kPQ * a.hd) % 128) return fail(IFX_ERR_UNSUPPORTED, "prefill attention head_dim");
  const size_t smem =
      (size_t)(kPQ * a.hd + kPK * (a.hd + 1) + kPK * a.hd + kPQ * kPK + 3 * kPQ) * sizeof(float);
  static bool attr = false;
  if (!attr) {
    IFX_CUDA(cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  100 * 1024));
    attr = true;
  }
  dim3 grid(a.H, (a.n + kPQ - 1) / kPQ);
  prefill_attn_kernel<<<grid, 128, smem, st>>>(a);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

}  // namespace ifx
