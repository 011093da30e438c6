// Op-level kernels: mirrors of src/ops.rs plus argmax and the sampler.
// These back the op-level C ABI used by parity tests; the token loop uses
// the fused kernels (gemv.cu, attention.cu, model.cu) instead.
#include <algorithm>
#include <mutex>
#include <string>

#include "ops.cuh"
#include "quant.cuh"

namespace ifx {

namespace {

inline unsigned nblk(size_t n, int t) { return (unsigned)std::min<size_t>((n + t - 1) / t, 1u << 20); }

__global__ void dequant_kernel(int type, const uint8_t *__restrict__ src, float *__restrict__ out,
                               size_t n) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n;
       e += (size_t)gridDim.x * blockDim.x)
    out[e] = dequant_elem(type, src, e);
}

// C = A B (ops.rs:15-26). One thread per output; k-sequential FMAs in the
// same order as matmul_avx2's per-element accumulation (c += a[i,l]*b[l,j]).
__global__ void matmul_kernel(const float *a, const float *b, float *c, size_t m, size_t n,
                              size_t k) {
  size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (idx >= m * n) return;
  size_t i = idx / n, j = idx % n;
  float acc = 0.f;
  size_t j8 = (n / 8) * 8;
  for (size_t l = 0; l < k; ++l) {
    float p = a[i * k + l];
    if (j < j8) acc = __fmaf_rn(p, b[l * n + j], acc);
    else acc = __fadd_rn(acc, __fmul_rn(p, b[l * n + j]));
  }
  c[idx] = acc;
}

// C = A B^T (ops.rs:33-44). One warp per output: eight lanes accumulate with
// FMA over k = lane mod 8 (the AVX2 lanes of matmul_t_avx2), combined with
// hsum256_ps's order ((l0+l4)+(l1+l5))+((l2+l6)+(l3+l7)), then the scalar
// tail. This reproduces the reference's bits.
__global__ void matmul_t_kernel(const float *a, const float *b, float *c, size_t m, size_t n,
                                size_t k) {
  size_t w = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x & 31;
  if (w >= m * n) return;
  size_t i = w / n, j = w % n;
  const float *ar = a + i * k, *br = b + j * k;
  size_t k8 = (k / 8) * 8;
  float acc = 0.f;
  if (lane < 8)
    for (size_t l = lane; l < k8; l += 8) acc = __fmaf_rn(ar[l], br[l], acc);
  float l0 = __shfl_sync(0xffffffffu, acc, 0), l1 = __shfl_sync(0xffffffffu, acc, 1);
  float l2 = __shfl_sync(0xffffffffu, acc, 2), l3 = __shfl_sync(0xffffffffu, acc, 3);
  float l4 = __shfl_sync(0xffffffffu, acc, 4), l5 = __shfl_sync(0xffffffffu, acc, 5);
  float l6 = __shfl_sync(0xffffffffu, acc, 6), l7 = __shfl_sync(0xffffffffu, acc, 7);
  if (lane == 0) {
    float s = __fadd_rn(__fadd_rn(__fadd_rn(l0, l4), __fadd_rn(l1, l5)),
                        __fadd_rn(__fadd_rn(l2, l6), __fadd_rn(l3, l7)));
    for (size_t l = k8; l < k; ++l) s = __fadd_rn(s, __fmul_rn(ar[l], br[l]));
    c[i * n + j] = s;
  }
}

// rms_norm_rows (ops.rs:155-180): one CTA per row.
__global__ void rms_norm_kernel(float *x, const float *w, float eps, size_t hidden) {
  float *r = x + blockIdx.x * hidden;
  __shared__ float red[32];
  float ss = 0.f;
  for (size_t i = threadIdx.x; i < hidden; i += blockDim.x) ss += r[i] * r[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  float scale = 1.0f / sqrtf(red[0] / (float)hidden + eps);
  for (size_t i = threadIdx.x; i < hidden; i += blockDim.x) r[i] = __fmul_rn(__fmul_rn(r[i], scale), w[i]);
}

__device__ __forceinline__ float sigmoid_ref(float v) {
  v = fminf(fmaxf(v, -80.0f), 80.0f);
  return 1.0f / (1.0f + expf(-v));
}

__global__ void silu_kernel(float *x, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = __fmul_rn(x[i], sigmoid_ref(x[i]));
}

__global__ void swiglu_kernel(const float *g, const float *u, float *o, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    o[i] = __fmul_rn(__fmul_rn(g[i], sigmoid_ref(g[i])), u[i]);
}

__global__ void add_kernel(float *o, const float *b, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    o[i] = __fadd_rn(o[i], b[i]);
}

// softmax_rows (ops.rs:223-239): one CTA per row.
__global__ void softmax_kernel(float *x, size_t cols) {
  float *r = x + blockIdx.x * cols;
  __shared__ float red[32];
  float mx = -INFINITY;
  for (size_t i = threadIdx.x; i < cols; i += blockDim.x) mx = fmaxf(mx, r[i]);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float s = 0.f;
  for (size_t i = threadIdx.x; i < cols; i += blockDim.x) {
    float e = expf(r[i] - mx);
    r[i] = e;
    s += e;
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  s = red[0];
  for (size_t i = threadIdx.x; i < cols; i += blockDim.x) r[i] = r[i] / s;
}

__global__ void embedding_kernel(const float *emb, size_t emb_len, const uint32_t *ids,
                                 size_t hidden, float *out, int *err) {
  size_t p = blockIdx.x;
  size_t src = (size_t)ids[p] * hidden;
  if (src + hidden > emb_len) {
    if (threadIdx.x == 0) atomicExch(err, 1);
    return;
  }
  for (size_t i = threadIdx.x; i < hidden; i += blockDim.x) out[p * hidden + i] = emb[src + i];
}

// rope (ops.rs:265-287): inv = 1/base^(i/rope_dim), angle = pos*inv,
// x0' = x0 cos - x1 sin, x1' = x0 sin + x1 cos.
__global__ void rope_kernel(float *x, size_t seq, size_t heads, size_t hd, size_t rope_dim,
                            float base, size_t pos0) {
  size_t pairs = rope_dim / 2;
  size_t total = seq * heads * pairs;
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < total;
       t += (size_t)gridDim.x * blockDim.x) {
    size_t i = (t % pairs) * 2, rest = t / pairs, h = rest % heads, pos = rest / heads;
    float *v = x + (pos * heads + h) * hd + i;
    float inv = 1.0f / powf(base, (float)i / (float)rope_dim);
    float ang = __fmul_rn((float)(pos + pos0), inv);
    float s, c;
    sincosf(ang, &s, &c);
    float a = v[0], b = v[1];
    v[0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    v[1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  }
}

// Argmax, last index on ties (Iterator::max_by): key = (ordered(v) << 32) | idx,
// the maximum key picks the largest value and, among equals, the largest index.
__global__ void argmax_kernel(const float *x, size_t n, unsigned long long *key) {
  unsigned long long best = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float v = x[i];
    if (v != v) continue;  // the reference panics on NaN; skip it here
    unsigned long long k = ((unsigned long long)ordered_bits(v) << 32) | (unsigned long long)i;
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(key, best);
}

__global__ void key_to_token_kernel(unsigned long long *key, uint32_t *out) {
  *out = (uint32_t)(*key & 0xffffffffull);
  *key = 0;
}

// ---------------------------------------------------------------- sampler
// Sampler::sample (sampler.rs:28-73) in one CTA of 1024 threads. Every
// "sorted descending, stable" cut of the reference is found without a sort:
// a radix search over the ordered bits of p picks the threshold value, and
// elements equal to it are taken in ascending index order (what a stable
// descending sort does with ties).
//
// Every sum of probability mass is exact and therefore independent of the
// order of additions (the same logits and draw always give the same token):
// p_i = exp(z_i / T) is held as the 64-bit fixed-point mass
// m_i = round(p_i * 2^50 / S), S the sum of all p_i, and the cumulative sums
// behind the top-p cut and the weighted draw are integer sums of m_i. The
// reference sums f32 values one after another (normalise, cumulative
// `>= top_p`, renormalise, WeightedIndex's cumulative weights); its pick and
// this one can differ only where u or top_p lies within that f32 rounding of
// a cumulative boundary.
constexpr int kSampThreads = 1024;
constexpr double kMassOne = 1125899906842624.0;  // 2^50: fixed-point mass of probability 1

struct Cut {
  uint32_t key;   // ordered bits of the threshold value
  uint32_t idx;   // last index (in ascending order) among keys == key that is kept
  int found;
};

__device__ __forceinline__ bool kept(const float *p, size_t i, const Cut &c1, const Cut &c2) {
  uint32_t k = ordered_bits(p[i]);
  if (c1.found && (k < c1.key || (k == c1.key && i > c1.idx))) return false;
  if (c2.found && (k < c2.key || (k == c2.key && i > c2.idx))) return false;
  return true;
}

// Fixed-point mass of one probability (scale = 2^50 / S).
__device__ __forceinline__ unsigned long long mass_of(float p, double scale) {
  return __double2ull_rn((double)p * scale);
}

// Exact block sum of 64-bit integers (every thread gets the total).
__device__ unsigned long long block_sum_u64(unsigned long long v, unsigned long long *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long t = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const unsigned long long r = red[0];
  __syncthreads();
  return r;
}

// Block sum of doubles in a fixed order (thread partials over a fixed element
// mapping, then a fixed shuffle tree), so the result never varies.
__device__ double block_sum_f64(double v, double *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    double t = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const double r = red[0];
  __syncthreads();
  return r;
}

// First element (desc value, asc index) at which the running weight reaches
// the target (>= when inclusive, > otherwise); weight = 1 (count) or the
// element's fixed-point mass. Integer histograms: exact in any order.
__device__ Cut find_cut(const float *p, size_t n, const Cut &c1, const Cut &c2, bool by_count,
                        unsigned long long target, bool inclusive, double scale,
                        unsigned long long *hist, unsigned long long *scan) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, pmask = 0;
  unsigned long long above = 0;
  for (int b = 3; b >= 0; --b) {
    for (int j = tid; j < 256; j += kSampThreads) hist[j] = 0;
    __syncthreads();
    for (size_t i = tid; i < n; i += kSampThreads) {
      if (!kept(p, i, c1, c2)) continue;
      const uint32_t k = ordered_bits(p[i]);
      if ((k & pmask) != prefix) continue;
      atomicAdd(&hist[(k >> (8 * b)) & 255u], by_count ? 1ull : mass_of(p[i], scale));
    }
    __syncthreads();
    if (tid == 0) {
      unsigned long long cum = above;
      int sel = -1;
      for (int j = 255; j >= 0; --j) {
        const unsigned long long nc = cum + hist[j];
        if (inclusive ? (nc >= target) : (nc > target)) {
          sel = j;
          break;
        }
        cum = nc;
      }
      scan[0] = (unsigned long long)(long long)sel;
      scan[1] = cum;
    }
    __syncthreads();
    const int sel = (int)(long long)scan[0];
    if (sel < 0) {
      Cut none{0, 0, 0};
      return none;
    }
    above = scan[1];
    prefix |= (uint32_t)sel << (8 * b);
    pmask |= 255u << (8 * b);
    __syncthreads();
  }
  // ties at `prefix`: walk indices in order (each thread a contiguous chunk)
  const size_t per = (n + kSampThreads - 1) / kSampThreads;
  const size_t lo = tid * per, hi = lo + per < n ? lo + per : n;
  unsigned long long mine = 0;
  for (size_t i = lo; i < hi; ++i)
    if (kept(p, i, c1, c2) && ordered_bits(p[i]) == prefix) mine += by_count ? 1ull : mass_of(p[i], scale);
  scan[2 + tid] = mine;
  __syncthreads();
  if (tid == 0) {
    unsigned long long run = above;
    for (int t = 0; t < kSampThreads; ++t) {
      const unsigned long long v = scan[2 + t];
      scan[2 + t] = run;  // exclusive prefix
      run += v;
    }
  }
  __syncthreads();
  __shared__ unsigned long long best;
  if (tid == 0) best = ~0ull;
  __syncthreads();
  unsigned long long run = scan[2 + tid];
  for (size_t i = lo; i < hi; ++i) {
    if (!(kept(p, i, c1, c2) && ordered_bits(p[i]) == prefix)) continue;
    run += by_count ? 1ull : mass_of(p[i], scale);
    if (inclusive ? (run >= target) : (run > target)) {
      atomicMin(&best, (unsigned long long)i);
      break;
    }
  }
  __syncthreads();
  Cut c{prefix, (uint32_t)(best == ~0ull ? 0xffffffffu : best), 1};
  __syncthreads();
  return c;
}

// Largest value, last index on ties (the argmax of the reference).
__device__ uint32_t block_argmax(const float *x, size_t n, unsigned long long *red) {
  unsigned long long best = 0;
  for (size_t i = threadIdx.x; i < n; i += kSampThreads) {
    const float v = x[i];
    if (v != v) continue;
    const unsigned long long k = ((unsigned long long)ordered_bits(v) << 32) | (unsigned long long)i;
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long t = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, t, o);
      t = other > t ? other : t;
    }
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const uint32_t r = (uint32_t)(red[0] & 0xffffffffull);
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kSampThreads) sample_kernel(
    const float *logits, float *p, size_t n, float temperature, uint64_t top_k, float top_p,
    float u, int use_hash, uint64_t seed, uint64_t offset, uint32_t *out) {
  __shared__ unsigned long long hist[256];
  __shared__ unsigned long long scan[2 + kSampThreads];
  __shared__ unsigned long long ured[32];
  __shared__ double dred[32];
  const int tid = threadIdx.x;
  if (use_hash) {
    // counter-based uniform in [0,1) with 23 random mantissa bits
    uint64_t z = seed + 0x9E3779B97F4A7C15ull * (offset + 1);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    u = (float)(z >> 41) * (1.0f / 8388608.0f);
  }
  // sampler.rs:34-38: exp(z / T) with no max subtraction; the exponential is
  // taken in double and rounded once to f32
  double s = 0.0;
  for (size_t i = tid; i < n; i += kSampThreads) {
    const float e = (float)exp((double)__fdiv_rn(logits[i], temperature));
    p[i] = e;
    s += (double)e;
  }
  __syncthreads();
  const double S = block_sum_f64(s, dred);
  if (!(S > 0.0) || !(S <= 1.7e308)) {
    // every p underflowed or some overflowed (the reference's normalisation
    // then yields NaN and its sort panics): take the largest logit instead
    const uint32_t t = block_argmax(logits, n, ured);
    if (tid == 0) *out = t;
    return;
  }
  const double scale = kMassOne / S;
  unsigned long long m = 0;
  for (size_t i = tid; i < n; i += kSampThreads) m += mass_of(p[i], scale);
  const unsigned long long M = block_sum_u64(m, ured);
  Cut none{0, 0, 0};
  Cut ck = none, cp = none;
  if (top_k > 0 && top_k < n)
    ck = find_cut(p, n, none, none, true, (unsigned long long)top_k, true, scale, hist, scan);
  if (top_p < 1.0f) {
    // cumulative normalised mass >= top_p (sampler.rs:49-62); top_p <= 0
    // keeps the first element, as the reference's first comparison does
    const double t = (double)top_p * (double)M;
    const unsigned long long target = t > 0.0 ? (unsigned long long)ceil(t) : 0ull;
    Cut c = find_cut(p, n, ck, none, false, target, true, scale, hist, scan);
    if (c.found) cp = c;
  }
  unsigned long long s2 = 0;
  for (size_t i = tid; i < n; i += kSampThreads)
    if (kept(p, i, ck, cp)) s2 += mass_of(p[i], scale);
  const unsigned long long S2 = block_sum_u64(s2, ured);
  // the draw: first candidate whose cumulative mass exceeds u * S2 (rand
  // 0.8.6 WeightedIndex: partition_point of cumulative weights <= chosen)
  const unsigned long long target = (unsigned long long)floor((double)u * (double)S2);
  if (top_k == 0 && !(top_p < 1.0f)) {
    // Neither filter sorted the candidates, so WeightedIndex walks them in
    // index order (sampler.rs:45-71), else the last index.
    const size_t per = (n + kSampThreads - 1) / kSampThreads;
    const size_t lo = tid * per, hi = lo + per < n ? lo + per : n;
    unsigned long long mine = 0;
    for (size_t i = lo; i < hi; ++i) mine += mass_of(p[i], scale);
    scan[2 + tid] = mine;
    __syncthreads();
    if (tid == 0) {
      unsigned long long run = 0;
      for (int t = 0; t < kSampThreads; ++t) {
        const unsigned long long v = scan[2 + t];
        scan[2 + t] = run;
        run += v;
      }
    }
    __shared__ unsigned long long first;
    if (tid == 0) first = ~0ull;
    __syncthreads();
    unsigned long long run = scan[2 + tid];
    for (size_t i = lo; i < hi; ++i) {
      run += mass_of(p[i], scale);
      if (run > target) {
        atomicMin(&first, (unsigned long long)i);
        break;
      }
    }
    __syncthreads();
    if (tid == 0) *out = (first == ~0ull) ? (uint32_t)(n - 1) : (uint32_t)first;
    return;
  }
  const Cut pick = find_cut(p, n, ck, cp, false, target, false, scale, hist, scan);
  __shared__ int resolved;
  if (tid == 0) {
    resolved = pick.found && pick.idx != 0xffffffffu;
    if (resolved) *out = pick.idx;
  }
  __syncthreads();
  if (!resolved) {
    // target beyond the kept mass (not reached for u < 1): WeightedIndex
    // returns the last weight, i.e. the smallest kept element (largest index
    // among ties)
    __shared__ unsigned long long low;
    if (tid == 0) low = ~0ull;
    __syncthreads();
    for (size_t i = tid; i < n; i += kSampThreads)
      if (kept(p, i, ck, cp)) {
        unsigned long long k = ((unsigned long long)ordered_bits(p[i]) << 32) | (0xffffffffu - (uint32_t)i);
        atomicMin(&low, k);
      }
    __syncthreads();
    if (tid == 0) *out = 0xffffffffu - (uint32_t)(low & 0xffffffffu);
  }
}

}  // namespace

ifx_status op_dequantize(int type, const uint8_t *src, size_t nbytes, float *out, size_t n,
                         cudaStream_t st) {
  BlockInfo b = block_info(type);
  if (!b.elems) return fail(IFX_ERR_UNKNOWN_TENSOR_TYPE, "dequantize: unsupported type");
  size_t expected = (n + b.elems - 1) / b.elems * b.bytes;
  if (nbytes != expected) return fail(IFX_ERR_UNEXPECTED_EOF, "dequantize: byte count");
  if (n == 0) return IFX_OK;
  size_t nfull = (nbytes / b.bytes) * b.elems;  // elements fully covered by blocks
  dequant_kernel<<<nblk(std::min(n, nfull), 256), 256, 0, st>>>(type, src, out, std::min(n, nfull));
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_matmul(const float *a, const float *b, float *c, size_t m, size_t n, size_t k,
                     cudaStream_t st) {
  if (!m || !n) return IFX_OK;
  matmul_kernel<<<nblk(m * n, 128), 128, 0, st>>>(a, b, c, m, n, k);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_matmul_t(const float *a, const float *b, float *c, size_t m, size_t n, size_t k,
                       cudaStream_t st) {
  if (!m || !n) return IFX_OK;
  size_t warps = m * n;
  matmul_t_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(a, b, c, m, n, k);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_rms_norm_rows(float *x, const float *w, float eps, size_t rows, size_t hidden,
                            cudaStream_t st) {
  if (!rows || !hidden) return IFX_OK;
  rms_norm_kernel<<<(unsigned)rows, 256, 0, st>>>(x, w, eps, hidden);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_silu(float *x, size_t n, cudaStream_t st) {
  if (!n) return IFX_OK;
  silu_kernel<<<nblk(n, 256), 256, 0, st>>>(x, n);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_swiglu(const float *g, const float *u, float *o, size_t n, cudaStream_t st) {
  if (!n) return IFX_OK;
  swiglu_kernel<<<nblk(n, 256), 256, 0, st>>>(g, u, o, n);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_add(float *o, const float *b, size_t n, cudaStream_t st) {
  if (!n) return IFX_OK;
  add_kernel<<<nblk(n, 256), 256, 0, st>>>(o, b, n);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_softmax_rows(float *x, size_t rows, size_t cols, cudaStream_t st) {
  if (!rows || !cols) return IFX_OK;
  softmax_kernel<<<(unsigned)rows, 256, 0, st>>>(x, cols);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_embedding_lookup(const float *emb, size_t emb_len, const uint32_t *ids,
                               size_t n_ids, size_t hidden, float *out, int *err_dev,
                               cudaStream_t st) {
  if (!n_ids) return IFX_OK;
  embedding_kernel<<<(unsigned)n_ids, 256, 0, st>>>(emb, emb_len, ids, hidden, out, err_dev);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_rope(float *x, size_t seq, size_t heads, size_t hd, size_t rope_dim, float base,
                   size_t pos0, cudaStream_t st) {
  if (rope_dim > hd || rope_dim % 2) return fail(IFX_ERR_SHAPE, "rope: rope_dim");
  size_t total = seq * heads * (rope_dim / 2);
  if (!total) return IFX_OK;
  rope_kernel<<<nblk(total, 256), 256, 0, st>>>(x, seq, heads, hd, rope_dim, base, pos0);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status op_argmax(const float *x, size_t n, unsigned long long *key_dev, uint32_t *out_dev,
                     cudaStream_t st) {
  if (!n) return fail(IFX_ERR_SHAPE, "argmax: empty input");
  argmax_kernel<<<std::min<unsigned>(nblk(n, 256), kNumSMs * 4), 256, 0, st>>>(x, n, key_dev);
  key_to_token_kernel<<<1, 1, 0, st>>>(key_dev, out_dev);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

static ifx_status sample_common(const float *logits, size_t n, float temperature, uint64_t top_k,
                                float top_p, float u, int use_hash, uint64_t seed,
                                uint64_t offset, uint32_t *out_dev, cudaStream_t st) {
  if (!n) return fail(IFX_ERR_SHAPE, "sample: empty logits");
  float *p = nullptr;
  IFX_CUDA(cudaMallocAsync(&p, n * sizeof(float), st));
  sample_kernel<<<1, kSampThreads, 0, st>>>(logits, p, n, temperature, top_k, top_p, u, use_hash,
                                             seed, offset, out_dev);
  cudaError_t e = cudaGetLastError();
  cudaFreeAsync(p, st);
  if (e != cudaSuccess) return cuda_fail(e, "sample_kernel");
  return IFX_OK;
}

ifx_status op_sample_u(const float *logits, size_t n, float temperature, uint64_t top_k,
                       float top_p, float u, uint32_t *out_dev, cudaStream_t st) {
  return sample_common(logits, n, temperature, top_k, top_p, u, 0, 0, 0, out_dev, st);
}

ifx_status op_sample_philox(const float *logits, size_t n, float temperature, uint64_t top_k,
                            float top_p, uint64_t seed, uint64_t offset, uint32_t *out_dev,
                            cudaStream_t st) {
  return sample_common(logits, n, temperature, top_k, top_p, 0.f, 1, seed, offset, out_dev, st);
}

// ------------------------------------------- sampler with static scratch --
// Backing store of op_sample_u_static: one file-scope device array, so that
// call allocates nothing. Layout: kStaticSampleMax f32 probabilities, then
// (at byte offset 4 * kStaticSampleMax, a multiple of 256) the 64-bit argmax
// key of the greedy case. 1 MiB + 256 B per device, reserved at module load.
static __device__ __align__(256) float g_sample_scratch[kStaticSampleMax + 64];
static_assert(kStaticSampleMax == IFX_SAMPLE_STATIC_MAX, "header and library limits differ");

namespace {
constexpr int kStaticMaxDevices = 64;
std::mutex g_scratch_mu;
float *g_scratch_ptr[kStaticMaxDevices] = {};

// Address of g_sample_scratch on the current device, looked up once per
// device (the first call on a device does the lookup with that device
// current; later calls only read the cached pointer).
ifx_status static_scratch(float **out) {
  int dev = 0;
  IFX_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kStaticMaxDevices)
    return fail(IFX_ERR_UNSUPPORTED, "sample_u_static: device ordinal " + std::to_string(dev) +
                                         " beyond the " + std::to_string(kStaticMaxDevices) +
                                         " devices this build tracks");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_sample_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_sample_scratch)");
    g_scratch_ptr[dev] = static_cast<float *>(ptr);
  }
  *out = g_scratch_ptr[dev];
  return IFX_OK;
}
}  // namespace

ifx_status op_sample_u_static(const float *logits, size_t n, float temperature, uint64_t top_k,
                              float top_p, float u, uint32_t *out_dev, cudaStream_t st) {
  if (!n) return fail(IFX_ERR_SHAPE, "sample: empty logits");
  if (n > kStaticSampleMax)
    return fail(IFX_ERR_INVALID_ARGUMENT,
                "sample_u_static: " + std::to_string(n) + " logits exceed the static scratch of " +
                    std::to_string(kStaticSampleMax) + " entries; use ifx_op_sample_u");
  float *scratch = nullptr;
  IFX_TRY(static_scratch(&scratch));
  if (temperature == 0.0f) {
    // the argmax key is combined with atomicMax and must start at zero
    auto *key = reinterpret_cast<unsigned long long *>(scratch + kStaticSampleMax);
    IFX_CUDA(cudaMemsetAsync(key, 0, sizeof(unsigned long long), st));
    return op_argmax(logits, n, key, out_dev, st);
  }
  // p (the first n floats) is written in full before it is read: no clearing
  sample_kernel<<<1, kSampThreads, 0, st>>>(logits, scratch, n, temperature, top_k, top_p, u, 0,
                                             0, 0, out_dev);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

}  // namespace ifx
