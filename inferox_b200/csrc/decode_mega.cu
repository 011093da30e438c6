// Persistent batch-1 decode kernel (one cooperative launch per token).
//
// 148 CTAs x (16 consumer warps + 1 producer warp). The token step is a list
// of phases (embed; per layer QKV GEMV, attention, Wo GEMV, W1/W3 GEMV, W2
// GEMV; logits GEMV; argmax). The attention phase's split-K partials are
// combined by the CTA that finishes each kv head's last split, and the cached
// K/V rows of each CTA's first attention item are bulk-copied into shared
// memory by the producer warp ahead of the QKV phase. Phases that read the previous phase's
// output are separated by a grid barrier (atomic counter with a bounded
// spin). The producer warp does not take part in the barriers: weights do
// not depend on activations, so it streams every GEMV phase's units for its
// CTA into the shared-memory ring back to back, running ahead across phase
// boundaries by as many stages as the ring holds. Barrier and staging time
// of the consumers is therefore overlapped with weight streaming, which is
// what separate kernel launches could not do.
#include <algorithm>
#include <vector>

#include "decode_mega.cuh"
#include "gemv_dev.cuh"
#include "ops.cuh"
#include "quant.cuh"

namespace ifx {

namespace {

using namespace gemvdev;

constexpr int kMaxGrp = 8;
constexpr size_t kMegaRingBytes = 90 * 1024;
constexpr int kMaxSplitsMega = 128;

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Generic addressing: the peer buffers are CUDA IPC mappings.
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait (one thread) until the epoch at `flag`, written by another
// rank, reaches e; false (error flag set to `code`) after limit_ns of wall
// time (another rank may legitimately start its step later than this one)
// or as soon as another thread has raised the error flag.
__device__ bool wait_epoch(const unsigned *flag, unsigned e, int *err, int code, uint64_t limit_ns) {
  const uint64_t t0 = global_ns();
  uint32_t spins = 0;
  while ((int)(ld_acquire_sys(flag) - e) < 0) {
    if ((++spins & 63u) == 0) {
      if (*(volatile int *)err) return false;
      if (global_ns() - t0 > limit_ns) {
        atomicExch(err, code);
        return false;
      }
      if (spins > 4096u) __nanosleep(256);
    }
  }
  return true;
}

// Copies phase record `src` into shared memory with plain 16-byte loads
// (one warp; no bulk copy, so nothing queues behind the weight ring's copies
// in the CTA's copy engine).
__device__ __forceinline__ void load_record(MegaPhase *dst, const MegaPhase *src, int lane) {
  constexpr int kWords = (int)(sizeof(MegaPhase) / 16);
  const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
  uint4 *d4 = reinterpret_cast<uint4 *>(dst);
  for (int i = lane; i < kWords; i += 32) d4[i] = __ldg(s4 + i);
}

// Grid barrier over all CTAs (consumer warps only). Bounded: polling stops
// after 2^24 polls (well over a second) or as soon as any thread has raised
// the error flag, which every poll reads beside the counter (the flag costs
// no extra round trip once the counter is reached).
// Returns false (the same value in every consumer thread of the CTA) when the
// error flag is set, so the CTA's consumers leave together; the host then
// reports IFX_ERR_TIMEOUT.
//
// While thread 0 waits, warp 1 copies the next phase's record `next` into
// `rec` (the buffer of two phases back, which every consumer has finished).
__device__ bool grid_barrier(unsigned *bar, unsigned target, int *err, MegaPhase *rec,
                             const MegaPhase *next) {
  __shared__ int s_err;
  consumer_sync();
  if (threadIdx.x == 0) {
    // release: the CTA's writes (ordered before this thread by the barrier
    // above) become visible to any CTA that acquires the counter
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
    uint32_t spins = 0;
    int e = 0;
    while (true) {
      const unsigned c = ld_acquire(bar);
      e = *(volatile int *)err;
      if (c >= target || e) break;
      if (++spins > (1u << 24)) {
        atomicExch(err, 401);
        e = 401;
        break;
      }
    }
    s_err = e;
  } else if ((threadIdx.x >> 5) == 1) {
    load_record(rec, next, threadIdx.x & 31);
  }
  consumer_sync();
  return s_err == 0;
}

__device__ __forceinline__ void rope_pair_m(float &a, float &b, int i, int rope_dim, float base,
                                            int pos) {
  const float inv = 1.0f / powf(base, (float)i / (float)rope_dim);
  const float ang = __fmul_rn((float)pos, inv);
  float s, c;
  sincosf(ang, &s, &c);
  const float x0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  const float x1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  a = x0;
  b = x1;
}

// ---------------------------------------------------------------- phases --
__device__ __noinline__ void phase_embed(const MegaArgs &A) {
  const int tid = threadIdx.x;
  const uint64_t base = (uint64_t)(*A.next_token) * (uint64_t)A.D;
  for (int i = blockIdx.x * kConsumerThreads + tid; i < A.D; i += gridDim.x * kConsumerThreads)
    A.x[i] = dequant_elem(A.emb_type, A.emb, base + i);
}

// Split-K decode attention. Item (h, s) covers cache rows [t0, t1) of kv
// head h: chunk = ceil((pos + 1) / nsa), t0 = s * chunk. Rows below pos are
// already in the cache; row pos (this token) is appended from qkv.
struct AttnSpan {
  int t0, t1, nk, nold;
};

// Cache rows one item can hold (the largest split plus this token's row),
// rounded up to whole 16-row MMA tiles.
__host__ __device__ __forceinline__ int attn_cap(int max_seq, int nsa) {
  return ((max_seq + nsa - 1) / nsa + 1 + 15) & ~15;
}

// Splits per kv head for this step: the fewest that keep every item within
// the rows one item's buffer holds (ceil(max_seq / A.nsa), A.nsa splits of
// a full cache), but at least A.nsa_base (the count that spreads the items
// over the SMs). A short context in a large cache thus takes fewer rounds of
// items and a smaller combine.
__device__ __forceinline__ int step_splits(const MegaArgs &A, int pos) {
  const int rmax = (A.max_seq + A.nsa - 1) / A.nsa;
  return min(A.nsa, max(A.nsa_base, (pos + 1 + rmax - 1) / rmax));
}

__device__ __forceinline__ AttnSpan attn_span(int pos, int nsa, int s) {
  const int len = pos + 1;
  const int chunk = (len + nsa - 1) / nsa;
  AttnSpan r;
  r.t0 = s * chunk;
  r.t1 = min(len, r.t0 + chunk);
  r.nk = max(0, r.t1 - r.t0);
  r.nold = max(0, min(r.t1, pos) - r.t0);
  return r;
}

// Thread 0: bulk-copy the cached K and V rows [t0, t0 + nold) of kv head h
// (layer `layer`) into the attention buffer, completing on `kvbar`. With no
// rows the barrier is completed by a plain arrive.
__device__ __noinline__ void attn_fetch(const MegaArgs &A, int layer, int h, int s, int pos, int ns,
                                       uint8_t *abuf, uint64_t *kvbar) {
  const AttnSpan sp = attn_span(pos, ns, s);
  const int hd = A.hd;
  const int cap = attn_cap(A.max_seq, A.nsa);
  const uint32_t bytes = (uint32_t)sp.nold * (uint32_t)hd * 2u;
  if (bytes == 0) {
    mbar_arrive(kvbar);
    return;
  }
  const size_t row0 = (size_t)layer * A.kv_layer_elems + ((size_t)h * A.max_seq + sp.t0) * hd;
  mbar_arrive_expect_tx(kvbar, 2u * bytes);
  bulk_g2s(abuf, A.kc0 + row0, bytes, kvbar);
  bulk_g2s(abuf + (size_t)cap * hd * 2, A.vc0 + row0, bytes, kvbar);
}

// One (kv head, split) item: scores of the grp query heads against the
// item's rows (cached rows from the attention buffer, this token's row from
// qkv), softmax statistics, P.V; partial (max, sum, output) to global.
// The cached rows must have landed (kvbar waited by the caller).
__device__ __noinline__ void attn_item(const MegaArgs &A, const MegaAttn &at, int h, int s, int pos,
                                      int NS, uint8_t *abuf) {
  const int tid = threadIdx.x;
  const int hd = A.hd, grp = A.H / A.G;
  const AttnSpan sp = attn_span(pos, NS, s);
  const int t0 = sp.t0, nk = sp.nk;
  const int cap = attn_cap(A.max_seq, A.nsa);
  const int n16 = hd / 8;  // 16-byte chunks per row
  const uint4 *Ks = reinterpret_cast<const uint4 *>(abuf);             // [cap][n16]
  uint4 *Vs4 = reinterpret_cast<uint4 *>(abuf + (size_t)cap * hd * 2);  // [cap][n16]
  float *qs = reinterpret_cast<float *>(abuf + (size_t)cap * hd * 4);    // [grp][hd]
  float *sc = qs + grp * hd;                                              // [grp][cap]
  float *stat = sc + grp * cap;                                           // [grp][2]
  // RoPE at position 0 is the identity (the reference's decode, forward.rs:371-372)
  const int rpos = A.rope_compat ? 0 : pos;
  const float *q = A.qkv + (size_t)h * grp * hd;
  for (int e = tid; e < grp * hd / 2; e += kConsumerThreads) {
    const int j = e / (hd / 2), i = 2 * (e % (hd / 2));
    float x0 = __ldcg(q + j * hd + i), x1 = __ldcg(q + j * hd + i + 1);
    if (rpos != 0 && i < A.rope_dim) rope_pair_m(x0, x1, i, A.rope_dim, A.rope_base, rpos);
    qs[j * hd + i] = x0;
    qs[j * hd + i + 1] = x1;
  }
  if (t0 <= pos && pos < sp.t1) {  // append this token's K/V (forward.rs:375-378)
    const float *kn = A.qkv + (size_t)A.H * hd + (size_t)h * hd;
    const float *vn = A.qkv + (size_t)(A.H + A.G) * hd + (size_t)h * hd;
    const int r = pos - t0;
    __half *kcp = at.kc + ((size_t)h * A.max_seq + pos) * hd;
    __half *vcp = at.vc + ((size_t)h * A.max_seq + pos) * hd;
    __half *Kh = reinterpret_cast<__half *>(abuf) + (size_t)r * hd;
    __half *Vh = reinterpret_cast<__half *>(Vs4) + (size_t)r * hd;
    for (int e = tid; e < hd / 2; e += kConsumerThreads) {
      const int i = 2 * e, ip = kv_col(pos, i, hd);
      float x0 = __ldcg(kn + i), x1 = __ldcg(kn + i + 1);
      if (rpos != 0 && i < A.rope_dim) rope_pair_m(x0, x1, i, A.rope_dim, A.rope_base, rpos);
      const __half2 kh = __floats2half2_rn(x0, x1);
      const __half2 vh = __floats2half2_rn(__ldcg(vn + i), __ldcg(vn + i + 1));
      *reinterpret_cast<__half2 *>(kcp + ip) = kh;
      *reinterpret_cast<__half2 *>(vcp + ip) = vh;
      *reinterpret_cast<__half2 *>(Kh + ip) = kh;
      *reinterpret_cast<__half2 *>(Vh + ip) = vh;
    }
  }
  consumer_sync();
  // scores: four adjacent threads share one (head j, row t); thread qtr
  // takes chunks qtr, qtr + 4, ... of the row, rotated by t & 7 so the eight
  // rows a warp reads at once fall on different banks
  const float isq = 1.0f / sqrtf((float)hd);
  for (int base = 0; base < grp * nk * 4; base += kConsumerThreads) {
    const int e = base + tid;
    const bool ok = e < grp * nk * 4;
    float acc = 0.f;
    int j = 0, t = 0;
    if (ok) {
      const int qtr = e & 3, jt = e >> 2;
      j = jt / nk;
      t = jt - j * nk;
      const float4 *q4 = reinterpret_cast<const float4 *>(qs + j * hd);
      int c = qtr + (t & 7);  // any rotation keeps each quarter's chunk set a partition
      const int key = kv_col(t0 + t, 0, hd) >> 3;  // chunk permutation of this cache row
      for (int cc = qtr; cc < n16; cc += 4) {
        while (c >= n16) c -= n16;
        const uint4 kv = Ks[t * n16 + (c ^ key)];
        const float4 qa = q4[2 * c], qb = q4[2 * c + 1];
        const float2 k0 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.x));
        const float2 k1 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.y));
        const float2 k2 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.z));
        const float2 k3 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.w));
        acc = fmaf(qa.x, k0.x, acc);
        acc = fmaf(qa.y, k0.y, acc);
        acc = fmaf(qa.z, k1.x, acc);
        acc = fmaf(qa.w, k1.y, acc);
        acc = fmaf(qb.x, k2.x, acc);
        acc = fmaf(qb.y, k2.y, acc);
        acc = fmaf(qb.z, k3.x, acc);
        acc = fmaf(qb.w, k3.y, acc);
        c += 4;
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (ok && (tid & 3) == 0) sc[j * cap + t] = acc * isq;
  }
  consumer_sync();
  const int warp = tid >> 5, lane = tid & 31;
  if (warp < grp) {  // softmax statistics of this split, head j = warp
    const int j = warp;
    float m = -INFINITY;
    for (int t = lane; t < nk; t += 32) m = fmaxf(m, sc[j * cap + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < nk; t += 32) {
      const float p = expf(sc[j * cap + t] - m);
      sc[j * cap + t] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stat[2 * j] = m;
      stat[2 * j + 1] = l;
    }
  }
  consumer_sync();
  float *po = A.part_o + (size_t)(h * NS + s) * grp * hd;
  const __half *Vh = reinterpret_cast<const __half *>(Vs4);
  for (int e = tid; e < grp * hd; e += kConsumerThreads) {
    const int j = e / hd, d = e % hd;
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    int t = 0;
    for (; t + 3 < nk; t += 4) {
      o0 = fmaf(sc[j * cap + t], __half2float(Vh[(size_t)t * hd + kv_col(t0 + t, d, hd)]), o0);
      o1 = fmaf(sc[j * cap + t + 1], __half2float(Vh[(size_t)(t + 1) * hd + kv_col(t0 + t + 1, d, hd)]), o1);
      o2 = fmaf(sc[j * cap + t + 2], __half2float(Vh[(size_t)(t + 2) * hd + kv_col(t0 + t + 2, d, hd)]), o2);
      o3 = fmaf(sc[j * cap + t + 3], __half2float(Vh[(size_t)(t + 3) * hd + kv_col(t0 + t + 3, d, hd)]), o3);
    }
    for (; t < nk; ++t)
      o0 = fmaf(sc[j * cap + t], __half2float(Vh[(size_t)t * hd + kv_col(t0 + t, d, hd)]), o0);
    po[e] = (o0 + o1) + (o2 + o3);
  }
  if (tid < grp) {
    const float m = nk > 0 ? stat[2 * tid] : -INFINITY, l = nk > 0 ? stat[2 * tid + 1] : 0.f;
    A.part_ml[(h * NS + s) * grp + tid] = make_float2(m, l);
  }
  consumer_sync();  // the buffer is reused by the next item
}

// The same item on tensor cores (head size a multiple of 64, at most eight
// query heads per kv head): S = K Q^T with the cached K rows as the A operand
// (ldmatrix from the chunk-swizzled rows, conflict-free) and the query heads
// as B columns carrying each head's hi and lo f16 planes (about 22 bits),
// added afterwards; softmax statistics over the item's rows; O = V^T P with
// V^T from ldmatrix.trans and P as hi/lo columns the same way. Up to four
// heads share one 8-column tile (column j the hi plane of head j, column
// 4 + j its lo plane, added across lanes); five to eight heads take two
// tiles (hi planes, lo planes). Output format as attn_item.
template <int W>
__device__ __noinline__ void attn_item_tc(const MegaArgs &A, const MegaAttn &at, int h, int s,
                                          int pos, int NS, uint8_t *abuf) {
  static_assert(W == 4 || W == 8, "head slots per plane");
  constexpr int NT = W / 4;  // 8-column B tiles per MMA step
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int hd = A.hd, grp = A.H / A.G;
  const AttnSpan sp = attn_span(pos, NS, s);
  const int t0 = sp.t0, nk = sp.nk, nk16 = (nk + 15) & ~15;
  const int cap = attn_cap(A.max_seq, A.nsa);
  const int qs = hd + 8, ps = cap + 8;  // padded row strides (conflict-free B loads)
  __half *Ks = reinterpret_cast<__half *>(abuf);  // [cap][hd], rows chunk-swizzled
  __half *Vs = Ks + (size_t)cap * hd;               // [cap][hd]
  __half *qh = Vs + (size_t)cap * hd;               // [2][W][qs]: plane, head
  float *sc = reinterpret_cast<float *>(qh + 2 * W * qs);  // [W][cap]
  __half *ph = reinterpret_cast<__half *>(sc + W * cap);   // [2][W][ps]
  float *stat = reinterpret_cast<float *>(ph + 2 * W * ps);  // [W][2]
  // RoPE at position 0 is the identity (the reference's decode, forward.rs:371-372)
  const int rpos = A.rope_compat ? 0 : pos;
  const float *q = A.qkv + (size_t)h * grp * hd;
  for (int e = tid; e < W * hd / 2; e += kConsumerThreads) {
    const int j = e / (hd / 2), i = 2 * (e % (hd / 2));
    float x0 = 0.f, x1 = 0.f;
    if (j < grp) {
      x0 = __ldcg(q + j * hd + i);
      x1 = __ldcg(q + j * hd + i + 1);
      if (rpos != 0 && i < A.rope_dim) rope_pair_m(x0, x1, i, A.rope_dim, A.rope_base, rpos);
    }
    const __half2 hi = __floats2half2_rn(x0, x1);
    *reinterpret_cast<__half2 *>(qh + j * qs + i) = hi;
    *reinterpret_cast<__half2 *>(qh + (W + j) * qs + i) =
        __floats2half2_rn(x0 - __low2float(hi), x1 - __high2float(hi));
  }
  if (t0 <= pos && pos < sp.t1) {  // append this token's K/V (forward.rs:375-378)
    const float *kn = A.qkv + (size_t)A.H * hd + (size_t)h * hd;
    const float *vn = A.qkv + (size_t)(A.H + A.G) * hd + (size_t)h * hd;
    const int r = pos - t0;
    __half *kcp = at.kc + ((size_t)h * A.max_seq + pos) * hd;
    __half *vcp = at.vc + ((size_t)h * A.max_seq + pos) * hd;
    for (int e = tid; e < hd / 2; e += kConsumerThreads) {
      const int i = 2 * e, ip = kv_col(pos, i, hd);
      float x0 = __ldcg(kn + i), x1 = __ldcg(kn + i + 1);
      if (rpos != 0 && i < A.rope_dim) rope_pair_m(x0, x1, i, A.rope_dim, A.rope_base, rpos);
      const __half2 kh = __floats2half2_rn(x0, x1);
      const __half2 vh = __floats2half2_rn(__ldcg(vn + i), __ldcg(vn + i + 1));
      *reinterpret_cast<__half2 *>(kcp + ip) = kh;
      *reinterpret_cast<__half2 *>(vcp + ip) = vh;
      *reinterpret_cast<__half2 *>(Ks + (size_t)r * hd + ip) = kh;
      *reinterpret_cast<__half2 *>(Vs + (size_t)r * hd + ip) = vh;
    }
  }
  // V rows [nk, nk16) enter P V with p = 0: they must be finite
  for (int e = tid; e < (nk16 - nk) * hd / 2; e += kConsumerThreads)
    *reinterpret_cast<__half2 *>(Vs + (size_t)nk * hd + 2 * e) = __floats2half2_rn(0.f, 0.f);
  consumer_sync();
  // scores: warp w takes 16-row tile w
  const float isq = 1.0f / sqrtf((float)hd);
  for (int mt = warp; mt < nk16 / 16; mt += kConsumerWarps) {
    float D[NT][4] = {};
    const int row = 16 * mt + (lane & 7) + 8 * ((lane >> 3) & 1);
    const int key = kv_col(t0 + row, 0, hd) >> 3;
    for (int ks = 0; ks < hd / 16; ++ks) {
      uint32_t a[4];
      ldsm_x4(a, smem_u32(Ks + (size_t)row * hd + (((2 * ks + (lane >> 4)) ^ key) << 3)));
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        // tile t, column g: row 8 t + g of qh (W = 4: plane g / 4, head g % 4)
        const __half *qp = qh + (8 * t + g) * qs + 2 * c + 16 * ks;
        mma_16816(D[t], a[0], a[1], a[2], a[3], *reinterpret_cast<const uint32_t *>(qp),
                  *reinterpret_cast<const uint32_t *>(qp + 8), D[t]);
      }
    }
    float S[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)  // hi + lo
      S[i] = NT == 2 ? D[0][i] + D[NT - 1][i] : D[0][i] + __shfl_xor_sync(0xffffffffu, D[0][i], 2);
    if (NT == 2 || c < 2) {
      const int ra = 16 * mt + g, rb = ra + 8;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = 2 * c + jj;
        if (j < grp) {
          sc[j * cap + ra] = ra < nk ? S[jj] * isq : -INFINITY;
          sc[j * cap + rb] = rb < nk ? S[2 + jj] * isq : -INFINITY;
        }
      }
    }
  }
  consumer_sync();
  if (warp < W) {  // softmax statistics of this split, head j = warp; p as hi/lo planes
    const int j = warp;
    float m = -INFINITY;
    if (j < grp)
      for (int t = lane; t < nk; t += 32) m = fmaxf(m, sc[j * cap + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < nk16; t += 32) {
      const float p = (j < grp && t < nk) ? expf(sc[j * cap + t] - m) : 0.f;
      const __half hp = __float2half_rn(p);
      ph[j * ps + t] = hp;
      ph[(W + j) * ps + t] = __float2half_rn(p - __half2float(hp));
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stat[2 * j] = m;
      stat[2 * j + 1] = l;
    }
  }
  consumer_sync();
  // O^T = V^T P: warp w takes dims [16 w, 16 w + 16)
  float *po = A.part_o + (size_t)(h * NS + s) * grp * hd;
  for (int mt = warp; mt < hd / 16; mt += kConsumerWarps) {
    float D[NT][4] = {};
    for (int ks = 0; ks < nk16 / 16; ++ks) {
      const int t = 16 * ks + (lane & 7) + 8 * (lane >> 4);
      const int chunk = (2 * mt + ((lane >> 3) & 1)) ^ (kv_col(t0 + t, 0, hd) >> 3);
      uint32_t a[4];
      ldsm_x4_t(a, smem_u32(Vs + (size_t)t * hd + (chunk << 3)));
#pragma unroll
      for (int tt = 0; tt < NT; ++tt) {
        const __half *pp = ph + (8 * tt + g) * ps + 2 * c + 16 * ks;
        mma_16816(D[tt], a[0], a[1], a[2], a[3], *reinterpret_cast<const uint32_t *>(pp),
                  *reinterpret_cast<const uint32_t *>(pp + 8), D[tt]);
      }
    }
    float O[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      O[i] = NT == 2 ? D[0][i] + D[NT - 1][i] : D[0][i] + __shfl_xor_sync(0xffffffffu, D[0][i], 2);
    if (NT == 2 || c < 2) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = 2 * c + jj;
        if (j < grp) {
          po[j * hd + 16 * mt + g] = O[jj];
          po[j * hd + 16 * mt + g + 8] = O[2 + jj];
        }
      }
    }
  }
  if (tid < grp) {
    const float m = nk > 0 ? stat[2 * tid] : -INFINITY, l = nk > 0 ? stat[2 * tid + 1] : 0.f;
    A.part_ml[(h * NS + s) * grp + tid] = make_float2(m, l);
  }
  consumer_sync();  // the buffer is reused by the next item
}

// Combine of the splits of kv head h (its grp query heads), run by the CTA
// that finished the head's last split: attn[hq][d] = sum_s w_s o_s[d] with
// w_s = exp(m_s - M) / sum_s' exp(m_s' - M) l_s' (splits with no rows carry
// l = 0 and weight 0). Two load rounds: the (m, l) pairs, then the partial
// outputs. `wbuf` holds 3 * grp * nsa floats.
// Fast form for grp * hd <= 512 and nsa <= 2 * kCombineLoads: warps 0-7
// own the output float4s (two threads each, alternate splits), and issue all
// their partial loads at once, while warps 8-11 fetch the (m, l) pairs and
// form the weights; one memory round trip instead of three.
constexpr int kCombineLoads = 12;

__device__ __forceinline__ void combine_kv_head_fast(const MegaArgs &A, int h, int NS, float *wbuf) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hd = A.hd, grp = A.H / A.G;
  float2 *ml = reinterpret_cast<float2 *>(wbuf);  // [grp][NS]
  float *wn = wbuf + 2 * grp * NS;                 // [grp][NS]
  const int F = grp * hd / 4;                      // output float4s
  const int f = tid >> 1, half = tid & 1;
  const bool mine = tid < 256 && f < F;
  const int j = mine ? (4 * f) / hd : 0;
  const float4 *po4 = reinterpret_cast<const float4 *>(A.part_o + (size_t)h * NS * grp * hd) + f;
  const size_t s4 = (size_t)grp * hd / 4;  // float4s between splits
  float4 v[kCombineLoads];
#pragma unroll
  for (int i = 0; i < kCombineLoads; ++i) {
    const int sp = half + 2 * i;
    v[i] = (mine && sp < NS) ? __ldcg(po4 + sp * s4) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (warp >= 8 && warp < 8 + grp) {  // the weights of head warp - 8
    const int jj = warp - 8;
    float2 t[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int sp = lane + 32 * r;
      t[r] = sp < NS ? __ldcg(&A.part_ml[(h * NS + sp) * grp + jj]) : make_float2(-INFINITY, 0.f);
    }
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < 4; ++r)
      if (t[r].y > 0.f) M = fmaxf(M, t[r].x);
    M = warp_max(M);
    float L = 0.f, w[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      w[r] = t[r].y > 0.f ? expf(t[r].x - M) : 0.f;
      L = fmaf(t[r].y, w[r], L);
    }
    L = warp_sum(L);
    const float invL = 1.0f / L;
#pragma unroll
    for (int r = 0; r < 4; ++r)
      if (lane + 32 * r < NS) wn[jj * NS + lane + 32 * r] = w[r] * invL;
  }
  consumer_sync();
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  if (mine) {
    const float *w = wn + j * NS;
#pragma unroll
    for (int i = 0; i < kCombineLoads; ++i) {
      const int sp = half + 2 * i;
      const float ws = sp < NS ? w[sp] : 0.f;
      o.x = fmaf(ws, v[i].x, o.x);
      o.y = fmaf(ws, v[i].y, o.y);
      o.z = fmaf(ws, v[i].z, o.z);
      o.w = fmaf(ws, v[i].w, o.w);
    }
  }
  // the two threads of a float4 (lanes 2k, 2k + 1) add their halves of the splits
  o.x += __shfl_xor_sync(0xffffffffu, o.x, 1);
  o.y += __shfl_xor_sync(0xffffffffu, o.y, 1);
  o.z += __shfl_xor_sync(0xffffffffu, o.z, 1);
  o.w += __shfl_xor_sync(0xffffffffu, o.w, 1);
  if (mine && half == 0) reinterpret_cast<float4 *>(A.attn + (size_t)h * grp * hd)[f] = o;
}

__device__ __noinline__ void combine_kv_head(const MegaArgs &A, int h, int NS, float *wbuf) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hd = A.hd, grp = A.H / A.G;
  if (grp * hd <= 512 && NS <= 2 * kCombineLoads && NS <= 128 && grp <= 8) {
    combine_kv_head_fast(A, h, NS, wbuf);
    return;
  }
  float2 *ml = reinterpret_cast<float2 *>(wbuf);  // [grp][NS]
  float *wn = wbuf + 2 * grp * NS;                 // [grp][NS]
  for (int e = tid; e < grp * NS; e += kConsumerThreads) {
    const int j = e / NS, s = e - j * NS;
    ml[e] = __ldcg(&A.part_ml[(h * NS + s) * grp + j]);
  }
  consumer_sync();
  if (warp < grp) {
    const int j = warp;
    float M = -INFINITY;
    for (int s = lane; s < NS; s += 32)
      if (ml[j * NS + s].y > 0.f) M = fmaxf(M, ml[j * NS + s].x);
    M = warp_max(M);
    float L = 0.f;
    for (int s = lane; s < NS; s += 32) {
      const float2 v = ml[j * NS + s];
      const float w = v.y > 0.f ? expf(v.x - M) : 0.f;
      wn[j * NS + s] = w;
      L = fmaf(v.y, w, L);
    }
    L = warp_sum(L);
    const float invL = 1.0f / L;
    __syncwarp();
    for (int s = lane; s < NS; s += 32) wn[j * NS + s] *= invL;
  }
  consumer_sync();
  const size_t sstride = (size_t)grp * hd;  // floats between splits
  for (int e = tid; e < grp * hd; e += kConsumerThreads) {
    const int j = e / hd, d = e - j * hd;
    const float *po = A.part_o + ((size_t)h * NS * grp + j) * hd + d;
    const float *w = wn + j * NS;
    float o0 = 0.f, o1 = 0.f;
    int s = 0;
#pragma unroll 4
    for (; s + 1 < NS; s += 2) {
      o0 = fmaf(w[s], __ldcg(po + s * sstride), o0);
      o1 = fmaf(w[s + 1], __ldcg(po + (s + 1) * sstride), o1);
    }
    if (s < NS) o0 = fmaf(w[s], __ldcg(po + s * sstride), o0);
    A.attn[(size_t)(h * grp + j) * hd + d] = o0 + o1;
  }
}

// All-reduce of one vector across the ranks, inside the step. Each element
// travels as one 64-bit word, the epoch in the high half and the f32 bits
// in the low half, written with a single relaxed system-scope store into
// every rank's receive row for this rank: a receiver that reads the epoch
// in a word has that word's value too, so no fence and no separate flag
// sit between a push and its use (one NVLink crossing). CTA b owns a slice
// of the elements; its threads push their elements, zero them in ar_src,
// then wait (bounded) for every rank's word of each element and add the
// ranks' values in rank order into ar_dst, so ar_dst stays identical on
// all ranks. Receive rows alternate between two parities: a rank pushes
// epoch e + 1 only after it has read every rank's epoch-e words of its
// slice, which every rank wrote after finishing epoch e - 1.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait for the word of epoch e at p (written by another rank);
// false (error flag set to `code`) after limit_ns or once another thread
// has raised the error flag.
__device__ bool wait_word(const unsigned long long *p, unsigned e, unsigned long long *out, int *err,
                          int code, uint64_t limit_ns) {
  uint64_t t0 = 0;
  for (uint32_t spins = 0;; ++spins) {
    const unsigned long long w = ld_relaxed_sys_u64(p);
    if ((unsigned)(w >> 32) == e) {
      *out = w;
      return true;
    }
    if ((spins & 63u) == 63u) {
      if (*(volatile int *)err) return false;
      const uint64_t t = global_ns();
      if (!t0) t0 = t;
      else if (t - t0 > limit_ns) {
        atomicExch(err, code);
        return false;
      }
    }
  }
}

__device__ __noinline__ void phase_allreduce(const MegaArgs &A, const MegaPhase &P, unsigned ar0) {
  const int tid = threadIdx.x, b = blockIdx.x, N = A.nranks, me = A.rank;
  const MegaPeers &pr = A.peers;
  const unsigned e = ar0 + (unsigned)P.ar_index;
  const size_t row = (size_t)pr.row_floats;
  const int n = P.ar_n, per = (n + (int)gridDim.x - 1) / (int)gridDim.x;
  const int lo = min(n, b * per), hi = min(n, lo + per);
  const size_t par_off = (size_t)(e & 1u) * kMaxRanks * row;
  for (int i = lo + tid; i < hi; i += kConsumerThreads) {
    const float v = __ldcg(P.ar_src + i);
    P.ar_src[i] = 0.f;
    const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(v);
    for (int r = 0; r < N; ++r)
      st_relaxed_sys_u64(reinterpret_cast<unsigned long long *>(pr.buf[r]) + par_off + (size_t)me * row + i, w);
  }
  const unsigned long long *rv = reinterpret_cast<const unsigned long long *>(pr.buf[me]) + par_off;
  for (int i = lo + tid; i < hi; i += kConsumerThreads) {
    float t = 0.f;
    for (int r = 0; r < N; ++r) {
      unsigned long long w = 0;
      wait_word(rv + (size_t)r * row + i, e, &w, A.err, 410, pr.wait_ns);  // on failure the step reports it
      const float u = __uint_as_float((unsigned)w);
      t = r == 0 ? u : t + u;
    }
    P.ar_dst[i] += t;
  }
}

// The maximum argmax key over the ranks (one thread of one CTA per rank):
// each rank's key goes to every rank, then each takes the maximum.
__device__ unsigned long long keys_max(const MegaArgs &A, unsigned long long k, unsigned e) {
  const MegaPeers &pr = A.peers;
  const int N = A.nranks, me = A.rank;
  const size_t slot = (size_t)(e & 1u) * kMaxRanks;
  for (int r = 0; r < N; ++r)
    reinterpret_cast<volatile unsigned long long *>(pr.buf[r] + pr.off_keys)[slot + me] = k;
  __threadfence_system();
  for (int r = 0; r < N; ++r) st_release_sys(reinterpret_cast<unsigned *>(pr.buf[r] + pr.off_kflags) + me, e);
  for (int r = 0; r < N; ++r)
    if (!wait_epoch(reinterpret_cast<const unsigned *>(pr.buf[me] + pr.off_kflags) + r, e, A.err, 411,
                    pr.wait_ns))
      return k;
  const volatile unsigned long long *keys =
      reinterpret_cast<const volatile unsigned long long *>(pr.buf[me] + pr.off_keys) + slot;
  for (int r = 0; r < N; ++r) k = keys[r] > k ? keys[r] : k;
  return k;
}

__device__ __noinline__ void phase_argmax(const MegaArgs &A, float *scr) {
  const int tid = threadIdx.x;
  unsigned long long best = 0;
  for (int i = blockIdx.x * kConsumerThreads + tid; i < A.V; i += gridDim.x * kConsumerThreads) {
    const float v = __ldcg(&A.logits[i]);
    if (v != v) continue;
    // the global index (this rank's vocab slice starts at v0)
    const unsigned long long k = ((unsigned long long)ordered_bits(v) << 32) | (unsigned)(i + A.v0);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((tid & 31) == 0 && best) atomicMax(A.amax_key, best);
  consumer_sync();
  __shared__ int last;
  if (tid == 0) {
    __threadfence();
    last = (atomicAdd(A.amax_count, 1) == (int)gridDim.x - 1);
    if (last) {
      __threadfence();
      unsigned long long k = atomicAdd(A.amax_key, 0ull);
      if (A.nranks > 1) {
        // every CTA read the epochs when the step began, grid barriers ago
        k = keys_max(A, k, A.peers.epoch[1] + 1u);
        A.peers.epoch[0] += (unsigned)A.n_ar;
        A.peers.epoch[1] += 1u;
      }
      const uint32_t tok = (uint32_t)(k & 0xffffffffull);
      *A.next_token = tok;
      A.tokens[*A.n_out] = tok;
      *A.n_out = *A.n_out + 1;
      *A.pos = *A.pos + 1;
      *A.amax_key = 0;
      *A.amax_count = 0;
    }
  }
  (void)scr;
}

__global__ void __launch_bounds__(kGemvThreads, 1) decode_mega_kernel(const __grid_constant__ MegaArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty_bar = full_bar + kGemvMaxStages;
  // [0] cached K/V rows of a CTA's first attention item of a layer (fetched
  // by the producer), [1] ranges, [2] cached K/V rows of further items
  uint64_t *xbar = reinterpret_cast<uint64_t *>(smem + kGemvBarBytes);
  MegaPhase *s_ph = reinterpret_cast<MegaPhase *>(smem + A.off_ph);     // two records
  const int2 *s_rg = reinterpret_cast<const int2 *>(smem + A.off_rg);   // this CTA's ranges
  uint32_t *tab = reinterpret_cast<uint32_t *>(smem + A.off_tab);       // ring offsets, lengths
  uint8_t *ring = smem + A.off_ring;
  uint8_t *abuf = smem + A.off_scr;   // attention item buffer
  uint8_t *scr = smem + A.off_stage;  // x staging of the GEMV phases
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the phase the consumers have entered (written by consumer thread 0 after
  // each grid barrier; read by the producer before it refills abuf)
  __shared__ volatile int s_phase;
  if (threadIdx.x == 0) {
    g_xzero = make_uint4(0u, 0u, 0u, 0u);
    s_phase = -1;
    for (int s = 0; s < kRingPos; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 8);
    }
    mbar_init(&xbar[0], 1);
    mbar_init(&xbar[1], 1);
    mbar_init(&xbar[2], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // this CTA's range table
    const uint32_t rg_bytes = (uint32_t)(A.nph_pad * sizeof(int2));
    mbar_arrive_expect_tx(&xbar[1], rg_bytes);
    bulk_g2s(smem + A.off_rg, A.rg + (size_t)blockIdx.x * A.nph_pad, rg_bytes, &xbar[1]);
  }
  if (warp == 1) load_record(&s_ph[0], &A.ph[0], lane);  // the first phase record
  // every thread waits for the range table; the CTA then agrees on the outcome
  // (the barrier also publishes the first record)
  const bool have_rg = __syncthreads_and(mbar_wait(&xbar[1], 0u, A.err, 403)) != 0;
  if (!have_rg) return;

  const int pos = *A.pos;  // this step's position (advanced after the last phase)
  const int nsa = step_splits(A, pos);                // attention splits per kv head this step
  const bool has_item = (int)blockIdx.x < A.G * nsa;  // the CTA's first attention item
  if (warp == kConsumerWarps) {
    // producer: every GEMV phase's units for this CTA, back to back; at each
    // QKV phase, first the cached K/V rows of the CTA's first attention item
    // of that layer (once the consumers have left the previous attention
    // phase, whose items used the buffer)
    if (lane == 0) {
      uint32_t it = 0;
      RingState rs{0u, 0u, 0u};
      const RingTab rt{tab};
      int last_attn = -1, kv_fetches = 0;
      bool ok = true;
      for (int p = 0; p < A.nph && ok; ++p) {
        const MegaPhase &P = A.ph[p];
        if (P.kind == PH_ATTN) last_attn = p;
        if (P.kind != PH_GEMV) continue;
        if (P.attn_prefetch && has_item) {
          uint32_t spins = 0;
          while (s_phase <= last_attn) {
            if (++spins > kSpinLimit || ((spins & 1023u) == 0 && *(volatile int *)A.err)) {
              ok = false;
              break;
            }
            __nanosleep(64);
          }
          if (!ok) break;
          fence_proxy_async_smem();  // the consumers' reads of abuf come before the copy
          attn_fetch(A, P.attn_prefetch - 1, blockIdx.x % A.G, blockIdx.x / A.G, pos, nsa, abuf, &xbar[0]);
          ++kv_fetches;
        }
        const int2 rg = s_rg[p];
        const int n = rg.y - rg.x;
        if (!gemv_produce(P.g, rg.x, n, it, ring, (uint32_t)A.ring_bytes, rt, rs, full_bar,
                          empty_bar, A.err)) {
          ok = false;  // gemv_produce drained its copies
          break;
        }
        it += (uint32_t)n;
      }
      if (ok) ring_drain(full_bar, kRingPos, it);
      // leave no K/V copy in flight (its phase completes when its bytes land)
      if (kv_fetches > 0) mbar_wait(&xbar[0], (uint32_t)(kv_fetches - 1) & 1u, nullptr, 0);
    }
    return;
  }

  uint32_t it = 0;
  int kv_issued = 0, kv_done = 0;  // K/V row fetches of further items (thread 0's view)
  int kv_first = 0;                // producer-fetched first items consumed
  // all-reduces done before this step (advanced by the argmax phase's last CTA)
  const unsigned ar0 = A.nranks > 1 ? *(volatile unsigned *)A.peers.epoch : 0u;
  __shared__ int s_kv_ok, s_last;
  for (int p = 0; p < A.nph; ++p) {
    // the record of phase p is loaded during the barrier into the buffer of
    // phase p - 2, which every consumer finished before the last barrier
    if (p > 0 && !grid_barrier(A.bar, (unsigned)p * gridDim.x, A.err, &s_ph[p & 1], &A.ph[p]))
      break;  // the same answer in every consumer thread
    if (threadIdx.x == 0) s_phase = p;
    const MegaPhase &P = s_ph[p & 1];
    if (P.zero_ptr)
      for (int i = blockIdx.x * kConsumerThreads + threadIdx.x; i < P.zero_n;
           i += gridDim.x * kConsumerThreads)
        P.zero_ptr[i] = 0.f;
    switch (P.kind) {
      case PH_EMBED:
        phase_embed(A);
        break;
      case PH_GEMV: {
        const int2 rg = s_rg[p];
        const int n = rg.y - rg.x;
        if (n > 0) {
          const bool full = n >= P.g.kunits;
          stage_x(P.g, rg.x, n, full, scr);
          consumer_sync();
          // on a failed wait the warp carries on to the next grid barrier,
          // which sees the error flag and ends the CTA's consumers together
          gemv_consume(P.g, rg.x, n, it, ring, tab, full_bar, empty_bar, scr, full, A.err);
          it += (uint32_t)n;
        }
        break;
      }
      case PH_ATTN: {
        const int items = A.G * nsa;
        for (int item = blockIdx.x; item < items; item += gridDim.x) {
          if (threadIdx.x == 0) {
            // the first item's rows were fetched by the producer ahead of the
            // QKV phase; further items' rows are fetched here.
            // A failed wait leaves garbage rows; the next grid barrier then
            // ends the step with the error flag set
            if (item == (int)blockIdx.x) {
              s_kv_ok = mbar_wait(&xbar[0], (uint32_t)kv_first & 1u, A.err, 405);
              ++kv_first;
            } else {
              attn_fetch(A, P.at.layer, item % A.G, item / A.G, pos, nsa, abuf, &xbar[2]);
              ++kv_issued;
              s_kv_ok = mbar_wait(&xbar[2], (uint32_t)kv_done & 1u, A.err, 405);
              ++kv_done;
            }
          }
          consumer_sync();
          const int h = item % A.G;
          if (A.attn_tc == 8)
            attn_item_tc<8>(A, P.at, h, item / A.G, pos, nsa, abuf);
          else if (A.attn_tc)
            attn_item_tc<4>(A, P.at, h, item / A.G, pos, nsa, abuf);
          else
            attn_item(A, P.at, h, item / A.G, pos, nsa, abuf);
          // split-K fixup: the CTA that finishes kv head h's last split
          // combines the head (release by every item, acquire by the last)
          if (threadIdx.x == 0) {
            __threadfence();
            // the counters run over all layers of the step (zeroed per launch)
            s_last = atomicAdd(&A.bar[1 + h], 1u) ==
                     (unsigned)((P.at.layer + 1) * nsa) - 1u;
          }
          consumer_sync();
          if (s_last) {
            __threadfence();
            combine_kv_head(A, h, nsa, reinterpret_cast<float *>(abuf));
            consumer_sync();  // the buffer is reused by the next item
          }
        }
        break;
      }
      case PH_ARGMAX:
        phase_argmax(A, reinterpret_cast<float *>(scr));
        break;
      case PH_ALLREDUCE:
        phase_allreduce(A, P, ar0);
        break;
      default:
        break;
    }
  }
  // leave no K/V copy of this thread in flight
  if (threadIdx.x == 0 && kv_issued > kv_done) mbar_wait(&xbar[2], (uint32_t)kv_done & 1u, nullptr, 0);
  (void)s_kv_ok;
}

}  // namespace

int mega_attn_splits_base(int G, int num_sms) {
  // at most 18 splits per kv head unless the rows demand more: the split
  // combine of the last CTA per kv head grows with the split count (37
  // splits at 4 kv heads per rank made it a 7 us tail per layer)
  return std::max(1, std::min(num_sms / std::max(1, G), 18));
}

int mega_attn_splits(int G, int max_seq, int num_sms) {
  int ns = mega_attn_splits_base(G, num_sms);
  ns = std::max(ns, (max_seq + 79) / 80);  // at most ~80 cached rows per item
  return std::min(ns, kMaxSplitsMega);
}

size_t mega_attn_scratch(int grp, int hd, int max_seq, int nsa) {
  const size_t cap = (size_t)attn_cap(max_seq, nsa);
  const size_t scalar = 2 * cap * hd * 2 + (size_t)grp * hd * 4 + (size_t)grp * cap * 4 + (size_t)grp * 8 + 64;
  // tensor-core items: K, V | q hi/lo [2][W][hd + 8] | scores [W][cap] | p hi/lo [2][W][cap + 8]
  // | stats, W = 4 or 8 head slots per plane
  const size_t W = grp <= 4 ? 4 : 8;
  const size_t tc = 2 * cap * hd * 2 + 2 * W * ((size_t)hd + 8) * 2 + W * cap * 4 +
                    2 * W * (cap + 8) * 2 + W * 8 + 64;
  return std::max(scalar, tc);
}

size_t mega_peer_bytes(int n, int grid, MegaPeers *layout) {
  const size_t row = ((size_t)n + 63) / 64 * 64;  // elements (64-bit words), 512-byte rows
  layout->row_floats = (int)row;
  layout->off_flags = 2 * kMaxRanks * row * sizeof(unsigned long long);
  layout->off_keys = layout->off_flags + ((size_t)grid * kMaxRanks * sizeof(unsigned) + 255) / 256 * 256;
  layout->off_kflags = layout->off_keys + 2 * kMaxRanks * sizeof(unsigned long long);
  return layout->off_kflags + 256;
}

ifx_status mega_finalize(MegaPlan *plan, const std::vector<MegaPhase> &phases, int num_sms) {
  MegaArgs &A = plan->args;
  static_assert(sizeof(MegaPhase) % 16 == 0, "phase records move by bulk copy");
  if (A.H / A.G > kMaxGrp || A.hd % 8 || A.hd > 256 || A.nsa > kMaxSplitsMega)
    return fail(IFX_ERR_UNSUPPORTED, "persistent decode: unsupported head geometry");
  size_t slot = 0, win = 0;
  for (const MegaPhase &p : phases)
    if (p.kind == PH_GEMV) {
      slot = std::max<size_t>(slot, (size_t)p.g.slot_bytes);
      size_t w = (size_t)p.g.win_units * xs_slot_bytes(p.g.kc);  // activation planes, sums
      win = std::max<size_t>(win, w);
    }
  // attention buffer (filled during the QKV phase) and staging area side by side
  const size_t attn_bytes =
      (std::max(mega_attn_scratch(A.H / A.G, A.hd, A.max_seq, A.nsa),
                (size_t)3 * (A.H / A.G) * A.nsa * sizeof(float)) +  // the head combine
       127) & ~(size_t)127;
  const size_t scratch = attn_bytes + win;
  constexpr size_t kCap = 220 * 1024;
  A.nph = (int)phases.size();
  A.nph_pad = (A.nph + 1) & ~1;
  // carve-up: stage barriers | 3 extra barriers | 2 phase records | ranges |
  // ring offsets and lengths | weight ring | scratch
  const size_t off_ph = kGemvBarBytes + 64;
  const size_t off_rg = off_ph + 2 * sizeof(MegaPhase);
  const size_t off_tab = (off_rg + (size_t)A.nph_pad * sizeof(int2) + 15) & ~(size_t)15;
  const size_t off_ring = (off_tab + kGemvTabBytes + 127) & ~(size_t)127;
  // the weight ring takes the rest (units packed back to back), up to
  // kMegaRingBytes: it must hold two of the largest units, and a deeper ring
  // measured slower (the bytes still in flight at a phase boundary delay the
  // staging loads and the grid barrier that come next)
  if (off_ring + scratch + 2 * slot > kCap)
    return fail(IFX_ERR_UNSUPPORTED, "persistent decode: shared memory plan too large");
  const size_t ring = std::max<size_t>(2 * slot, std::min<size_t>(kMegaRingBytes, kCap - off_ring - scratch)) &
                      ~(size_t)127;
  A.ring_bytes = (int)ring;
  A.slot_bytes = (int)slot;
  A.scratch_bytes = (int)scratch;
  A.off_ph = (int)off_ph;
  A.off_rg = (int)off_rg;
  A.off_tab = (int)off_tab;
  A.off_ring = (int)off_ring;
  A.off_scr = (int)(off_ring + ring);
  A.off_stage = (int)(A.off_scr + attn_bytes);
  // per-CTA unit ranges of every phase (zero-length outside GEMV phases)
  std::vector<int2> rg((size_t)num_sms * A.nph_pad, make_int2(0, 0));
  std::vector<int2> sched(num_sms);
  for (int p = 0; p < A.nph; ++p) {
    if (phases[p].kind != PH_GEMV) continue;
    IFX_CUDA(cudaMemcpy(sched.data(), phases[p].g.sched, sizeof(int2) * num_sms,
                        cudaMemcpyDeviceToHost));
    for (int b = 0; b < num_sms; ++b) rg[(size_t)b * A.nph_pad + p] = sched[b];
  }
  IFX_CUDA(cudaMalloc(&plan->d_rg, sizeof(int2) * rg.size()));
  IFX_CUDA(cudaMemcpy(plan->d_rg, rg.data(), sizeof(int2) * rg.size(), cudaMemcpyHostToDevice));
  A.rg = plan->d_rg;
  IFX_CUDA(cudaMalloc(&plan->d_phases, sizeof(MegaPhase) * phases.size()));
  IFX_CUDA(cudaMemcpy(plan->d_phases, phases.data(), sizeof(MegaPhase) * phases.size(),
                      cudaMemcpyHostToDevice));
  A.ph = plan->d_phases;
  plan->smem = (size_t)A.off_scr + scratch;
  plan->grid = num_sms;
  IFX_CUDA(cudaFuncSetAttribute(decode_mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kCap));
  int per_sm = 0;
  IFX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mega_kernel, kGemvThreads,
                                                         plan->smem));
  if (per_sm < 1) return fail(IFX_ERR_UNSUPPORTED, "persistent decode kernel does not fit on an SM");
  return IFX_OK;
}

ifx_status mega_launch(const MegaPlan &plan, cudaStream_t st) {
  IFX_CUDA(cudaMemsetAsync(plan.args.bar, 0, sizeof(unsigned) * (1 + plan.args.G), st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident (grid barriers)
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  IFX_CUDA(cudaLaunchKernelEx(&cfg, decode_mega_kernel, plan.args));
  return IFX_OK;
}

void mega_free(MegaPlan *plan) {
  if (plan->d_phases) cudaFree(plan->d_phases);
  if (plan->d_rg) cudaFree(plan->d_rg);
  plan->d_phases = nullptr;
  plan->d_rg = nullptr;
}

}  // namespace ifx
