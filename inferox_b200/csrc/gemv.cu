// Batch-1 fused dequant GEMV for sm_100a.
//
// Structure (one CTA per SM, 288 threads):
//  * warp 8 lane 0 is the producer: it streams this CTA's contiguous range of
//    weight units (128 rows x kc columns, see qlayout.cuh) from HBM into a
//    shared-memory ring with 1-D bulk async copies (cp.async.bulk, completion
//    on an mbarrier). It starts BEFORE griddepcontrol.wait, so with
//    programmatic dependent launch the weights of this GEMV stream in while
//    the previous kernel drains.
//  * warps 0-7 are consumers: after griddepcontrol.wait they stage f(x)
//    (plain / RMSNorm / SwiGLU) as f16 tensor-core B fragments plus per-group
//    sums in shared memory, then each warp owns one 16-row warp tile of every
//    unit: 128-bit conflict-free shared loads, in-register dequant to f16
//    subnormals (one AND/PRMT per register), mma.m16n8k16 with f32
//    accumulation, and per-group scale/min epilogues in f32.
//  * Batch-1 trick: the MMA's 8 B columns carry one quantisation group each
//    (column n = x restricted to group n, the other groups masked to zero),
//    so one MMA chain yields every group's partial dot at once and the
//    per-group scales are applied once per unit instead of once per chunk.
//  * Rows are accumulated into y with red.global.add.f32: a CTA range may
//    start or end inside a CTA tile; the caller pre-initialises y (zero, or
//    the residual for Wo/W2, which makes the residual add free).
#include <algorithm>
#include <cstring>

#include "gemv.cuh"

namespace ifx {

namespace {

__device__ __forceinline__ float silu_f(float v) {
  // ops.rs:199-209: clamp to [-80, 80], x * 1/(1 + exp(-x))
  float c = fminf(fmaxf(v, -80.0f), 80.0f);
  return v * (1.0f / (1.0f + expf(-c)));
}

__device__ __forceinline__ int find_seg(const GemvArgs &a, int u) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < kGemvMaxSegs; ++i)
    if (i < a.nseg && u >= a.seg[i].unit_begin) s = i;
  return s;
}

struct Acc2 {
  float r0, r1;  // rows g and g+8
};

// ------------------------------------------------------------------ Q4_K --
__device__ __forceinline__ void unit_q4k(const uint8_t *wt, const uint4 *xf, const float *s16,
                                         const uint32_t (&mk)[8], int lane, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3;
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const uint4 *sv = reinterpret_cast<const uint4 *>(wt + 2048);
  // four independent accumulator chains (one per 64-column step); each step
  // only fills its own two group columns, so summing them is exact
  float Ds[4][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f},
                    {0.f, 0.f, 0.f, 0.f}};
  uint4 q[4], xb[8];
#pragma unroll
  for (int s = 0; s < 4; ++s) q[s] = qv[s * 32 + lane];
#pragma unroll
  for (int p = 0; p < 8; ++p) xb[p] = xf[p * 4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t wds[4] = {q[s].x, q[s].y, q[s].z, q[s].w};
#pragma unroll
    for (int p2 = 0; p2 < 2; ++p2) {
      const int pair = 2 * s + p2;  // chunk pair == quant group (32 columns)
      const uint32_t m = mk[pair];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t wd = wds[2 * p2 + e];
        const uint32_t hi = wd >> 8;
        const uint32_t b0 = (e ? xb[pair].z : xb[pair].x) & m;
        const uint32_t b1 = (e ? xb[pair].w : xb[pair].y) & m;
        mma_16816(Ds[s], wd & 0x000F000Fu, wd & 0x00F000F0u, hi & 0x000F000Fu, hi & 0x00F000F0u,
                  b0, b1, Ds[s]);
      }
    }
  }
  float D[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) D[i] = (Ds[0][i] + Ds[1][i]) + (Ds[2][i] + Ds[3][i]);
  // D[0] = (g, group 2c), D[1] = (g, 2c+1), D[2] = (g+8, 2c), D[3] = (g+8, 2c+1)
  const float Sa = s16[4 * c] + s16[4 * c + 1];
  const float Sb = s16[4 * c + 2] + s16[4 * c + 3];
  const int bi = (2 * c) & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 hd = sv[g + 8 * h];
    const float d = h2f((uint16_t)(hd.x & 0xffffu)) * (h ? 1048576.0f : 16777216.0f);
    const float dm = h2f((uint16_t)(hd.x >> 16));
    const uint32_t w0 = hd.y, w1 = hd.z, w2 = hd.w;
    // 6-bit scale/min unpack of dequant.rs:141-149, four groups per word
    const uint32_t sc_lo = w0 & 0x3F3F3F3Fu, mn_lo = w1 & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u);
    const uint32_t mn_hi = ((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u);
    const uint32_t scw = (c < 2) ? sc_lo : sc_hi;
    const uint32_t mnw = (c < 2) ? mn_lo : mn_hi;
    const float sca = (float)((scw >> (8 * bi)) & 0xffu), scb = (float)((scw >> (8 * bi + 8)) & 0xffu);
    const float mna = (float)((mnw >> (8 * bi)) & 0xffu), mnb = (float)((mnw >> (8 * bi + 8)) & 0xffu);
    float r = h ? acc.r1 : acc.r0;
    r = fmaf(d * sca, D[2 * h + 0], r);
    r = fmaf(-(dm * mna), Sa, r);
    r = fmaf(d * scb, D[2 * h + 1], r);
    r = fmaf(-(dm * mnb), Sb, r);
    if (h) acc.r1 = r; else acc.r0 = r;
  }
}

// ------------------------------------------------------------------ Q6_K --
__device__ __forceinline__ void unit_q6k(const uint8_t *wt, const uint4 *xf, const float *s16,
                                         const uint32_t (&mk)[8], int lane, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3;
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const uint4 *hv = reinterpret_cast<const uint4 *>(wt + 2048);
  // eight independent chains: {low plane, 2-bit plane} x set (chunks 0-7 /
  // 8-15) x chunk parity; parities fill disjoint columns, so they add exactly
  float DLp[2][2][4], DHp[2][2][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int i = 0; i < 4; ++i) DLp[a][b][i] = DHp[a][b][i] = 0.f;
  uint4 q[4], hq[2];
#pragma unroll
  for (int s = 0; s < 4; ++s) q[s] = qv[s * 32 + lane];
#pragma unroll
  for (int t = 0; t < 2; ++t) hq[t] = hv[t * 32 + lane];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t wds[4] = {q[s].x, q[s].y, q[s].z, q[s].w};
    const uint4 hh = hq[s >> 1];
    const uint32_t hws[4] = {hh.x, hh.y, hh.z, hh.w};
#pragma unroll
    for (int p2 = 0; p2 < 2; ++p2) {
      const int pair = 2 * s + p2;
      const uint4 xb = xf[pair * 4];
      const uint32_t Hw = hws[pair & 3];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int ch = 2 * pair + e;  // 16-column group index 0..15
        const int set = ch >> 3, col = ch & 7;
        const uint32_t m = mk[col];
        const uint32_t wd = wds[2 * p2 + e];
        const uint32_t hi = wd >> 8;
        const uint32_t b0 = (e ? xb.z : xb.x) & m;
        const uint32_t b1 = (e ? xb.w : xb.y) & m;
        const uint32_t H = e ? (Hw >> 8) : Hw;
        const uint32_t H4 = H >> 4;
        mma_16816(DLp[set][e], wd & 0x000F000Fu, wd & 0x00F000F0u, hi & 0x000F000Fu,
                  hi & 0x00F000F0u, b0, b1, DLp[set][e]);
        mma_16816(DHp[set][e], H & 0x00030003u, H & 0x000C000Cu, H4 & 0x00030003u,
                  H4 & 0x000C000Cu, b0, b1, DHp[set][e]);
      }
    }
  }
  float DL[2][4], DH[2][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      DL[a][i] = DLp[a][0][i] + DLp[a][1][i];
      DH[a][i] = DHp[a][0][i] + DHp[a][1][i];
    }
  const uint8_t *scb = wt + 3072;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = g + 8 * h;
    const float d = h2f(*reinterpret_cast<const uint16_t *>(scb + 256 + 2 * row));
    const uint4 sv = *reinterpret_cast<const uint4 *>(scb + 16 * row);
    // scales for groups 2c, 2c+1 (set 0) and 8+2c, 9+2c (set 1)
    const uint32_t w_lo = (c < 2) ? sv.x : sv.y;
    const uint32_t w_hi = (c < 2) ? sv.z : sv.w;
    const int sh = 16 * (c & 1);
    float r = h ? acc.r1 : acc.r0;
#pragma unroll
    for (int set = 0; set < 2; ++set) {
      const uint32_t sw = set ? w_hi : w_lo;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int grp = 8 * set + 2 * c + j;
        const float sc = (float)((sw >> (sh + 8 * j)) & 0xffu);
        const float lo = DL[set][2 * h + j], hv2 = DH[set][2 * h + j];
        const float dot = h ? (lo + 64.0f * hv2) * 1048576.0f : (lo + 16.0f * hv2) * 16777216.0f;
        r = fmaf(d * sc, dot - 32.0f * s16[grp], r);
      }
    }
    if (h) acc.r1 = r; else acc.r0 = r;
  }
}

// ------------------------------------------------------- Q4_0 and Q8_0 --
// Generic (runtime chunk count) paths; used by the tiny config and tests.
__device__ __forceinline__ void unit_q4_0(const uint8_t *wt, int kc, int wt_qbytes,
                                          const uint4 *xf, const float *s16, int lane, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3;
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const int nsteps = kc / 64, nb = kc / 32;
  float D[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int s = 0; s < nsteps; ++s) {
    const uint4 q = qv[s * 32 + lane];
    const uint32_t wds[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int p2 = 0; p2 < 2; ++p2) {
      const int pair = 2 * s + p2;
      const uint4 xb = xf[pair * 4];
      const uint32_t m = (g == pair) ? 0xffffffffu : 0u;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t wd = wds[2 * p2 + e];
        const uint32_t hi = wd >> 8;
        mma_16816(D, wd & 0x000F000Fu, wd & 0x00F000F0u, hi & 0x000F000Fu, hi & 0x00F000F0u,
                  (e ? xb.z : xb.x) & m, (e ? xb.w : xb.y) & m, D);
      }
    }
  }
  const uint8_t *sc = wt + wt_qbytes;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = g + 8 * h;
    float r = h ? acc.r1 : acc.r0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int blk = 2 * c + j;
      if (blk < nb) {
        const float d = h2f(*reinterpret_cast<const uint16_t *>(sc + (row * nb + blk) * 2));
        const float S = s16[2 * blk] + s16[2 * blk + 1];
        const float T = D[2 * h + j] * (h ? 1048576.0f : 16777216.0f);
        r = fmaf(d, T - 8.0f * S, r);
      }
    }
    if (h) acc.r1 = r; else acc.r0 = r;
  }
}

__device__ __forceinline__ void unit_q8_0(const uint8_t *wt, int kc, int wt_qbytes,
                                          const uint4 *xf, const float *s16, int lane, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3;
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const int nb = kc / 32;
  float D[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int s = 0; s < nb; ++s) {  // chunk pair s == block s
    const uint4 q = qv[s * 32 + lane];
    const uint4 xb = xf[s * 4];
    const uint32_t m = (g == s) ? 0xffffffffu : 0u;
    mma_16816(D, prmt(q.x, 0u, 0x4140u), prmt(q.x, 0u, 0x4342u), prmt(q.y, 0u, 0x4140u),
              prmt(q.y, 0u, 0x4342u), xb.x & m, xb.y & m, D);
    mma_16816(D, prmt(q.z, 0u, 0x4140u), prmt(q.z, 0u, 0x4342u), prmt(q.w, 0u, 0x4140u),
              prmt(q.w, 0u, 0x4342u), xb.z & m, xb.w & m, D);
  }
  const uint8_t *sc = wt + wt_qbytes;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = g + 8 * h;
    float r = h ? acc.r1 : acc.r0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int blk = 2 * c + j;
      if (blk < nb) {
        const float d = h2f(*reinterpret_cast<const uint16_t *>(sc + (row * nb + blk) * 2));
        const float S = s16[2 * blk] + s16[2 * blk + 1];
        r = fmaf(d, D[2 * h + j] * 16777216.0f - 128.0f * S, r);
      }
    }
    if (h) acc.r1 = r; else acc.r0 = r;
  }
}

// Consumer-side input staging: f(x) as f16 B fragments + 16-column sums.
__device__ void stage_x(const GemvArgs &a, int u0, int n, bool full, uint8_t *xw, float *s16) {
  const int tid = threadIdx.x;  // 0..255
  const int nslots = full ? a.kunits : n;
  float inv = 1.0f;
  if (a.mode == GEMV_RMSNORM) {
    __shared__ float red[8];
    float ss = 0.f;
    for (int k = tid; k < a.K; k += 256) {
      const float v = a.x[k];
      ss += v * v;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    inv = 1.0f / sqrtf(tot / (float)a.K + a.eps);
  }
  auto fx = [&](int k) -> float {
    if (a.mode == GEMV_RMSNORM) return (a.x[k] * inv) * a.normw[k];
    if (a.mode == GEMV_SWIGLU) return silu_f(a.x[k]) * a.x2[k];
    return a.x[k];
  };
  auto slot_kunit = [&](int j) -> int {
    if (full) return j;
    const int u = u0 + j;
    const int s = find_seg(a, u);
    return (u - a.seg[s].unit_begin) % a.kunits;
  };
  const int ent = a.kc / 8;  // 16-byte entries per slot
  for (int e = tid; e < nslots * ent; e += 256) {
    const int j = e / ent, q = e % ent, p = q >> 2, c = q & 3;
    const int k0 = slot_kunit(j) * a.kc + 32 * p + 2 * c;
    __half2 h0 = __floats2half2_rn(fx(k0), fx(k0 + 1));
    __half2 h1 = __floats2half2_rn(fx(k0 + 8), fx(k0 + 9));
    __half2 h2 = __floats2half2_rn(fx(k0 + 16), fx(k0 + 17));
    __half2 h3 = __floats2half2_rn(fx(k0 + 24), fx(k0 + 25));
    uint4 v;
    v.x = *reinterpret_cast<uint32_t *>(&h0);
    v.y = *reinterpret_cast<uint32_t *>(&h1);
    v.z = *reinterpret_cast<uint32_t *>(&h2);
    v.w = *reinterpret_cast<uint32_t *>(&h3);
    reinterpret_cast<uint4 *>(xw)[(j * (a.kc / 32) + p) * 4 + c] = v;
  }
  const int g16 = a.kc / 16;
  for (int e = tid; e < nslots * g16; e += 256) {
    const int j = e / g16, h = e % g16;
    const int k0 = slot_kunit(j) * a.kc + 16 * h;
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < 16; ++t) s += __half2float(__float2half_rn(fx(k0 + t)));
    s16[e] = s;
  }
}

__global__ void __launch_bounds__(kGemvThreads, 2) gemv_b1_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty_bar = full_bar + kGemvMaxStages;
  uint8_t *ring = smem + 128;
  uint8_t *xw = ring + (size_t)a.nstages * a.slot_bytes;
  float *s16 = reinterpret_cast<float *>(xw + (size_t)a.win_units * a.kc * 2);

  const int2 rg = a.sched[blockIdx.x];
  const int u0 = rg.x, n = rg.y - rg.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = a.nstages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 8);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 8) {
    // ---------------- producer: weights only, safe before griddepcontrol.wait
    if (lane == 0) {
      for (int i = 0; i < n; ++i) {
        const int st = i % NS;
        const uint32_t ph = (uint32_t)(i / NS) & 1u;
        if (i >= NS && !mbar_wait(&empty_bar[st], ph ^ 1u, a.err, 101)) break;
        const int u = u0 + i;
        const int sg = find_seg(a, u);
        const GemvSeg &S = a.seg[sg];
        const uint8_t *src = S.w + (size_t)(u - S.unit_begin) * S.unit_bytes;
        mbar_arrive_expect_tx(&full_bar[st], (uint32_t)S.unit_bytes);
        bulk_g2s(ring + (size_t)st * a.slot_bytes, src, (uint32_t)S.unit_bytes, &full_bar[st]);
      }
    }
    return;
  }

  // ---------------- consumers
  pdl_wait();
  pdl_launch();
  if (a.zero_ptr)
    for (int i = blockIdx.x * 256 + threadIdx.x; i < a.zero_n; i += gridDim.x * 256)
      a.zero_ptr[i] = 0.f;
  if (n <= 0) return;
  const bool full = n >= a.kunits;
  stage_x(a, u0, n, full, xw, s16);
  asm volatile("bar.sync 1, 256;" ::: "memory");

  const int g = lane >> 2, c = lane & 3;
  uint32_t mk[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mk[i] = (g == i) ? 0xffffffffu : 0u;

  Acc2 acc{0.f, 0.f};
  int sg = find_seg(a, u0);
  int local = u0 - a.seg[sg].unit_begin;
  for (int i = 0; i < n; ++i) {
    const int st = i % NS;
    const uint32_t ph = (uint32_t)(i / NS) & 1u;
    const GemvSeg &S = a.seg[sg];
    const int kunit = local % a.kunits;
    const int slot = full ? kunit : i;
    if (!mbar_wait(&full_bar[st], ph, a.err, 102)) return;
    const uint8_t *wt = ring + (size_t)st * a.slot_bytes + (size_t)warp * S.wt_bytes;
    const uint4 *xf = reinterpret_cast<const uint4 *>(xw) + (size_t)slot * (a.kc / 32) * 4 + c;
    const float *sl = s16 + (size_t)slot * (a.kc / 16);
    switch (S.type) {
      case IFX_TYPE_Q4_K: unit_q4k(wt, xf, sl, mk, lane, acc); break;
      case IFX_TYPE_Q6_K: unit_q6k(wt, xf, sl, mk, lane, acc); break;
      case IFX_TYPE_Q4_0: unit_q4_0(wt, a.kc, S.wt_qbytes, xf, sl, lane, acc); break;
      case IFX_TYPE_Q8_0: unit_q8_0(wt, a.kc, S.wt_qbytes, xf, sl, lane, acc); break;
      default: break;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);

    // advance; flush when the CTA tile (or segment) changes or the range ends
    const int ctile = local / a.kunits;
    int nsg = sg, nlocal = local + 1;
    if (sg + 1 < a.nseg && u0 + i + 1 >= a.seg[sg + 1].unit_begin) {
      nsg = sg + 1;
      nlocal = 0;
    }
    const bool flush = (i == n - 1) || nsg != sg || (nlocal / a.kunits) != ctile;
    if (flush) {
      float r0 = acc.r0, r1 = acc.r1;
      r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
      r0 += __shfl_xor_sync(0xffffffffu, r0, 2);
      r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
      r1 += __shfl_xor_sync(0xffffffffu, r1, 2);
      if (c == 0) {
        const int row = ctile * kCtaRows + warp * 16 + g;
        if (row < S.rows) red_add_f32(S.y + row, r0);
        if (row + 8 < S.rows) red_add_f32(S.y + row + 8, r1);
      }
      acc.r0 = acc.r1 = 0.f;
    }
    sg = nsg;
    local = nlocal;
  }
}

}  // namespace

ifx_status gemv_plan(const QMatrix *const *mats, float *const *ys, int nseg, int mode,
                     const float *x, const float *x2, const float *normw, float eps, int *err,
                     GemvPlan *plan) {
  if (nseg < 1 || nseg > kGemvMaxSegs) return fail(IFX_ERR_INVALID_ARGUMENT, "gemv: nseg");
  GemvArgs a{};
  a.nseg = nseg;
  a.kc = mats[0]->L.kc;
  a.kunits = mats[0]->L.kunits;
  a.K = (int)mats[0]->L.cols;
  std::vector<int64_t> seg_units(nseg), seg_bytes(nseg);
  int64_t total_units = 0;
  int slot = 0;
  uint64_t wbytes = 0;
  for (int i = 0; i < nseg; ++i) {
    const QLayout &L = mats[i]->L;
    if (L.kc != a.kc || L.cols != a.K)
      return fail(IFX_ERR_SHAPE, "gemv: segments must share K and unit width");
    GemvSeg &S = a.seg[i];
    S.w = mats[i]->d;
    S.y = ys[i];
    S.type = L.type;
    S.rows = (int)L.rows;
    S.unit_bytes = L.unit_bytes;
    S.wt_bytes = L.wt_bytes;
    S.wt_qbytes = L.wt_qbytes;
    S.unit_begin = (int)total_units;
    seg_units[i] = (int64_t)L.ctiles * L.kunits;
    total_units += seg_units[i];
    slot = std::max(slot, L.unit_bytes);
    wbytes += mats[i]->gguf_bytes();
  }
  if (total_units >= (1ll << 31)) return fail(IFX_ERR_SHAPE, "gemv: too many units");
  a.mode = mode;
  a.x = x;
  a.x2 = x2;
  a.normw = normw;
  a.eps = eps;
  a.err = err;
  a.slot_bytes = slot;
  a.nstages = std::min(kGemvMaxStages, std::max(2, kGemvRingBytes / slot));

  // byte-balanced contiguous ranges, one per CTA
  const int G = (int)std::min<int64_t>(kNumSMs, total_units);
  std::vector<int64_t> cum(total_units + 1, 0);
  {
    int64_t u = 0;
    for (int i = 0; i < nseg; ++i)
      for (int64_t k = 0; k < seg_units[i]; ++k, ++u) cum[u + 1] = cum[u] + a.seg[i].unit_bytes;
  }
  std::vector<int2> sched(G);
  int64_t prev = 0;
  int win = 1;
  for (int b = 0; b < G; ++b) {
    int64_t target = (cum[total_units] * (b + 1)) / G;
    int64_t e = (b == G - 1) ? total_units
                             : (int64_t)(std::lower_bound(cum.begin(), cum.end(), target) - cum.begin());
    e = std::max<int64_t>(e, prev);
    if (b < G - 1 && e == prev && prev < total_units) e = prev + 1;
    sched[b] = make_int2((int)prev, (int)e);
    const int n = (int)(e - prev);
    win = std::max(win, n >= a.kunits ? a.kunits : n);
    prev = e;
  }
  a.win_units = win;
  IFX_CUDA(cudaMalloc(&plan->d_sched, sizeof(int2) * G));
  IFX_CUDA(cudaMemcpy(plan->d_sched, sched.data(), sizeof(int2) * G, cudaMemcpyHostToDevice));
  a.sched = plan->d_sched;
  plan->args = a;
  plan->grid = G;
  plan->smem = 128 + (size_t)a.nstages * a.slot_bytes + (size_t)win * (a.kc * 2 + a.kc / 16 * 4);
  plan->weight_bytes = wbytes;
  static bool attr_set = false;
  if (!attr_set) {
    IFX_CUDA(cudaFuncSetAttribute(gemv_b1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  200 * 1024));
    attr_set = true;
  }
  if (plan->smem > 200 * 1024) return fail(IFX_ERR_SHAPE, "gemv: shared memory plan too large");
  return IFX_OK;
}

void gemv_plan_rebind(GemvPlan *plan, const QMatrix *const *mats, float *const *ys,
                      const float *x, const float *x2, const float *normw) {
  for (int i = 0; i < plan->args.nseg; ++i) {
    plan->args.seg[i].w = mats[i]->d;
    plan->args.seg[i].y = ys[i];
  }
  plan->args.x = x;
  plan->args.x2 = x2;
  plan->args.normw = normw;
}

void gemv_plan_free(GemvPlan *plan) {
  if (plan->d_sched) cudaFree(plan->d_sched);
  plan->d_sched = nullptr;
}

ifx_status gemv_launch(const GemvPlan &plan, cudaStream_t stream, bool pdl) {
  IFX_CUDA(launch(gemv_b1_kernel, dim3(plan.grid), dim3(kGemvThreads), plan.smem, stream, pdl,
                  plan.args));
  return IFX_OK;
}

}  // namespace ifx
