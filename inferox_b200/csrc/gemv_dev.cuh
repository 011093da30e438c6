// Device-side building blocks of the fused dequant GEMV, shared by the
// standalone GEMV kernel (gemv.cu) and the persistent decode kernel
// (decode_mega.cu): per-type unit consumers (mma.m16n8k16 over the
// fragment-ordered layout of qlayout.cuh) and the activation staging.
#pragma once
#include "gemv.cuh"

namespace ifx {
namespace gemvdev {

// 16 zero bytes in shared memory (set by the kernels at start): the B
// fragment of a lane whose MMA column is not the current quantisation group
// is loaded from here instead of being masked after the load.
__shared__ uint4 g_xzero;

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

// (float)v for 0 <= v < 2^23 without the conversion pipe: place v in the
// mantissa of 2^23 and subtract 2^23 (both steps exact).
__device__ __forceinline__ float u2f_small(uint32_t v) {
  return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}
// A scale byte v as u8 (smask 0) or int8 (smask 0x80): (v ^ smask) placed in
// the mantissa of 2^23, minus bias = 2^23 + smask (both exact).
__device__ __forceinline__ float sc2f(uint32_t v, uint32_t smask, float bias) {
  return __uint_as_float(0x4B000000u | (v ^ smask)) - bias;
}

struct Acc2 {
  float r0, r1;  // rows g and g+8
};

// x is staged as two f16 planes, x ~= hi + lo (hi = f16(x), lo = f16(x - hi)),
// `xlo` uint4s after the hi plane; the integer weights are exact in f16, so
// A.hi + A.lo carries x to about 22 bits and the products to f32 accuracy.
//
// Column layout of every MMA below: a k-step covers one quantisation group,
// and of the eight B columns only two are non-zero: column (group & 3)
// carries the hi plane and column (group & 3) + 4 the lo plane, so one MMA
// takes both planes. An accumulator therefore holds at most four groups;
// groups 0-3 and 4-7 of a unit go to different accumulators (E and F), and
// fold_hilo adds the hi and lo columns of each group across lanes c and
// c ^ 2. Lane g loads its B fragment from the hi plane (g < 4) or the lo
// plane (g >= 4) when g & 3 is the group's column, and from the shared zero
// vector otherwise.
__device__ __forceinline__ const uint4 *xplane(const uint4 *xf, int xlo, int g) {
  return g < 4 ? xf : xf + xlo;
}

// E: groups 0-3 (hi in columns 0-3, lo in 4-7); F: groups 4-7, likewise.
// Returns in lane c = lane & 3 the totals of groups 2c and 2c + 1 for rows
// g (D[0], D[1]) and g + 8 (D[2], D[3]), the C-fragment layout of a single
// group-per-column accumulation.
__device__ __forceinline__ void fold_hilo(const float (&E)[4], const float (&F)[4], int c,
                                          float (&D)[4]) {
  const bool lowc = c < 2;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float recv = __shfl_xor_sync(0xffffffffu, lowc ? F[i] : E[i], 2);
    D[i] = (lowc ? E[i] : F[i]) + recv;
  }
}

// ------------------------------------------------------------------ Q4_K --
__device__ __forceinline__ void unit_q4k(const uint8_t *wt, const uint4 *xf, int xlo,
                                         const float *s16, int lane, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3, gq = g & 3;
  const uint4 *xp = xplane(xf, xlo, g);
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const uint4 *sv = reinterpret_cast<const uint4 *>(wt + 2048);
  // four independent accumulator chains, one per 64-column step (two
  // groups); steps 0-1 hold groups 0-3, steps 2-3 groups 4-7
  float Ds[4][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f},
                    {0.f, 0.f, 0.f, 0.f}};
  uint4 q[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) q[s] = qv[s * 32 + lane];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t wds[4] = {q[s].x, q[s].y, q[s].z, q[s].w};
#pragma unroll
    for (int p2 = 0; p2 < 2; ++p2) {
      const int grp = 2 * s + p2;  // chunk pair == quant group (32 columns)
      const uint4 xb = *(gq == (grp & 3) ? xp + grp * 4 : &g_xzero);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t wd = wds[2 * p2 + e];
        const uint32_t hi = wd >> 8;
        const uint32_t a0 = wd & 0x000F000Fu, a1 = wd & 0x00F000F0u;
        const uint32_t a2 = hi & 0x000F000Fu, a3 = hi & 0x00F000F0u;
        mma_16816(Ds[s], a0, a1, a2, a3, e ? xb.z : xb.x, e ? xb.w : xb.y, Ds[s]);
      }
    }
  }
  float E[4], F[4], D[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // disjoint columns: these sums are exact
    E[i] = Ds[0][i] + Ds[1][i];
    F[i] = Ds[2][i] + Ds[3][i];
  }
  fold_hilo(E, F, c, D);
  // D[0] = (g, group 2c), D[1] = (g, 2c+1), D[2] = (g+8, 2c), D[3] = (g+8, 2c+1)
  const float Sa = s16[4 * c] + s16[4 * c + 1];
  const float Sb = s16[4 * c + 2] + s16[4 * c + 3];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 hd = sv[g + 8 * h];
    // repacked header (repack.cu): word c = this lane's 24-bit scale/min field
    // | byte c of (d, dmin) in the top byte
    const float d = h2f((uint16_t)prmt(hd.x, hd.y, 0x0073u)) * (h ? 1048576.0f : 16777216.0f);
    const float dm = h2f((uint16_t)prmt(hd.z, hd.w, 0x0073u));
    const uint32_t f = (c & 2) ? ((c & 1) ? hd.w : hd.z) : ((c & 1) ? hd.y : hd.x);
    const float sca = u2f_small(f & 63u), scb = u2f_small((f >> 6) & 63u);
    const float mna = u2f_small((f >> 12) & 63u), mnb = u2f_small((f >> 18) & 63u);
    float r = h ? acc.r1 : acc.r0;
    r = fmaf(d * sca, D[2 * h + 0], r);
    r = fmaf(-(dm * mna), Sa, r);
    r = fmaf(d * scb, D[2 * h + 1], r);
    r = fmaf(-(dm * mnb), Sb, r);
    if (h) acc.r1 = r; else acc.r0 = r;
  }
}

// ------------------------------------------------------------------ Q6_K --
// Sixteen 16-column groups per unit; accumulator set t = chunk >> 2 holds
// chunks 4t..4t+3 (hi columns 0-3, lo columns 4-7), one set per 64-column
// step, separately for the low-nibble plane (DL) and the 2-bit plane (DH).
// smask 0x80 reads the scale bytes as int8 (llama.cpp), 0 as u8 (the
// reference): (b ^ smask) - smask.
__device__ __forceinline__ void unit_q6k(const uint8_t *wt, const uint4 *xf, int xlo,
                                         const float *s16, int lane, uint32_t smask, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3, gq = g & 3;
  const uint4 *xp = xplane(xf, xlo, g);
  const uint2 *zero2 = reinterpret_cast<const uint2 *>(&g_xzero);
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const uint4 *hv = reinterpret_cast<const uint4 *>(wt + 2048);
  float DL[4][4], DH[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int i = 0; i < 4; ++i) DL[a][i] = DH[a][i] = 0.f;
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
      const uint32_t Hw = hws[pair & 3];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int ch = 2 * pair + e;  // 16-column group index 0..15; set = s
        const uint2 xb =
            *(gq == (ch & 3) ? reinterpret_cast<const uint2 *>(xp + pair * 4) + e : zero2);
        const uint32_t wd = wds[2 * p2 + e];
        const uint32_t hi = wd >> 8;
        const uint32_t H = e ? (Hw >> 8) : Hw;
        const uint32_t H4 = H >> 4;
        const uint32_t a0 = wd & 0x000F000Fu, a1 = wd & 0x00F000F0u;
        const uint32_t a2 = hi & 0x000F000Fu, a3 = hi & 0x00F000F0u;
        const uint32_t h0 = H & 0x00030003u, h1 = H & 0x000C000Cu;
        const uint32_t h2 = H4 & 0x00030003u, h3 = H4 & 0x000C000Cu;
        mma_16816(DL[s], a0, a1, a2, a3, xb.x, xb.y, DL[s]);
        mma_16816(DH[s], h0, h1, h2, h3, xb.x, xb.y, DH[s]);
      }
    }
  }
  // q = low + 16 * high; rows g + 8 carry both planes scaled by 16 and 4
  float T[4][4];
#pragma unroll
  for (int t = 0; t < 4; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i)
      T[t][i] = i < 2 ? (DL[t][i] + 16.0f * DH[t][i]) * 16777216.0f
                      : (DL[t][i] + 64.0f * DH[t][i]) * 1048576.0f;
  // U[0]: chunks 2c, 2c+1 (sets 0, 1); U[1]: chunks 8+2c, 9+2c (sets 2, 3)
  float U[2][4];
  fold_hilo(T[0], T[1], c, U[0]);
  fold_hilo(T[2], T[3], c, U[1]);
  const uint8_t *scb = wt + 3072;
  const float sbias = 8388608.0f + (float)smask;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = g + 8 * h;
    const float d = h2f(*reinterpret_cast<const uint16_t *>(scb + 256 + 2 * row));
    const uint4 sv = *reinterpret_cast<const uint4 *>(scb + 16 * row);
    // scales for groups 2c, 2c+1 (chunks 0-7) and 8+2c, 9+2c (chunks 8-15)
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
        const float sc = sc2f((sw >> (sh + 8 * j)) & 0xffu, smask, sbias);
        r = fmaf(d * sc, U[set][2 * h + j] - 32.0f * s16[grp], r);
      }
    }
    if (h) acc.r1 = r; else acc.r0 = r;
  }
}

// ------------------------------------------------------- Q4_0 and Q8_0 --
// Runtime chunk count (kc <= 256: at most eight 32-column blocks per unit).
__device__ __forceinline__ void unit_q4_0(const uint8_t *wt, int kc, int wt_qbytes,
                                          const uint4 *xf, int xlo, const float *s16, int lane,
                                          Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3, gq = g & 3;
  const uint4 *xp = xplane(xf, xlo, g);
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const int nsteps = kc / 64, nb = kc / 32;
  float E[4] = {0.f, 0.f, 0.f, 0.f}, F[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    if (s < nsteps) {
      const uint4 q = qv[s * 32 + lane];
      const uint32_t wds[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int p2 = 0; p2 < 2; ++p2) {
        const int blk = 2 * s + p2;
        const uint4 xb = *(gq == (blk & 3) ? xp + blk * 4 : &g_xzero);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const uint32_t wd = wds[2 * p2 + e];
          const uint32_t hi = wd >> 8;
          const uint32_t a0 = wd & 0x000F000Fu, a1 = wd & 0x00F000F0u;
          const uint32_t a2 = hi & 0x000F000Fu, a3 = hi & 0x00F000F0u;
          if (s < 2) mma_16816(E, a0, a1, a2, a3, e ? xb.z : xb.x, e ? xb.w : xb.y, E);
          else mma_16816(F, a0, a1, a2, a3, e ? xb.z : xb.x, e ? xb.w : xb.y, F);
        }
      }
    }
  }
  float D[4];
  fold_hilo(E, F, c, D);
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
                                          const uint4 *xf, int xlo, const float *s16, int lane,
                                          Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3, gq = g & 3;
  const uint4 *xp = xplane(xf, xlo, g);
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const int nb = kc / 32;
  float E[4] = {0.f, 0.f, 0.f, 0.f}, F[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < 8; ++s) {  // chunk pair s == block s
    if (s < nb) {
      const uint4 q = qv[s * 32 + lane];
      const uint4 xb = *(gq == (s & 3) ? xp + s * 4 : &g_xzero);
      const uint32_t a0 = prmt(q.x, 0u, 0x4140u), a1 = prmt(q.x, 0u, 0x4342u);
      const uint32_t a2 = prmt(q.y, 0u, 0x4140u), a3 = prmt(q.y, 0u, 0x4342u);
      const uint32_t a4 = prmt(q.z, 0u, 0x4140u), a5 = prmt(q.z, 0u, 0x4342u);
      const uint32_t a6 = prmt(q.w, 0u, 0x4140u), a7 = prmt(q.w, 0u, 0x4342u);
      if (s < 4) {
        mma_16816(E, a0, a1, a2, a3, xb.x, xb.y, E);
        mma_16816(E, a4, a5, a6, a7, xb.z, xb.w, E);
      } else {
        mma_16816(F, a0, a1, a2, a3, xb.x, xb.y, F);
        mma_16816(F, a4, a5, a6, a7, xb.z, xb.w, F);
      }
    }
  }
  float D[4];
  fold_hilo(E, F, c, D);
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

constexpr int kConsumerWarps = kGemvThreads / 32 - 1;
constexpr int kConsumerThreads = kConsumerWarps * 32;

// Named barrier over the consumer warps only (the producer warp has left).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory");
}

// One segment's fields, held in registers by the loops below. Reading
// GemvArgs through a reference (a __grid_constant__ parameter, or a phase
// record in global memory) inside a loop turns every field into a load that
// the mbarrier asm statements' memory clobbers force to be repeated; the
// loops therefore only touch these copies and re-read GemvArgs when a
// segment boundary is crossed.
struct SegView {
  const uint8_t *w;
  float *y;
  int type, rows, unit_bytes, wt_bytes, wt_qbytes, begin, units;  // type as in GemvSeg
};

__device__ __forceinline__ SegView load_seg(const GemvArgs &a, int s) {
  const GemvSeg &S = a.seg[s];
  return SegView{S.w, S.y, S.type, S.rows, S.unit_bytes, S.wt_bytes, S.wt_qbytes, S.unit_begin,
                 S.units};
}

// Consumer-side input staging: f(x) as f16 B fragments + 16-column sums.
// Every global read is a coalesced float4 issued up front. When the staged
// columns fit in one pass (up to 2 float4 per thread: K <= 4096 for a full
// CTA range) all loads go out in one round, the RMSNorm sum of squares is
// taken from those same values (or from one extra set of loads issued in the
// same round), and the normalised values are formed from registers after a
// single consumer barrier.
static __device__ __forceinline__ void emit_x4(float (&y)[4], bool valid, int f, int per_slot,
                                               int kc, __half *xh, float *s16, int tid, int xlo) {
  const __half2 h01 = __floats2half2_rn(y[0], y[1]), h23 = __floats2half2_rn(y[2], y[3]);
  const __half2 l01 = __floats2half2_rn(y[0] - __low2float(h01), y[1] - __high2float(h01));
  const __half2 l23 = __floats2half2_rn(y[2] - __low2float(h23), y[3] - __high2float(h23));
  // the 16-column sum of the values the MMAs see (hi + lo): 4 lanes per group
  float s = ((__low2float(h01) + __low2float(l01)) + (__high2float(h01) + __high2float(l01))) +
            ((__low2float(h23) + __low2float(l23)) + (__high2float(h23) + __high2float(l23)));
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  if (valid) {
    const int j = f / per_slot, o = (f % per_slot) * 4;  // o: column within the slot
    const int p = o / 32, rr = o % 32, hh = rr / 16, ss = rr % 16;  // ss = 0,4,8,12
    // element ss at half index ((j*kc/32 + p)*4 + c)*8 + hh*4 + (ss/8)*2 + ss%2
    const int c0 = (ss % 8) / 2;
    const size_t ent = ((size_t)(j * (kc / 32) + p) * 4) * 8 + hh * 4 + (ss / 8) * 2;
    *reinterpret_cast<__half2 *>(xh + ent + (size_t)c0 * 8) = h01;
    *reinterpret_cast<__half2 *>(xh + ent + (size_t)(c0 + 1) * 8) = h23;
    *reinterpret_cast<__half2 *>(xh + (size_t)xlo * 8 + ent + (size_t)c0 * 8) = l01;
    *reinterpret_cast<__half2 *>(xh + (size_t)xlo * 8 + ent + (size_t)(c0 + 1) * 8) = l23;
    if ((tid & 3) == 0) s16[j * (kc / 16) + o / 16] = s;
  }
}

static __device__ __noinline__ void stage_x(const GemvArgs &a, int u0, int n, bool full, uint8_t *xw, float *s16) {
  const int tid = threadIdx.x;  // 0..kConsumerThreads-1
  constexpr int T = kConsumerThreads;
  const int mode = a.mode, K = a.K, kc = a.kc, kunits = a.kunits, nseg = a.nseg;
  const float4 *x4 = reinterpret_cast<const float4 *>(a.x);
  const float4 *w4 = reinterpret_cast<const float4 *>(mode == GEMV_RMSNORM ? a.normw : a.x2);
  const float eps = a.eps;
  const bool norm = mode == GEMV_RMSNORM;
  int sb[kGemvMaxSegs];  // segment first units (increasing); unused ones never match
#pragma unroll
  for (int i = 0; i < kGemvMaxSegs; ++i) sb[i] = i < nseg ? a.seg[i].unit_begin : 0x7fffffff;
  const int nslots = full ? kunits : n;
  const int per_slot = kc / 4;  // float4s per slot
  const int total = nslots * per_slot;
  const int K4 = K / 4;
  __shared__ float red[kConsumerWarps];
  __half *xh = reinterpret_cast<__half *>(xw);
  constexpr int R = 2;  // float4s per thread per pass (kept small: no spills)
  const bool one_pass = total <= R * T;
  const int xlo = a.win_units * kc / 8;  // the lo plane, in uint4s after the hi plane
  float inv = 1.0f;
  if (norm && !one_pass) {  // sum of squares first (several staging passes follow)
    float ss = 0.f;
    for (int f = tid; f < K4; f += T) {
      const float4 v = __ldcg(x4 + f);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    consumer_sync();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kConsumerWarps; ++i) tot += red[i];
    inv = 1.0f / sqrtf(tot / (float)K + eps);
  }
  for (int base = 0; base < total; base += R * T) {
    float4 v[R], w[R];
    int kk[R];
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = w[r] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < R; ++r) {  // issue all loads first
      const int f = base + r * T + tid;
      kk[r] = -1;
      if (f < total) {
        const int j = f / per_slot, o = (f % per_slot) * 4;
        int kunit = j;
        if (!full) {
          const int u = u0 + j;
          int b = sb[0];
#pragma unroll
          for (int i = 1; i < kGemvMaxSegs; ++i) b = u >= sb[i] ? sb[i] : b;
          kunit = (u - b) % kunits;
        }
        kk[r] = kunit * kc + o;
        v[r] = __ldcg(x4 + kk[r] / 4);
        if (mode != GEMV_PLAIN) w[r] = mode == GEMV_SWIGLU ? __ldcg(w4 + kk[r] / 4) : w4[kk[r] / 4];
      }
    }
    if (norm && one_pass) {
      // a full range stages every column of x exactly once, so its loads
      // give the sum of squares; otherwise read x once more in this round
      float ss = 0.f;
      if (full) {
#pragma unroll
        for (int r = 0; r < R; ++r)
          ss += v[r].x * v[r].x + v[r].y * v[r].y + v[r].z * v[r].z + v[r].w * v[r].w;
      } else {
        for (int f = tid; f < K4; f += T) {
          const float4 t = __ldcg(x4 + f);
          ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        }
      }
      ss = warp_sum(ss);
      if ((tid & 31) == 0) red[tid >> 5] = ss;
      consumer_sync();
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kConsumerWarps; ++i) tot += red[i];
      inv = 1.0f / sqrtf(tot / (float)K + eps);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int f = base + r * T + tid;
      float y[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
      const float z[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
      if (kk[r] >= 0) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (mode == GEMV_RMSNORM) y[t] = (y[t] * inv) * z[t];
          else if (mode == GEMV_SWIGLU) y[t] = silu_f(y[t]) * z[t];
        }
      }
      emit_x4(y, kk[r] >= 0, f, per_slot, kc, xh, s16, tid, xlo);
    }
  }
}

// Unit ranges of the two consumer halves: half 0 takes the first
// ceil(n/2) units of the CTA's range [u0, u0 + n), half 1 the rest, each
// walking its run in order. Ring position p holds half (p & 1)'s unit p >> 1,
// so the positions alternate between the halves (with an odd n the last
// position, n - 1, is even and belongs to half 0).
__device__ __forceinline__ int half_begin(int n, int half) { return half ? (n + 1) >> 1 : 0; }
__device__ __forceinline__ int half_count(int n, int half) { return half ? n >> 1 : (n + 1) >> 1; }

// Walks the units of one half run, one segment at a time, for the producer.
struct UnitCursor {
  int sg, left;
  SegView S;
  const uint8_t *src;
  __device__ __forceinline__ void init(const GemvArgs &a, int u) {
    sg = find_seg(a, u);
    S = load_seg(a, sg);
    src = S.w + (size_t)(u - S.begin) * S.unit_bytes;
    left = S.begin + S.units - u;
  }
  // source of the current unit, then advance (the run never passes the
  // last segment)
  __device__ __forceinline__ const uint8_t *next(const GemvArgs &a, int &bytes) {
    if (left <= 0) {
      ++sg;
      S = load_seg(a, sg);
      src = S.w;
      left = S.units;
    }
    const uint8_t *p = src;
    bytes = S.unit_bytes;
    src += S.unit_bytes;
    --left;
    return p;
  }
};

// Producer side: stream the CTA's units [u0, u0 + n) of one GEMV into the
// ring, ring positions it, it + 1, ... (slot = position % NS), alternating
// between the two halves' runs. One thread calls this.
__device__ __forceinline__ bool gemv_produce(const GemvArgs &a, int u0, int n, uint32_t it,
                                             uint8_t *ring, int NS, int slot_bytes,
                                             uint64_t *full_bar, uint64_t *empty_bar, int *err) {
  if (n <= 0) return true;
  UnitCursor c0, c1;  // two named cursors: an indexed pair would live in local memory
  c0.init(a, u0);
  if (n > 1) c1.init(a, u0 + half_begin(n, 1));
  // slot and phase parity of ring position it + i, advanced without divisions
  int st = (int)(it % (uint32_t)NS);
  uint32_t ph = (it / (uint32_t)NS) & 1u;
  for (int i = 0; i < n; ++i) {
    const uint32_t rp = it + (uint32_t)i;
    if (rp >= (uint32_t)NS && !mbar_wait(&empty_bar[st], ph ^ 1u, err, 101)) {
      ring_drain(full_bar, NS, rp);
      return false;
    }
    int bytes;
    const uint8_t *src = (i & 1) ? c1.next(a, bytes) : c0.next(a, bytes);
    mbar_arrive_expect_tx(&full_bar[st], (uint32_t)bytes);
    bulk_g2s(ring + (size_t)st * slot_bytes, src, (uint32_t)bytes, &full_bar[st]);
    if (++st == NS) {
      st = 0;
      ph ^= 1u;
    }
  }
  return true;
}

// Adds a warp's row sums to the output rows of CTA tile `ctile`.
__device__ __forceinline__ void flush_rows(Acc2 &acc, const SegView &S, int ctile, int wti, int lane) {
  float r0 = acc.r0, r1 = acc.r1;
  r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
  r0 += __shfl_xor_sync(0xffffffffu, r0, 2);
  r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
  r1 += __shfl_xor_sync(0xffffffffu, r1, 2);
  if ((lane & 3) == 0) {
    const int row = ctile * kCtaRows + wti * 16 + (lane >> 2);
    if (row < S.rows) red_add_f32(S.y + row, r0);
    if (row + 8 < S.rows) red_add_f32(S.y + row + 8, r1);
  }
  acc.r0 = acc.r1 = 0.f;
}

// `cnt` consecutive units of one segment (type TYPE) for one warp: the k-th
// unit of the half's run sits at ring position it + 2 (k0 + k) + half.
template <int TYPE>
__device__ __forceinline__ bool consume_run(const SegView &S, int k0, int cnt, int half, int hbeg,
                                            uint32_t it, const uint8_t *ring, int NS,
                                            int slot_bytes, uint64_t *full_bar,
                                            uint64_t *empty_bar, const uint8_t *xw,
                                            const float *s16, bool full, int kc, int kunits,
                                            int xlo_uint4, int &ctile,
                                            int &kunit, Acc2 &acc, int *err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wti = warp & 7;
  const int xstep = (kc / 32) * 4, sstep = kc / 16;
  const int xlo = xlo_uint4;
  // slot and phase parity of this warp's ring positions (step 2, NS >= 2),
  // advanced without divisions
  const uint32_t rp0 = it + 2u * (uint32_t)k0 + (uint32_t)half;
  int st = (int)(rp0 % (uint32_t)NS);
  uint32_t ph = (rp0 / (uint32_t)NS) & 1u;
  for (int k = 0; k < cnt; ++k) {
    const int slot = full ? kunit : hbeg + k0 + k;
    if (!mbar_wait(&full_bar[st], ph, err, 102)) return false;
    const uint8_t *wt = ring + (size_t)st * slot_bytes + (size_t)wti * S.wt_bytes;
    const uint4 *xf = reinterpret_cast<const uint4 *>(xw) + (size_t)slot * xstep + (lane & 3);
    const float *sl = s16 + (size_t)slot * sstep;
    if (TYPE == IFX_TYPE_Q4_K) unit_q4k(wt, xf, xlo, sl, lane, acc);
    else if (TYPE == IFX_TYPE_Q6_K) unit_q6k(wt, xf, xlo, sl, lane, (uint32_t)S.type >> 8, acc);
    else if (TYPE == IFX_TYPE_Q4_0) unit_q4_0(wt, kc, S.wt_qbytes, xf, xlo, sl, lane, acc);
    else unit_q8_0(wt, kc, S.wt_qbytes, xf, xlo, sl, lane, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
    st += 2;
    if (st >= NS) {
      st -= NS;
      ph ^= 1u;
    }
    if (++kunit == kunits) {  // end of a CTA tile: its rows are complete here
      flush_rows(acc, S, ctile, wti, lane);
      kunit = 0;
      ++ctile;
    }
  }
  return true;
}

// Consumer side: the 16 consumer warps process the CTA's units [u0, u0 + n)
// in two halves of eight warps (see half_begin); warp w owns warp tile w % 8
// of every unit of its half's run, and row sums are flushed with
// red.global.add at each CTA-tile end and at the end of each segment run.
// x fragments / 16-column sums must already be staged in xw / s16.
__device__ __forceinline__ bool gemv_consume(const GemvArgs &a, int u0, int n, uint32_t it,
                                             const uint8_t *ring, int NS, int slot_bytes,
                                             uint64_t *full_bar, uint64_t *empty_bar,
                                             const uint8_t *xw, const float *s16, bool full,
                                             int *err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = warp >> 3, wti = warp & 7;
  const int hbeg = half_begin(n, half), hcnt = half_count(n, half);
  if (hcnt <= 0) return true;
  const int kunits = a.kunits, kc = a.kc;
  const int xlo = a.win_units * kc / 8;  // lo plane offset in uint4s
  int sg = find_seg(a, u0 + hbeg);
  SegView S = load_seg(a, sg);
  const int local = u0 + hbeg - S.begin;
  int ctile = local / kunits, kunit = local % kunits;
  int seg_left = S.units - local;
  Acc2 acc{0.f, 0.f};
  for (int k = 0; k < hcnt;) {
    const int cnt = min(hcnt - k, seg_left);
    bool ok;
    switch (S.type & 0xff) {
      case IFX_TYPE_Q4_K:
        ok = consume_run<IFX_TYPE_Q4_K>(S, k, cnt, half, hbeg, it, ring, NS, slot_bytes, full_bar,
                                        empty_bar, xw, s16, full, kc, kunits, xlo, ctile, kunit, acc, err);
        break;
      case IFX_TYPE_Q6_K:
        ok = consume_run<IFX_TYPE_Q6_K>(S, k, cnt, half, hbeg, it, ring, NS, slot_bytes, full_bar,
                                        empty_bar, xw, s16, full, kc, kunits, xlo, ctile, kunit, acc, err);
        break;
      case IFX_TYPE_Q4_0:
        ok = consume_run<IFX_TYPE_Q4_0>(S, k, cnt, half, hbeg, it, ring, NS, slot_bytes, full_bar,
                                        empty_bar, xw, s16, full, kc, kunits, xlo, ctile, kunit, acc, err);
        break;
      default:
        ok = consume_run<IFX_TYPE_Q8_0>(S, k, cnt, half, hbeg, it, ring, NS, slot_bytes, full_bar,
                                        empty_bar, xw, s16, full, kc, kunits, xlo, ctile, kunit, acc, err);
        break;
    }
    if (!ok) return false;
    if (kunit != 0) flush_rows(acc, S, ctile, wti, lane);  // a partial tile ends the run
    k += cnt;
    if (k < hcnt) {  // next segment, from its first unit
      ++sg;
      S = load_seg(a, sg);
      ctile = kunit = 0;
      seg_left = S.units;
    }
  }
  return true;
}

}  // namespace gemvdev
}  // namespace ifx
