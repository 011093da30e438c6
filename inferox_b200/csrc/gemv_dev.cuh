// Device-side building blocks of the fused dequant GEMV, shared by the
// standalone GEMV kernel (gemv.cu) and the persistent decode kernel
// (decode_mega.cu): per-type unit consumers (mma.m16n8k16 over the
// fragment-ordered layout of qlayout.cuh) and the activation staging.
#pragma once
#include "gemv.cuh"

namespace ifx {
namespace gemvdev {

// 16 zero bytes in shared memory (set by the kernels at start).
__shared__ uint4 g_xzero;
// Per-warp partial sums of squares of x written by stage_x in RMSNorm mode
// (summed in warp order by the consumers after the staging barrier).
__shared__ float g_ssq[16];

constexpr int kConsumerWarps = kGemvThreads / 32 - 1;
constexpr int kConsumerThreads = kConsumerWarps * 32;

// Named barrier over the consumer warps only (the producer warp has left).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory");
}


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

struct Acc2 {
  float r0, r1;  // rows g and g+8
};

// ----------------------------------------------------- staged activations --
// The batch-1 GEMV runs on the integer tensor cores: weights enter as their
// exact quantised integers (u8), activations as four int8 planes. The CTA
// stages f(x) (plain / RMSNorm / SwiGLU) as x = E * (p0 + p1/2^7 + p2/2^14 +
// p3/2^21), E a power of two with max|x / E| <= 127: p0 = rint(x/E), each
// later plane the rounded residual of the one before times 2^7, so the
// staged value is x to about 28 bits below the CTA's largest |x|, and every
// product of the MMA (u8 weight times s8 plane, summed in s32) is exact.
//
// E is chosen per 32-column group (for K-quant units, whose integer sums run
// over a whole 256-column unit, one E for the unit's eight groups). Per slot
// (one unit's kc columns): the planes, then per 16-column chunk the int16
// sums of each plane (planes 0-3, then four zeros), then per chunk the f32
// sum of the staged values, then per group E. Byte layout of the planes: for 32-column
// group gr, plane p and lane column c (0-3), 8 bytes at
// ((gr * 4 + p) * 4 + c) * 8: the chunk's columns {2c, 2c+8, 2c+1, 2c+9},
// then the same of the group's second chunk (+16). That order is the one in
// which the repacked weight words of qlayout.cuh hold a lane's values of one
// row (nibble j of byte j of the word, low nibbles row g, high nibbles row
// g+8), so one AND gives the MMA's A register and B is loaded as is.
__host__ __device__ constexpr size_t xs_plane_bytes(int kc) { return (size_t)kc * 4; }
__host__ __device__ constexpr size_t xs_isum_bytes(int kc) { return (size_t)(kc / 16) * 16; }
__host__ __device__ constexpr size_t xs_fsum_bytes(int kc) { return (size_t)(kc / 16) * 4; }
__host__ __device__ constexpr size_t xs_escale_bytes(int kc) { return (size_t)(kc / 32) * 4; }
__host__ __device__ constexpr size_t xs_slot_bytes(int kc) {
  return xs_plane_bytes(kc) + xs_isum_bytes(kc) + xs_fsum_bytes(kc) + xs_escale_bytes(kc);
}

// Where the three parts of a staging window of `win` slots start.
struct XStage {
  uint8_t *planes;
  int16_t *isum;
  float *fsum, *escale;
  __device__ __forceinline__ void init(uint8_t *base, int win, int kc) {
    planes = base;
    isum = reinterpret_cast<int16_t *>(base + (size_t)win * xs_plane_bytes(kc));
    fsum = reinterpret_cast<float *>(base + (size_t)win * (xs_plane_bytes(kc) + xs_isum_bytes(kc)));
    escale = fsum + (size_t)win * (kc / 16);
  }
};

// rint(t) through the f32 adder: t + 1.5 * 2^23 lies in [2^23, 2^24) for
// |t| < 2^22, whose ulp is 1, so the sum is t rounded to an integer (ties to
// even) and its low mantissa byte is that integer modulo 256 (two's
// complement). Returns the bits; `r` becomes the rounded value as f32.
__device__ __forceinline__ uint32_t round_bits(float t, float &r) {
  const float s = t + 12582912.0f;
  r = s - 12582912.0f;
  return __float_as_uint(s);
}

// The four planes of t = x / E (|t| <= 127): byte p of plane p in the low
// byte of bits[p]; rounded plane values (as exact f32) in v[p].
__device__ __forceinline__ void planes4(float t, uint32_t (&bits)[4], float (&v)[4]) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    bits[p] = round_bits(t, v[p]);
    t = (t - v[p]) * 128.0f;  // exact: the residual is at most 1/2 in magnitude
  }
}

// Bytes 0 of a, b, c, d as one word (a lowest).
__device__ __forceinline__ uint32_t pack4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return prmt(prmt(a, b, 0x0040u), prmt(c, d, 0x0040u), 0x5410u);
}

// Consumer-side input staging. Every global read is a coalesced float4
// issued up front. One work item is (slot, 16-column chunk, half q): the
// float4s at chunk columns 4q and 4q + 8, which fill the plane words of lane
// columns c = 2q and 2q + 1. Items run in order over threads, so the 32
// items of a 256-column slot are one warp and the 4 items of a 32-column
// group four adjacent lanes: E comes from warp shuffles, with no block-wide
// step. RMSNorm is staged as x * w; its scalar 1/rms(x) multiplies the row
// sums when they are flushed (W((x s) w) = s W(x w)), and its sum of squares
// is left per warp in g_ssq, read after the staging barrier.
static __device__ __noinline__ void stage_x(const GemvArgs &a, int u0, int n, bool full, uint8_t *xw) {
  const int tid = threadIdx.x;  // 0..kConsumerThreads-1
  constexpr int T = kConsumerThreads;
  const int mode = a.mode, K = a.K, kc = a.kc, kunits = a.kunits, nseg = a.nseg;
  const float4 *x4 = reinterpret_cast<const float4 *>(a.x);
  const float4 *w4 = reinterpret_cast<const float4 *>(mode == GEMV_RMSNORM ? a.normw : a.x2);
  const bool norm = mode == GEMV_RMSNORM;
  int sb[kGemvMaxSegs];  // segment first units (increasing); unused ones never match
#pragma unroll
  for (int i = 0; i < kGemvMaxSegs; ++i) sb[i] = i < nseg ? a.seg[i].unit_begin : 0x7fffffff;
  const int nslots = full ? kunits : n;
  const int cps = kc / 16;  // chunks per slot
  const int items = nslots * cps * 2;
  const int K4 = K / 4;
  // lanes that share one E: the unit (a warp) for K-quant slots, else the group
  const int ewidth = kc == 256 ? 32 : 4;
  XStage X;
  X.init(xw, a.win_units, kc);
  auto col_of = [&](int j, int o) {  // column (within K) of chunk offset o of slot j
    int kunit = j;
    if (!full) {
      const int u = u0 + j;
      int b = sb[0];
#pragma unroll
      for (int i = 1; i < kGemvMaxSegs; ++i) b = u >= sb[i] ? sb[i] : b;
      kunit = (u - b) % kunits;
    }
    return kunit * kc + o;
  };
  float ss = 0.f;
  if (norm && !full)  // the sum of squares of all of x (the staged columns are a subset)
    for (int f = tid; f < K4; f += T) {
      const float4 t = __ldcg(x4 + f);
      ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
    }
  for (int base = 0; base < items; base += T) {
    const int item = base + tid;
    const bool ok = item < items;
    // item -> (slot j, chunk h, half q); q is the fastest index
    const int q = item & 1, h = (item >> 1) % cps, j = (item >> 1) / cps;
    float4 v[2], w[2];
    v[0] = v[1] = w[0] = w[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {  // issue all loads first
        const int k = col_of(j, 16 * h + 4 * q + 8 * r) / 4;
        v[r] = __ldcg(x4 + k);
        if (mode != GEMV_PLAIN) w[r] = mode == GEMV_SWIGLU ? __ldcg(w4 + k) : w4[k];
      }
    }
    if (norm && full)  // a full range stages every column of x exactly once
#pragma unroll
      for (int r = 0; r < 2; ++r)
        ss += v[r].x * v[r].x + v[r].y * v[r].y + v[r].z * v[r].z + v[r].w * v[r].w;
    float y[8];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float xe[4] = {v[r].x, v[r].y, v[r].z, v[r].w}, we[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        y[4 * r + e] = mode == GEMV_RMSNORM ? xe[e] * we[e]
                       : mode == GEMV_SWIGLU ? silu_f(xe[e]) * we[e] : xe[e];
    }
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(y[i]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (ewidth == 32) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    }
    // E = 2^e with max |y| / E in [63.5, 127] (1 for an all-zero group)
    float E = 1.0f, invE = 1.0f;
    if (mx > 0.f && mx < 3.0e38f) {
      // 1/E = 2^(6 - floor(log2 mx)): biased exponent 127 + 6 - (b - 127)
      // for mx's biased exponent b, clamped to normal numbers
      const int eb = min(254, 260 - (int)((__float_as_uint(mx) >> 23) & 0xff));
      invE = __uint_as_float((uint32_t)eb << 23);
      if (mx * invE > 127.0f) invE *= 0.5f;
      E = 1.0f / invE;  // exact: a power of two
    }
    uint32_t bits[8][4];
    float pv[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) planes4(y[i] * invE, bits[i], pv[i]);  // a power of two: exact
    // the chunk's plane sums: these 8 values plus the partner half's 8
    float ps[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float t = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) t += pv[i][p];  // small integers: exact
      ps[p] = t + __shfl_xor_sync(0xffffffffu, t, 1);
    }
    if (ok) {
      // lane column c = 2q takes the float4 elements 0, 1 (columns 4q, 4q + 8,
      // then 4q + 1, 4q + 9); c = 2q + 1 takes elements 2, 3
      uint8_t *dst = X.planes + (size_t)j * xs_plane_bytes(kc) + (size_t)(h >> 1) * 128 + (h & 1) * 4;
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint32_t wa = pack4(bits[0][p], bits[4][p], bits[1][p], bits[5][p]);
        const uint32_t wb = pack4(bits[2][p], bits[6][p], bits[3][p], bits[7][p]);
        *reinterpret_cast<uint32_t *>(dst + (size_t)((p * 4 + 2 * q) * 8)) = wa;
        *reinterpret_cast<uint32_t *>(dst + (size_t)((p * 4 + 2 * q + 1) * 8)) = wb;
      }
      if (q == 0) {
        int16_t *is = X.isum + ((size_t)j * cps + h) * 8;
        *reinterpret_cast<uint4 *>(is) =
            make_uint4(((uint32_t)(uint16_t)(int16_t)ps[0]) | ((uint32_t)(uint16_t)(int16_t)ps[1] << 16),
                       ((uint32_t)(uint16_t)(int16_t)ps[2]) | ((uint32_t)(uint16_t)(int16_t)ps[3] << 16),
                       0u, 0u);
        X.fsum[(size_t)j * cps + h] =
            E * (ps[0] + (ps[1] + (ps[2] + ps[3] * 0.0078125f) * 0.0078125f) * 0.0078125f);
        if ((h & 1) == 0) X.escale[(size_t)j * (cps / 2) + (h >> 1)] = E;
      }
    }
  }
  if (norm) {
    ss = warp_sum(ss);
    if ((tid & 31) == 0) g_ssq[tid >> 5] = ss;
  }
}

// 1/rms(x) of the staged RMSNorm input (ops.rs:155-168: 1/sqrt(sum x^2 / n +
// eps)), from the per-warp sums stage_x left; call after the staging barrier.
__device__ __forceinline__ float staged_rms_inv(const GemvArgs &a) {
  if (a.mode != GEMV_RMSNORM) return 1.0f;
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) t += g_ssq[i];
  return 1.0f / sqrtf(t / (float)a.K + a.eps);
}

// ----------------------------------------------------------- unit consumers
// mma.sync m16n8k32 / m16n8k16 with u8 A (the weights' integers), s8 B (the
// activation planes) and s32 accumulation. A register layout: k = 4c + byte
// (c = lane & 3) for row g = lane >> 2 (a0) and g + 8 (a1), k + 16 for a2,
// a3 (k32 only). B: column n = g, the same k. D: rows g / g + 8, columns 2c
// and 2c + 1. Planes 0-3 sit in B columns 0-3 (lanes g < 4 load them, the
// others keep zeros), so lane c < 2 ends with planes 2c, 2c + 1 of its rows.
__device__ __forceinline__ void imma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void imma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%7,%7,%7,%7};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// What a consumer needs of one staged slot, for lane (g, c).
struct XSlot {
  const uint2 *b;     // this lane's B words of group 0 (group gr at b[gr * 16])
  const int16_t *is;  // int16 plane sums of chunk 0 (chunk h at is[h * 8])
  const float *fs;    // f32 sums per chunk
  const float *es;    // E per 32-column group
};

__device__ __forceinline__ uint32_t word4(const uint4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Plane sums (planes 2c, 2c + 1; zeros for c >= 2) of chunk h.
__device__ __forceinline__ void plane_sums(const XSlot &X, int h, int c, int &s0, int &s1) {
  const uint32_t v = *reinterpret_cast<const uint32_t *>(X.is + h * 8 + 2 * c);
  s0 = (int)(int16_t)(v & 0xffffu);
  s1 = (int)v >> 16;
}

constexpr uint32_t kNib = 0x0F0F0F0Fu;

// ------------------------------------------------------------------ Q4_K --
// dequant.rs:123-163: y = (d * sc_g) * q - (dmin * m_g). Per 32-column group
// one k32 MMA; the integer scale enters the s32 sum (sum_g sc_g * dot_g is
// exact), d once per unit, the mins through the f32 group sums.
// Every weight byte of the unit is in registers once the loads at its top
// have completed: the warp then releases its ring bytes (one arrive on
// `rel`), so the producer can refill them while the MMAs run.
__device__ __forceinline__ void release_unit(uint64_t *rel, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(rel);
}

__device__ __forceinline__ void unit_q4k(const uint8_t *wt, const XSlot &X, bool has_b, int lane,
                                         float cs, uint64_t *rel, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3;
  const float sa = X.es[0] * cs, sb = sa * 0.0078125f;  // planes 2c, 2c + 1
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const uint4 *sv = reinterpret_cast<const uint4 *>(wt + 2048);
  uint4 q[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) q[s] = qv[s * 32 + lane];
  // repacked header (repack.cu): word k = the 24-bit scale/min field of
  // groups 2k, 2k+1 (sc 6 bits each, then m) | byte k of (d, dmin) on top
  const uint4 hd0 = sv[g], hd1 = sv[g + 8];
  release_unit(rel, lane);
  int A0 = 0, A1 = 0, A2 = 0, A3 = 0;
#pragma unroll
  for (int gr = 0; gr < 8; ++gr) {
    const uint32_t w0 = word4(q[gr >> 1], 2 * (gr & 1)), w1 = word4(q[gr >> 1], 2 * (gr & 1) + 1);
    uint2 b = make_uint2(0u, 0u);
    if (has_b) b = X.b[gr * 16];
    int D[4];
    imma_k32(D, w0 & kNib, (w0 >> 4) & kNib, w1 & kNib, (w1 >> 4) & kNib, b.x, b.y);
    const int sh = 6 * (gr & 1);
    const int sc0 = (int)((word4(hd0, gr >> 1) >> sh) & 63u);
    const int sc1 = (int)((word4(hd1, gr >> 1) >> sh) & 63u);
    A0 += sc0 * D[0];
    A1 += sc0 * D[1];
    A2 += sc1 * D[2];
    A3 += sc1 * D[3];
  }
  const float d0 = h2f((uint16_t)prmt(hd0.x, hd0.y, 0x0073u)), dm0 = h2f((uint16_t)prmt(hd0.z, hd0.w, 0x0073u));
  const float d1 = h2f((uint16_t)prmt(hd1.x, hd1.y, 0x0073u)), dm1 = h2f((uint16_t)prmt(hd1.z, hd1.w, 0x0073u));
  // mins of this lane's groups 2c, 2c + 1 (chunks 4c .. 4c + 3)
  const float Sa = X.fs[4 * c] + X.fs[4 * c + 1], Sb = X.fs[4 * c + 2] + X.fs[4 * c + 3];
  const uint32_t f0 = word4(hd0, c), f1 = word4(hd1, c);
  const float m0 = fmaf(u2f_small((f0 >> 18) & 63u), Sb, u2f_small((f0 >> 12) & 63u) * Sa);
  const float m1 = fmaf(u2f_small((f1 >> 18) & 63u), Sb, u2f_small((f1 >> 12) & 63u) * Sa);
  acc.r0 = fmaf(d0, fmaf((float)A1, sb, (float)A0 * sa), fmaf(-dm0, m0, acc.r0));
  acc.r1 = fmaf(d1, fmaf((float)A3, sb, (float)A2 * sa), fmaf(-dm1, m1, acc.r1));
}

// ------------------------------------------------------------------ Q6_K --
// dequant.rs:174-199: q = low nibble | two bits << 4 (6 bits), y = (d * sc) *
// (q - 32), sc per 16 columns read as u8 (the reference) or int8 (smask
// 0x80, llama.cpp). One k16 MMA per 16-column chunk with sc applied in the
// s32 sum; the -32 bias as d * sum_h sc_h * S_h over the f32 chunk sums
// (lane c takes chunks 4c .. 4c + 3; the flush adds the lanes).
__device__ __forceinline__ int q6_scale(uint32_t word, int byte, uint32_t smask) {
  return (int)(((word >> (8 * byte)) & 0xffu) ^ smask) - (int)smask;
}

__device__ __forceinline__ void unit_q6k(const uint8_t *wt, const XSlot &X, bool has_b, int lane,
                                         float cs, uint32_t smask, uint64_t *rel, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3;
  const float sa = X.es[0] * cs, sb = sa * 0.0078125f;  // planes 2c, 2c + 1
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const uint4 *hv = reinterpret_cast<const uint4 *>(wt + 2048);
  const uint8_t *scb = wt + 3072;
  uint4 q[4], hq[2];
#pragma unroll
  for (int s = 0; s < 4; ++s) q[s] = qv[s * 32 + lane];
#pragma unroll
  for (int t = 0; t < 2; ++t) hq[t] = hv[t * 32 + lane];
  const uint4 sc0v = *reinterpret_cast<const uint4 *>(scb + 16 * g);
  const uint4 sc1v = *reinterpret_cast<const uint4 *>(scb + 16 * (g + 8));
  const float d0 = h2f(*reinterpret_cast<const uint16_t *>(scb + 256 + 2 * g));
  const float d1 = h2f(*reinterpret_cast<const uint16_t *>(scb + 256 + 2 * (g + 8)));
  release_unit(rel, lane);
  int A0 = 0, A1 = 0, A2 = 0, A3 = 0;
#pragma unroll
  for (int gr = 0; gr < 8; ++gr) {
    uint2 b = make_uint2(0u, 0u);
    if (has_b) b = X.b[gr * 16];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int h = 2 * gr + e;
      const uint32_t w = word4(q[h >> 2], h & 3);
      uint32_t H = word4(hq[h >> 3], (h >> 1) & 3);
      if (e) H >>= 8;
      // the 2-bit values sit at bit 2i (row g) / 2i + 2 (row g+8) of nibble i:
      // moved to bits 4-5 of the byte that holds the same element's nibble
      const uint32_t ag = (w & kNib) | ((H << 4) & 0x00300030u) | ((H << 8) & 0x30003000u);
      const uint32_t ag8 = ((w >> 4) & kNib) | ((H << 2) & 0x00300030u) | ((H << 6) & 0x30003000u);
      int D[4];
      imma_k16(D, ag, ag8, e ? b.y : b.x);
      const int scg = q6_scale(word4(sc0v, h >> 2), h & 3, smask);
      const int scg8 = q6_scale(word4(sc1v, h >> 2), h & 3, smask);
      A0 += scg * D[0];
      A1 += scg * D[1];
      A2 += scg8 * D[2];
      A3 += scg8 * D[3];
    }
  }
  // the bias of this lane's chunks 4c .. 4c + 3
  const uint32_t s0w = word4(sc0v, c), s1w = word4(sc1v, c);
  float b0 = 0.f, b1 = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float S = X.fs[4 * c + i];
    b0 = fmaf((float)q6_scale(s0w, i, smask), S, b0);
    b1 = fmaf((float)q6_scale(s1w, i, smask), S, b1);
  }
  acc.r0 = fmaf(d0, fmaf((float)A1, sb, fmaf((float)A0, sa, -32.0f * b0)), acc.r0);
  acc.r1 = fmaf(d1, fmaf((float)A3, sb, fmaf((float)A2, sa, -32.0f * b1)), acc.r1);
}

// ------------------------------------------------------- Q4_0 and Q8_0 --
// dequant.rs:62-111: y = (q - 8) d (Q4_0, nibbles) or q d (Q8_0, bytes
// stored as q + 128); d an f16 per row and 32-column block. Runtime block
// count (kc <= 256). The two plane columns of a lane are combined in s32
// (128 t0 + t1) before the block's f32 scale.
__device__ __forceinline__ void unit_q4_0(const uint8_t *wt, int kc, int wt_qbytes, const XSlot &X,
                                          bool has_b, int lane, float cs, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3;
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const int nb = kc / 32;
  const uint8_t *sc = wt + wt_qbytes;
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    if (2 * s < nb) {
      const uint4 Q = qv[s * 32 + lane];
#pragma unroll
      for (int p2 = 0; p2 < 2; ++p2) {
        const int blk = 2 * s + p2;
        if (blk < nb) {
          const uint32_t w0 = p2 ? Q.z : Q.x, w1 = p2 ? Q.w : Q.y;
          uint2 b = make_uint2(0u, 0u);
          if (has_b) b = X.b[blk * 16];
          int D[4];
          imma_k32(D, w0 & kNib, (w0 >> 4) & kNib, w1 & kNib, (w1 >> 4) & kNib, b.x, b.y);
          int a0, a1, c0, c1;
          plane_sums(X, 2 * blk, c, a0, a1);
          plane_sums(X, 2 * blk + 1, c, c0, c1);
          const int s0 = a0 + c0, s1 = a1 + c1;
          const int T0 = 128 * (D[0] - 8 * s0) + (D[1] - 8 * s1);
          const int T1 = 128 * (D[2] - 8 * s0) + (D[3] - 8 * s1);
          const float dA = h2f(*reinterpret_cast<const uint16_t *>(sc + (g * nb + blk) * 2));
          const float dB = h2f(*reinterpret_cast<const uint16_t *>(sc + ((g + 8) * nb + blk) * 2));
          const float sb = X.es[blk] * cs * 0.0078125f;  // plane 2c + 1 of the block
          acc.r0 = fmaf(dA * sb, (float)T0, acc.r0);
          acc.r1 = fmaf(dB * sb, (float)T1, acc.r1);
        }
      }
    }
  }
}

__device__ __forceinline__ void unit_q8_0(const uint8_t *wt, int kc, int wt_qbytes, const XSlot &X,
                                          bool has_b, int lane, float cs, Acc2 &acc) {
  const int g = lane >> 2, c = lane & 3;
  const uint4 *qv = reinterpret_cast<const uint4 *>(wt);
  const int nb = kc / 32;
  const uint8_t *sc = wt + wt_qbytes;
#pragma unroll
  for (int s = 0; s < 8; ++s) {  // block s: 16 bytes per lane, rows g, g+8
    if (s < nb) {
      const uint4 Q = qv[s * 32 + lane];
      // Q.x: (g, 2c) (g, 2c+1) (g+8, 2c) (g+8, 2c+1); Q.y: the same at 2c+8,
      // 2c+9; Q.z / Q.w: the block's second chunk
      uint2 b = make_uint2(0u, 0u);
      if (has_b) b = X.b[s * 16];
      int D[4];
      imma_k32(D, prmt(Q.x, Q.y, 0x5140u), prmt(Q.x, Q.y, 0x7362u), prmt(Q.z, Q.w, 0x5140u),
               prmt(Q.z, Q.w, 0x7362u), b.x, b.y);
      int a0, a1, c0, c1;
      plane_sums(X, 2 * s, c, a0, a1);
      plane_sums(X, 2 * s + 1, c, c0, c1);
      const int s0 = a0 + c0, s1 = a1 + c1;
      const int T0 = 128 * (D[0] - 128 * s0) + (D[1] - 128 * s1);
      const int T1 = 128 * (D[2] - 128 * s0) + (D[3] - 128 * s1);
      const float dA = h2f(*reinterpret_cast<const uint16_t *>(sc + (g * nb + s) * 2));
      const float dB = h2f(*reinterpret_cast<const uint16_t *>(sc + ((g + 8) * nb + s) * 2));
      const float sb = X.es[s] * cs * 0.0078125f;  // plane 2c + 1 of the block
      acc.r0 = fmaf(dA * sb, (float)T0, acc.r0);
      acc.r1 = fmaf(dB * sb, (float)T1, acc.r1);
    }
  }
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

// The weight ring is a byte ring: ring position p (one unit; positions
// alternate between the consumer halves) uses mbarrier slot p % kRingPos, and
// its bytes are packed right after the previous position's, wrapping to
// offset 0 when the unit does not fit before the end. The bytes in flight
// therefore do not depend on the unit size (fixed slots sized for the
// largest unit would hold far fewer of the small ones). The producer records
// each position's offset and length in shared memory (the consumers read the
// offset once the position's full barrier has completed) and, before placing
// a unit, waits in age order for every position in flight whose bytes it
// would overwrite, and for the previous user of its barrier slot.
constexpr int kRingPos = kGemvMaxStages;
static_assert(kRingPos % 2 == 0, "a slot must always belong to the same consumer half");

struct RingTab {  // shared memory: the offset of each position in flight, by slot
  uint32_t *off;
};

// Producer thread state that persists across the GEMVs of one kernel: where
// the next unit goes, the oldest position not yet seen released and where
// that position starts. The positions in flight occupy the ring from
// tail_off to head, in order (possibly wrapping past the end).
struct RingState {
  uint32_t head, tail, tail_off;
};

// Does [start, end) (which never wraps) meet the bytes in flight?
__device__ __forceinline__ bool ring_busy(const RingState &rs, uint32_t p, uint32_t start,
                                          uint32_t end) {
  if (rs.tail == p) return false;  // nothing in flight
  if (rs.tail_off < rs.head) return start < rs.head && rs.tail_off < end;
  // the bytes in flight wrap: [tail_off, ring end) and [0, head)
  return end > rs.tail_off || start < rs.head;
}

// Producer side: stream the CTA's units [u0, u0 + n) of one GEMV into the
// ring as positions it, it + 1, ..., alternating between the two halves'
// runs. One thread calls this.
__device__ __forceinline__ bool gemv_produce(const GemvArgs &a, int u0, int n, uint32_t it,
                                             uint8_t *ring, uint32_t ring_bytes, RingTab tab,
                                             RingState &rs, uint64_t *full_bar, uint64_t *empty_bar,
                                             int *err) {
  if (n <= 0) return true;
  UnitCursor c0, c1;  // two named cursors: an indexed pair would live in local memory
  c0.init(a, u0);
  if (n > 1) c1.init(a, u0 + half_begin(n, 1));
  for (int i = 0; i < n; ++i) {
    const uint32_t p = it + (uint32_t)i;
    int bytes;
    const uint8_t *src = (i & 1) ? c1.next(a, bytes) : c0.next(a, bytes);
    uint32_t start = rs.head;
    if (start + (uint32_t)bytes > ring_bytes) start = 0;
    const uint32_t end = start + (uint32_t)bytes;
    // release positions in age order until this one's bytes are free and
    // its barrier slot's previous user (position p - kRingPos) is done
    while (rs.tail + kRingPos <= p || ring_busy(rs, p, start, end)) {
      if (!mbar_wait(&empty_bar[rs.tail % kRingPos], (rs.tail / kRingPos) & 1u, err, 101)) {
        ring_drain(full_bar, kRingPos, p);
        return false;
      }
      ++rs.tail;
      rs.tail_off = rs.tail < p ? tab.off[rs.tail % kRingPos] : start;
    }
    const uint32_t ps = p % kRingPos;
    tab.off[ps] = start;
    mbar_arrive_expect_tx(&full_bar[ps], (uint32_t)bytes);
    bulk_g2s(ring + start, src, (uint32_t)bytes, &full_bar[ps]);
    if (rs.tail == p) rs.tail_off = start;  // the ring was empty
    rs.head = end;
  }
  return true;
}

// Adds a warp's row sums to the output rows of CTA tile `ctile`.
__device__ __forceinline__ void flush_rows(Acc2 &acc, const SegView &S, int ctile, int wti, int lane,
                                           float rscale) {
  float r0 = acc.r0 * rscale, r1 = acc.r1 * rscale;
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
                                            uint32_t it, const uint8_t *ring, const uint32_t *ring_off,
                                            uint64_t *full_bar,
                                            uint64_t *empty_bar, const XStage &X, bool full, int kc,
                                            int kunits, float cs, float rscale, int &ctile,
                                            int &kunit, Acc2 &acc, int *err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wti = warp & 7;
  const int g = lane >> 2, c = lane & 3;
  const bool has_b = g < 4;  // lanes that load a plane (B columns 0-3)
  const int cps = kc / 16;
  // barrier slot and phase parity of this warp's ring positions (step 2),
  // advanced without divisions
  const uint32_t rp0 = it + 2u * (uint32_t)k0 + (uint32_t)half;
  int st = (int)(rp0 % (uint32_t)kRingPos);
  uint32_t ph = (rp0 / (uint32_t)kRingPos) & 1u;
  for (int k = 0; k < cnt; ++k) {
    const int slot = full ? kunit : hbeg + k0 + k;
    if (!mbar_wait(&full_bar[st], ph, err, 102)) return false;
    const uint8_t *wt = ring + ring_off[st] + (size_t)wti * S.wt_bytes;
    XSlot xs;
    xs.b = reinterpret_cast<const uint2 *>(X.planes + (size_t)slot * xs_plane_bytes(kc)) +
           ((has_b ? g : 0) * 4 + c);
    xs.is = X.isum + (size_t)slot * cps * 8;
    xs.fs = X.fsum + (size_t)slot * cps;
    xs.es = X.escale + (size_t)slot * (cps / 2);
    // Q4_K / Q6_K release their ring bytes as soon as they hold them in
    // registers; Q4_0 / Q8_0 read scales block by block and release at the end
    if (TYPE == IFX_TYPE_Q4_K) unit_q4k(wt, xs, has_b, lane, cs, &empty_bar[st], acc);
    else if (TYPE == IFX_TYPE_Q6_K) unit_q6k(wt, xs, has_b, lane, cs, (uint32_t)S.type >> 8, &empty_bar[st], acc);
    else if (TYPE == IFX_TYPE_Q4_0) unit_q4_0(wt, kc, S.wt_qbytes, xs, has_b, lane, cs, acc);
    else unit_q8_0(wt, kc, S.wt_qbytes, xs, has_b, lane, cs, acc);
    if (TYPE == IFX_TYPE_Q4_0 || TYPE == IFX_TYPE_Q8_0) release_unit(&empty_bar[st], lane);
    st += 2;
    if (st >= kRingPos) {
      st -= kRingPos;
      ph ^= 1u;
    }
    if (++kunit == kunits) {  // end of a CTA tile: its rows are complete here
      flush_rows(acc, S, ctile, wti, lane, rscale);
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
// The activation planes and sums must already be staged in xw (stage_x).
__device__ __forceinline__ bool gemv_consume(const GemvArgs &a, int u0, int n, uint32_t it,
                                             const uint8_t *ring, const uint32_t *ring_off,
                                             uint64_t *full_bar, uint64_t *empty_bar,
                                             uint8_t *xw, bool full, int *err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = warp >> 3, wti = warp & 7;
  const int hbeg = half_begin(n, half), hcnt = half_count(n, half);
  if (hcnt <= 0) return true;
  const int kunits = a.kunits, kc = a.kc;
  XStage X;
  X.init(xw, a.win_units, kc);
  // the value of plane p is E * 2^-7p: lane c < 2 holds planes 2c, 2c + 1
  const int c = lane & 3;
  const float cs = c == 0 ? 1.0f : c == 1 ? 6.103515625e-05f : 0.f;  // 2^-14 for c = 1
  const float rscale = staged_rms_inv(a);
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
        ok = consume_run<IFX_TYPE_Q4_K>(S, k, cnt, half, hbeg, it, ring, ring_off, full_bar,
                                        empty_bar, X, full, kc, kunits, cs, rscale, ctile, kunit, acc, err);
        break;
      case IFX_TYPE_Q6_K:
        ok = consume_run<IFX_TYPE_Q6_K>(S, k, cnt, half, hbeg, it, ring, ring_off, full_bar,
                                        empty_bar, X, full, kc, kunits, cs, rscale, ctile, kunit, acc, err);
        break;
      case IFX_TYPE_Q4_0:
        ok = consume_run<IFX_TYPE_Q4_0>(S, k, cnt, half, hbeg, it, ring, ring_off, full_bar,
                                        empty_bar, X, full, kc, kunits, cs, rscale, ctile, kunit, acc, err);
        break;
      default:
        ok = consume_run<IFX_TYPE_Q8_0>(S, k, cnt, half, hbeg, it, ring, ring_off, full_bar,
                                        empty_bar, X, full, kc, kunits, cs, rscale, ctile, kunit, acc, err);
        break;
    }
    if (!ok) return false;
    if (kunit != 0) flush_rows(acc, S, ctile, wti, lane, rscale);  // a partial tile ends the run
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
