// Prefill fused dequant GEMM: the weight units of qlayout.cuh and the staged
// activations stream through a shared-memory ring with 1-D bulk async copies
// (producer warp, mbarriers). Each consumer warp turns its 16-row A fragments
// into exact small integers in f16 (the quantised values, bias removed) once
// per 16-column chunk and reuses them across the 8 token n-tiles of the
// CTA's 64-token block with mma.m16n8k16. x is staged as two f16 planes
// (x ~= hi + lo, about 22 bits), both multiplied into a per-scale-group f32
// accumulator, and each group's scale (and Q4_K's min, through per-token
// group sums of x) is applied in f32 — so the only rounding left is f32
// accumulation order.
#include <algorithm>

#include "gemm.cuh"
#include "dense.cuh"

namespace ifx {

namespace {

constexpr int kGThreads = 288;
constexpr int kGStages = 2;
// One 16-column chunk of a block of 8 * NT tokens, hi + lo planes: NT n-tiles
// x 32 lanes x 4 halves x 2 planes x 2 bytes.
__host__ __device__ constexpr int xchunk_bytes(int nt) { return nt * 512; }

__device__ __forceinline__ float silu_g(float v) {
  float c = fminf(fmaxf(v, -80.0f), 80.0f);
  return v * (1.0f / (1.0f + expf(-c)));
}

// X staging: CTA (t, y) computes the transform of columns [y * kStageCols,
// (y + 1) * kStageCols) of token row t (the RMSNorm statistic over the whole
// row) and writes them into the fragment layout [mblock][chunk][plane][nt]
// [lane][4 halves] of blocks of 8 * NT tokens, then the per-token 32-column
// sums.
constexpr int kStageCols = 256;  // 8 warps: one column per thread

__global__ void stage_x_kernel(const float *X, const float *X2, const float *normw, float eps,
                               int mode, int64_t M, int64_t K, int NT, __half *out, StageZero z) {
  // launched with programmatic serialization: X is read after the previous
  // grid completes; the next grid (a GEMM) may start fetching its weights
  pdl_wait();
  pdl_launch();
  {  // buffers the following GEMMs accumulate into start at zero
    const int64_t nb = (int64_t)gridDim.x * gridDim.y, b = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
    for (int i = 0; i < 2; ++i)
      if (z.p[i])
        for (int64_t e = b * blockDim.x + threadIdx.x; e < z.n[i]; e += nb * blockDim.x) z.p[i][e] = 0.f;
  }
  const int64_t t = blockIdx.x;  // token (row), may be >= M for padding
  const int64_t kbeg = (int64_t)blockIdx.y * kStageCols;
  const int64_t kend = std::min<int64_t>(K, kbeg + kStageCols);
  const int tid = threadIdx.x;
  __shared__ float red[32];
  __shared__ float s_inv;
  float inv = 1.0f;
  if (mode == GX_RMSNORM && t < M) {
    float ss = 0.f;
    for (int64_t k = tid; k < K; k += blockDim.x) {
      const float v = X[t * K + k];
      ss += v * v;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
      float v = tid < (int)(blockDim.x / 32) ? red[tid] : 0.f;
      v = warp_sum(v);
      if (tid == 0) s_inv = 1.0f / sqrtf(v / (float)K + eps);
    }
    __syncthreads();
    inv = s_inv;
  }
  const int tokb = 8 * NT;
  const int64_t mb = t / tokb, tt = t % tokb;
  const int nt = (int)(tt / 8), g = (int)(tt % 8);
  const int64_t nch = K / 16, ngr = K / 32;
  float *sums = reinterpret_cast<float *>(out + (size_t)((M + tokb - 1) / tokb) * (size_t)nch *
                                                    (size_t)(xchunk_bytes(NT) / 2));
  for (int64_t k0 = kbeg; k0 < kend; k0 += blockDim.x) {  // a warp covers one 32-column group
    const int64_t k = k0 + tid;
    float v = 0.f;
    if (t < M && k < kend) {
      if (mode == GX_RMSNORM) v = (X[t * K + k] * inv) * normw[k];
      else if (mode == GX_SWIGLU) v = silu_g(X[t * K + k]) * X2[t * K + k];
      else v = X[t * K + k];
    }
    const __half hv = __float2half_rn(v);
    const __half lv = __float2half_rn(v - __half2float(hv));
    float gs = __half2float(hv) + __half2float(lv);  // what the MMAs see
    gs = warp_sum(gs);
    if (k < kend) {
      const int64_t ch = k / 16;
      const int kk = (int)(k % 16);
      // B fragment: b0 = (k 2c, 2c+1), b1 = (k 2c+8, 2c+9) of column g
      const int c = (kk % 8) / 2, hi = kk / 8, e = kk % 2;
      const int lane = g * 4 + c;
      const int64_t idx = ((((mb * nch + ch) * 2) * NT + nt) * 32 + lane) * 4 + hi * 2 + e;
      out[idx] = hv;
      out[idx + NT * 32 * 4] = lv;  // the lo plane follows the hi plane of the chunk
      if ((tid & 31) == 0) sums[(mb * ngr + k / 32) * tokb + tt] = gs;
    }
  }
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// (float)(v & 63) and (float)(v & 255) on the FP32 pipe: the integer placed in
// the mantissa of 2^23, then 2^23 subtracted (both exact).
__device__ __forceinline__ float u2f6(uint32_t v) {
  return __uint_as_float(0x4B000000u | (v & 63u)) - 8388608.0f;
}
__device__ __forceinline__ float u2f8(uint32_t v) {
  return __uint_as_float(0x4B000000u | (v & 255u)) - 8388608.0f;
}
// A Q6_K scale byte as u8 (smask 0, the reference) or int8 (smask 0x80,
// llama.cpp): (v ^ smask) - smask, with bias = 2^23 + smask (exact).
__device__ __forceinline__ float s2f8(uint32_t v, uint32_t smask, float bias) {
  return __uint_as_float(0x4B000000u | ((v & 255u) ^ smask)) - bias;
}
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Word i of v by selects (a dynamic index into a register array would go
// through local memory).
__device__ __forceinline__ uint32_t word4(const uint4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// (v - sub) * scale + add with v the magic-biased f16 pair in `bits`.
__device__ __forceinline__ uint32_t deq(uint32_t bits, __half2 sub, __half2 scale, __half2 add) {
  return h2u(__hfma2(__hsub2(u2h(bits), sub), scale, add));
}

// One matrix of a launch: its row tiles are blockIdx.y in [ctile0, ctile0 +
// its ctiles).
struct GemmSeg {
  const uint8_t *w;
  float *C;
  int64_t ldc;
  int type, rows, unit_bytes, wt_bytes, wt_qbytes, ctile0;
  uint32_t smask;  // 0x80: Q6_K scale bytes are int8 (llama.cpp), else 0
};
constexpr int kGemmMaxSegs = 3;

struct GemmArgs {
  GemmSeg seg[kGemmMaxSegs];  // matrices sharing K and the staged input
  int nseg;
  const uint8_t *x;   // staged fragments
  const float *sums;  // per-token sums of x over 32-column groups
  int64_t M;
  int kc, kunits, nch_total;
  int max_unit;    // the largest unit of the segments: a stage's weight slot
  int accumulate;  // C += result (else C = result)
  int atomic;      // C += result with atomic adds (K split over gridDim.z CTAs)
  int *err;
};

// Q4_K unit with the 6-bit sub-scale folded into the A operand: sc * q
// (rows g) and 16 sc * q (rows g+8, high nibbles) are integers of at most 10
// significant bits, exact in f16, made by one f16x2 FMA per register
// ((1024 + q) sc - 1024 sc, a single rounding of an exact result). The
// MMAs then accumulate a whole 256-column unit, d is applied once per unit,
// and the mins term sum_g m_g S_g (S_g the staged group sums of x) is one
// more k16 MMA per token tile (A = the eight 6-bit mins of each row, B = the
// group sums as hi/lo f16), scaled by dmin. Two accumulators (even and odd
// chunks) keep the MMA chains short.
template <int NT>
__device__ __forceinline__ void gemm_unit_q4k(const uint8_t *wt, const uint8_t *xs, const float *sx,
                                              int lane, float (&acc)[NT][4]) {
  const int g = lane >> 2, c = lane & 3;
  const __half2 b1024 = __float2half2_rn(1024.f), m1024 = __float2half2_rn(-1024.f);
  const uint4 hA = *reinterpret_cast<const uint4 *>(wt + 2048 + 16 * g);
  const uint4 hB = *reinterpret_cast<const uint4 *>(wt + 2048 + 16 * (g + 8));
  const float dA = h2f((uint16_t)prmt(hA.x, hA.y, 0x0073u));
  const float dmA = h2f((uint16_t)prmt(hA.z, hA.w, 0x0073u));
  const float dB = h2f((uint16_t)prmt(hB.x, hB.y, 0x0073u)) * 0.0625f;
  const float dmB = h2f((uint16_t)prmt(hB.z, hB.w, 0x0073u));
  const uint4 *wq4 = reinterpret_cast<const uint4 *>(wt);  // a lane's 4 chunks per 16 bytes
  float ua[2][NT][4];
#pragma unroll
  for (int p = 0; p < 2; ++p)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) ua[p][nt][0] = ua[p][nt][1] = ua[p][nt][2] = ua[p][nt][3] = 0.f;
  uint4 q4 = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int gi = 0; gi < 8; ++gi) {
    if ((gi & 1) == 0) q4 = wq4[(gi >> 1) * 32 + lane];  // chunks 2 gi .. 2 gi + 3 (conflict-free)
    const int sh = 6 * (gi & 1);
    const uint32_t sa = (word4(hA, gi >> 1) >> sh) & 63u, sb = (word4(hB, gi >> 1) >> sh) & 63u;
    const __half2 scA = __hsub2(u2h(0x64006400u | sa | (sa << 16)), b1024);  // exact
    const __half2 scB = __hsub2(u2h(0x64006400u | sb | (sb << 16)), b1024);
    const __half2 ngA = __hmul2(scA, m1024), ngB = __hmul2(scB, m1024);      // -1024 sc, exact
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int ch = 2 * gi + cc;
      const uint32_t wd = word4(q4, ch & 3);
      const uint32_t hi = wd >> 8;
      const uint32_t a0 = h2u(__hfma2(u2h((wd & 0x000F000Fu) | 0x64006400u), scA, ngA));
      const uint32_t a1 = h2u(__hfma2(u2h((wd & 0x00F000F0u) | 0x64006400u), scB, ngB));
      const uint32_t a2 = h2u(__hfma2(u2h((hi & 0x000F000Fu) | 0x64006400u), scA, ngA));
      const uint32_t a3 = h2u(__hfma2(u2h((hi & 0x00F000F0u) | 0x64006400u), scB, ngB));
      const uint2 *xb = reinterpret_cast<const uint2 *>(xs + (size_t)ch * xchunk_bytes(NT)) + lane;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 bh = xb[nt * 32], bl = xb[NT * 32 + nt * 32];
        mma_16816(ua[cc][nt], a0, a1, a2, a3, bh.x, bh.y, ua[cc][nt]);
        mma_16816(ua[cc][nt], a0, a1, a2, a3, bl.x, bl.y, ua[cc][nt]);
      }
    }
  }
  // mins: A row g = (m_2c, m_2c+1) of row g, row g+8 the same of row g+8
  // (k = group, groups 8-15 absent); B = (S_2c, S_2c+1) of token g as hi/lo
  const uint32_t fA = word4(hA, c), fB = word4(hB, c);
  const uint32_t am0 = h2u(__hsub2(u2h(0x64006400u | ((fA >> 12) & 63u) | (((fA >> 18) & 63u) << 16)), b1024));
  const uint32_t am1 = h2u(__hsub2(u2h(0x64006400u | ((fB >> 12) & 63u) | (((fB >> 18) & 63u) << 16)), b1024));
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int tok = 8 * nt + g;
    const float s0 = sx[(2 * c) * (8 * NT) + tok], s1 = sx[(2 * c + 1) * (8 * NT) + tok];
    const __half2 sh2 = __floats2half2_rn(s0, s1);
    const __half2 sl2 = __floats2half2_rn(s0 - __low2float(sh2), s1 - __high2float(sh2));
    float mc[4] = {0.f, 0.f, 0.f, 0.f};
    mma_16816(mc, am0, am1, 0u, 0u, h2u(sh2), 0u, mc);
    mma_16816(mc, am0, am1, 0u, 0u, h2u(sl2), 0u, mc);
    acc[nt][0] = fmaf(dA, ua[0][nt][0] + ua[1][nt][0], fmaf(-dmA, mc[0], acc[nt][0]));
    acc[nt][1] = fmaf(dA, ua[0][nt][1] + ua[1][nt][1], fmaf(-dmA, mc[1], acc[nt][1]));
    acc[nt][2] = fmaf(dB, ua[0][nt][2] + ua[1][nt][2], fmaf(-dmB, mc[2], acc[nt][2]));
    acc[nt][3] = fmaf(dB, ua[0][nt][3] + ua[1][nt][3], fmaf(-dmB, mc[3], acc[nt][3]));
  }
}

// Q6_K, Q4_0 and Q8_0 units (Q4_K: gemm_unit_q4k). Weight words are read
// 16 bytes per lane (a lane's words of four 16-column chunks: conflict-free)
// in blocks of four chunks; each scale group's MMAs go into `tmp`, which
// the group's f32 scale then adds into `acc`.
template <int TYPE, int NT>
__device__ __forceinline__ void gemm_unit(const uint8_t *wt, const uint8_t *xs, const float *sx,
                                          int kc, int wt_qbytes, uint32_t smask, int lane,
                                          float (&acc)[NT][4]) {
  const int g = lane >> 2;
  // chunks per scale group: Q6_K scales every 16 columns, the others every 32
  constexpr int cpg = (TYPE == IFX_TYPE_Q6_K) ? 1 : 2;
  float dA = 0.f, dB = 0.f;
  if (TYPE == IFX_TYPE_Q6_K) {
    dA = h2f(*reinterpret_cast<const uint16_t *>(wt + 3072 + 256 + 2 * g));
    dB = h2f(*reinterpret_cast<const uint16_t *>(wt + 3072 + 256 + 2 * (g + 8))) * 0.0625f;
  }
  const uint4 *w4 = reinterpret_cast<const uint4 *>(wt);
  float tmp[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) tmp[nt][0] = tmp[nt][1] = tmp[nt][2] = tmp[nt][3] = 0.f;
  const int nch = kc / 16;  // Q8_0 units may end in a partial block (kc 32, 96, 160)
#pragma unroll 1
  for (int cb = 0; cb < (nch + 3) / 4; ++cb) {
    uint4 qa = make_uint4(0u, 0u, 0u, 0u), qb = qa, hw = qa;
    if (TYPE == IFX_TYPE_Q8_0) {  // a lane's 16 bytes hold two chunks
      qa = w4[(2 * cb) * 32 + lane];
      if (4 * cb + 2 < nch) qb = w4[(2 * cb + 1) * 32 + lane];
    } else {
      qa = w4[cb * 32 + lane];
    }
    if (TYPE == IFX_TYPE_Q6_K) hw = reinterpret_cast<const uint4 *>(wt + 2048)[(cb >> 1) * 32 + lane];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int ch = 4 * cb + j;
      if (ch >= nch) break;
      // exact integer A fragments; rows g+8 come from the high nibble and
      // carry a factor 16 (Q6_K, Q4_0), folded into their scale below
      uint32_t a[4];
      if (TYPE == IFX_TYPE_Q6_K) {
        const uint32_t wd = word4(qa, j);
        uint32_t H = word4(hw, 2 * (cb & 1) + (j >> 1));
        if (j & 1) H >>= 8;
        const __half2 sub0 = __float2half2_rn(1056.f), sub1 = __float2half2_rn(1536.f);
        const uint32_t hi = wd >> 8, H4 = H >> 4;
        a[0] = h2u(__hsub2(u2h((wd & 0x000F000Fu) | ((H & 0x00030003u) << 4) | 0x64006400u), sub0));
        a[1] = h2u(__hsub2(u2h((wd & 0x00F000F0u) | ((H & 0x000C000Cu) << 6) | 0x64006400u), sub1));
        a[2] = h2u(__hsub2(u2h((hi & 0x000F000Fu) | ((H4 & 0x00030003u) << 4) | 0x64006400u), sub0));
        a[3] = h2u(__hsub2(u2h((hi & 0x00F000F0u) | ((H4 & 0x000C000Cu) << 6) | 0x64006400u), sub1));
      } else if (TYPE == IFX_TYPE_Q4_0) {
        const uint32_t wd = word4(qa, j);
        const __half2 sub0 = __float2half2_rn(1032.f), sub1 = __float2half2_rn(1152.f);
        const uint32_t hi = wd >> 8;
        a[0] = h2u(__hsub2(u2h((wd & 0x000F000Fu) | 0x64006400u), sub0));
        a[1] = h2u(__hsub2(u2h((wd & 0x00F000F0u) | 0x64006400u), sub1));
        a[2] = h2u(__hsub2(u2h((hi & 0x000F000Fu) | 0x64006400u), sub0));
        a[3] = h2u(__hsub2(u2h((hi & 0x00F000F0u) | 0x64006400u), sub1));
      } else {  // Q8_0: bytes q + 128
        const uint4 &q = (j < 2) ? qa : qb;
        const uint32_t w0 = (j & 1) ? q.z : q.x, w1 = (j & 1) ? q.w : q.y;
        const __half2 sub = __float2half2_rn(1152.f);
        a[0] = h2u(__hsub2(u2h(prmt(w0, 0x64646464u, 0x4140u)), sub));
        a[1] = h2u(__hsub2(u2h(prmt(w0, 0x64646464u, 0x4342u)), sub));
        a[2] = h2u(__hsub2(u2h(prmt(w1, 0x64646464u, 0x4140u)), sub));
        a[3] = h2u(__hsub2(u2h(prmt(w1, 0x64646464u, 0x4342u)), sub));
      }
      const uint2 *xb = reinterpret_cast<const uint2 *>(xs + (size_t)ch * xchunk_bytes(NT)) + lane;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 bh = xb[nt * 32], bl = xb[NT * 32 + nt * 32];
        mma_16816(tmp[nt], a[0], a[1], a[2], a[3], bh.x, bh.y, tmp[nt]);
        mma_16816(tmp[nt], a[0], a[1], a[2], a[3], bl.x, bl.y, tmp[nt]);
      }
      if ((j + 1) % cpg) continue;
      // the group ends: its scales for rows g (sA) and g+8 (sB), f32
      const int gi = ch / cpg;
      float sA, sB;
      if (TYPE == IFX_TYPE_Q6_K) {
        const uint8_t *scb = wt + 3072;
        const float sbias = 8388608.0f + (float)smask;
        sA = dA * s2f8(scb[16 * g + gi], smask, sbias);
        sB = dB * s2f8(scb[16 * (g + 8) + gi], smask, sbias);
      } else {
        const int nb = kc / 32;
        sA = h2f(*reinterpret_cast<const uint16_t *>(wt + wt_qbytes + (g * nb + gi) * 2));
        sB = h2f(*reinterpret_cast<const uint16_t *>(wt + wt_qbytes + ((g + 8) * nb + gi) * 2));
        if (TYPE == IFX_TYPE_Q4_0) sB *= 0.0625f;
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[nt][0] = fmaf(sA, tmp[nt][0], acc[nt][0]);
        acc[nt][1] = fmaf(sA, tmp[nt][1], acc[nt][1]);
        acc[nt][2] = fmaf(sB, tmp[nt][2], acc[nt][2]);
        acc[nt][3] = fmaf(sB, tmp[nt][3], acc[nt][3]);
        tmp[nt][0] = tmp[nt][1] = tmp[nt][2] = tmp[nt][3] = 0.f;
      }
    }
  }
}

// Blocks of 8 * NT tokens x 128 weight rows; gridDim.z splits K (each z
// takes a contiguous share of the row tile's units, results added
// atomically).
template <int NT>
__global__ void __launch_bounds__(kGThreads, NT <= 2 ? 3 : 1) gemm_kernel(const __grid_constant__ GemmArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty_bar = full_bar + kGStages;
  constexpr int tokb = 8 * NT;
  const int xbytes = a.kc / 16 * xchunk_bytes(NT);           // x hi + lo of the unit's columns
  const int sbytes = a.kc / 32 * tokb * (int)sizeof(float);  // per-token group sums
  const int stage_bytes = a.max_unit + xbytes + sbytes;
  uint8_t *ring = smem + 128;
  int si = 0;  // this CTA's matrix
#pragma unroll
  for (int i = 1; i < kGemmMaxSegs; ++i)
    if (i < a.nseg && (int)blockIdx.y >= a.seg[i].ctile0) si = i;
  const GemmSeg S = a.seg[si];
  const int mb = blockIdx.x, ctile = blockIdx.y - S.ctile0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int upc = (a.kunits + gridDim.z - 1) / gridDim.z;  // units per K split
  const int u0 = blockIdx.z * upc, n = max(0, min(a.kunits, u0 + upc) - u0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 8);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // programmatic serialization: the next grid may start its weight fetch;
  // this grid's weights do not depend on the previous grid, its staged
  // activations do (read after griddepcontrol.wait)
  pdl_launch();
  if (warp == 8) {
    if (lane == 0) {
      auto xcopy = [&](int i) {
        const int st = i % kGStages, u = u0 + i;
        uint8_t *dst = ring + (size_t)st * stage_bytes;
        const uint8_t *xsrc =
            a.x + ((size_t)mb * a.nch_total + (size_t)u * (a.kc / 16)) * xchunk_bytes(NT);
        const uint8_t *ssrc = reinterpret_cast<const uint8_t *>(
            a.sums + ((size_t)mb * (a.nch_total / 2) + (size_t)u * (a.kc / 32)) * tokb);
        bulk_g2s(dst + a.max_unit, xsrc, (uint32_t)xbytes, &full_bar[st]);
        bulk_g2s(dst + a.max_unit + xbytes, ssrc, (uint32_t)sbytes, &full_bar[st]);
      };
      const int pre = min(n, kGStages);
      for (int i = 0; i < n; ++i) {
        const int st = i % kGStages;
        const uint32_t ph = (uint32_t)(i / kGStages) & 1u;
        if (i >= kGStages && !mbar_wait(&empty_bar[st], ph ^ 1u, a.err, 201)) break;
        uint8_t *dst = ring + (size_t)st * stage_bytes;
        const uint8_t *wsrc = S.w + ((size_t)ctile * a.kunits + u0 + i) * S.unit_bytes;
        mbar_arrive_expect_tx(&full_bar[st], (uint32_t)(S.unit_bytes + xbytes + sbytes));
        bulk_g2s(dst, wsrc, (uint32_t)S.unit_bytes, &full_bar[st]);
        if (i + 1 == pre) {  // the first stages' weights are on their way
          pdl_wait();
          for (int k = 0; k < pre; ++k) xcopy(k);
        } else if (i >= pre) {
          xcopy(i);
        }
      }
    }
    return;
  }

  if (n == 0) return;  // an empty K split (the producer issued nothing either)
  pdl_wait();  // the outputs were zeroed (or hold the residual) by earlier grids
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  for (int i = 0; i < n; ++i) {
    const int st = i % kGStages;
    const uint32_t ph = (uint32_t)(i / kGStages) & 1u;
    if (!mbar_wait(&full_bar[st], ph, a.err, 202)) return;
    const uint8_t *base = ring + (size_t)st * stage_bytes;
    const uint8_t *wt = base + (size_t)warp * S.wt_bytes;
    const uint8_t *xs = base + a.max_unit;
    const float *sx = reinterpret_cast<const float *>(xs + a.kc / 16 * xchunk_bytes(NT));
    switch (S.type) {
      case IFX_TYPE_Q4_K: gemm_unit_q4k<NT>(wt, xs, sx, lane, acc); break;
      case IFX_TYPE_Q6_K: gemm_unit<IFX_TYPE_Q6_K, NT>(wt, xs, sx, a.kc, S.wt_qbytes, S.smask, lane, acc); break;
      case IFX_TYPE_Q4_0: gemm_unit<IFX_TYPE_Q4_0, NT>(wt, xs, sx, a.kc, S.wt_qbytes, S.smask, lane, acc); break;
      default: gemm_unit<IFX_TYPE_Q8_0, NT>(wt, xs, sx, a.kc, S.wt_qbytes, S.smask, lane, acc); break;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
  }
  // D[nt] = rows (g, g+8) x tokens (8nt + 2c, 8nt + 2c + 1)
  const int g = lane >> 2, c = lane & 3;
  const int r0 = ctile * 128 + warp * 16 + g;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int row = r0 + ((j & 2) ? 8 : 0);
      const int64_t tok = (int64_t)mb * tokb + nt * 8 + 2 * c + (j & 1);
      if (row < S.rows && tok < a.M) {
        float *p = S.C + tok * S.ldc + row;
        if (a.atomic) red_add_f32(p, acc[nt][j]);
        else *p = a.accumulate ? (*p + acc[nt][j]) : acc[nt][j];
      }
    }
}

}  // namespace

// Staged x of an M x K input in blocks of 8 * NT tokens: the hi/lo
// fragments of every 16-column chunk of every block, then the per-token
// 32-column group sums.
static size_t xfrag_frag_bytes(int64_t M, int64_t K, int NT) {
  const int64_t tokb = 8 * NT, mblocks = (M + tokb - 1) / tokb;
  return (size_t)mblocks * (size_t)(K / 16) * (size_t)xchunk_bytes(NT);
}

static size_t xfrag_bytes(int64_t M, int64_t K, int NT) {
  const int64_t tokb = 8 * NT, mblocks = (M + tokb - 1) / tokb;
  return xfrag_frag_bytes(M, K, NT) + (size_t)mblocks * (size_t)(K / 32) * tokb * sizeof(float);
}

static int small_nt(int64_t M) { return M <= 16 ? 2 : 4; }

size_t gemm_xfrag_bytes(int64_t M, int64_t K) {
  const size_t sync_bytes = xfrag_bytes(M, K, kGemmTokens / 8);
  return tc_gemm_eligible(K) ? std::max(sync_bytes, tc_xtile_bytes(M, K)) : sync_bytes;
}

size_t gemm_small_xfrag_bytes(int64_t M, int64_t K) { return xfrag_bytes(M, K, small_nt(M)); }

static ifx_status stage_sync(const float *X, const float *X2, const float *normw, float eps,
                             int mode, int64_t M, int64_t K, int NT, void *xfrag, cudaStream_t st,
                             StageZero z = StageZero{}, bool pdl = false) {
  if (K % 32) return fail(IFX_ERR_SHAPE, "gemm: K must be a multiple of 32");
  const int64_t tokb = 8 * NT, mpad = (M + tokb - 1) / tokb * tokb;
  const dim3 grid((unsigned)mpad, (unsigned)((K + kStageCols - 1) / kStageCols));
  IFX_CUDA(launch(stage_x_kernel, grid, dim3(256), 0, st, pdl, X, X2, normw, eps, mode, M, K, NT,
                  reinterpret_cast<__half *>(xfrag), z));
  return IFX_OK;
}

ifx_status gemm_stage_x(const float *X, const float *X2, const float *normw, float eps, int mode,
                        int64_t M, int64_t K, void *xfrag, cudaStream_t st) {
  if (K % 32) return fail(IFX_ERR_SHAPE, "gemm: K must be a multiple of 32");
  if (tc_gemm_eligible(K)) return tc_stage_x(X, X2, normw, eps, mode, M, K, xfrag, st);
  return stage_sync(X, X2, normw, eps, mode, M, K, kGemmTokens / 8, xfrag, st);
}

ifx_status gemm_small_stage_x(const float *X, const float *X2, const float *normw, float eps,
                              int mode, int64_t M, int64_t K, void *xfrag, cudaStream_t st,
                              StageZero zero, bool pdl) {
  if (M > kGemmSmallMax) return fail(IFX_ERR_UNSUPPORTED, "gemm: small batch above 32 tokens");
  return stage_sync(X, X2, normw, eps, mode, M, K, small_nt(M), xfrag, st, zero, pdl);
}

// n (<= 3) matrices with the same K and unit width over one staged input:
// their row tiles side by side in one launch (blockIdx.y), K split over
// gridDim.z CTAs (results added atomically when ksplit > 1).
template <int NT>
static ifx_status launch_sync(const QMatrix *const *W, float *const *C, const int64_t *ldc, int n,
                              const void *xfrag, int64_t M, int accumulate, int ksplit, int *err,
                              cudaStream_t st, bool pdl = false) {
  if (n < 1 || n > kGemmMaxSegs) return fail(IFX_ERR_INVALID_ARGUMENT, "gemm: 1 to 3 matrices");
  GemmArgs a{};
  a.nseg = n;
  a.x = reinterpret_cast<const uint8_t *>(xfrag);
  a.sums = reinterpret_cast<const float *>(a.x + xfrag_frag_bytes(M, W[0]->L.cols, NT));
  a.M = M;
  a.kc = W[0]->L.kc;
  a.kunits = W[0]->L.kunits;
  a.nch_total = (int)(W[0]->L.cols / 16);
  int ctiles = 0;
  for (int i = 0; i < n; ++i) {
    const QLayout &L = W[i]->L;
    if (L.kc != a.kc || L.cols != W[0]->L.cols)
      return fail(IFX_ERR_SHAPE, "gemm: fused matrices must share K and unit width");
    GemmSeg &S = a.seg[i];
    S.w = W[i]->d;
    S.C = C[i];
    S.ldc = ldc[i];
    S.type = L.type;
    S.rows = (int)L.rows;
    S.unit_bytes = L.unit_bytes;
    S.wt_bytes = L.wt_bytes;
    S.wt_qbytes = L.wt_qbytes;
    S.smask = L.q6_s8 ? 0x80u : 0u;
    S.ctile0 = ctiles;
    ctiles += L.ctiles;
    a.max_unit = std::max(a.max_unit, L.unit_bytes);
  }
  a.accumulate = accumulate;
  a.atomic = ksplit > 1 ? 1 : 0;
  a.err = err;
  const size_t smem = 128 + (size_t)kGStages * (a.max_unit + a.kc / 16 * xchunk_bytes(NT) +
                                                a.kc / 32 * 8 * NT * sizeof(float));
  if (smem > 226 * 1024) return fail(IFX_ERR_UNSUPPORTED, "gemm: shared memory plan too large");
  static size_t attr = 0;
  if (smem > attr) {
    IFX_CUDA(cudaFuncSetAttribute(gemm_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    attr = smem;
  }
  dim3 grid((unsigned)((M + 8 * NT - 1) / (8 * NT)), (unsigned)ctiles, (unsigned)ksplit);
  IFX_CUDA(launch(gemm_kernel<NT>, grid, dim3(kGThreads), smem, st, pdl, a));
  return IFX_OK;
}

template <int NT>
static ifx_status launch_sync(const QMatrix &W, const void *xfrag, int64_t M, float *C,
                              int64_t ldc, int accumulate, int ksplit, int *err, cudaStream_t st,
                              bool pdl = false) {
  const QMatrix *w[1] = {&W};
  float *c[1] = {C};
  const int64_t l[1] = {ldc};
  return launch_sync<NT>(w, c, l, 1, xfrag, M, accumulate, ksplit, err, st, pdl);
}

ifx_status gemm_run_multi(const QMatrix *const *W, float *const *C, const int64_t *ldc, int n,
                          const void *xfrag, int64_t M, int accumulate, int *err,
                          cudaStream_t st) {
  if (n >= 1 && W[0]->L.dense) {
    for (int i = 0; i < n; ++i) IFX_TRY(dense_gemm(*W[i], xfrag, M, C[i], ldc[i], accumulate, st));
    return IFX_OK;
  }
  if (n >= 1 && tc_gemm_eligible(W[0]->L.cols))
    return tc_gemm_run_multi(W, C, ldc, n, xfrag, M, accumulate, err, st);
  for (int i = 0; i < n; ++i) IFX_TRY(gemm_run(*W[i], xfrag, M, C[i], ldc[i], accumulate, err, st));
  return IFX_OK;
}

ifx_status gemm_run(const QMatrix &W, const void *xfrag, int64_t M, float *C, int64_t ldc,
                    int accumulate, int *err, cudaStream_t st) {
  if (W.L.dense) return dense_gemm(W, xfrag, M, C, ldc, accumulate, st);
  if (tc_gemm_eligible(W.L.cols)) return tc_gemm_run(W, xfrag, M, C, ldc, accumulate, err, st);
  return launch_sync<kGemmTokens / 8>(W, xfrag, M, C, ldc, accumulate, 1, err, st);
}

ifx_status gemm_small_run_multi(const QMatrix *const *W, float *const *C, const int64_t *ldc,
                                int n, const void *xfrag, int64_t M, int *err, cudaStream_t st) {
  if (n >= 1 && W[0]->L.dense) {
    for (int i = 0; i < n; ++i) IFX_TRY(dense_gemm(*W[i], xfrag, M, C[i], ldc[i], 1, st));
    return IFX_OK;
  }
  if (M > kGemmSmallMax) return fail(IFX_ERR_UNSUPPORTED, "gemm: small batch above 32 tokens");
  for (int i = 1; i < n; ++i)  // different unit widths run as separate launches
    if (W[i]->L.kc != W[0]->L.kc) {
      for (int k = 0; k < n; ++k) IFX_TRY(gemm_small_run(*W[k], xfrag, M, C[k], ldc[k], err, st));
      return IFX_OK;
    }
  int ctiles = 0;
  for (int i = 0; i < n; ++i) ctiles += W[i]->L.ctiles;
  const int ksplit = std::max(1, std::min(W[0]->L.kunits, (2 * kNumSMs + ctiles - 1) / ctiles));
  if (small_nt(M) == 2) return launch_sync<2>(W, C, ldc, n, xfrag, M, 1, ksplit, err, st, true);
  return launch_sync<4>(W, C, ldc, n, xfrag, M, 1, ksplit, err, st, true);
}

ifx_status gemm_small_run(const QMatrix &W, const void *xfrag, int64_t M, float *C, int64_t ldc,
                          int *err, cudaStream_t st) {
  if (W.L.dense) return dense_gemm(W, xfrag, M, C, ldc, 1, st);
  if (M > kGemmSmallMax) return fail(IFX_ERR_UNSUPPORTED, "gemm: small batch above 32 tokens");
  // enough K splits for about two CTAs per SM, never more than the units
  const int ksplit = std::max(1, std::min(W.L.kunits, (2 * kNumSMs + W.L.ctiles - 1) / W.L.ctiles));
  if (small_nt(M) == 2) return launch_sync<2>(W, xfrag, M, C, ldc, 1, ksplit, err, st, true);
  return launch_sync<4>(W, xfrag, M, C, ldc, 1, ksplit, err, st, true);
}

}  // namespace ifx
