// Prefill GEMM on the 5th-generation tensor cores: C[M, rows] (+)= f(X) . W^T
// with tcgen05.mma (kind::f16, 128 x N x 16 per instruction, f32
// accumulators in tensor memory).
//
// One CTA computes a 128-row x N-token tile (N <= 256) over the whole K:
//   * warp 0 (one lane) bulk-copies the activation tiles of each 32-column
//     k-block into shared memory (pre-swizzled images written by
//     tc_stage_x_kernel, so a 1-D bulk copy lands them in the canonical
//     64-byte-swizzle K-major layout the MMA reads);
//   * warps 4-11 dequantise the weight rows of the k-block from the
//     repacked units (qlayout.cuh) straight into the same layout, one
//     16-row warp tile each;
//   * warp 1 (one lane) issues the MMAs and commits their completion to
//     the stage's "empty" barrier; warp 2 owns the tensor-memory allocation;
//   * warps 4-7 (one per 32-lane quarter of tensor memory) read the
//     accumulators back with tcgen05.ld and write C.
//
// Precision: the reference dequantises to f32 and multiplies in f32. Here
// each dequantised weight w (f32, the reference's formula) is split as
// w * 2^8 ~= a_hi + a_lo (two f16, about 22 bits) and each activation as
// x ~= x_hi + x_lo; three MMAs accumulate a_hi x_hi + a_hi x_lo + a_lo x_hi
// in f32 (the dropped a_lo x_lo term is below 2^-22 relative), and the
// epilogue removes the 2^8. Weight magnitudes up to 255 are representable.
#include <algorithm>

#include "gemm.cuh"

namespace ifx {

namespace {

constexpr int kTcRows = 128;   // weight rows per CTA (MMA M)
constexpr int kTcKB = 32;      // k per pipeline stage: one 64-byte swizzle row of f16
constexpr int kTcStages = 4;   // four stages of 48 KB at N = 256: copies land well ahead
constexpr int kTcThreads = 384;
constexpr int kTcDeq0 = 4;     // first dequantising warp; warps 4..11, one 16-row tile each
constexpr float kTcAScale = 256.0f;
constexpr int kTcFetch = 64;   // columns a dequantising lane fetches at once (two stages)
constexpr int kATile = kTcRows * kTcKB * 2;  // bytes of one A plane per stage (8 KB)

// Byte offset of element (r, k), 0 <= k < 32, in a K-major tile with the
// 64-byte swizzle: 8-row atoms of 64-byte rows, stacked every 512 bytes;
// 16-byte chunk k/8 of row r sits at chunk (k/8) ^ ((r % 8) / 2) (address
// bits [4, 6) XOR bits [7, 9) of a 512-byte aligned atom).
__host__ __device__ __forceinline__ uint32_t sw64(int r, int k) {
  return (uint32_t)((r >> 3) * 512 + (r & 7) * 64 + ((((k >> 3) ^ ((r & 7) >> 1)) & 3) << 4) +
                    (k & 7) * 2);
}

// Shared-memory matrix descriptor (tcgen05): start address >> 4, leading
// byte offset 16 (unused by swizzled K-major layouts), stride byte offset
// 512 (between 8-row atoms), descriptor version 1, 64-byte swizzle (4).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}

// Instruction descriptor, kind::f16: f32 accumulator, f16 A and B, both
// K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Starts pulling [p, p + bytes) into L2 (16-byte aligned, multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Generic-proxy shared-memory writes become visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Sixteen consecutive 32-bit columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float silu_t(float v) {
  float c = fminf(fmaxf(v, -80.0f), 80.0f);
  return v * (1.0f / (1.0f + expf(-c)));
}

// Activation staging: token t's row of f(X) as hi/lo f16 planes in the tile
// images [token tile][k-block][plane][ntile x 32 f16, swizzled]. One CTA per
// token (padding tokens of the last tile are zero); each thread writes
// 16-byte chunks (8 consecutive columns) of both planes.
__global__ void tc_stage_x_kernel(const float *X, const float *X2, const float *normw, float eps,
                                  int mode, int64_t M, int64_t K, int ntile, uint8_t *out) {
  const int64_t t = blockIdx.x;
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
  const int64_t tt = t / ntile;
  const int n = (int)(t % ntile);
  const int64_t nkb = K / kTcKB;
  const size_t tile = (size_t)ntile * kTcKB * 2;
  for (int64_t c8 = tid; c8 < K / 8; c8 += blockDim.x) {
    const int64_t k0 = c8 * 8;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float y = 0.f;
      if (t < M) {
        const int64_t k = k0 + j;
        if (mode == GX_RMSNORM) y = (X[t * K + k] * inv) * normw[k];
        else if (mode == GX_SWIGLU) y = silu_t(X[t * K + k]) * X2[t * K + k];
        else y = X[t * K + k];
      }
      v[j] = y;
    }
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
      const __half2 l = __floats2half2_rn(v[2 * j] - __low2float(h), v[2 * j + 1] - __high2float(h));
      hw[j] = *reinterpret_cast<const uint32_t *>(&h);
      lw[j] = *reinterpret_cast<const uint32_t *>(&l);
    }
    const int64_t kb = k0 / kTcKB;
    const size_t base = (size_t)((tt * nkb + kb) * 2) * tile + sw64(n, (int)(k0 % kTcKB));
    *reinterpret_cast<uint4 *>(out + base) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4 *>(out + base + tile) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}

constexpr int kTcMaxSegs = 3;

// One weight matrix of a launch; its row tiles are CTAs [ctile0, ctile0 + ctiles).
struct TcSeg {
  const uint8_t *w;  // repacked units
  float *C;
  int64_t ldc;
  int type, rows, kc, kunits, unit_bytes, wt_bytes, wt_qbytes, ctile0, ctiles;
  uint32_t smask;  // 0x80: Q6_K scale bytes are int8 (llama.cpp), else 0
};

struct TcArgs {
  TcSeg seg[kTcMaxSegs];  // matrices sharing K and the staged input
  int nseg;
  const uint8_t *xt;  // staged activation tiles
  int M, nkb, ntile, tmem_cols;
  int accumulate;
  int *err;
};

// Raw words of one 64-column fetch block (four 16-column chunks, two
// stages) for lane (g, c) of a warp tile: loaded one block ahead of use.
struct TcRaw {
  uint4 q, q2;        // quantised words (q2: second half of a Q8_0 block)
  uint32_t s0, s1;    // per-row scale words (rows g, g + 8)
  uint2 h;            // Q6_K 2-bit plane words
  uint4 hd0, hd1;     // Q4_K row headers (rows g, g + 8)
};

template <int TYPE>
__device__ __forceinline__ void tc_fetch(const TcSeg &a, int ctile, int wt, int kb, int lane,
                                         TcRaw &R) {
  const int g = lane >> 2;
  const int bpu = a.kc / kTcFetch;  // fetch blocks per unit
  const int unit = kb / bpu, sub = kb - unit * bpu;
  const uint8_t *wp = a.w + ((size_t)ctile * a.kunits + unit) * a.unit_bytes + (size_t)wt * a.wt_bytes;
  if (TYPE == IFX_TYPE_Q8_0) {
    const uint4 *qv = reinterpret_cast<const uint4 *>(wp);
    R.q = qv[(2 * sub) * 32 + lane];
    R.q2 = qv[(2 * sub + 1) * 32 + lane];
  } else {
    R.q = reinterpret_cast<const uint4 *>(wp)[sub * 32 + lane];
  }
  if (TYPE == IFX_TYPE_Q4_K) {
    const uint4 *hd = reinterpret_cast<const uint4 *>(wp + 2048);
    R.hd0 = hd[g];
    R.hd1 = hd[g + 8];
  } else if (TYPE == IFX_TYPE_Q6_K) {
    const uint32_t *hp = reinterpret_cast<const uint32_t *>(wp + 2048);
    R.h = *reinterpret_cast<const uint2 *>(hp + ((sub / 2) * 32 + lane) * 4 + (2 * sub) % 4);
    const uint8_t *scb = wp + 3072;
    R.s0 = *reinterpret_cast<const uint32_t *>(scb + 16 * g + 4 * sub);
    R.s1 = *reinterpret_cast<const uint32_t *>(scb + 16 * (g + 8) + 4 * sub);
    R.hd0.x = *reinterpret_cast<const uint16_t *>(scb + 256 + 2 * g);
    R.hd0.y = *reinterpret_cast<const uint16_t *>(scb + 256 + 2 * (g + 8));
  } else {  // Q4_0, Q8_0: f16 scales of the two 32-column blocks of the k-block
    const int nb = a.kc / 32;
    const uint8_t *sc = wp + a.wt_qbytes;
    R.s0 = *reinterpret_cast<const uint32_t *>(sc + (g * nb + 2 * sub) * 2);
    R.s1 = *reinterpret_cast<const uint32_t *>(sc + ((g + 8) * nb + 2 * sub) * 2);
  }
}

__device__ __forceinline__ __half2 u2h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Splits w * 2^8 for a pair of weights into hi/lo f16 pairs and stores them.
__device__ __forceinline__ void tc_store_pair(float x0, float x1, uint8_t *ahi, uint8_t *alo,
                                              uint32_t off) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 hf = __half22float2(h);
  *reinterpret_cast<__half2 *>(ahi + off) = h;
  *reinterpret_cast<__half2 *>(alo + off) = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
}

// Dequantises half `half` (chunks 2 half, 2 half + 1) of the fetched block
// into one stage's A planes (rows 16 wt + {g, g+8}, 32 columns). The
// quantised values become exact small integers in f16 first (the bits OR-ed
// under the exponent of 1024, then 1024 plus the type's bias subtracted —
// rows g + 8 come from the high nibble and carry a factor 16, folded into
// their scale), as the repacked A-fragment layout allows: register a0 holds
// (row g, columns 2c, 2c+1), a1 (row g+8, same columns), a2 (row g, 2c+8,
// 2c+9), a3 (row g+8, 2c+8, 2c+9) of the chunk. One 32-column stage is one
// Q4_K group, two Q6_K scale groups, one Q4_0 / Q8_0 block: the scales are
// decoded once per stage, pre-multiplied by 2^8.
template <int TYPE>
__device__ __forceinline__ void tc_emit(const TcSeg &a, const TcRaw &R, int wt, int kb, int half,
                                        int lane, uint8_t *ahi, uint8_t *alo) {
  const int g = lane >> 2, c = lane & 3;
  const int bpu = a.kc / kTcFetch;
  const int sub = kb % bpu;
  const uint32_t words[4] = {R.q.x, R.q.y, R.q.z, R.q.w};
  const int r0 = 16 * wt + g;
  // per-row (g, g+8) multiplier and offset of this stage: w = mul * q' - off
  float mul0, mul1, off0 = 0.f, off1 = 0.f;
  if (TYPE == IFX_TYPE_Q4_K) {
    // dequant.rs:151-158: dall = d * sc, dm = dmin * mn, y = dall * q - dm
    const int gi = 2 * sub + half, j = gi & 1;  // the stage's 32-column group
    float dall[2], dmn[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 hd = h ? R.hd1 : R.hd0;
      const float d = h2f((uint16_t)prmt(hd.x, hd.y, 0x0073u));
      const float dm = h2f((uint16_t)prmt(hd.z, hd.w, 0x0073u));
      const uint32_t f = sub == 0 ? hd.x : sub == 1 ? hd.y : sub == 2 ? hd.z : hd.w;
      dall[h] = d * (float)((f >> (6 * j)) & 63u);
      dmn[h] = dm * (float)((f >> (12 + 6 * j)) & 63u);
    }
    mul0 = dall[0] * kTcAScale;
    mul1 = dall[1] * (kTcAScale / 16.f);
    off0 = dmn[0] * kTcAScale;
    off1 = dmn[1] * kTcAScale;
  } else if (TYPE == IFX_TYPE_Q6_K) {
    mul0 = h2f((uint16_t)R.hd0.x) * kTcAScale;  // d; the 16-column scales follow per chunk
    mul1 = h2f((uint16_t)R.hd0.y) * (kTcAScale / 16.f);
  } else {  // Q4_0 / Q8_0: the f16 scale of the stage's 32-column block
    mul0 = h2f((uint16_t)(half ? (R.s0 >> 16) : (R.s0 & 0xffffu))) * kTcAScale;
    mul1 = h2f((uint16_t)(half ? (R.s1 >> 16) : (R.s1 & 0xffffu))) *
           (TYPE == IFX_TYPE_Q4_0 ? kTcAScale / 16.f : kTcAScale);
  }
#pragma unroll
  for (int ii = 0; ii < 2; ++ii) {
    const int i = 2 * half + ii;  // 16-column chunk of the fetch block
    uint32_t av[4];
    float m0 = mul0, m1 = mul1;
    if (TYPE == IFX_TYPE_Q4_K || TYPE == IFX_TYPE_Q4_0) {
      const uint32_t wd = words[i], hi = wd >> 8;
      const __half2 sub0 = __float2half2_rn(TYPE == IFX_TYPE_Q4_K ? 1024.f : 1032.f);
      const __half2 sub1 = __float2half2_rn(TYPE == IFX_TYPE_Q4_K ? 1024.f : 1152.f);
      av[0] = wd & 0x000F000Fu;
      av[1] = wd & 0x00F000F0u;
      av[2] = hi & 0x000F000Fu;
      av[3] = hi & 0x00F000F0u;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const __half2 v = __hsub2(u2h2(av[r] | 0x64006400u), (r & 1) ? sub1 : sub0);
        av[r] = *reinterpret_cast<const uint32_t *>(&v);
      }
    } else if (TYPE == IFX_TYPE_Q6_K) {
      // dequant.rs:189-196: q = low nibble | 2 high bits << 4, y = (d * sc) * (q - 32)
      const uint32_t wd = words[i], hi = wd >> 8;
      uint32_t H = (i >> 1) ? R.h.y : R.h.x;
      if (i & 1) H >>= 8;
      const uint32_t H4 = H >> 4;
      const __half2 sub0 = __float2half2_rn(1056.f), sub1 = __float2half2_rn(1536.f);
      av[0] = (wd & 0x000F000Fu) | ((H & 0x00030003u) << 4);
      av[1] = (wd & 0x00F000F0u) | ((H & 0x000C000Cu) << 6);
      av[2] = (hi & 0x000F000Fu) | ((H4 & 0x00030003u) << 4);
      av[3] = (hi & 0x00F000F0u) | ((H4 & 0x000C000Cu) << 6);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const __half2 v = __hsub2(u2h2(av[r] | 0x64006400u), (r & 1) ? sub1 : sub0);
        av[r] = *reinterpret_cast<const uint32_t *>(&v);
      }
      // scale of the 16-column chunk: u8 (the reference) or int8 (smask 0x80)
      m0 *= (float)(int)(((R.s0 >> (8 * i)) & 0xffu) ^ a.smask) - (float)a.smask;
      m1 *= (float)(int)(((R.s1 >> (8 * i)) & 0xffu) ^ a.smask) - (float)a.smask;
    } else {  // Q8_0, dequant.rs:93-111: q * d (bytes stored as q + 128)
      const uint4 Q = (i >> 1) ? R.q2 : R.q;  // chunk pair (i / 2), chunk i % 2 of it
      const uint32_t wa = (i & 1) ? Q.z : Q.x, wb = (i & 1) ? Q.w : Q.y;
      const __half2 sub = __float2half2_rn(1152.f);
      av[0] = prmt(wa, 0x64646464u, 0x4140u);
      av[1] = prmt(wa, 0x64646464u, 0x4342u);
      av[2] = prmt(wb, 0x64646464u, 0x4140u);
      av[3] = prmt(wb, 0x64646464u, 0x4342u);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const __half2 v = __hsub2(u2h2(av[r]), sub);
        av[r] = *reinterpret_cast<const uint32_t *>(&v);
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {  // r: (g, 2c) (g+8, 2c) (g, 2c+8) (g+8, 2c+8)
      const float2 q = __half22float2(u2h2(av[r]));
      const float m = (r & 1) ? m1 : m0, o = (r & 1) ? off1 : off0;
      const float x0 = fmaf(m, q.x, -o), x1 = fmaf(m, q.y, -o);
      tc_store_pair(x0, x1, ahi, alo, sw64(r0 + 8 * (r & 1), 16 * ii + 2 * c + 8 * (r >> 1)));
    }
  }
}

template <int TYPE>
__device__ __forceinline__ void tc_dequant_loop(const TcArgs &a, const TcSeg &S, int ctile, int wt,
                                                int lane, uint8_t *stages, int stage_bytes,
                                                uint64_t *a_full, uint64_t *empty) {
  TcRaw R{}, Rn{};
  const int nfb = a.nkb / 2;  // fetch blocks (two stages each)
  tc_fetch<TYPE>(S, ctile, wt, 0, lane, R);
  for (int fb = 0; fb < nfb; ++fb) {
    if (fb + 1 < nfb) tc_fetch<TYPE>(S, ctile, wt, fb + 1, lane, Rn);  // one block ahead
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int kb = 2 * fb + half;
      const int s = kb % kTcStages;
      const uint32_t ph = (uint32_t)(kb / kTcStages) & 1u;
      if (kb >= kTcStages && !mbar_wait(&empty[s], ph ^ 1u, a.err, 302)) return;
      uint8_t *ahi = stages + (size_t)s * stage_bytes;
      tc_emit<TYPE>(S, R, wt, fb, half, lane, ahi, ahi + kATile);
      fence_async_smem();
      mbar_arrive(&a_full[s]);
    }
    R = Rn;
  }
}

__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t a_full[kTcStages], b_full[kTcStages], empty[kTcStages], done;
  __shared__ uint32_t tmem_slot;
  // 1024-byte alignment for the swizzled tiles
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t *stages = smem_raw + pad;
  const int btile = a.ntile * kTcKB * 2;            // bytes of one B plane per stage
  const int stage_bytes = 2 * kATile + 2 * btile;   // A hi, A lo, B hi, B lo
  int si = 0;  // this CTA's matrix
#pragma unroll
  for (int i = 1; i < kTcMaxSegs; ++i)
    if (i < a.nseg && (int)blockIdx.x >= a.seg[i].ctile0) si = i;
  const TcSeg &S = a.seg[si];
  const int ctile = (int)blockIdx.x - S.ctile0, tt = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&a_full[s], 32 * (kTcThreads / 32 - kTcDeq0));
      mbar_init(&b_full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  if (warp == 2) {  // tensor-memory allocation (whole warp)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_slot)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // activation tiles; the row tile's weight units are pulled into L2
      // two units ahead of the dequantising warps, so their loads hit L2
      const int kpu = S.kc / kTcKB;  // k-blocks per unit
      const uint8_t *wrow = S.w + (size_t)ctile * S.kunits * S.unit_bytes;
      for (int u = 0; u < 2 && u < S.kunits; ++u)
        prefetch_l2(wrow + (size_t)u * S.unit_bytes, (uint32_t)S.unit_bytes);
      int issued = 0;
      for (int kb = 0; kb < a.nkb; ++kb) {
        const int s = kb % kTcStages;
        const uint32_t ph = (uint32_t)(kb / kTcStages) & 1u;
        if (kb % kpu == 0 && kb / kpu + 2 < S.kunits)
          prefetch_l2(wrow + (size_t)(kb / kpu + 2) * S.unit_bytes, (uint32_t)S.unit_bytes);
        if (kb >= kTcStages && !mbar_wait(&empty[s], ph ^ 1u, a.err, 301)) break;
        uint8_t *bdst = stages + (size_t)s * stage_bytes + 2 * kATile;
        const uint8_t *src = a.xt + (size_t)(((int64_t)tt * a.nkb + kb) * 2) * btile;
        mbar_arrive_expect_tx(&b_full[s], (uint32_t)(2 * btile));
        bulk_g2s(bdst, src, (uint32_t)(2 * btile), &b_full[s]);
        issued = kb + 1;
      }
      // no copy may outlive the CTA: wait (bounded) for the last ones to land
      for (int kb = std::max(0, issued - kTcStages); kb < issued; ++kb)
        mbar_wait(&b_full[kb % kTcStages], (uint32_t)(kb / kTcStages) & 1u, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issue
      const uint32_t idesc = idesc_f16(a.ntile);
      for (int kb = 0; kb < a.nkb; ++kb) {
        const int s = kb % kTcStages;
        const uint32_t ph = (uint32_t)(kb / kTcStages) & 1u;
        if (!mbar_wait(&a_full[s], ph, a.err, 303)) break;
        if (!mbar_wait(&b_full[s], ph, a.err, 304)) break;
        tc_fence_after();
        const uint32_t base = smem_u32(stages + (size_t)s * stage_bytes);
        const uint32_t ah = base, al = base + kATile, bh = base + 2 * kATile, bl = bh + btile;
#pragma unroll
        for (int j = 0; j < kTcKB / 16; ++j) {  // 32 bytes of K per MMA
          const uint32_t o = 32u * j;
          umma_f16(tmem, umma_desc(ah + o), umma_desc(bh + o), idesc, (kb | j) != 0);
          umma_f16(tmem, umma_desc(ah + o), umma_desc(bl + o), idesc, 1u);
          umma_f16(tmem, umma_desc(al + o), umma_desc(bh + o), idesc, 1u);
        }
        umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
      }
      umma_commit(&done);  // every MMA issued above has completed
    }
  } else if (warp >= kTcDeq0) {
    const int wt = warp - kTcDeq0;
    switch (S.type) {
      case IFX_TYPE_Q4_K:
        tc_dequant_loop<IFX_TYPE_Q4_K>(a, S, ctile, wt, lane, stages, stage_bytes, a_full, empty);
        break;
      case IFX_TYPE_Q6_K:
        tc_dequant_loop<IFX_TYPE_Q6_K>(a, S, ctile, wt, lane, stages, stage_bytes, a_full, empty);
        break;
      case IFX_TYPE_Q4_0:
        tc_dequant_loop<IFX_TYPE_Q4_0>(a, S, ctile, wt, lane, stages, stage_bytes, a_full, empty);
        break;
      default:
        tc_dequant_loop<IFX_TYPE_Q8_0>(a, S, ctile, wt, lane, stages, stage_bytes, a_full, empty);
        break;
    }
    if (warp < kTcDeq0 + 4) {  // epilogue: warp w reads tensor-memory lanes 32 (w % 4) ..
      const bool ok = mbar_wait(&done, 0u, a.err, 305);
      tc_fence_after();
      const int q = warp & 3;
      const int row = ctile * kTcRows + 32 * q + lane;
      for (int c0 = 0; c0 < a.ntile; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
        if (ok && row < S.rows) {
          const int64_t tok0 = (int64_t)tt * a.ntile + c0;
          const int64_t ldc = S.ldc;
          float *p = S.C + tok0 * ldc + row;
          if (a.accumulate) {  // all 16 reads in flight before the first write
            float old[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) old[j] = tok0 + j < a.M ? p[(int64_t)j * ldc] : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (tok0 + j < a.M) p[(int64_t)j * ldc] = old[j] + v[j] * (1.0f / kTcAScale);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (tok0 + j < a.M) p[(int64_t)j * ldc] = v[j] * (1.0f / kTcAScale);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(a.tmem_cols)
                 : "memory");
  }
}

}  // namespace

int tc_gemm_ntile(int64_t M) {
  const int64_t n = (M + 31) / 32 * 32;
  return (int)std::min<int64_t>(256, std::max<int64_t>(32, n));
}

bool tc_gemm_eligible(int64_t K) { return K % kTcFetch == 0; }

size_t tc_xtile_bytes(int64_t M, int64_t K) {
  const int nt = tc_gemm_ntile(M);
  const int64_t tiles = (M + nt - 1) / nt;
  return (size_t)tiles * (size_t)(K / kTcKB) * 2 * (size_t)nt * kTcKB * 2;
}

ifx_status tc_stage_x(const float *X, const float *X2, const float *normw, float eps, int mode,
                      int64_t M, int64_t K, void *xt, cudaStream_t st) {
  const int nt = tc_gemm_ntile(M);
  const int64_t mpad = (M + nt - 1) / nt * nt;
  tc_stage_x_kernel<<<(unsigned)mpad, 256, 0, st>>>(X, X2, normw, eps, mode, M, K, nt,
                                                    reinterpret_cast<uint8_t *>(xt));
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status tc_gemm_run_multi(const QMatrix *const *W, float *const *C, const int64_t *ldc, int n,
                             const void *xt, int64_t M, int accumulate, int *err,
                             cudaStream_t st) {
  if (n < 1 || n > kTcMaxSegs) return fail(IFX_ERR_INVALID_ARGUMENT, "tc gemm: 1 to 3 matrices");
  TcArgs a{};
  int ct = 0;
  for (int i = 0; i < n; ++i) {
    const QLayout &L = W[i]->L;
    if (L.kc % kTcFetch || L.cols % kTcFetch || L.cols != W[0]->L.cols)
      return fail(IFX_ERR_UNSUPPORTED, "tc gemm: K blocks must be multiples of 64 columns");
    TcSeg &S = a.seg[i];
    S.w = W[i]->d;
    S.C = C[i];
    S.ldc = ldc[i];
    S.type = L.type;
    S.rows = (int)L.rows;
    S.kc = L.kc;
    S.kunits = L.kunits;
    S.unit_bytes = L.unit_bytes;
    S.wt_bytes = L.wt_bytes;
    S.wt_qbytes = L.wt_qbytes;
    S.smask = L.q6_s8 ? 0x80u : 0u;
    S.ctile0 = ct;
    S.ctiles = L.ctiles;
    ct += L.ctiles;
  }
  a.nseg = n;
  a.xt = reinterpret_cast<const uint8_t *>(xt);
  a.M = (int)M;
  a.nkb = (int)(W[0]->L.cols / kTcKB);
  a.ntile = tc_gemm_ntile(M);
  a.tmem_cols = a.ntile <= 32 ? 32 : a.ntile <= 64 ? 64 : a.ntile <= 128 ? 128 : 256;
  a.accumulate = accumulate;
  a.err = err;
  const size_t smem = 1024 + (size_t)kTcStages * (2 * kATile + 2 * (size_t)a.ntile * kTcKB * 2);
  if (smem > 226 * 1024) return fail(IFX_ERR_UNSUPPORTED, "tc gemm: shared memory plan too large");
  static size_t attr = 0;  // the kernel's opt-in dynamic shared memory so far
  if (smem > attr) {
    IFX_CUDA(cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    attr = smem;
  }
  dim3 grid((unsigned)ct, (unsigned)((M + a.ntile - 1) / a.ntile));
  tc_gemm_kernel<<<grid, kTcThreads, smem, st>>>(a);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

ifx_status tc_gemm_run(const QMatrix &W, const void *xt, int64_t M, float *C, int64_t ldc,
                       int accumulate, int *err, cudaStream_t st) {
  const QMatrix *w[1] = {&W};
  float *c[1] = {C};
  const int64_t l[1] = {ldc};
  return tc_gemm_run_multi(w, c, l, 1, xt, M, accumulate, err, st);
}

}  // namespace ifx
