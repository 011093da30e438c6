// One-time repack of GGUF quantised blocks (reference byte semantics,
// src/gguf/dequant.rs:62-199) into the fragment-ordered layout of
// qlayout.cuh. Runs once per weight at load; never on the token path.
#include "qlayout.cuh"
#include "repack.h"

namespace ifx {

namespace {

struct Src {
  const uint8_t *p;
  int64_t cols;
  int type;
};

// 4-bit value (Q4_K / Q4_0) or low nibble of the 6-bit value (Q6_K) at (row, k).
__device__ __forceinline__ uint32_t nib_at(const Src &s, int64_t row, int64_t k) {
  if (s.type == IFX_TYPE_Q4_K) {
    const uint8_t *b = s.p + (row * (s.cols / 256) + k / 256) * 144;
    int j = (int)(k % 256), g = j / 32, l = j % 32;
    uint8_t byte = b[16 + g * 16 + l / 2];
    return (l % 2 == 0) ? (byte & 15u) : (byte >> 4);
  } else if (s.type == IFX_TYPE_Q4_0) {
    const uint8_t *b = s.p + (row * (s.cols / 32) + k / 32) * 18;
    int j = (int)(k % 32);
    uint8_t byte = b[2 + (j & 15)];
    return (j < 16) ? (byte & 15u) : (byte >> 4);
  } else {  // Q6_K low nibble
    const uint8_t *b = s.p + (row * (s.cols / 256) + k / 256) * 210;
    int j = (int)(k % 256);
    uint8_t byte = b[18 + j / 2];
    return (j % 2 == 0) ? (byte & 15u) : (byte >> 4);
  }
}

__device__ __forceinline__ uint32_t q6_hi_at(const Src &s, int64_t row, int64_t k) {
  const uint8_t *b = s.p + (row * (s.cols / 256) + k / 256) * 210;
  int j = (int)(k % 256);
  return (b[146 + j / 4] >> (2 * (j % 4))) & 3u;
}

__device__ __forceinline__ uint32_t q8_u_at(const Src &s, int64_t row, int64_t k) {
  const uint8_t *b = s.p + (row * (s.cols / 32) + k / 32) * 34;
  return (uint32_t)((int)(int8_t)b[2 + k % 32] + 128);
}

// One CTA per (unit, warp tile); threads stride over the tile's words.
__global__ void repack_kernel(QLayout L, const uint8_t *__restrict__ src,
                              uint8_t *__restrict__ dst) {
  const int64_t unit = blockIdx.x;
  const int w = blockIdx.y;
  const int ctile = (int)(unit / L.kunits), kunit = (int)(unit % L.kunits);
  uint8_t *out = dst + unit * L.unit_bytes + (int64_t)w * L.wt_bytes;
  const int64_t row0 = (int64_t)ctile * kCtaRows + w * 16;
  const int64_t k0 = (int64_t)kunit * L.kc;
  Src s{src, L.cols, L.type};
  const int nchunks = L.kc / 16;

  auto valid = [&](int r) { return row0 + r < L.rows; };

  if (L.type == IFX_TYPE_Q4_K || L.type == IFX_TYPE_Q4_0 || L.type == IFX_TYPE_Q6_K) {
    // nibble plane: word (lane, chunk) at ((chunk/4)*32 + lane)*16 + (chunk%4)*4
    for (int idx = threadIdx.x; idx < 32 * nchunks; idx += blockDim.x) {
      int lane = idx % 32, ch = idx / 32;
      int g = lane / 4, c = lane % 4;
      uint32_t word = 0;
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        int r = (p & 1) ? g + 8 : g;
        int col = 2 * c + ((p & 2) ? 8 : 0) + ((p & 4) ? 1 : 0);
        uint32_t q = valid(r) ? nib_at(s, row0 + r, k0 + 16 * ch + col) : 0u;
        word |= q << (4 * p);
      }
      *reinterpret_cast<uint32_t *>(out + ((ch / 4) * 32 + lane) * 16 + (ch % 4) * 4) = word;
    }
    if (L.type == IFX_TYPE_Q6_K) {
      // 2-bit plane: word per (lane, chunk pair t) at 2048 + ((t/4)*32+lane)*16 + (t%4)*4;
      // chunk parity cp, register r, element e at bit 8*cp + 16*e + 2*r.
      for (int idx = threadIdx.x; idx < 32 * (nchunks / 2); idx += blockDim.x) {
        int lane = idx % 32, t = idx / 32;
        int g = lane / 4, c = lane % 4;
        uint32_t word = 0;
        for (int cp = 0; cp < 2; ++cp)
          for (int r = 0; r < 4; ++r)
            for (int e = 0; e < 2; ++e) {
              int row = (r & 1) ? g + 8 : g;
              int col = 2 * c + ((r & 2) ? 8 : 0) + e;
              int ch = 2 * t + cp;
              uint32_t h = valid(row) ? q6_hi_at(s, row0 + row, k0 + 16 * ch + col) : 0u;
              word |= h << (8 * cp + 16 * e + 2 * r);
            }
        *reinterpret_cast<uint32_t *>(out + 2048 + ((t / 4) * 32 + lane) * 16 + (t % 4) * 4) =
            word;
      }
    }
  } else if (L.type == IFX_TYPE_Q8_0) {
    // W0 = [u(g,2c), u(g,2c+1), u(g+8,2c), u(g+8,2c+1)], W1 = same at +8;
    // at ((chunk/2)*32 + lane)*16 + (chunk%2)*8 + wsel*4.
    for (int idx = threadIdx.x; idx < 32 * nchunks * 2; idx += blockDim.x) {
      int lane = idx % 32, rest = idx / 32, wsel = rest % 2, ch = rest / 2;
      int g = lane / 4, c = lane % 4;
      uint32_t word = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        int r = (b & 2) ? g + 8 : g;
        int col = 2 * c + (b & 1) + (wsel ? 8 : 0);
        uint32_t u = valid(r) ? q8_u_at(s, row0 + r, k0 + 16 * ch + col) : 0u;
        word |= u << (8 * b);
      }
      *reinterpret_cast<uint32_t *>(out + ((ch / 2) * 32 + lane) * 16 + (ch % 2) * 8 + wsel * 4) =
          word;
    }
  }

  // scales
  uint8_t *sc = out + L.wt_qbytes;
  if (L.type == IFX_TYPE_Q4_K) {
    // 16 bytes per row = four 32-bit words; word c holds the 24-bit field
    // sc[2c] | sc[2c+1] << 6 | mn[2c] << 12 | mn[2c+1] << 18 (the two groups
    // lane c of the GEMV epilogue needs, unpacked from the 6-bit encoding of
    // dequant.rs:141-149) and, in its top byte, byte c of (d, dmin) as f16.
    for (int r = threadIdx.x; r < 16; r += blockDim.x) {
      uint8_t *o = sc + 16 * r;
      if (!valid(r)) {
        for (int b = 0; b < 16; ++b) o[b] = 0;
        continue;
      }
      const uint8_t *blk = src + ((row0 + r) * (L.cols / 256) + kunit) * 144;
      const uint8_t *s = blk + 4;
      uint32_t scv[8], mnv[8];
      for (int g = 0; g < 8; ++g) {
        if (g < 4) {
          scv[g] = s[g] & 63;
          mnv[g] = s[g + 4] & 63;
        } else {
          scv[g] = (s[g + 4] & 15) | ((s[g - 4] >> 6) << 4);
          mnv[g] = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
        }
      }
      for (int c = 0; c < 4; ++c) {
        const uint32_t f = scv[2 * c] | (scv[2 * c + 1] << 6) | (mnv[2 * c] << 12) | (mnv[2 * c + 1] << 18);
        o[4 * c + 0] = (uint8_t)(f & 0xff);
        o[4 * c + 1] = (uint8_t)((f >> 8) & 0xff);
        o[4 * c + 2] = (uint8_t)((f >> 16) & 0xff);
        o[4 * c + 3] = blk[c];  // d (bytes 0-1) and dmin (bytes 2-3)
      }
    }
  } else if (L.type == IFX_TYPE_Q6_K) {
    for (int idx = threadIdx.x; idx < 16 * 16; idx += blockDim.x) {
      int r = idx / 16, b = idx % 16;
      sc[idx] = valid(r) ? src[((row0 + r) * (L.cols / 256) + kunit) * 210 + 2 + b] : 0;
    }
    for (int idx = threadIdx.x; idx < 32; idx += blockDim.x) {
      int r = idx / 2, b = idx % 2;
      sc[256 + idx] = valid(r) ? src[((row0 + r) * (L.cols / 256) + kunit) * 210 + b] : 0;
    }
  } else {  // Q4_0 / Q8_0: f16 d per 32-block
    const int bb = (L.type == IFX_TYPE_Q4_0) ? 18 : 34;
    const int nb = L.kc / 32;
    for (int idx = threadIdx.x; idx < 16 * nb * 2; idx += blockDim.x) {
      int r = idx / (nb * 2), rem = idx % (nb * 2), blk = rem / 2, b = rem % 2;
      sc[idx] = valid(r) ? src[((row0 + r) * (L.cols / 32) + (int64_t)kunit * nb + blk) * bb + b]
                         : 0;
    }
  }
}

}  // namespace

ifx_status repack_to_device(const QLayout &L, const uint8_t *src_dev, uint8_t *dst_dev,
                            cudaStream_t stream) {
  dim3 grid((unsigned)((int64_t)L.ctiles * L.kunits), kWarpTiles);
  repack_kernel<<<grid, 128, 0, stream>>>(L, src_dev, dst_dev);
  IFX_CUDA(cudaGetLastError());
  return IFX_OK;
}

}  // namespace ifx
