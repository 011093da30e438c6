// Exact per-element dequantisation under the reference's byte semantics
// (src/gguf/dequant.rs). Every multiply/subtract is an explicitly rounded
// __fmul_rn/__fsub_rn so nvcc cannot contract them into an FMA: the Rust
// code rounds each operation separately, and these must match bit for bit.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace ifx {

struct BlockInfo {
  int elems, bytes;
};

// Internal type id (never in a file): Q6_K blocks in the reference's byte
// order whose sixteen scale bytes are int8, as llama.cpp writes and reads
// them (the reference reads them as u8, dequant.rs:195). Loads with
// kquant_layout = IFX_KQUANT_GGML permute llama.cpp's Q6_K blocks into the
// reference's order and tag them with this id.
constexpr int kTypeQ6KS8 = 0x100 | IFX_TYPE_Q6_K;

__host__ __device__ inline BlockInfo block_info(int type) {
  switch (type) {
    case IFX_TYPE_F32: return {1, 4};
    case IFX_TYPE_F16: return {1, 2};
    case IFX_TYPE_Q4_0: return {32, 18};
    case IFX_TYPE_Q8_0: return {32, 34};
    case IFX_TYPE_Q4_K: return {256, 144};
    case IFX_TYPE_Q6_K: return {256, 210};
    case kTypeQ6KS8: return {256, 210};
    case IFX_TYPE_Q8_K: return {256, 292};
    default: return {0, 0};
  }
}

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) {
  return (uint16_t)(p[0] | (p[1] << 8));
}

// Element e of a tensor of `type` stored as GGUF blocks at `src`.
__device__ __forceinline__ float dequant_elem(int type, const uint8_t *src, uint64_t e) {
  switch (type) {
    case IFX_TYPE_F32: {
      uint32_t b = (uint32_t)src[4 * e] | ((uint32_t)src[4 * e + 1] << 8) |
                   ((uint32_t)src[4 * e + 2] << 16) | ((uint32_t)src[4 * e + 3] << 24);
      return __uint_as_float(b);
    }
    case IFX_TYPE_F16:
      return h2f_exact(ld_u16(src + 2 * e));
    case IFX_TYPE_Q4_0: {  // dequant.rs:62-84
      const uint8_t *c = src + (e / 32) * 18;
      int j = (int)(e % 32);
      float delta = h2f_exact(ld_u16(c));
      uint8_t byte = c[2 + (j & 15)];
      int q = (j < 16) ? (byte & 15) : (byte >> 4);
      return __fmul_rn((float)(q - 8), delta);
    }
    case IFX_TYPE_Q8_0: {  // dequant.rs:93-111
      const uint8_t *c = src + (e / 32) * 34;
      float delta = h2f_exact(ld_u16(c));
      return __fmul_rn((float)(int8_t)c[2 + e % 32], delta);
    }
    case IFX_TYPE_Q4_K: {  // dequant.rs:123-163
      const uint8_t *c = src + (e / 256) * 144;
      int j = (int)(e % 256), g = j / 32, l = j % 32;
      float d = h2f_exact(ld_u16(c)), dmin = h2f_exact(ld_u16(c + 2));
      const uint8_t *s = c + 4;
      uint32_t sc, mn;
      if (g < 4) {
        sc = s[g] & 63;
        mn = s[g + 4] & 63;
      } else {
        sc = (s[g + 4] & 15) | ((s[g - 4] >> 6) << 4);
        mn = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
      }
      float dall = __fmul_rn(d, (float)sc);
      float dmv = __fmul_rn(dmin, (float)mn);
      uint8_t byte = c[16 + g * 16 + l / 2];
      uint32_t q = (l % 2 == 0) ? (byte & 15) : (byte >> 4);
      return __fsub_rn(__fmul_rn(dall, (float)q), dmv);
    }
    case IFX_TYPE_Q6_K: {  // dequant.rs:174-199 (scale byte read as u8)
      const uint8_t *c = src + (e / 256) * 210;
      int j = (int)(e % 256);
      float d = h2f_exact(ld_u16(c));
      uint8_t qlb = c[18 + j / 2];
      uint32_t nib = (j % 2 == 0) ? (qlb & 15) : (qlb >> 4);
      uint32_t hb = (c[146 + j / 4] >> (2 * (j % 4))) & 3;
      int q = (int)(nib | (hb << 4));
      return __fmul_rn(__fmul_rn(d, (float)c[2 + j / 16]), (float)(q - 32));
    }
    case kTypeQ6KS8: {  // the same with int8 scales: y = (d * sc) * (q - 32)
      const uint8_t *c = src + (e / 256) * 210;
      int j = (int)(e % 256);
      float d = h2f_exact(ld_u16(c));
      uint8_t qlb = c[18 + j / 2];
      uint32_t nib = (j % 2 == 0) ? (qlb & 15) : (qlb >> 4);
      uint32_t hb = (c[146 + j / 4] >> (2 * (j % 4))) & 3;
      int q = (int)(nib | (hb << 4));
      return __fmul_rn(__fmul_rn(d, (float)(int8_t)c[2 + j / 16]), (float)(q - 32));
    }
    case IFX_TYPE_Q8_K: {  // dequant.rs:210-232
      const uint8_t *c = src + (e / 256) * 292;
      int j = (int)(e % 256);
      float d = h2f_exact(ld_u16(c)), dmin = h2f_exact(ld_u16(c + 2));
      float v = __fmul_rn(__fmul_rn(d, (float)c[4 + j / 8]), (float)(int8_t)c[36 + j]);
      return __fsub_rn(v, dmin);
    }
    default:
      return 0.0f;
  }
}

}  // namespace ifx
