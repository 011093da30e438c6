// llama.cpp (ggml) GGUF files on the reference's kernels: type ids and
// K-quant byte orders.
//
// The reference numbers tensor types its own way from Q5_0 on
// (src/gguf/types.rs:70-100: Q5_0 = 5, Q5_1 = 6, Q8_0 = 7, Q8_1 = 8) and
// decodes Q4_K and Q6_K blocks in its own element order
// (src/gguf/dequant.rs:123-199). Files written by llama.cpp use ggml's ids
// (Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9) and ggml's block layouts:
//
//   Q4_K (144 bytes, d, dmin, 12 scale bytes as in the reference): the 128
//     quant bytes hold four 64-element chunks; element 64c + e is the low
//     nibble of byte 32c + e for e < 32 and the high nibble of byte
//     32c + e - 32 otherwise (the reference: byte 16g + l/2 of 32-element
//     group g, even l in the low nibble). Group j / 32 selects the scale and
//     min in both.
//   Q6_K (210 bytes): ql[128], qh[64], int8 scales[16], then f16 d (the
//     reference: d, scales, ql, qh). Element j = 128n + 32t + l takes the
//     low (t < 2) or high (t >= 2) nibble of ql[64n + 32(t & 1) + l] and
//     bits 2t, 2t+1 of qh[32n + l]; scale j / 16 in both layouts, but
//     llama.cpp reads the scale byte as int8 where the reference reads u8.
//
// ggml_to_reference() permutes blocks into the reference's byte order so
// the repack and every kernel run unchanged; Q6_K blocks come back tagged
// with the internal id kTypeQ6KS8 so the kernels read their scales as int8.
// Q4_0 and Q8_0 blocks are byte-identical in the two formats.
#include <cstring>
#include <string>

#include "kquant.h"
#include "quant.cuh"
#include "status.h"

namespace ifx {

int ggml_type_to_reference(uint32_t ggml_type) {
  switch (ggml_type) {
    case 0: return IFX_TYPE_F32;
    case 1: return IFX_TYPE_F16;
    case 2: return IFX_TYPE_Q4_0;
    case 3: return 3;  // Q4_1
    case 6: return 5;  // Q5_0
    case 7: return 6;  // Q5_1
    case 8: return IFX_TYPE_Q8_0;
    case 9: return 8;  // Q8_1
    case 10: case 11: case 12: case 13: case 14: case 15: return (int)ggml_type;  // Q2_K..Q8_K
    default: return -1;  // IQ*, integer, BF16 ...: nothing on this path reads them
  }
}

namespace {

void q4k_block(const uint8_t *s, uint8_t *d) {
  memcpy(d, s, 16);  // d, dmin, scales: same place, same meaning
  uint8_t *qs = d + 16;
  memset(qs, 0, 128);
  for (int j = 0; j < 256; ++j) {
    const int c = j / 64, e = j % 64;
    const uint8_t b = s[16 + 32 * c + (e & 31)];
    const uint32_t q = e < 32 ? (b & 15u) : (b >> 4);
    const int g = j / 32, l = j % 32;
    qs[16 * g + l / 2] |= (uint8_t)(l % 2 == 0 ? q : q << 4);
  }
}

void q6k_block(const uint8_t *s, uint8_t *d) {
  const uint8_t *ql = s, *qh = s + 128, *sc = s + 192;
  memcpy(d, s + 208, 2);  // f16 d
  memcpy(d + 2, sc, 16);  // scales (int8 bytes, kept as they are)
  uint8_t *rql = d + 18, *rqh = d + 146;
  memset(rql, 0, 128 + 64);
  for (int j = 0; j < 256; ++j) {
    const int n = j / 128, t = (j % 128) / 32, l = j % 32;
    const uint8_t b = ql[64 * n + 32 * (t & 1) + l];
    const uint32_t lo = t < 2 ? (b & 15u) : (b >> 4);
    const uint32_t hi = (qh[32 * n + l] >> (2 * t)) & 3u;
    rql[j / 2] |= (uint8_t)(j % 2 == 0 ? lo : lo << 4);
    rqh[j / 4] |= (uint8_t)(hi << (2 * (j % 4)));
  }
}

}  // namespace

ifx_status ggml_to_reference(int type, const uint8_t *src, size_t nbytes, uint8_t *dst,
                             int *type_out) {
  const BlockInfo b = block_info(type);
  if (type == IFX_TYPE_Q4_K || type == IFX_TYPE_Q6_K) {
    if (nbytes % (size_t)b.bytes)
      return fail(IFX_ERR_SHAPE, "llama.cpp K-quant data is not a whole number of blocks");
    uint8_t blk[256];  // one source block, so dst may overlap src
    for (size_t i = 0; i < nbytes; i += (size_t)b.bytes) {
      memcpy(blk, src + i, (size_t)b.bytes);
      if (type == IFX_TYPE_Q4_K) q4k_block(blk, dst + i);
      else q6k_block(blk, dst + i);
    }
    *type_out = type == IFX_TYPE_Q6_K ? kTypeQ6KS8 : type;
    return IFX_OK;
  }
  if (src != dst && nbytes) memmove(dst, src, nbytes);
  *type_out = type;
  return IFX_OK;
}

}  // namespace ifx

extern "C" ifx_status ifx_kquant_from_ggml(uint32_t ggml_type, const void *src, size_t nbytes,
                                           void *dst, int *type_out, int *signed_scales_out) {
  using namespace ifx;
  if (!type_out || !signed_scales_out || (nbytes && (!src || !dst)))
    return fail(IFX_ERR_INVALID_ARGUMENT, "ifx_kquant_from_ggml: null argument");
  const int t = ggml_type_to_reference(ggml_type);
  if (t < 0 || !block_info(t).elems)
    return fail(IFX_ERR_UNSUPPORTED, "ifx_kquant_from_ggml: ggml type " + std::to_string(ggml_type) +
                                         " is not one of F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, Q8_K");
  if (t == IFX_TYPE_Q8_K)
    return fail(IFX_ERR_UNSUPPORTED, "ifx_kquant_from_ggml: Q8_K layouts differ beyond a permutation");
  int out = 0;
  IFX_TRY(ggml_to_reference(t, static_cast<const uint8_t *>(src), nbytes, static_cast<uint8_t *>(dst),
                            &out));
  *type_out = out == kTypeQ6KS8 ? IFX_TYPE_Q6_K : out;
  *signed_scales_out = out == kTypeQ6KS8;
  return IFX_OK;
}
