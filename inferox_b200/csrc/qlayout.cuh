// Repacked HBM layout of a quantised weight matrix W[rows, cols] for the
// fused dequant kernels.
//
// The matrix is cut into "units": 128 output rows (a CTA tile of eight
// 16-row warp tiles) x `kc` input columns. Units are stored contiguously in
// CTA-tile-major order (unit = ctile * kunits + kunit) so one bulk async copy
// moves one unit into shared memory. Inside a unit, warp tile w occupies
// bytes [w * wt_bytes, (w + 1) * wt_bytes): first the quantised values
// pre-permuted into mma.m16n8k16 A-fragment order (one 16-byte vector per
// lane per step, so each lane's load is a single conflict-free 128-bit
// access), then that warp tile's scales.
//
// A-fragment order: lane (g = lane / 4, c = lane % 4) of a 16-row warp tile
// holds, for each 16-column chunk, the 8 values at rows {g, g+8} x chunk
// columns {2c, 2c+1, 2c+8, 2c+9}. Values are placed so that a single AND
// (4-bit types) or PRMT (8-bit) turns them into f16 subnormals q * 2^-24
// (rows g) or 16 q * 2^-24 (4-bit rows g+8) that the tensor core multiplies
// exactly; the power-of-two factors are folded into the group scales.
//
// The layout holds exactly the bytes of the GGUF blocks (no padding except
// rows beyond `rows` in the last CTA tile, which are zero).
#pragma once
#include <stdint.h>

#include "quant.cuh"

namespace ifx {

constexpr int kCtaRows = 128;   // rows per CTA tile (8 warp tiles of 16)
constexpr int kWarpTiles = 8;

struct QLayout {
  int type = 0;
  int64_t rows = 0, cols = 0;
  int ctiles = 0;    // ceil(rows / 128)
  int kc = 0;        // columns per unit
  int kunits = 0;    // cols / kc
  int wt_qbytes = 0; // quantised bytes per warp tile per unit
  int wt_sbytes = 0; // scale bytes per warp tile per unit
  int wt_bytes = 0;
  int unit_bytes = 0;
  uint64_t total_bytes = 0;
  int q6_s8 = 0;     // Q6_K scale bytes are int8 (llama.cpp), not u8
  int dense = 0;     // row-major f32 (dequantised F32 / F16 / Q8_K), not units
};

// Largest unit that still fits the GEMV's shared-memory stage.
constexpr int kMaxUnitBytes = 27 * 1024;

// Fills `L` for a [rows, cols] matrix of `type`; false if unsupported.
// kTypeQ6KS8 gives the Q6_K layout with q6_s8 set.
inline bool make_layout(int type, int64_t rows, int64_t cols, QLayout *L) {
  if (type == kTypeQ6KS8) {
    if (!make_layout(IFX_TYPE_Q6_K, rows, cols, L)) return false;
    L->q6_s8 = 1;
    return true;
  }
  QLayout q;
  q.type = type;
  q.rows = rows;
  q.cols = cols;
  q.ctiles = (int)((rows + kCtaRows - 1) / kCtaRows);
  switch (type) {
    case IFX_TYPE_Q4_K:
    case IFX_TYPE_Q6_K:
      if (cols % 256) return false;
      q.kc = 256;
      break;
    case IFX_TYPE_Q4_0:
      if (cols % 64) return false;
      q.kc = (cols % 256 == 0) ? 256 : (cols % 128 == 0 ? 128 : 64);
      break;
    case IFX_TYPE_Q8_0: {
      if (cols % 32) return false;
      q.kc = 0;
      // multiples of 64 first: the tensor-memory GEMM stages 64-column k-blocks
      for (int kc = 192; kc >= 64 && !q.kc; kc -= 64)
        if (cols % kc == 0 && kc * 17 * kWarpTiles <= kMaxUnitBytes) q.kc = kc;
      for (int kc = 192; kc >= 32 && !q.kc; kc -= 32)
        if (cols % kc == 0 && kc * 17 * kWarpTiles <= kMaxUnitBytes) q.kc = kc;
      if (!q.kc) return false;
      break;
    }
    default:
      return false;
  }
  q.kunits = (int)(cols / q.kc);
  switch (type) {
    case IFX_TYPE_Q4_K:
      q.wt_qbytes = 2048;  // 16 chunks x 4 B x 32 lanes
      q.wt_sbytes = 256;   // 16 rows x {d, dmin, scales[12]}
      break;
    case IFX_TYPE_Q6_K:
      q.wt_qbytes = 3072;  // nibble plane 2048 + 2-bit plane 1024
      q.wt_sbytes = 288;   // 16 rows x 16 u8 scales, then 16 x f16 d
      break;
    case IFX_TYPE_Q4_0:
      q.wt_qbytes = q.kc / 16 * 4 * 32;
      q.wt_sbytes = 16 * (q.kc / 32) * 2;
      break;
    case IFX_TYPE_Q8_0:
      q.wt_qbytes = q.kc / 16 * 8 * 32;
      q.wt_sbytes = 16 * (q.kc / 32) * 2;
      break;
  }
  q.wt_bytes = q.wt_qbytes + q.wt_sbytes;
  q.unit_bytes = q.wt_bytes * kWarpTiles;
  q.total_bytes = (uint64_t)q.ctiles * q.kunits * q.unit_bytes;
  *L = q;
  return true;
}

}  // namespace ifx
