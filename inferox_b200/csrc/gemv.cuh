// Batch-1 fused dequant GEMV: y[rows] (+)= W[rows, K] . f(x)[K]
// (replaces Weights::tensor_f32_by_index + ops::matmul_t at m = 1,
// src/model/forward.rs:366-368, 418, 431-434, 575).
#pragma once
#include <vector>

#include "repack.h"

namespace ifx {

// Input transform applied while staging x in shared memory.
enum GemvMode {
  GEMV_PLAIN = 0,    // x
  GEMV_RMSNORM = 1,  // rms_norm(x) * w   (ops.rs:155-168)
  GEMV_SWIGLU = 2,   // silu(x) * x2      (ops.rs:190-209)
};

constexpr int kGemvMaxSegs = 4;
constexpr int kGemvMaxStages = 16;
constexpr int kGemvThreads = 544;  // 16 consumer warps + 1 producer warp
constexpr int kGemvRingBytes = 176 * 1024;
constexpr int kGemvBarBytes = 2 * kGemvMaxStages * 8;  // full + empty mbarriers
constexpr int kGemvTabBytes = 2 * kGemvMaxStages * 4;  // ring offsets + lengths

struct GemvSeg {
  const uint8_t *w;  // repacked weights (device)
  float *y;          // output, accumulated with red.global.add
  int type;          // low byte: IFX_TYPE_*; bits 8-15: Q6_K scale mask (0x80:
                     // int8 scale bytes as llama.cpp writes them, 0: u8)
  int rows;          // valid output rows
  int unit_bytes, wt_bytes, wt_qbytes;
  int unit_begin;    // first global unit index of this segment
  int units;         // units in this segment (ctiles * kunits)
};

struct GemvArgs {
  GemvSeg seg[kGemvMaxSegs];
  int nseg;
  int kc, kunits, K;
  int mode;
  const float *x, *x2, *normw;
  float eps;
  const int2 *sched;  // per CTA [unit_begin, unit_end)
  int slot_bytes;  // largest unit of the plan
  int ring_bytes;  // weight ring (bytes; units packed back to back)
  int win_units;   // staged activation slots
  int *err;
  float *zero_ptr;    // zeroed by the consumers after griddepcontrol.wait
  int zero_n;         // (a buffer a later kernel accumulates into)
};

struct GemvPlan {
  GemvArgs args{};
  int grid = 0;
  size_t smem = 0;
  int2 *d_sched = nullptr;  // owned by the plan's creator
  uint64_t weight_bytes = 0;
  int dense = 0;  // dense f32 segments (dense.cu): no unit schedule
};

// Builds a byte-balanced schedule over `mats` (all with the same K and
// unit width). Output pointers ys[i] receive W_i . f(x).
ifx_status gemv_plan(const QMatrix *const *mats, float *const *ys, int nseg, int mode,
                     const float *x, const float *x2, const float *normw, float eps, int *err,
                     GemvPlan *plan);
void gemv_plan_free(GemvPlan *plan);
ifx_status gemv_launch(const GemvPlan &plan, cudaStream_t stream, bool pdl);
// Re-point an existing plan (same shapes) at other weights/outputs/inputs.
void gemv_plan_rebind(GemvPlan *plan, const QMatrix *const *mats, float *const *ys,
                      const float *x, const float *x2, const float *normw);

}  // namespace ifx
