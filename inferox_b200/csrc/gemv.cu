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
#include "dense.cuh"
#include "gemv_dev.cuh"

namespace ifx {

namespace {
using namespace gemvdev;

__global__ void __launch_bounds__(kGemvThreads, 1) gemv_b1_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty_bar = full_bar + kGemvMaxStages;
  uint32_t *tab = reinterpret_cast<uint32_t *>(smem + kGemvBarBytes);
  uint8_t *ring = smem + kGemvBarBytes + kGemvTabBytes;
  uint8_t *xw = ring + a.ring_bytes;  // staged activations (stage_x)

  const int2 rg = a.sched[blockIdx.x];
  const int u0 = rg.x, n = rg.y - rg.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    g_xzero = make_uint4(0u, 0u, 0u, 0u);
    for (int s = 0; s < kRingPos; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 8);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // producer: weights only, so it is safe before griddepcontrol.wait
    if (lane == 0) {
      RingState rs{0u, 0u, 0u};
      if (gemv_produce(a, u0, n, 0u, ring, (uint32_t)a.ring_bytes, RingTab{tab}, rs,
                       full_bar, empty_bar, a.err))
        ring_drain(full_bar, kRingPos, (uint32_t)max(n, 0));
    }
    return;
  }

  // consumers
  pdl_wait();
  pdl_launch();
  if (a.zero_ptr)
    for (int i = blockIdx.x * kConsumerThreads + threadIdx.x; i < a.zero_n;
         i += gridDim.x * kConsumerThreads)
      a.zero_ptr[i] = 0.f;
  if (n <= 0) return;
  const bool full = n >= a.kunits;
  stage_x(a, u0, n, full, xw);
  consumer_sync();
  gemv_consume(a, u0, n, 0u, ring, tab, full_bar, empty_bar, xw, full, a.err);
}

}  // namespace

ifx_status gemv_plan(const QMatrix *const *mats, float *const *ys, int nseg, int mode,
                     const float *x, const float *x2, const float *normw, float eps, int *err,
                     GemvPlan *plan) {
  if (nseg < 1 || nseg > kGemvMaxSegs) return fail(IFX_ERR_INVALID_ARGUMENT, "gemv: nseg");
  if (mats[0]->L.dense) {  // dense f32 matrices (dense.cu): no units, no schedule
    GemvArgs a{};
    a.nseg = nseg;
    a.K = (int)mats[0]->L.cols;
    uint64_t wbytes = 0;
    for (int i = 0; i < nseg; ++i) {
      if (!mats[i]->L.dense || mats[i]->L.cols != a.K)
        return fail(IFX_ERR_SHAPE, "gemv: dense segments must share K");
      a.seg[i].w = mats[i]->d;
      a.seg[i].y = ys[i];
      a.seg[i].rows = (int)mats[i]->L.rows;
      wbytes += mats[i]->L.total_bytes;
    }
    a.mode = mode;
    a.x = x;
    a.x2 = x2;
    a.normw = normw;
    a.eps = eps;
    a.err = err;
    *plan = GemvPlan{};
    plan->dense = 1;
    plan->weight_bytes = wbytes;
    IFX_TRY(dense_gemv_plan(a, &plan->grid, &plan->smem));
    plan->args = a;
    return IFX_OK;
  }
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
    S.type = L.type | (L.q6_s8 ? 0x80 << 8 : 0);
    S.rows = (int)L.rows;
    S.unit_bytes = L.unit_bytes;
    S.wt_bytes = L.wt_bytes;
    S.wt_qbytes = L.wt_qbytes;
    S.unit_begin = (int)total_units;
    S.units = (int)((int64_t)L.ctiles * L.kunits);
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

  // byte-balanced contiguous ranges, one per CTA
  // one schedule entry per SM (the persistent decode kernel indexes it by
  // CTA); CTAs beyond the unit count get empty ranges
  const int G = kNumSMs;
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
  // the weight ring takes what the staging window leaves of the shared
  // memory cap (at most kGemvRingBytes), and must hold two of the largest units
  constexpr size_t kSmemCap = 220 * 1024;
  const size_t win_bytes = (size_t)win * gemvdev::xs_slot_bytes(a.kc);  // activation planes, sums
  const size_t fixed = kGemvBarBytes + kGemvTabBytes + win_bytes;
  const size_t ring = fixed < kSmemCap ? std::min<size_t>(kGemvRingBytes, (kSmemCap - fixed) & ~(size_t)15) : 0;
  if (ring < 2 * (size_t)slot) return fail(IFX_ERR_SHAPE, "gemv: shared memory plan too large");
  a.ring_bytes = (int)ring;
  const size_t smem = fixed + ring;
  IFX_CUDA(cudaMalloc(&plan->d_sched, sizeof(int2) * G));
  IFX_CUDA(cudaMemcpy(plan->d_sched, sched.data(), sizeof(int2) * G, cudaMemcpyHostToDevice));
  a.sched = plan->d_sched;
  plan->args = a;
  plan->grid = G;
  plan->smem = smem;
  plan->weight_bytes = wbytes;
  static bool attr_set = false;
  if (!attr_set) {
    IFX_CUDA(cudaFuncSetAttribute(gemv_b1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kSmemCap));
    attr_set = true;
  }
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
  if (plan.dense) return dense_gemv_launch(plan.args, plan.grid, plan.smem, stream, pdl);
  IFX_CUDA(launch(gemv_b1_kernel, dim3(plan.grid), dim3(kGemvThreads), plan.smem, stream, pdl,
                  plan.args));
  return IFX_OK;
}

}  // namespace ifx
