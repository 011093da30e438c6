// Shared helpers for the sm_100a kernels: status plumbing, PTX wrappers for
// mbarriers, bulk async copies (TMA, 1-D, one destination CTA), programmatic
// dependent launch, and the m16n8k16 f16 tensor-core MMA.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "status.h"

namespace ifx {

ifx_status cuda_fail(cudaError_t e, const char *what);

#define IFX_CUDA(call)                                           \
  do {                                                           \
    cudaError_t _e = (call);                                     \
    if (_e != cudaSuccess) return ::ifx::cuda_fail(_e, #call);   \
  } while (0)

constexpr int kNumSMs = 148;

// Position of element i (0 <= i < hd) of K/V cache row t (t: the row's
// position in the cache) inside that row. For head sizes that are a multiple
// of 64 the 16-byte chunks of a row are XOR-permuted by t % 8, so eight
// consecutive rows read at one logical chunk fall on eight different
// shared-memory bank groups (the tensor-core decode attention reads them with
// ldmatrix); other head sizes keep the plain order. Even i and i + 1 stay
// adjacent, so half2 accesses are unaffected.
__host__ __device__ __forceinline__ int kv_col(int t, int i, int hd) {
  return (hd & 63) ? i : (i ^ ((t & 7) << 3));
}

// ---------------------------------------------------------------- PTX ----
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: every spin in this library gives up after kSpinLimit polls,
// raises a device error flag and lets the kernel return, so a lost arrival
// can never hang the GPU. try_wait itself suspends for a while per poll.
constexpr uint32_t kSpinLimit = 1u << 24;

// A wait also gives up early once another thread has raised the flag, so
// one lost arrival ends every waiter in the grid quickly.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err_flag,
                                          int code) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (err_flag && (i & 1023u) == 1023u && *(volatile int *)err_flag) return false;
  }
  if (err_flag) atomicExch(err_flag, code);
  return false;
}

// Wait for the bulk copies of ring positions [max(0, end - NS), end) to land
// (positions before that had their slot refilled, so they completed). Used
// before a producer leaves, so no copy into shared memory outlives the CTA.
__device__ __forceinline__ void ring_drain(uint64_t *full_bar, int NS, uint32_t end) {
  const uint32_t b = end > (uint32_t)NS ? end - (uint32_t)NS : 0u;
  for (uint32_t rp = b; rp < end; ++rp) {
    uint64_t *bar = &full_bar[rp % (uint32_t)NS];
    const uint32_t ph = (rp / (uint32_t)NS) & 1u;
    for (uint32_t i = 0; i < kSpinLimit && !mbar_try_wait(bar, ph); ++i) {
    }
  }
}

// Orders this thread's view of earlier shared-memory accesses (generic
// proxy) before bulk copies it issues next (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk async copy global -> shared, completion counted on an mbarrier.
// dst, src and bytes must be 16-byte aligned / multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch (PDL). wait: block until the preceding grid
// in the stream has completed and its writes are visible. launch: allow the
// next grid to start its pre-wait prologue (weight prefetch).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C (f32).
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1,
                                          const float (&c)[4]) {
  // not volatile: the MMA has no side effects, so the scheduler may move
  // independent work (scale unpack, loads) across it
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

// Four 8x8 b16 matrices from shared memory (lanes 8q..8q+7 give the row
// addresses of matrix q), in the mma.m16n8k16 fragment layout; `_t`
// transposes each matrix.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ void red_add_f32(float *addr, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// f16 bits -> f32 (exact, subnormals kept). NaN payloads are not preserved;
// use h2f_exact where bit-exactness with the `half` crate matters.
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// The `half` crate's to_f32 bit for bit: NaNs keep their payload and get the
// quiet bit set (0x7FC0_0000), which __half2float does not do.
__device__ __forceinline__ float h2f_exact(uint16_t h) {
  if ((h & 0x7c00u) == 0x7c00u && (h & 0x3ffu))
    return __uint_as_float(((uint32_t)(h & 0x8000u) << 16) | 0x7fc00000u | ((uint32_t)(h & 0x3ffu) << 13));
  return __half2float(__ushort_as_half(h));
}

// Launch helper: optionally attach the programmatic-stream-serialization
// attribute so the kernel may begin while its predecessor drains.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, bool pdl, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace ifx
