// Host-side view of a repacked quantised matrix on the device.
#pragma once
#include <cuda_runtime.h>

#include "qlayout.cuh"

namespace ifx {

struct QMatrix {
  QLayout L;
  uint8_t *d = nullptr;  // repacked bytes (device)
  int device = 0;
  // Quantised bytes of the original GGUF blocks for this matrix (what a
  // decode step must stream from HBM).
  uint64_t gguf_bytes() const {
    if (L.dense) return L.total_bytes;  // streamed as f32
    BlockInfo b = block_info(L.type);
    return (uint64_t)(L.rows * L.cols / b.elems) * b.bytes;
  }
};

ifx_status repack_to_device(const QLayout &L, const uint8_t *src_dev, uint8_t *dst_dev,
                            cudaStream_t stream);

}  // namespace ifx
