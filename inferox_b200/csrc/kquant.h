// llama.cpp (ggml) type ids and K-quant byte orders mapped onto the
// reference's (kquant.cu).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "../../include/inferox.h"

namespace ifx {

// The reference's TensorType id (src/gguf/types.rs:70-100) for a ggml type
// id, or -1 for types with no counterpart on this path.
int ggml_type_to_reference(uint32_t ggml_type);

// Blocks of `type` (a reference id) written in llama.cpp's order, permuted
// into the reference's order (dst may be src: converted in place).
// *type_out is `type`, except kTypeQ6KS8 for Q6_K (int8 scales).
ifx_status ggml_to_reference(int type, const uint8_t *src, size_t nbytes, uint8_t *dst,
                             int *type_out);

}  // namespace ifx
