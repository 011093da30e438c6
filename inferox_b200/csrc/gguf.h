// Host-side GGUF reader used at model load (restates src/gguf/file.rs,
// tensor.rs, value.rs and types.rs; errors map onto gguf::Error).
#pragma once
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/inferox.h"

namespace ifx {

struct GgufValue {
  uint32_t vt = 0;  // ValueType id (types.rs:8-22)
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  // arrays: element type, length and the first kArrayPreview items (what
  // Value's Display shows, value.rs:86-99); the rest are parsed and dropped
  uint32_t arr_type = 0;
  uint64_t arr_len = 0;
  std::vector<GgufValue> items;
  static constexpr uint64_t kArrayPreview = 9;
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> shape;
  uint32_t type = 0;
  uint64_t offset = 0;  // relative to the data region
  uint64_t n_elements() const {
    uint64_t n = 1;
    for (uint64_t d : shape) n *= d;
    return n;
  }
};

struct GgufFile {
  uint32_t version = 0;
  std::vector<std::pair<std::string, GgufValue>> kv;
  std::vector<GgufTensor> tensors;
  uint64_t data_offset = 0;

  const GgufValue *get(const std::string &key) const;
  bool get_u32(const std::string &key, uint32_t *out) const;
  bool get_u64(const std::string &key, uint64_t *out) const;
  bool get_f32(const std::string &key, float *out) const;
  bool get_string(const std::string &key, std::string *out) const;
  int tensor_index(const std::string &name) const;
};

// GgufFile::read (file.rs:57-116) over an in-memory image.
ifx_status gguf_parse(const uint8_t *p, size_t len, GgufFile *out);
// TensorInfo::byte_size (tensor.rs:30-40); -1 when the type is unknown.
int64_t gguf_type_bytes(uint32_t type, uint64_t n_elements);
// Weights::tensor_bytes bounds checks (weights.rs:97-112).
ifx_status gguf_tensor_range(const GgufFile &f, size_t file_len, int idx, uint64_t *start,
                             uint64_t *size);
// Config::from_gguf (config.rs:34-84).
ifx_status gguf_config(const GgufFile &f, ifx_config *c);

}  // namespace ifx
