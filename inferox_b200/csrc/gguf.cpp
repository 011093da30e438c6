// GGUF parsing for model load. Follows src/gguf/file.rs:57-116 (header,
// metadata, tensor infos, 32-byte aligned data region), value.rs:45-113,
// tensor.rs:30-75, types.rs:110-229, weights.rs:97-112 and
// model/config.rs:34-84, with the same error for each failure.
#include "gguf.h"

#include <cstring>

#include "status.h"

namespace ifx {

namespace {

struct Reader {
  const uint8_t *p;
  size_t len, pos = 0;
  ifx_status err = IFX_OK;
  bool read(void *dst, size_t n) {
    if (err != IFX_OK) return false;
    if (n > len - pos) {
      err = IFX_ERR_IO;  // read_exact's io::Error (file.rs:73)
      return false;
    }
    memcpy(dst, p + pos, n);
    pos += n;
    return true;
  }
  uint32_t u32() {
    uint32_t v = 0;
    read(&v, 4);
    return v;
  }
  uint64_t u64() {
    uint64_t v = 0;
    read(&v, 8);
    return v;
  }
};

bool utf8_ok(const std::string &s) {
  size_t i = 0, n = s.size();
  const unsigned char *b = reinterpret_cast<const unsigned char *>(s.data());
  while (i < n) {
    unsigned c = b[i];
    size_t k;
    uint32_t cp;
    if (c < 0x80) {
      ++i;
      continue;
    } else if ((c & 0xe0) == 0xc0) {
      k = 1;
      cp = c & 0x1f;
    } else if ((c & 0xf0) == 0xe0) {
      k = 2;
      cp = c & 0x0f;
    } else if ((c & 0xf8) == 0xf0) {
      k = 3;
      cp = c & 0x07;
    } else {
      return false;
    }
    for (size_t t = 1; t <= k; ++t) {
      if (i + t >= n || (b[i + t] & 0xc0) != 0x80) return false;
      cp = (cp << 6) | (b[i + t] & 0x3f);
    }
    if ((k == 1 && cp < 0x80) || (k == 2 && cp < 0x800) || (k == 3 && cp < 0x10000) ||
        cp > 0x10ffff || (cp >= 0xd800 && cp <= 0xdfff))
      return false;
    i += k + 1;
  }
  return true;
}

bool read_string(Reader &r, std::string *s) {
  uint64_t n = r.u64();
  if (r.err) return false;
  if (n > r.len - r.pos) {
    r.err = IFX_ERR_IO;
    return false;
  }
  s->assign(reinterpret_cast<const char *>(r.p + r.pos), (size_t)n);
  r.pos += (size_t)n;
  if (!utf8_ok(*s)) {
    r.err = IFX_ERR_INVALID_UTF8;
    return false;
  }
  return true;
}

bool read_value(Reader &r, uint32_t vt, GgufValue *v) {
  if (v) v->vt = vt;
  switch (vt) {
    case 0: { uint8_t x = 0; r.read(&x, 1); if (v) v->u = x; break; }
    case 1: { int8_t x = 0; r.read(&x, 1); if (v) v->i = x; break; }
    case 2: { uint16_t x = 0; r.read(&x, 2); if (v) v->u = x; break; }
    case 3: { int16_t x = 0; r.read(&x, 2); if (v) v->i = x; break; }
    case 4: { uint32_t x = 0; r.read(&x, 4); if (v) v->u = x; break; }
    case 5: { int32_t x = 0; r.read(&x, 4); if (v) v->i = x; break; }
    case 6: { float x = 0; r.read(&x, 4); if (v) v->f = x; break; }
    case 7: { uint8_t x = 0; r.read(&x, 1); if (v) v->u = x != 0; break; }
    case 8: {
      std::string s;
      read_string(r, &s);
      if (v) v->s = std::move(s);
      break;
    }
    case 9: {
      uint32_t it = r.u32();
      if (r.err) return false;
      if (it > 12) {
        r.err = IFX_ERR_UNKNOWN_VALUE_TYPE;
        return false;
      }
      uint64_t n = r.u64();
      if (v) {
        v->arr_type = it;
        v->arr_len = n;
      }
      for (uint64_t k = 0; k < n && !r.err; ++k) {
        if (v && k < GgufValue::kArrayPreview) {
          v->items.emplace_back();
          read_value(r, it, &v->items.back());
        } else {
          read_value(r, it, nullptr);
        }
      }
      break;
    }
    case 10: { uint64_t x = 0; r.read(&x, 8); if (v) v->u = x; break; }
    case 11: { int64_t x = 0; r.read(&x, 8); if (v) v->i = x; break; }
    case 12: { double x = 0; r.read(&x, 8); if (v) v->f = x; break; }
    default: r.err = IFX_ERR_UNKNOWN_VALUE_TYPE;
  }
  return r.err == IFX_OK;
}

bool valid_type(uint32_t v) { return v <= 30 && v != 4 && v != 9; }  // types.rs:110-142

}  // namespace

int64_t gguf_type_bytes(uint32_t type, uint64_t n) {
  switch (type) {
    case 0: return (int64_t)(n * 4);
    case 1: return (int64_t)(n * 2);
    case 16: return (int64_t)n;
    case 17: return (int64_t)(n * 2);
    case 18: return (int64_t)(n * 4);
    case 19: case 20: return (int64_t)(n * 8);
    default: break;
  }
  int e = 0, b = 0;
  switch (type) {
    case 2: e = 32; b = 18; break;
    case 3: e = 32; b = 20; break;
    case 5: e = 32; b = 22; break;
    case 6: e = 32; b = 24; break;
    case 7: e = 32; b = 34; break;
    case 8: e = 32; b = 36; break;
    case 29: e = 32; b = 18; break;
    case 10: e = 256; b = 96; break;
    case 11: e = 256; b = 110; break;
    case 12: e = 256; b = 144; break;
    case 13: e = 256; b = 176; break;
    case 14: e = 256; b = 210; break;
    case 15: e = 256; b = 292; break;
    case 21: e = 256; b = 166; break;
    case 22: e = 256; b = 184; break;
    case 23: e = 256; b = 66; break;
    case 24: e = 256; b = 104; break;
    case 25: e = 256; b = 176; break;
    case 26: e = 256; b = 98; break;
    case 27: e = 256; b = 166; break;
    case 28: e = 256; b = 136; break;
    case 30: e = 256; b = 116; break;
    default: return -1;
  }
  return (int64_t)((n + e - 1) / e * b);
}

const GgufValue *GgufFile::get(const std::string &key) const {
  for (auto &kv_ : kv)
    if (kv_.first == key) return &kv_.second;
  return nullptr;
}

bool GgufFile::get_u32(const std::string &key, uint32_t *out) const {
  uint64_t v;
  if (!get_u64(key, &v)) return false;
  *out = (uint32_t)v;
  return true;
}

bool GgufFile::get_u64(const std::string &key, uint64_t *out) const {
  const GgufValue *v = get(key);
  if (!v) return false;
  switch (v->vt) {
    case 0: case 2: case 4: case 10: *out = v->u; return true;
    case 1: case 3: case 5: case 11: *out = (uint64_t)v->i; return true;
    default: return false;
  }
}

bool GgufFile::get_f32(const std::string &key, float *out) const {
  const GgufValue *v = get(key);
  if (!v) return false;
  switch (v->vt) {
    case 6: case 12: *out = (float)v->f; return true;
    case 0: case 2: case 4: case 10: *out = (float)v->u; return true;
    case 1: case 3: case 5: case 11: *out = (float)v->i; return true;
    default: return false;
  }
}

bool GgufFile::get_string(const std::string &key, std::string *out) const {
  const GgufValue *v = get(key);
  if (!v || v->vt != 8) return false;
  *out = v->s;
  return true;
}

int GgufFile::tensor_index(const std::string &name) const {
  for (size_t i = 0; i < tensors.size(); ++i)
    if (tensors[i].name == name) return (int)i;
  return -1;
}

ifx_status gguf_parse(const uint8_t *p, size_t len, GgufFile *out) {
  Reader r{p, len};
  char magic[4];
  if (!r.read(magic, 4)) return fail(r.err, "gguf: reading magic");
  if (memcmp(magic, "GGUF", 4) != 0) return fail(IFX_ERR_INVALID_MAGIC, "gguf: invalid magic");
  out->version = r.u32();
  if (r.err) return fail(r.err, "gguf: header");
  if (out->version != 2 && out->version != 3)
    return fail(IFX_ERR_UNSUPPORTED_VERSION, "gguf: unsupported version");
  uint64_t n_tensors = r.u64(), n_kv = r.u64();
  if (r.err) return fail(r.err, "gguf: header");
  if (n_kv > len || n_tensors > len) return fail(IFX_ERR_IO, "gguf: counts exceed file size");
  out->kv.clear();
  out->tensors.clear();
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key;
    if (!read_string(r, &key)) return fail(r.err, "gguf: metadata key");
    uint32_t vt = r.u32();
    if (r.err) return fail(r.err, "gguf: metadata type");
    if (vt > 12) return fail(IFX_ERR_UNKNOWN_VALUE_TYPE, "gguf: unknown value type");
    GgufValue v;
    if (!read_value(r, vt, &v)) return fail(r.err, "gguf: metadata value");
    out->kv.emplace_back(std::move(key), std::move(v));
  }
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensor t;
    if (!read_string(r, &t.name)) return fail(r.err, "gguf: tensor name");
    uint32_t nd = r.u32();
    if (r.err) return fail(r.err, "gguf: tensor dims");
    if (nd > 4) return fail(IFX_ERR_INVALID_SHAPE, "gguf: more than 4 dims");
    for (uint32_t d = 0; d < nd; ++d) t.shape.push_back(r.u64());
    t.type = r.u32();
    if (!r.err && !valid_type(t.type)) return fail(IFX_ERR_UNKNOWN_TENSOR_TYPE, "gguf: tensor type");
    t.offset = r.u64();
    if (r.err) return fail(r.err, "gguf: tensor info");
    out->tensors.push_back(std::move(t));
  }
  out->data_offset = (r.pos + 31) / 32 * 32;
  return IFX_OK;
}

ifx_status gguf_tensor_range(const GgufFile &f, size_t file_len, int idx, uint64_t *start,
                             uint64_t *size) {
  if (idx < 0 || (size_t)idx >= f.tensors.size())
    return fail(IFX_ERR_INVALID_TENSOR_INDEX, "tensor index out of bounds");
  const GgufTensor &t = f.tensors[idx];
  int64_t sz = gguf_type_bytes(t.type, t.n_elements());
  if (sz < 0) return fail(IFX_ERR_UNKNOWN_TENSOR_TYPE, "tensor " + t.name + ": unknown type");
  uint64_t s = f.data_offset + t.offset;
  if (s < f.data_offset) return fail(IFX_ERR_TENSOR_OFFSET_OVERFLOW, "tensor " + t.name + ": offset");
  uint64_t e = s + (uint64_t)sz;
  if (e < s) return fail(IFX_ERR_TENSOR_OFFSET_OVERFLOW, "tensor " + t.name + ": size");
  if (e > file_len) return fail(IFX_ERR_UNEXPECTED_EOF, "tensor " + t.name + ": past end of file");
  *start = s;
  *size = (uint64_t)sz;
  return IFX_OK;
}

ifx_status gguf_config(const GgufFile &f, ifx_config *c) {
  memset(c, 0, sizeof(*c));
  std::string arch;
  if (!f.get_string("general.architecture", &arch))
    return fail(IFX_ERR_TENSOR_NOT_FOUND, "tensor not found: general.architecture");
  strncpy(c->architecture, arch.c_str(), sizeof(c->architecture) - 1);
  if (arch != "llama") return fail(IFX_ERR_UNSUPPORTED_ARCHITECTURE, "unsupported architecture: " + arch);
  auto need = [&](const char *k, uint64_t *v) -> bool { return f.get_u64(k, v); };
  if (!need("llama.embedding_length", &c->hidden_size))
    return fail(IFX_ERR_TENSOR_NOT_FOUND, "tensor not found: llama.embedding_length");
  if (!need("llama.block_count", &c->n_layers))
    return fail(IFX_ERR_TENSOR_NOT_FOUND, "tensor not found: llama.block_count");
  if (!need("llama.attention.head_count", &c->n_heads))
    return fail(IFX_ERR_TENSOR_NOT_FOUND, "tensor not found: llama.attention.head_count");
  uint32_t v32;
  c->n_kv_heads = f.get_u32("llama.attention.head_count_kv", &v32) ? v32 : c->n_heads;
  if (c->n_heads == 0) return fail(IFX_ERR_INVALID_SHAPE, "head_count is 0");
  c->head_dim = f.get_u32("llama.attention.key_length", &v32) ? v32 : c->hidden_size / c->n_heads;
  if (!need("llama.feed_forward_length", &c->intermediate_size))
    return fail(IFX_ERR_TENSOR_NOT_FOUND, "tensor not found: llama.feed_forward_length");
  if (!f.get_f32("llama.attention.layer_norm_rms_epsilon", &c->norm_eps)) c->norm_eps = 1e-5f;
  if (!f.get_f32("llama.rope.freq_base", &c->rope_base)) c->rope_base = 10000.0f;
  c->rope_dim = f.get_u32("llama.rope.dimension_count", &v32) ? v32 : c->head_dim;
  c->context_length = f.get_u32("llama.context_length", &v32) ? v32 : 4096;
  c->vocab_size = f.get_u32("llama.vocab_size", &v32) ? v32 : 0;
  return IFX_OK;
}

}  // namespace ifx
