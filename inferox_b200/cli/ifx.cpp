// `ifx`: the reference's command-line program (src/main.rs) on the B200
// library.
//
//   ifx <model.gguf>                                   inspect the file
//   ifx <model.gguf> <tokenizer.json> <prompt> [max_tokens] [temperature]
//
// Generate mode follows main.rs:39-95 step for step: load the model and the
// tokenizer, encode the prompt, make a KV cache of the model's full
// context_length, feed every prompt token through decode_step (not prefill),
// then max_tokens times sample the latest logits (temperature as given,
// top_k 0, top_p 1) and feed the sampled token back; print the decoded
// tokens with no trailing newline. The reference draws from an unseeded
// thread_rng; here the draws come from the device sampler's counter-based
// generator, seeded from IFX_SEED when set, else from std::random_device.
// Greedy output (temperature 0, the default) is deterministic either way.
// IFX_KQUANT_LAYOUT=ggml loads a file written by llama.cpp (ggml type ids and
// K-quant byte orders; the default, "reference", reads the reference's).
//
// Inspect mode prints the header, metadata, tensor table, data layout and
// the first five tensors' byte ranges in the reference's format
// (main.rs:97-186), reading the file through a read-only mapping.
//
// Exit status 1 with "error: ..." on stderr for every failure main.rs
// reports that way; usage errors likewise.
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cerrno>
#include <cmath>
#include <random>
#include <string>
#include <vector>

#include "../../include/inferox.h"
#include "../csrc/gguf.h"

namespace {

[[noreturn]] void die(const std::string &msg) {
  fprintf(stderr, "%s\n", msg.c_str());
  exit(1);
}

std::string last_error() {
  const char *e = ifx_last_error();
  return e ? e : "";
}

// ------------------------------------------------------ argument parsing --

// usize::from_str: an optional '+', then decimal digits, no overflow.
bool parse_usize(const char *s, uint64_t *out) {
  if (*s == '+') ++s;
  if (!*s) return false;
  uint64_t v = 0;
  for (; *s; ++s) {
    if (*s < '0' || *s > '9') return false;
    const uint64_t d = (uint64_t)(*s - '0');
    if (v > (UINT64_MAX - d) / 10) return false;
    v = v * 10 + d;
  }
  *out = v;
  return true;
}

// f32::from_str: decimal or exponent notation, inf/infinity/nan in any case;
// no surrounding space and no hexadecimal form.
bool parse_f32(const char *s, float *out) {
  if (!*s || isspace((unsigned char)*s)) return false;
  const char *p = (*s == '+' || *s == '-') ? s + 1 : s;
  if (p[0] == '0' && (p[1] == 'x' || p[1] == 'X')) return false;
  if (strchr(s, '(')) return false;
  char *end = nullptr;
  const float v = strtof(s, &end);
  if (end == s || *end) return false;
  *out = v;
  return true;
}

// ------------------------------------------------------- value display --

// Rust's Display for f32/f64: the shortest decimal that reads back to the
// same value, written out positionally (never with an exponent).
std::string rust_float(double v, bool single) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v < 0 ? "-inf" : "inf";
  char buf[64];
  const int maxp = single ? 9 : 17;
  int p = 1;
  for (; p < maxp; ++p) {
    snprintf(buf, sizeof buf, "%.*e", p - 1, v);
    if (single ? (strtof(buf, nullptr) == (float)v) : (strtod(buf, nullptr) == v)) break;
  }
  snprintf(buf, sizeof buf, "%.*e", p - 1, v);
  // buf = [-]d[.ddd]e[+-]XX
  std::string m(buf), digits;
  const bool neg = m[0] == '-';
  const size_t epos = m.find('e');
  for (size_t i = neg ? 1 : 0; i < epos; ++i)
    if (m[i] != '.') digits.push_back(m[i]);
  const int exp10 = atoi(m.c_str() + epos + 1);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  std::string out = neg ? "-" : "";
  if (digits == "0") return out + "0";
  const int n = (int)digits.size();
  if (exp10 >= n - 1) {
    out += digits + std::string((size_t)(exp10 - (n - 1)), '0');
  } else if (exp10 >= 0) {
    out += digits.substr(0, (size_t)exp10 + 1) + "." + digits.substr((size_t)exp10 + 1);
  } else {
    out += "0." + std::string((size_t)(-exp10 - 1), '0') + digits;
  }
  return out;
}

const char *value_type_name(uint32_t vt) {  // ValueType's Display (types.rs:44-63)
  static const char *n[] = {"uint8", "int8",  "uint16", "int16",  "uint32", "int32",  "float32",
                            "bool",  "string", "array", "uint64", "int64",  "float64"};
  return vt < 13 ? n[vt] : "?";
}

std::string show_value(const ifx::GgufValue &v) {  // Value's Display (value.rs:74-106)
  switch (v.vt) {
    case 0: case 2: case 4: case 10: return std::to_string(v.u);
    case 1: case 3: case 5: case 11: return std::to_string(v.i);
    case 6: return rust_float(v.f, true);
    case 12: return rust_float(v.f, false);
    case 7: return v.u ? "true" : "false";
    case 8: return v.s;
    case 9: {
      std::string s = std::string(value_type_name(v.arr_type)) + "[" + std::to_string(v.arr_len) + "] [";
      const uint64_t max_preview = 8;
      for (uint64_t i = 0; i < v.arr_len; ++i) {
        if (i >= max_preview && v.arr_len > max_preview + 1) {
          s += ", ...";
          break;
        }
        if (i > 0) s += ", ";
        if (i < v.items.size()) s += show_value(v.items[i]);
      }
      return s + "]";
    }
  }
  return "";
}

const char *tensor_type_name(uint32_t t) {  // TensorType::name (types.rs:146-178)
  switch (t) {
    case 0: return "F32";     case 1: return "F16";     case 2: return "Q4_0";
    case 3: return "Q4_1";    case 5: return "Q5_0";    case 6: return "Q5_1";
    case 7: return "Q8_0";    case 8: return "Q8_1";    case 10: return "Q2_K";
    case 11: return "Q3_K";   case 12: return "Q4_K";   case 13: return "Q5_K";
    case 14: return "Q6_K";   case 15: return "Q8_K";   case 16: return "I8";
    case 17: return "I16";    case 18: return "I32";    case 19: return "I64";
    case 20: return "F64";    case 21: return "IQ1_S";  case 22: return "IQ1_M";
    case 23: return "IQ2_XXS"; case 24: return "IQ2_XS"; case 25: return "IQ2_S";
    case 26: return "IQ3_XXS"; case 27: return "IQ3_S";  case 28: return "IQ4_XS";
    case 29: return "IQ4_NL";  case 30: return "IQ4_XSS";
  }
  return "?";
}

// Left-aligned in `width` characters (Rust pads by characters, not bytes).
std::string pad(const std::string &s, size_t width) {
  size_t chars = 0;
  for (unsigned char c : s) chars += (c & 0xC0) != 0x80;
  return chars >= width ? s : s + std::string(width - chars, ' ');
}

void section(const char *title) {
  const std::string rule(72, '-');
  printf("%s\n%s\n%s\n", rule.c_str(), title, rule.c_str());
}

// gguf::Error's Display (error.rs:47-76) for a failed open of `bytes`.
std::string gguf_error_text(ifx_status st, const uint8_t *bytes, size_t len) {
  switch (st) {
    case IFX_ERR_INVALID_MAGIC: {
      std::string s = "invalid magic: expected 'GGUF', got [";
      for (int i = 0; i < 4; ++i) s += (i ? ", " : "") + std::to_string(i < (int)len ? bytes[i] : 0);
      return s + "]";
    }
    case IFX_ERR_UNSUPPORTED_VERSION: {
      uint32_t v = 0;
      if (len >= 8) memcpy(&v, bytes + 4, 4);
      return "unsupported GGUF version: " + std::to_string(v) + " (expected 2 or 3)";
    }
    case IFX_ERR_UNEXPECTED_EOF: return "unexpected end of file";
    case IFX_ERR_TENSOR_OFFSET_OVERFLOW: return "tensor byte range overflows file bounds";
    default: break;
  }
  const std::string msg = last_error();
  return st == IFX_ERR_IO && msg.rfind("io error", 0) != 0 ? "io error: " + msg : msg;
}

// ------------------------------------------------------------- inspect --

void inspect(const char *path) {  // main.rs:97-116
  const std::string fail = std::string("error: failed to open '") + path + "': ";
  const int fd = open(path, O_RDONLY);
  if (fd < 0) die(fail + "io error: " + strerror(errno) + " (os error " + std::to_string(errno) + ")");
  struct stat sb;
  if (fstat(fd, &sb) != 0) die(fail + "io error: " + strerror(errno) + " (os error " + std::to_string(errno) + ")");
  const size_t len = (size_t)sb.st_size;
  const uint8_t *bytes = nullptr;
  if (len) {
    void *mp = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
    if (mp == MAP_FAILED) die(fail + "io error: " + strerror(errno) + " (os error " + std::to_string(errno) + ")");
    bytes = static_cast<const uint8_t *>(mp);
  }
  close(fd);
  static const uint8_t empty = 0;
  ifx::GgufFile f;
  const ifx_status st = ifx::gguf_parse(bytes ? bytes : &empty, len, &f);
  if (st != IFX_OK) die(fail + gguf_error_text(st, bytes, len));

  section("Header");
  printf("  version:     %u\n", f.version);
  printf("  n_tensors:   %zu\n", f.tensors.size());
  printf("  n_kv:        %zu\n", f.kv.size());

  section(("Metadata (" + std::to_string(f.kv.size()) + " entries)").c_str());
  for (size_t i = 0; i < f.kv.size(); ++i)
    printf("  [%3zu] %s (%s) => %s\n", i, pad(f.kv[i].first, 50).c_str(),
           value_type_name(f.kv[i].second.vt), show_value(f.kv[i].second).c_str());

  section(("Tensors (" + std::to_string(f.tensors.size()) + " tensors)").c_str());
  bool all_known = true;
  uint64_t total = 0;
  for (size_t i = 0; i < f.tensors.size(); ++i) {
    const ifx::GgufTensor &t = f.tensors[i];
    std::string shape;
    for (size_t d = 0; d < t.shape.size(); ++d) shape += (d ? " x " : "") + std::to_string(t.shape[d]);
    printf("  [%3zu] %s\n", i, t.name.c_str());
    printf("        type:    %s (id=%u)\n", tensor_type_name(t.type), t.type);
    printf("        shape:   [%s]\n", shape.c_str());
    printf("        elems:   %llu\n", (unsigned long long)t.n_elements());
    printf("        offset:  %llu bytes\n", (unsigned long long)t.offset);
    const int64_t size = ifx::gguf_type_bytes(t.type, t.n_elements());
    if (size >= 0) {
      printf("        size:    %lld bytes\n", (long long)size);
      total += (uint64_t)size;
    } else {
      printf("        size:    <unknown type size>\n");
      all_known = false;
    }
  }

  section("Layout");
  printf("  file:                 %s\n", path);
  printf("  tensor data offset:   %llu bytes\n", (unsigned long long)f.data_offset);
  if (all_known) printf("  total tensor bytes:   %llu bytes\n", (unsigned long long)total);
  else printf("  total tensor bytes:   <unknown>\n");

  section("Raw tensor bytes (mmap)");
  if (f.tensors.empty()) {
    printf("  (no tensors)\n");
  } else {
    for (size_t i = 0; i < f.tensors.size() && i < 5; ++i) {
      uint64_t start = 0, size = 0;
      const ifx_status s = ifx::gguf_tensor_range(f, len, (int)i, &start, &size);
      if (s == IFX_OK) {
        printf("  %s -> %llu bytes\n", pad(f.tensors[i].name, 40).c_str(), (unsigned long long)size);
      } else {
        std::string e = s == IFX_ERR_UNKNOWN_TENSOR_TYPE
                            ? "unknown tensor type id: " + std::to_string(f.tensors[i].type)
                            : gguf_error_text(s, bytes, len);
        printf("  %s -> error: %s\n", pad(f.tensors[i].name, 40).c_str(), e.c_str());
      }
    }
    if (f.tensors.size() > 5) printf("  ... and %zu more tensor(s)\n", f.tensors.size() - 5);
  }
  if (bytes) munmap(const_cast<uint8_t *>(bytes), len);
}

// ------------------------------------------------------------ generate --

void generate(const char *model_path, const char *tok_path, const char *prompt, uint64_t max_tokens,
              float temperature) {  // main.rs:39-95
  ifx_load_opts o;
  ifx_load_opts_default(&o);
  // the arguments stay main.rs's; a file written by llama.cpp is announced
  // through the environment
  if (const char *k = getenv("IFX_KQUANT_LAYOUT")) {
    if (!strcmp(k, "ggml")) o.kquant_layout = IFX_KQUANT_GGML;
    else if (strcmp(k, "reference") != 0)
      die(std::string("error: IFX_KQUANT_LAYOUT must be 'reference' or 'ggml', not '") + k + "'");
  }
  ifx_model *m = nullptr;
  if (ifx_model_load(model_path, &o, &m) != IFX_OK)
    die(std::string("error: failed to load model '") + model_path + "': " + last_error());
  ifx_tokenizer *tok = nullptr;
  if (ifx_tokenizer_load(tok_path, &tok) != IFX_OK)
    die(std::string("error: failed to load tokenizer '") + tok_path + "': " + last_error());

  const size_t plen = strlen(prompt);
  size_t n = 0;
  std::vector<uint32_t> ids(plen + 16);
  ifx_status st = ifx_tokenizer_encode(tok, prompt, plen, ids.data(), ids.size(), &n);
  if (st == IFX_ERR_SHAPE) {
    ids.resize(n);
    st = ifx_tokenizer_encode(tok, prompt, plen, ids.data(), ids.size(), &n);
  }
  if (st != IFX_OK) die("error: " + last_error());
  ids.resize(n);

  ifx_config cfg;
  if (ifx_model_config(m, &cfg) != IFX_OK) die("error: " + last_error());
  ifx_kv *kv = nullptr;  // KvCache::new(n_layers, context_length) (main.rs:66-67)
  if (ifx_kv_create(m, (size_t)cfg.context_length, &kv) != IFX_OK) die("error: " + last_error());

  uint64_t seed;
  if (const char *e = getenv("IFX_SEED")) {
    seed = strtoull(e, nullptr, 10);
  } else {
    std::random_device rd;
    seed = ((uint64_t)rd() << 32) ^ rd();
  }
  ifx_sampler s{temperature, 0, 1.0f};

  for (uint32_t t : ids)
    if (ifx_decode_step(m, kv, t, nullptr) != IFX_OK) die("error: decode failed: " + last_error());

  std::vector<uint32_t> generated;
  for (uint64_t i = 0; i < max_tokens; ++i) {
    uint32_t next = 0;
    if (ifx_sample(m, &s, seed, i, &next) != IFX_OK) die("error: " + last_error());
    generated.push_back(next);
    if (ifx_decode_step(m, kv, next, nullptr) != IFX_OK) die("error: decode failed: " + last_error());
  }

  size_t tl = 0;
  std::string text(generated.size() * 8 + 16, '\0');
  st = ifx_tokenizer_decode(tok, generated.data(), generated.size(), &text[0], text.size(), &tl);
  if (st == IFX_ERR_SHAPE) {
    text.resize(tl);
    st = ifx_tokenizer_decode(tok, generated.data(), generated.size(), &text[0], text.size(), &tl);
  }
  if (st != IFX_OK) die("error: " + last_error());
  fwrite(text.data(), 1, tl, stdout);
  fflush(stdout);
  ifx_kv_free(kv);
  ifx_tokenizer_free(tok);
  ifx_model_free(m);
}

}  // namespace

int main(int argc, char **argv) {  // main.rs:9-37
  if (argc < 2) die(std::string("usage: ") + argv[0] +
                    " <model.gguf> [tokenizer.json] [prompt] [max_tokens] [temperature]");
  if (argc < 4) {
    inspect(argv[1]);
    return 0;
  }
  uint64_t max_tokens = 32;
  float temperature = 0.0f;
  if (argc > 4 && !parse_usize(argv[4], &max_tokens)) max_tokens = 32;
  if (argc > 5 && !parse_f32(argv[5], &temperature)) temperature = 0.0f;
  generate(argv[1], argv[2], argv[3], max_tokens, temperature);
  return 0;
}
