// Byte-level BPE tokenizer over a Hugging Face tokenizer.json: the
// reference's BpeTokenizer (src/tokenizer/mod.rs:23-226) and its GPT-2 byte
// tables (src/tokenizer/bytes.rs:10-35), as host C++ behind the C ABI.
//
// Behaviour kept from the reference:
//   * the schema its serde structs accept (mod.rs:37-57): `model.type`,
//     `model.vocab` (string -> u32), `model.merges` (strings "a b") are
//     required, `model.unk_token` may be null or absent, `added_tokens`
//     defaults to empty and each entry needs `content`; unknown fields are
//     ignored, a known field given twice is an error, and any schema error
//     is a JSON error that comes before the "BPE" type check (mod.rs:69-73);
//   * merge ranks are line indices, a line splits on Unicode white space
//     and keeps its first two parts, a later duplicate pair overwrites the
//     earlier rank (mod.rs:80-88); unk_id = vocab[unk_token] else 0
//     (mod.rs:97-101);
//   * encode splits out added tokens first (mod.rs:157-191), maps every
//     other byte through the byte encoder and merges repeatedly the adjacent
//     pair of lowest rank, leftmost among equals (mod.rs:114-140); pieces
//     outside the vocabulary become unk_id (mod.rs:150-154);
//   * decode maps each character of each known token back through the byte
//     decoder (other characters contribute their UTF-8 bytes), skips unknown
//     ids and converts the bytes lossily: each maximal invalid subsequence
//     becomes one U+FFFD (String::from_utf8_lossy, mod.rs:206-225).
//
// Where the reference is not deterministic or does not return, this file
// picks one behaviour: two added tokens found at the same position resolve
// to the longer one (the reference's HashSet order decides), an empty added
// token is ignored when splitting (the reference loops forever on it), and
// an id held by two vocabulary entries decodes to the later entry in the
// file (HashMap order in the reference).
//
// The merge loop runs on a heap of candidate pairs keyed by (rank, start
// offset) with lazily invalidated entries, which performs the same merges in
// the same order as the reference's rescan of all pairs after each merge,
// in O(n log n) instead of O(n^2) for a prompt that is one long piece (the
// reference has no pre-tokenizer).
#include <cstring>
#include <fstream>
#include <queue>
#include <sstream>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "../../include/inferox.h"
#include "status.h"

namespace ifx {

namespace {

// ------------------------------------------------------------- UTF-8 ----

void put_utf8(uint32_t cp, std::string *out) {
  if (cp < 0x80) {
    out->push_back((char)cp);
  } else if (cp < 0x800) {
    out->push_back((char)(0xC0 | (cp >> 6)));
    out->push_back((char)(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    out->push_back((char)(0xE0 | (cp >> 12)));
    out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back((char)(0x80 | (cp & 0x3F)));
  } else {
    out->push_back((char)(0xF0 | (cp >> 18)));
    out->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
    out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back((char)(0x80 | (cp & 0x3F)));
  }
}

// Length of the valid UTF-8 sequence at b[i] (1-4), or 0 with *bad set to
// the number of bytes of the maximal prefix of a valid sequence (at least 1)
// when the bytes there are not valid UTF-8 (Unicode's "maximal subpart"
// rule, which String::from_utf8_lossy follows).
size_t utf8_seq(const uint8_t *b, size_t n, size_t i, size_t *bad) {
  const uint8_t c = b[i];
  if (c < 0x80) return 1;
  auto at = [&](size_t k) -> int { return i + k < n ? b[i + k] : -1; };
  auto cont = [](int x) { return x >= 0x80 && x <= 0xBF; };
  size_t w;
  bool second_ok;
  const int s = at(1);
  if (c >= 0xC2 && c <= 0xDF) {
    w = 2;
    second_ok = cont(s);
  } else if (c >= 0xE0 && c <= 0xEF) {
    w = 3;
    second_ok = (c == 0xE0) ? (s >= 0xA0 && s <= 0xBF)
                : (c == 0xED) ? (s >= 0x80 && s <= 0x9F)
                              : cont(s);
  } else if (c >= 0xF0 && c <= 0xF4) {
    w = 4;
    second_ok = (c == 0xF0) ? (s >= 0x90 && s <= 0xBF)
                : (c == 0xF4) ? (s >= 0x80 && s <= 0x8F)
                              : cont(s);
  } else {
    *bad = 1;
    return 0;
  }
  if (!second_ok) {
    *bad = 1;
    return 0;
  }
  for (size_t k = 2; k < w; ++k) {
    if (!cont(at(k))) {
      *bad = k;
      return 0;
    }
  }
  return w;
}

bool utf8_valid(const uint8_t *b, size_t n) {
  size_t i = 0, bad = 0;
  while (i < n) {
    const size_t w = utf8_seq(b, n, i, &bad);
    if (!w) return false;
    i += w;
  }
  return true;
}

uint32_t utf8_cp(const uint8_t *b, size_t w) {
  if (w == 1) return b[0];
  uint32_t cp = b[0] & (w == 2 ? 0x1F : w == 3 ? 0x0F : 0x07);
  for (size_t k = 1; k < w; ++k) cp = (cp << 6) | (b[k] & 0x3F);
  return cp;
}

// Code points of a valid UTF-8 string.
std::vector<uint32_t> code_points(const std::string &s) {
  std::vector<uint32_t> cps;
  const uint8_t *b = reinterpret_cast<const uint8_t *>(s.data());
  size_t i = 0, bad = 0;
  while (i < s.size()) {
    const size_t w = utf8_seq(b, s.size(), i, &bad);
    if (!w) break;  // strings here come from validated JSON
    cps.push_back(utf8_cp(b + i, w));
    i += w;
  }
  return cps;
}

// Unicode White_Space (what str::split_whitespace splits on).
bool is_white_space(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F ||
         c == 0x205F || c == 0x3000;
}

// -------------------------------------------------------------- JSON ----

struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } k = Null;
  bool b = false;
  bool integer = false;  // number without fraction or exponent
  bool negative = false;
  uint64_t u = 0;        // magnitude of an integer (saturates past 2^64)
  std::string s;         // string value
  std::vector<JVal> a;
  std::vector<std::pair<std::string, JVal>> o;
};

// Strict RFC 8259 parser (what serde_json accepts when reading into
// strings, integers, sequences and maps): no trailing commas, no comments,
// no NaN, no lone surrogates, no raw control characters in strings, nothing
// after the top-level value, at most 128 levels of nesting.
class JsonParser {
 public:
  JsonParser(const char *p, size_t n) : p_(p), n_(n) {}
  bool parse(JVal *out) {
    ws();
    if (!value(out, 0)) return false;
    ws();
    if (i_ != n_) return err("trailing characters");
    return true;
  }
  std::string error() const {
    std::ostringstream m;
    m << msg_ << " at byte " << i_;
    return m.str();
  }

 private:
  const char *p_;
  size_t n_, i_ = 0;
  std::string msg_;

  bool err(const char *m) {
    if (msg_.empty()) msg_ = m;
    return false;
  }
  void ws() {
    while (i_ < n_ && (p_[i_] == ' ' || p_[i_] == '\t' || p_[i_] == '\n' || p_[i_] == '\r')) ++i_;
  }
  bool lit(const char *w) {
    const size_t l = strlen(w);
    if (n_ - i_ < l || memcmp(p_ + i_, w, l) != 0) return err("invalid literal");
    i_ += l;
    return true;
  }
  bool value(JVal *v, int depth) {
    if (i_ >= n_) return err("EOF while parsing a value");
    const char c = p_[i_];
    if (c == '{' || c == '[') {
      if (depth >= 128) return err("recursion limit exceeded");
      return c == '{' ? object(v, depth + 1) : array(v, depth + 1);
    }
    if (c == '"') {
      v->k = JVal::Str;
      return string(&v->s);
    }
    if (c == 't') {
      v->k = JVal::Bool;
      v->b = true;
      return lit("true");
    }
    if (c == 'f') {
      v->k = JVal::Bool;
      return lit("false");
    }
    if (c == 'n') {
      v->k = JVal::Null;
      return lit("null");
    }
    if (c == '-' || (c >= '0' && c <= '9')) return number(v);
    return err("expected value");
  }
  bool number(JVal *v) {
    v->k = JVal::Num;
    if (p_[i_] == '-') {
      v->negative = true;
      ++i_;
    }
    if (i_ >= n_ || p_[i_] < '0' || p_[i_] > '9') return err("invalid number");
    v->integer = true;
    if (p_[i_] == '0') {
      ++i_;
    } else {
      while (i_ < n_ && p_[i_] >= '0' && p_[i_] <= '9') {
        const uint64_t d = (uint64_t)(p_[i_] - '0');
        v->u = (v->u > (UINT64_MAX - d) / 10) ? UINT64_MAX : v->u * 10 + d;
        ++i_;
      }
    }
    if (i_ < n_ && p_[i_] == '.') {
      v->integer = false;
      ++i_;
      if (i_ >= n_ || p_[i_] < '0' || p_[i_] > '9') return err("invalid number");
      while (i_ < n_ && p_[i_] >= '0' && p_[i_] <= '9') ++i_;
    }
    if (i_ < n_ && (p_[i_] == 'e' || p_[i_] == 'E')) {
      v->integer = false;
      ++i_;
      if (i_ < n_ && (p_[i_] == '+' || p_[i_] == '-')) ++i_;
      if (i_ >= n_ || p_[i_] < '0' || p_[i_] > '9') return err("invalid number");
      while (i_ < n_ && p_[i_] >= '0' && p_[i_] <= '9') ++i_;
    }
    return true;
  }
  bool hex4(uint32_t *out) {
    if (n_ - i_ < 4) return err("EOF while parsing a string");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = p_[i_ + k];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return err("invalid escape");
    }
    i_ += 4;
    *out = v;
    return true;
  }
  bool string(std::string *s) {
    ++i_;  // opening quote
    s->clear();
    while (true) {
      if (i_ >= n_) return err("EOF while parsing a string");
      const unsigned char c = (unsigned char)p_[i_];
      if (c == '"') {
        ++i_;
        return true;
      }
      if (c < 0x20) return err("control character in string");
      if (c != '\\') {
        s->push_back((char)c);
        ++i_;
        continue;
      }
      ++i_;
      if (i_ >= n_) return err("EOF while parsing a string");
      const char e = p_[i_++];
      switch (e) {
        case '"': s->push_back('"'); break;
        case '\\': s->push_back('\\'); break;
        case '/': s->push_back('/'); break;
        case 'b': s->push_back('\b'); break;
        case 'f': s->push_back('\f'); break;
        case 'n': s->push_back('\n'); break;
        case 'r': s->push_back('\r'); break;
        case 't': s->push_back('\t'); break;
        case 'u': {
          uint32_t cp;
          if (!hex4(&cp)) return false;
          if (cp >= 0xDC00 && cp <= 0xDFFF) return err("lone trailing surrogate");
          if (cp >= 0xD800 && cp <= 0xDBFF) {
            if (n_ - i_ < 2 || p_[i_] != '\\' || p_[i_ + 1] != 'u')
              return err("lone leading surrogate");
            i_ += 2;
            uint32_t lo;
            if (!hex4(&lo)) return false;
            if (lo < 0xDC00 || lo > 0xDFFF) return err("lone leading surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(cp, s);
          break;
        }
        default: return err("invalid escape");
      }
    }
  }
  bool array(JVal *v, int depth) {
    v->k = JVal::Arr;
    ++i_;
    ws();
    if (i_ < n_ && p_[i_] == ']') {
      ++i_;
      return true;
    }
    while (true) {
      v->a.emplace_back();
      ws();
      if (!value(&v->a.back(), depth)) return false;
      ws();
      if (i_ >= n_) return err("EOF while parsing a list");
      if (p_[i_] == ',') {
        ++i_;
        continue;
      }
      if (p_[i_] == ']') {
        ++i_;
        return true;
      }
      return err("expected `,` or `]`");
    }
  }
  bool object(JVal *v, int depth) {
    v->k = JVal::Obj;
    ++i_;
    ws();
    if (i_ < n_ && p_[i_] == '}') {
      ++i_;
      return true;
    }
    while (true) {
      ws();
      if (i_ >= n_ || p_[i_] != '"') return err("key must be a string");
      v->o.emplace_back();
      if (!string(&v->o.back().first)) return false;
      ws();
      if (i_ >= n_ || p_[i_] != ':') return err("expected `:`");
      ++i_;
      ws();
      if (!value(&v->o.back().second, depth)) return false;
      ws();
      if (i_ >= n_) return err("EOF while parsing an object");
      if (p_[i_] == ',') {
        ++i_;
        continue;
      }
      if (p_[i_] == '}') {
        ++i_;
        return true;
      }
      return err("expected `,` or `}`");
    }
  }
};

// One named field of a struct-like object: null when absent; an error
// message when it appears twice (serde's "duplicate field").
bool field(const JVal &obj, const char *name, const JVal **out, std::string *why) {
  *out = nullptr;
  for (const auto &kv : obj.o) {
    if (kv.first != name) continue;
    if (*out) {
      *why = std::string("duplicate field `") + name + "`";
      return false;
    }
    *out = &kv.second;
  }
  return true;
}

// ------------------------------------------------------------ tables ----

// bytes.rs:10-27: bytes 0x21-0x7E, 0xA1-0xAC and 0xAE-0xFF map to the same
// code point; the other 68 bytes, in order, to U+0100, U+0101, ...
const std::vector<uint32_t> &byte_encoder() {
  static const std::vector<uint32_t> t = [] {
    std::vector<uint32_t> e(256);
    uint32_t n = 0;
    for (uint32_t b = 0; b < 256; ++b) {
      const bool keep = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE);
      e[b] = keep ? b : 0x100 + n++;
    }
    return e;
  }();
  return t;
}

struct PairHash {
  size_t operator()(const std::pair<std::string, std::string> &p) const {
    return std::hash<std::string>()(p.first) * 1000003u ^ std::hash<std::string>()(p.second);
  }
};

}  // namespace

}  // namespace ifx

struct ifx_tokenizer {
  std::unordered_map<std::string, uint32_t> vocab;
  std::unordered_map<uint32_t, std::string> id_to_token;
  std::unordered_map<std::pair<std::string, std::string>, size_t, ifx::PairHash> merges;
  std::vector<std::string> special;  // distinct added tokens, file order
  std::unordered_set<std::string> special_set;
  uint32_t unk_id = 0;
  std::vector<std::string> byte_str;             // byte -> its encoder character as UTF-8
  std::unordered_map<uint32_t, uint8_t> decoder;  // byte_decoder (bytes.rs:30-35)
};

namespace ifx {

namespace {

ifx_status json_fail(const std::string &why) {
  return fail(IFX_ERR_JSON, "json error: " + why);
}

// BpeTokenizer::from_json (mod.rs:67-110).
ifx_status tokenizer_from_json(const char *text, size_t len, ifx_tokenizer **out) {
  JVal root;
  JsonParser jp(text, len);
  if (!jp.parse(&root)) return json_fail(jp.error());
  if (root.k != JVal::Obj) return json_fail("expected struct TokenizerJson");
  std::string why;
  const JVal *added = nullptr, *model = nullptr;
  if (!field(root, "added_tokens", &added, &why) || !field(root, "model", &model, &why))
    return json_fail(why);
  if (!model) return json_fail("missing field `model`");
  if (model->k != JVal::Obj) return json_fail("invalid type for `model`, expected struct Model");
  std::vector<std::string> added_contents;
  if (added) {
    if (added->k != JVal::Arr) return json_fail("invalid type for `added_tokens`, expected a sequence");
    for (const JVal &t : added->a) {
      if (t.k != JVal::Obj) return json_fail("invalid type for an added token, expected struct AddedToken");
      const JVal *content = nullptr;
      if (!field(t, "content", &content, &why)) return json_fail(why);
      if (!content) return json_fail("missing field `content`");
      if (content->k != JVal::Str) return json_fail("invalid type for `content`, expected a string");
      added_contents.push_back(content->s);
    }
  }
  const JVal *kind = nullptr, *vocab = nullptr, *merges = nullptr, *unk = nullptr;
  if (!field(*model, "type", &kind, &why) || !field(*model, "vocab", &vocab, &why) ||
      !field(*model, "merges", &merges, &why) || !field(*model, "unk_token", &unk, &why))
    return json_fail(why);
  if (!kind) return json_fail("missing field `type`");
  if (kind->k != JVal::Str) return json_fail("invalid type for `type`, expected a string");
  if (!vocab) return json_fail("missing field `vocab`");
  if (vocab->k != JVal::Obj) return json_fail("invalid type for `vocab`, expected a map");
  if (!merges) return json_fail("missing field `merges`");
  if (merges->k != JVal::Arr) return json_fail("invalid type for `merges`, expected a sequence");
  for (const JVal &m : merges->a)
    if (m.k != JVal::Str) return json_fail("invalid type for a merge, expected a string");
  if (unk && unk->k != JVal::Null && unk->k != JVal::Str)
    return json_fail("invalid type for `unk_token`, expected a string");
  for (const auto &kv : vocab->o) {
    const JVal &v = kv.second;
    if (v.k != JVal::Num || !v.integer || (v.negative && v.u != 0) || v.u > 0xFFFFFFFFull)
      return json_fail("invalid value for vocabulary entry, expected u32");
  }
  if (kind->s != "BPE")
    return fail(IFX_ERR_UNSUPPORTED_MODEL, "unsupported tokenizer model: " + kind->s);

  auto *t = new ifx_tokenizer();
  for (const auto &kv : vocab->o) {
    t->vocab[kv.first] = (uint32_t)kv.second.u;  // a repeated key: the later value
  }
  for (const auto &kv : vocab->o) {
    auto it = t->vocab.find(kv.first);
    if (it->second == (uint32_t)kv.second.u) t->id_to_token[it->second] = kv.first;
  }
  for (size_t rank = 0; rank < merges->a.size(); ++rank) {
    const std::vector<uint32_t> cps = code_points(merges->a[rank].s);
    std::string parts[2];
    int np = 0;
    bool in = false;
    for (uint32_t c : cps) {
      if (is_white_space(c)) {
        if (in) {
          in = false;
          if (++np == 2) break;
        }
        continue;
      }
      in = true;
      put_utf8(c, &parts[np]);
    }
    if (!parts[0].empty() && !parts[1].empty()) t->merges[{parts[0], parts[1]}] = rank;
  }
  for (const std::string &s : added_contents)
    if (t->special_set.insert(s).second) t->special.push_back(s);
  if (unk && unk->k == JVal::Str) {
    auto it = t->vocab.find(unk->s);
    if (it != t->vocab.end()) t->unk_id = it->second;
  }
  const std::vector<uint32_t> &enc = byte_encoder();
  t->byte_str.resize(256);
  for (int b = 0; b < 256; ++b) {
    put_utf8(enc[b], &t->byte_str[b]);
    t->decoder[enc[b]] = (uint8_t)b;
  }
  *out = t;
  return IFX_OK;
}

// BpeTokenizer::bpe (mod.rs:114-140): merge the adjacent pair of lowest
// rank, the leftmost of equal ranks, until no adjacent pair has a rank.
std::vector<std::string> bpe(const ifx_tokenizer &t, std::vector<std::string> pieces) {
  const size_t n = pieces.size();
  if (n < 2) return pieces;
  struct Node {
    std::string s;
    int prev, next;
    uint32_t ver;
    bool alive;
  };
  std::vector<Node> nodes(n);
  for (size_t i = 0; i < n; ++i)
    nodes[i] = Node{std::move(pieces[i]), (int)i - 1, i + 1 < n ? (int)i + 1 : -1, 0, true};
  // (rank, left node = its start position among the original pieces)
  struct Cand {
    size_t rank;
    int left, right;
    uint32_t lver, rver;
    bool operator>(const Cand &o) const {
      return rank != o.rank ? rank > o.rank : left > o.left;
    }
  };
  std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
  auto push = [&](int l, int r) {
    if (l < 0 || r < 0) return;
    auto it = t.merges.find({nodes[l].s, nodes[r].s});
    if (it != t.merges.end()) heap.push(Cand{it->second, l, r, nodes[l].ver, nodes[r].ver});
  };
  for (size_t i = 0; i + 1 < n; ++i) push((int)i, (int)i + 1);
  while (!heap.empty()) {
    const Cand c = heap.top();
    heap.pop();
    Node &L = nodes[c.left], &R = nodes[c.right];
    if (!L.alive || !R.alive || L.next != c.right || L.ver != c.lver || R.ver != c.rver) continue;
    L.s += R.s;
    R.alive = false;
    L.next = R.next;
    if (R.next >= 0) nodes[R.next].prev = c.left;
    ++L.ver;
    push(L.prev, c.left);
    push(c.left, L.next);
  }
  std::vector<std::string> outp;
  for (int i = 0; i >= 0; i = nodes[i].next) outp.push_back(std::move(nodes[i].s));
  return outp;
}

// BpeTokenizer::encode_piece (mod.rs:142-155).
void encode_piece(const ifx_tokenizer &t, const std::string &text, std::vector<uint32_t> *ids) {
  std::vector<std::string> initial;
  initial.reserve(text.size());
  for (unsigned char b : text) initial.push_back(t.byte_str[b]);
  for (const std::string &s : bpe(t, std::move(initial))) {
    auto it = t.vocab.find(s);
    ids->push_back(it != t.vocab.end() ? it->second : t.unk_id);
  }
}

// Tokenizer::encode (mod.rs:194-204) with split_special (mod.rs:157-191).
void encode(const ifx_tokenizer &t, const std::string &text, std::vector<uint32_t> *ids) {
  if (t.special.empty()) {
    encode_piece(t, text, ids);
    return;
  }
  auto special_id = [&](const std::string &s) {
    auto it = t.vocab.find(s);
    ids->push_back(it != t.vocab.end() ? it->second : t.unk_id);
  };
  size_t at = 0;
  while (at < text.size()) {
    size_t best = std::string::npos;
    const std::string *tok = nullptr;
    for (const std::string &s : t.special) {
      if (s.empty()) continue;
      const size_t p = text.find(s, at);
      if (p == std::string::npos) continue;
      if (p < best || (p == best && s.size() > tok->size())) {
        best = p;
        tok = &s;
      }
    }
    if (!tok) {
      encode_piece(t, text.substr(at), ids);
      break;
    }
    if (best > at) encode_piece(t, text.substr(at, best - at), ids);
    special_id(*tok);
    at = best + tok->size();
  }
}

// Tokenizer::decode (mod.rs:206-225), then String::from_utf8_lossy.
std::string decode(const ifx_tokenizer &t, const uint32_t *ids, size_t n) {
  std::string bytes;
  for (size_t i = 0; i < n; ++i) {
    auto it = t.id_to_token.find(ids[i]);
    if (it == t.id_to_token.end()) continue;
    for (uint32_t c : code_points(it->second)) {
      auto d = t.decoder.find(c);
      if (d != t.decoder.end()) bytes.push_back((char)d->second);
      else put_utf8(c, &bytes);
    }
  }
  std::string out;
  out.reserve(bytes.size());
  const uint8_t *b = reinterpret_cast<const uint8_t *>(bytes.data());
  size_t i = 0;
  while (i < bytes.size()) {
    size_t bad = 0;
    const size_t w = utf8_seq(b, bytes.size(), i, &bad);
    if (w) {
      out.append(bytes, i, w);
      i += w;
    } else {
      put_utf8(0xFFFD, &out);
      i += bad;
    }
  }
  return out;
}

}  // namespace

}  // namespace ifx

using namespace ifx;

extern "C" {

ifx_status ifx_tokenizer_load_json(const char *json, size_t len, ifx_tokenizer **out) {
  if (!out || (!json && len)) return fail(IFX_ERR_INVALID_ARGUMENT, "ifx_tokenizer_load_json: null argument");
  *out = nullptr;
  if (!utf8_valid(reinterpret_cast<const uint8_t *>(json), len))
    return fail(IFX_ERR_INVALID_UTF8, "ifx_tokenizer_load_json: text is not UTF-8");
  try {
    return tokenizer_from_json(json, len, out);
  } catch (const std::bad_alloc &) {
    return fail(IFX_ERR_OUT_OF_MEMORY, "ifx_tokenizer_load_json: out of host memory");
  }
}

ifx_status ifx_tokenizer_load(const char *path, ifx_tokenizer **out) {
  if (!path || !out) return fail(IFX_ERR_INVALID_ARGUMENT, "ifx_tokenizer_load: null argument");
  *out = nullptr;
  std::ifstream f(path, std::ios::binary);
  if (!f) return fail(IFX_ERR_IO, std::string("io error: cannot open ") + path);
  std::string text((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  if (f.bad()) return fail(IFX_ERR_IO, std::string("io error: cannot read ") + path);
  // fs::read_to_string reports bytes that are not UTF-8 as an io error
  if (!utf8_valid(reinterpret_cast<const uint8_t *>(text.data()), text.size()))
    return fail(IFX_ERR_IO, "io error: stream did not contain valid UTF-8");
  try {
    return tokenizer_from_json(text.data(), text.size(), out);
  } catch (const std::bad_alloc &) {
    return fail(IFX_ERR_OUT_OF_MEMORY, "ifx_tokenizer_load: out of host memory");
  }
}

void ifx_tokenizer_free(ifx_tokenizer *t) { delete t; }

ifx_status ifx_tokenizer_encode(const ifx_tokenizer *t, const char *text, size_t len, uint32_t *ids,
                                size_t cap, size_t *n_ids) {
  if (!t || !n_ids || (!text && len) || (!ids && cap))
    return fail(IFX_ERR_INVALID_ARGUMENT, "ifx_tokenizer_encode: null argument");
  *n_ids = 0;
  if (!utf8_valid(reinterpret_cast<const uint8_t *>(text), len))
    return fail(IFX_ERR_INVALID_UTF8, "ifx_tokenizer_encode: text is not UTF-8");
  std::vector<uint32_t> v;
  try {
    encode(*t, std::string(text ? text : "", len), &v);
  } catch (const std::bad_alloc &) {
    return fail(IFX_ERR_OUT_OF_MEMORY, "ifx_tokenizer_encode: out of host memory");
  }
  *n_ids = v.size();
  if (v.size() > cap)
    return fail(IFX_ERR_SHAPE, "ifx_tokenizer_encode: " + std::to_string(v.size()) +
                                   " ids do not fit a buffer of " + std::to_string(cap));
  if (!v.empty()) memcpy(ids, v.data(), v.size() * sizeof(uint32_t));
  return IFX_OK;
}

ifx_status ifx_tokenizer_decode(const ifx_tokenizer *t, const uint32_t *ids, size_t n, char *text,
                                size_t cap, size_t *len) {
  if (!t || !len || (!ids && n) || (!text && cap))
    return fail(IFX_ERR_INVALID_ARGUMENT, "ifx_tokenizer_decode: null argument");
  *len = 0;
  std::string s;
  try {
    s = decode(*t, ids, n);
  } catch (const std::bad_alloc &) {
    return fail(IFX_ERR_OUT_OF_MEMORY, "ifx_tokenizer_decode: out of host memory");
  }
  *len = s.size();
  if (s.size() > cap)
    return fail(IFX_ERR_SHAPE, "ifx_tokenizer_decode: " + std::to_string(s.size()) +
                                   " bytes do not fit a buffer of " + std::to_string(cap));
  if (!s.empty()) memcpy(text, s.data(), s.size());
  return IFX_OK;
}

ifx_status ifx_tokenizer_vocab_size(const ifx_tokenizer *t, size_t *n) {
  if (!t || !n) return fail(IFX_ERR_INVALID_ARGUMENT, "ifx_tokenizer_vocab_size: null argument");
  *n = t->vocab.size();
  return IFX_OK;
}

}  // extern "C"
