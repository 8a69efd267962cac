// efg_efq.cpp - .efq reader: a strict JSON parser and the reference's validation of the
// header and tensor table (src/qfile.cpp:125-223, src/model_config.cpp), with the same
// error messages, so a file the reference rejects is rejected here for the same reason.
#include "efg_efq.h"

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <numeric>
#include <unordered_map>

namespace efg::efq {

namespace {

[[noreturn]] void bad(const std::string& msg) { throw FormatError(msg); }

// ------------------------------------------------------------------ JSON
class Parser {
 public:
  explicit Parser(std::string_view t) : t_(t) {}
  Json document() {
    Json v = value(0);
    ws();
    if (p_ != t_.size()) err("trailing characters after the JSON value");
    return v;
  }

 private:
  std::string_view t_;
  size_t p_ = 0;

  [[noreturn]] void err(const char* what) {
    size_t line = 1, col = 1;
    for (size_t i = 0; i < p_ && i < t_.size(); ++i) {
      if (t_[i] == '\n') {
        ++line;
        col = 1;
      } else {
        ++col;
      }
    }
    char buf[160];
    std::snprintf(buf, sizeof buf, "%s at line %zu, column %zu", what, line, col);
    bad(buf);
  }
  void ws() {
    while (p_ < t_.size() && (t_[p_] == ' ' || t_[p_] == '\n' || t_[p_] == '\r' || t_[p_] == '\t')) ++p_;
  }
  bool lit(const char* s) {
    const size_t n = std::strlen(s);
    if (t_.substr(p_, n) == s) {
      p_ += n;
      return true;
    }
    return false;
  }
  Json value(int depth) {
    if (depth > 256) err("nesting too deep");
    ws();
    if (p_ >= t_.size()) err("unexpected end of input");
    const char c = t_[p_];
    Json v;
    if (c == '{') {
      v.t = Json::T::Obj;
      ++p_;
      ws();
      if (p_ < t_.size() && t_[p_] == '}') {
        ++p_;
        return v;
      }
      for (;;) {
        ws();
        if (p_ >= t_.size() || t_[p_] != '"') err("expected a string key");
        std::string k = string();
        for (const auto& e : v.keys)
          if (e == k) err("duplicate object key");
        ws();
        if (p_ >= t_.size() || t_[p_] != ':') err("expected ':'");
        ++p_;
        v.items.push_back(value(depth + 1));
        v.keys.push_back(std::move(k));
        ws();
        if (p_ < t_.size() && t_[p_] == ',') {
          ++p_;
          continue;
        }
        if (p_ < t_.size() && t_[p_] == '}') {
          ++p_;
          return v;
        }
        err("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.t = Json::T::Arr;
      ++p_;
      ws();
      if (p_ < t_.size() && t_[p_] == ']') {
        ++p_;
        return v;
      }
      for (;;) {
        v.items.push_back(value(depth + 1));
        ws();
        if (p_ < t_.size() && t_[p_] == ',') {
          ++p_;
          continue;
        }
        if (p_ < t_.size() && t_[p_] == ']') {
          ++p_;
          return v;
        }
        err("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.t = Json::T::Str;
      v.s = string();
      return v;
    }
    if (lit("true")) {
      v.t = Json::T::Bool;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.t = Json::T::Bool;
      return v;
    }
    if (lit("null")) return v;
    if (c == '-' || (c >= '0' && c <= '9')) return number();
    err("unexpected character");
  }
  std::string string() {
    ++p_;  // opening quote
    std::string out;
    while (p_ < t_.size()) {
      const char c = t_[p_++];
      if (c == '"') return out;
      if (static_cast<unsigned char>(c) < 0x20) err("control character in string");
      if (c != '\\') {
        out += c;
        continue;
      }
      if (p_ >= t_.size()) break;
      const char e = t_[p_++];
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          if (p_ + 4 > t_.size()) err("bad \\u escape");
          unsigned cp = 0;
          for (int i = 0; i < 4; ++i) {
            const char h = t_[p_++];
            cp <<= 4;
            if (h >= '0' && h <= '9') cp |= h - '0';
            else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
            else err("bad \\u escape");
          }
          if (cp < 0x80) {
            out += static_cast<char>(cp);
          } else if (cp < 0x800) {
            out += static_cast<char>(0xC0 | (cp >> 6));
            out += static_cast<char>(0x80 | (cp & 0x3F));
          } else {  // tensor names and policy labels are ASCII; other code points kept as UTF-8
            out += static_cast<char>(0xE0 | (cp >> 12));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
          }
          break;
        }
        default: err("bad escape");
      }
    }
    err("unterminated string");
  }
  Json number() {
    const size_t start = p_;
    if (t_[p_] == '-') ++p_;
    if (p_ >= t_.size() || !std::isdigit(static_cast<unsigned char>(t_[p_]))) err("bad number");
    if (t_[p_] == '0' && p_ + 1 < t_.size() && std::isdigit(static_cast<unsigned char>(t_[p_ + 1])))
      err("leading zero in number");
    while (p_ < t_.size() && std::isdigit(static_cast<unsigned char>(t_[p_]))) ++p_;
    bool integral = true;
    if (p_ < t_.size() && t_[p_] == '.') {
      integral = false;
      ++p_;
      if (p_ >= t_.size() || !std::isdigit(static_cast<unsigned char>(t_[p_]))) err("bad number");
      while (p_ < t_.size() && std::isdigit(static_cast<unsigned char>(t_[p_]))) ++p_;
    }
    if (p_ < t_.size() && (t_[p_] == 'e' || t_[p_] == 'E')) {
      integral = false;
      ++p_;
      if (p_ < t_.size() && (t_[p_] == '+' || t_[p_] == '-')) ++p_;
      if (p_ >= t_.size() || !std::isdigit(static_cast<unsigned char>(t_[p_]))) err("bad number");
      while (p_ < t_.size() && std::isdigit(static_cast<unsigned char>(t_[p_]))) ++p_;
    }
    Json v;
    v.t = Json::T::Num;
    v.s = std::string(t_.substr(start, p_ - start));
    v.d = std::strtod(v.s.c_str(), nullptr);
    if (integral) {
      errno = 0;
      const long long ll = std::strtoll(v.s.c_str(), nullptr, 10);
      if (errno == 0) {
        v.is_int = true;
        v.i = ll;
      }
    }
    return v;
  }
};

const char* json_type(Json::T t) {
  switch (t) {
    case Json::T::Null: return "null";
    case Json::T::Bool: return "bool";
    case Json::T::Num: return "number";
    case Json::T::Str: return "string";
    case Json::T::Arr: return "array";
    case Json::T::Obj: return "object";
  }
  return "?";
}

std::string shape_str(const std::vector<uint64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

uint64_t read_le(const uint8_t* p, int n) {
  uint64_t v = 0;
  for (int i = n - 1; i >= 0; --i) v = (v << 8) | p[i];
  return v;
}

// ------------------------------------------------------------------ config.json fields
const Json* member(const Json& root, const char* key) { return root.find(key); }

int64_t req_int(const Json& root, const char* key, int64_t lo, int64_t hi) {
  const Json* v = member(root, key);
  if (!v) bad(std::string("config.json: missing required field '") + key + "'");
  if (v->t != Json::T::Num || !v->is_int)
    bad(std::string("config.json: '") + key + "' must be an integer, got " +
        (v->t == Json::T::Num ? v->s : json_type(v->t)));
  if (v->i < lo || v->i > hi)
    bad(std::string("config.json: '") + key + "' = " + std::to_string(v->i) + " is outside [" + std::to_string(lo) +
        ", " + std::to_string(hi) + "]");
  return v->i;
}
int64_t opt_int(const Json& root, const char* key, int64_t def, int64_t lo, int64_t hi) {
  const Json* v = member(root, key);
  if (!v || v->t == Json::T::Null) return def;
  return req_int(root, key, lo, hi);
}
double req_num(const Json& root, const char* key) {
  const Json* v = member(root, key);
  if (!v) bad(std::string("config.json: missing required field '") + key + "'");
  if (v->t != Json::T::Num) bad(std::string("config.json: '") + key + "' must be a number, got " + json_type(v->t));
  return v->d;
}
double opt_num(const Json& root, const char* key, double def) {
  const Json* v = member(root, key);
  if (!v || v->t == Json::T::Null) return def;
  return req_num(root, key);
}
bool opt_bool(const Json& root, const char* key, bool def) {
  const Json* v = member(root, key);
  if (!v || v->t == Json::T::Null) return def;
  if (v->t != Json::T::Bool) bad(std::string("config.json: '") + key + "' must be true or false");
  return v->b;
}
std::string opt_str(const Json& root, const char* key, const std::string& def) {
  const Json* v = member(root, key);
  if (!v || v->t == Json::T::Null) return def;
  if (v->t != Json::T::Str) bad(std::string("config.json: '") + key + "' must be a string");
  return v->s;
}

bool is_norm(const std::string& name) { return name.find("norm") != std::string::npos; }

}  // namespace

// ------------------------------------------------------------------ Json accessors
const Json* Json::find(std::string_view key) const {
  if (t != T::Obj) return nullptr;
  for (size_t k = 0; k < keys.size(); ++k)
    if (keys[k] == key) return &items[k];
  return nullptr;
}
const Json& Json::at(std::string_view key) const {
  if (t != T::Obj) bad(std::string("expected a JSON object, got ") + json_type(t));
  if (const Json* v = find(key)) return *v;
  bad("missing key '" + std::string(key) + "'");
}
const std::string& Json::str() const {
  if (t != T::Str) bad(std::string("expected a string, got ") + json_type(t));
  return s;
}
uint64_t Json::u64() const {
  if (t != T::Num || !is_int || i < 0) bad("expected a non-negative integer, got " + (t == T::Num ? s : json_type(t)));
  return static_cast<uint64_t>(i);
}
double Json::num() const {
  if (t != T::Num) bad(std::string("expected a number, got ") + json_type(t));
  return d;
}

Json parse_json(std::string_view text) { return Parser(text).document(); }

// ------------------------------------------------------------------ types
const char* type_name(int t) {
  switch (t) {
    case 0: return "F32";
    case 1: return "F16";
    case 2: return "BF16";
    case 3: return "Q8_0";
    case 4: return "Q4_0";
    default: return "?";
  }
}

int type_from_string(std::string_view s) {
  for (int t = 0; t <= 4; ++t) {
    std::string lower = type_name(t);
    for (char& c : lower) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
    if (s == type_name(t) || s == lower) return t;
  }
  return -1;
}

uint64_t row_bytes(int t, uint64_t cols) {
  switch (t) {
    case 0: return cols * 4;
    case 1:
    case 2: return cols * 2;
    case 3:
    case 4:
      if (cols % 32 != 0)
        bad(std::string(type_name(t)) + " needs a row length divisible by 32, got " + std::to_string(cols));
      return cols / 32 * (t == 3 ? 34 : 18);
    default: bad("unknown type");
  }
}

// ------------------------------------------------------------------ config
Config parse_config(const Json& root) {
  if (root.t != Json::T::Obj) bad("config.json: top level must be a JSON object");
  const std::string model_type = opt_str(root, "model_type", "");
  if (model_type != "llama")
    bad("config.json: model_type '" + model_type + "' is not supported (EdgeForge targets 'llama')");
  const std::string act = opt_str(root, "hidden_act", "silu");
  if (act != "silu") bad("config.json: hidden_act '" + act + "' is not supported (expected 'silu')");
  constexpr int64_t kMaxDim = 1 << 20;
  Config c;
  c.hidden = req_int(root, "hidden_size", 1, kMaxDim);
  c.intermediate = req_int(root, "intermediate_size", 1, kMaxDim);
  c.layers = req_int(root, "num_hidden_layers", 1, 4096);
  c.heads = req_int(root, "num_attention_heads", 1, 4096);
  c.kv_heads = opt_int(root, "num_key_value_heads", c.heads, 1, 4096);
  c.vocab = req_int(root, "vocab_size", 1, 1 << 24);
  c.max_position = opt_int(root, "max_position_embeddings", 2048, 1, 1 << 24);
  c.rms_eps = req_num(root, "rms_norm_eps");
  c.rope_theta = opt_num(root, "rope_theta", 10000.0);
  c.tie_embeddings = opt_bool(root, "tie_word_embeddings", false);
  const bool attn_bias = opt_bool(root, "attention_bias", false), mlp_bias = opt_bool(root, "mlp_bias", false);
  if (c.hidden % c.heads != 0)
    bad("config.json: hidden_size " + std::to_string(c.hidden) + " is not divisible by num_attention_heads " +
        std::to_string(c.heads));
  c.head_dim = opt_int(root, "head_dim", c.hidden / c.heads, 1, kMaxDim);
  if (c.head_dim * c.heads != c.hidden) bad("config.json: head_dim * num_attention_heads must equal hidden_size");
  if (c.head_dim % 2 != 0) bad("config.json: head_dim must be even for RoPE");
  if (c.heads % c.kv_heads != 0)
    bad("config.json: num_attention_heads " + std::to_string(c.heads) + " is not divisible by num_key_value_heads " +
        std::to_string(c.kv_heads));
  if (!(c.rms_eps > 0.0) || !std::isfinite(c.rms_eps)) bad("config.json: rms_norm_eps must be a positive finite number");
  if (!(c.rope_theta > 0.0) || !std::isfinite(c.rope_theta))
    bad("config.json: rope_theta must be a positive finite number");
  if (const Json* rs = member(root, "rope_scaling"); rs && rs->t != Json::T::Null)
    bad("config.json: rope_scaling is set; scaled RoPE is not supported yet");
  if (attn_bias) bad("config.json: attention_bias=true is not supported");
  if (mlp_bias) bad("config.json: mlp_bias=true is not supported");
  return c;
}

std::vector<std::pair<std::string, std::vector<uint64_t>>> expected_tensors(const Config& c) {
  const auto D = static_cast<uint64_t>(c.hidden), F = static_cast<uint64_t>(c.intermediate),
             V = static_cast<uint64_t>(c.vocab), KV = static_cast<uint64_t>(c.kv_dim());
  std::vector<std::pair<std::string, std::vector<uint64_t>>> out;
  out.push_back({"model.embed_tokens.weight", {V, D}});
  for (int64_t l = 0; l < c.layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    out.push_back({p + "self_attn.q_proj.weight", {D, D}});
    out.push_back({p + "self_attn.k_proj.weight", {KV, D}});
    out.push_back({p + "self_attn.v_proj.weight", {KV, D}});
    out.push_back({p + "self_attn.o_proj.weight", {D, D}});
    out.push_back({p + "mlp.gate_proj.weight", {F, D}});
    out.push_back({p + "mlp.up_proj.weight", {F, D}});
    out.push_back({p + "mlp.down_proj.weight", {D, F}});
    out.push_back({p + "input_layernorm.weight", {D}});
    out.push_back({p + "post_attention_layernorm.weight", {D}});
  }
  out.push_back({"model.norm.weight", {D}});
  if (!c.tie_embeddings) out.push_back({"lm_head.weight", {V, D}});
  return out;
}

// ------------------------------------------------------------------ policy
bool glob_match(std::string_view p, std::string_view s) {
  size_t pi = 0, si = 0, star = std::string_view::npos, mark = 0;
  while (si < s.size()) {
    if (pi < p.size() && p[pi] == '*') {
      star = pi++;
      mark = si;
    } else if (pi < p.size() && p[pi] == s[si]) {
      ++pi;
      ++si;
    } else if (star != std::string_view::npos) {
      pi = star + 1;
      si = ++mark;
    } else {
      return false;
    }
  }
  while (pi < p.size() && p[pi] == '*') ++pi;
  return pi == p.size();
}

std::pair<int, std::string> policy_choice(const Policy& p, const std::string& name, uint64_t cols,
                                          bool use_overrides) {
  if (is_norm(name)) return {0, "norm"};
  std::pair<int, std::string> c{p.layers, "layers"};
  if (name == "model.embed_tokens.weight") c = {p.embed, "embed"};
  if (name == "lm_head.weight") c = {p.lm_head, "lm_head"};
  if (use_overrides)
    for (const auto& o : p.overrides)
      if (glob_match(o.first, name)) c = {o.second, "override"};
  if ((c.first == 3 || c.first == 4) && cols % 32 != 0) c = {2, "fallback-bf16"};
  return c;
}

// ------------------------------------------------------------------ the file
const Tensor* Layout::find(std::string_view name) const {
  for (const auto& t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}
const Tensor& Layout::at(std::string_view name) const {
  if (const Tensor* t = find(name)) return *t;
  bad("tensor '" + std::string(name) + "' not found");
}

Layout parse(const uint8_t* file, uint64_t size) {
  if (size < 16) bad("file too small to be an .efq model (" + std::to_string(size) + " bytes)");
  if (std::memcmp(file, "EFQ1", 4) != 0) bad("not an EdgeForge .efq file (bad magic)");
  const uint64_t version = read_le(file + 4, 4);
  if (version != 1) bad("unsupported .efq version " + std::to_string(version) + " (this build reads 1)");
  Layout L;
  L.header_len = read_le(file + 8, 8);
  if (L.header_len == 0 || L.header_len > 100000000ull || L.header_len > size - 16)
    bad("invalid .efq header length " + std::to_string(L.header_len));
  Json h;
  try {
    h = parse_json(std::string_view(reinterpret_cast<const char*>(file + 16), L.header_len));
  } catch (const FormatError& e) {
    bad(std::string("invalid .efq header: ") + e.what());
  }
  if (h.at("format").str() != "edgeforge-quant") bad(".efq header: wrong \"format\"");
  L.cfg = parse_config(h.at("config"));
  L.data_start = 16 + L.header_len;
  const Json& tl = h.at("tensors");
  if (tl.t != Json::T::Arr) bad(".efq header: \"tensors\" must be an array");
  for (const Json& e : tl.items) {
    Tensor t;
    t.name = e.at("name").str();
    t.type = type_from_string(e.at("type").str());
    if (t.type < 0) bad("tensor '" + t.name + "': unknown type " + e.at("type").str());
    if (const Json* r = e.find("rule")) t.rule = r->str();
    for (const Json& d : e.at("shape").items) t.shape.push_back(d.u64());
    if (t.shape.empty() || t.shape.size() > 2) bad("tensor '" + t.name + "': shape must be 1-D or 2-D");
    t.offset = e.at("offset").u64();
    t.bytes = e.at("bytes").u64();
    const uint64_t row = row_bytes(t.type, t.cols());
    if (t.rows() != 0 && row > std::numeric_limits<uint64_t>::max() / t.rows())
      bad("tensor '" + t.name + "': size overflows");
    if (row * t.rows() != t.bytes)
      bad("tensor '" + t.name + "': " + type_name(t.type) + " " + shape_str(t.shape) + " needs " +
          std::to_string(row * t.rows()) + " bytes, header says " + std::to_string(t.bytes));
    if (t.offset % 64 != 0) bad("tensor '" + t.name + "': offset is not 64-byte aligned");
    if (t.offset < L.data_start) bad("tensor '" + t.name + "': data overlaps the header");
    if (t.offset > size || t.bytes > size - t.offset)
      bad("tensor '" + t.name + "': data runs past the end of the file (truncated?)");
    L.tensors.push_back(std::move(t));
  }
  std::vector<size_t> order(L.tensors.size());
  std::iota(order.begin(), order.end(), size_t{0});
  std::sort(order.begin(), order.end(), [&](size_t a, size_t b) { return L.tensors[a].offset < L.tensors[b].offset; });
  for (size_t i = 1; i < order.size(); ++i) {
    const Tensor& p = L.tensors[order[i - 1]];
    const Tensor& c = L.tensors[order[i]];
    if (c.offset < p.offset + p.bytes) bad("tensors '" + p.name + "' and '" + c.name + "' overlap");
  }
  std::unordered_map<std::string, const Tensor*> by_name;
  for (const auto& t : L.tensors)
    if (!by_name.emplace(t.name, &t).second) bad("duplicate tensor '" + t.name + "'");
  const auto expected = expected_tensors(L.cfg);
  for (const auto& e : expected) {
    const auto it = by_name.find(e.first);
    if (it == by_name.end()) bad("missing tensor '" + e.first + "'");
    if (it->second->shape != e.second)
      bad("tensor '" + e.first + "' has shape " + shape_str(it->second->shape) + ", config needs " +
          shape_str(e.second));
  }
  if (by_name.size() != expected.size()) bad(".efq file has tensors the config does not use");

  const Json& qs = h.at("quant");
  const Json* ov = qs.find("overrides");
  if (!ov)
    bad(".efq header has no \"overrides\" table: written by an older pre-release build, re-run edgeforge quantize");
  auto type_field = [&](const Json& v, const char* what) {
    const int t = type_from_string(v.str());
    if (t < 0) bad(std::string(".efq header: unknown ") + what + " type " + v.str());
    return t;
  };
  L.policy.layers = type_field(qs.at("layers"), "layers");
  L.policy.lm_head = type_field(qs.at("lm_head"), "lm_head");
  L.policy.embed = type_field(qs.at("embed"), "embed");
  if (qs.at("norms").str() != "F32") bad(".efq header: norms must be F32");
  if (const Json* n = qs.find("policy")) L.policy.name = n->str();
  for (const Json& o : ov->items) L.policy.overrides.push_back({o.at("pattern").str(), type_field(o.at("type"), "override")});
  for (const auto& o : L.policy.overrides) {  // src/qfile.cpp:79-92
    if (o.first.empty()) bad("override with an empty tensor pattern");
    size_t hits = 0;
    for (const auto& e : expected) {
      if (!glob_match(o.first, e.first)) continue;
      if (is_norm(e.first))
        bad("override '" + o.first + "' matches norm tensor '" + e.first + "' (norms are always F32)");
      ++hits;
    }
    if (hits == 0) bad("override '" + o.first + "' matches no tensor of this model");
  }
  for (const auto& t : L.tensors) {
    const auto c = policy_choice(L.policy, t.name, t.cols());
    if (t.type != c.first || t.rule != c.second)
      bad("tensor '" + t.name + "' is stored as " + type_name(t.type) + " (rule \"" + t.rule +
          "\") but the file's quantization policy gives " + type_name(c.first) + " (rule \"" + c.second + "\")");
  }
  return L;
}

}  // namespace efg::efq
