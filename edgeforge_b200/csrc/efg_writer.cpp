// efg_writer.cpp - the .efq writer on the GPU: config.json + model.safetensors (BF16, F16 or
// F32 tensors) -> .efq, byte-identical to the reference's ef::quantize_model
// (src/quantizer.cpp:151-290) for the same policy.
//
// Per tensor, in forward-pass order: Q4_0 / Q8_0 targets are widened to FP32, quantized and
// measured on the device (launch_dequantize, launch_quantize, launch_quant_stats: all
// bit-exact with the reference's quantize_row and its double error sums); F32 / F16 / BF16
// targets are converted on the host (a plain copy for the usual BF16 embedding and the F32
// norms). The header is laid out as the reference lays it out: a placeholder with zeroed
// statistics sizes the data region, the tensors follow at 64-byte aligned offsets, and the
// header is rewritten with the measured rel_rmse / max_abs_err in fixed-width fields.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/efg.h"
#include "efg_efq.h"
#include "efg_host.h"
#include "efg_quant.cuh"

namespace efg::writer {
namespace {

using efq::FormatError;

// ---------------------------------------------------------------- host conversions

uint32_t bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}
float from_bits(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// Exact binary16 -> binary32 (include/ef/fp16.h:44-66).
float half_to_float(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  if (e == 0) return from_bits(bits(static_cast<float>(m) * 5.9604644775390625e-08f) | sign);
  if (e == 31) return from_bits(sign | 0x7F800000u | (m << 13));
  return from_bits(sign | ((e + 112u) << 23) | (m << 13));
}

// binary32 -> binary16, nearest-even, |x| >= 65520 -> inf, NaN quieted (include/ef/fp16.h:69-92).
uint16_t float_to_half(float f) {
  const uint32_t u = bits(f), a = u & 0x7FFFFFFFu;
  const uint16_t sign = static_cast<uint16_t>((u >> 16) & 0x8000u);
  if (a > 0x7F800000u) return static_cast<uint16_t>(sign | 0x7E00u | ((a >> 13) & 0x3FFu));
  if (a >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);
  if (a < 0x38800000u) return static_cast<uint16_t>(sign | static_cast<uint16_t>(std::nearbyint(from_bits(a) * 16777216.0f)));
  const uint32_t x = a - 0x38000000u, dropped = x & 0x1FFFu;
  uint32_t r = x >> 13;
  if (dropped > 0x1000u || (dropped == 0x1000u && (r & 1u))) ++r;
  return static_cast<uint16_t>(sign | r);
}

// binary32 -> bfloat16, nearest-even, NaN quieted (include/ef/fp16.h:94-104).
uint16_t float_to_bf16(float f) {
  uint32_t u = bits(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((u >> 16) | 0x0040u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

// ---------------------------------------------------------------- safetensors (read-only map)

struct SrcTensor {
  int dtype = 0;  // 0 F32, 1 F16, 2 BF16
  std::vector<uint64_t> shape;
  const uint8_t* data = nullptr;
  uint64_t bytes = 0;
  uint64_t numel() const {
    uint64_t n = 1;
    for (uint64_t d : shape) n *= d;
    return n;
  }
};

struct Mapped {
  void* p = MAP_FAILED;
  size_t n = 0;
  ~Mapped() {
    if (p != MAP_FAILED && n) munmap(p, n);
  }
};

struct Safetensors {
  Mapped map;
  uint64_t size = 0;
  std::map<std::string, SrcTensor> tensors;
  std::vector<std::string> order;
};

std::string shape_str(const std::vector<uint64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

void open_safetensors(const std::string& path, Safetensors& st) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw FormatError("cannot open '" + path + "': " + std::strerror(errno));
  struct stat sb {};
  if (fstat(fd, &sb) != 0) {
    ::close(fd);
    throw FormatError("cannot stat '" + path + "'");
  }
  st.size = static_cast<uint64_t>(sb.st_size);
  if (st.size) {
    st.map.p = mmap(nullptr, st.size, PROT_READ, MAP_PRIVATE, fd, 0);
    st.map.n = st.size;
  }
  ::close(fd);
  if (st.size && st.map.p == MAP_FAILED) throw FormatError("cannot map '" + path + "'");
  const auto* f = static_cast<const uint8_t*>(st.map.p);
  if (st.size < 8) throw FormatError("'" + path + "' is too small to be a safetensors file");
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | f[i];
  if (hlen > st.size - 8) throw FormatError("'" + path + "': header length runs past the end of the file");
  const efq::Json h = efq::parse_json(std::string_view(reinterpret_cast<const char*>(f + 8), hlen));
  if (h.t != efq::Json::T::Obj) throw FormatError("'" + path + "': header is not a JSON object");
  const uint64_t base = 8 + hlen;
  for (size_t i = 0; i < h.keys.size(); ++i) {
    const std::string& name = h.keys[i];
    if (name == "__metadata__") continue;
    const efq::Json& e = h.items[i];
    SrcTensor t;
    const std::string dt = e.at("dtype").str();
    t.dtype = dt == "F32" ? 0 : dt == "F16" ? 1 : dt == "BF16" ? 2 : -1;
    for (const efq::Json& d : e.at("shape").items) t.shape.push_back(d.u64());
    const efq::Json& off = e.at("data_offsets");
    if (off.items.size() != 2) throw FormatError("tensor '" + name + "': bad data_offsets");
    const uint64_t b = off.items[0].u64(), en = off.items[1].u64();
    if (en < b || en > st.size - base) throw FormatError("tensor '" + name + "': data runs past the end of the file");
    t.data = f + base + b;
    t.bytes = en - b;
    if (t.dtype >= 0 && t.bytes != t.numel() * (t.dtype == 0 ? 4 : 2))
      throw FormatError("tensor '" + name + "': byte size does not match dtype and shape");
    st.tensors.emplace(name, std::move(t));
    st.order.push_back(name);
  }
}

// ---------------------------------------------------------------- policies

struct NamedPolicy {
  const char* name;
  std::vector<std::pair<std::string, int>> overrides;
  int64_t hidden, intermediate, layers, heads, kv_heads, vocab;  // all zero: any model
};

// The reference's version-controlled policies (src/quantizer.cpp:64-90): "uniform" and the
// TinyLlama-1.1B-Chat recipe that keeps six attention matrices in Q8_0, guarded by the
// architecture it was measured on.
const std::vector<NamedPolicy>& named_policies() {
  static const std::vector<NamedPolicy> v = {
      {"uniform", {}, 0, 0, 0, 0, 0, 0},
      {"tinyllama-1.1b-chat-v1.0",
       {{"model.layers.0.self_attn.k_proj.weight", 3},
        {"model.layers.0.self_attn.v_proj.weight", 3},
        {"model.layers.1.self_attn.v_proj.weight", 3},
        {"model.layers.2.self_attn.v_proj.weight", 3},
        {"model.layers.17.self_attn.v_proj.weight", 3},
        {"model.layers.18.self_attn.v_proj.weight", 3}},
       2048, 5632, 22, 32, 4, 32000},
  };
  return v;
}

bool policy_matches(const NamedPolicy& p, const efq::Config& c) {
  if (p.hidden == 0) return true;
  return c.hidden == p.hidden && c.intermediate == p.intermediate && c.layers == p.layers && c.heads == p.heads &&
         c.kv_heads == p.kv_heads && c.vocab == p.vocab && !c.tie_embeddings;
}

std::string lower(std::string s) {
  for (char& ch : s) ch = static_cast<char>(std::tolower(static_cast<unsigned char>(ch)));
  return s;
}

// ef::parse_overrides (src/qfile.cpp:94-115): "TENSOR=TYPE,..." or "none".
std::vector<std::pair<std::string, int>> parse_overrides(std::string_view spec) {
  std::vector<std::pair<std::string, int>> out;
  if (lower(std::string(spec)) == "none") return out;
  size_t pos = 0;
  while (pos <= spec.size()) {
    const size_t comma = std::min(spec.find(',', pos), spec.size());
    const std::string_view item = spec.substr(pos, comma - pos);
    const size_t eq = item.rfind('=');
    if (item.empty() || eq == std::string_view::npos || eq == 0 || eq + 1 == item.size())
      throw std::invalid_argument("override '" + std::string(item) +
                                  "' must look like TENSOR=TYPE (e.g. model.layers.0.self_attn.v_proj.weight=q8_0), "
                                  "or be 'none'");
    const int t = efq::type_from_string(lower(std::string(item.substr(eq + 1))));
    if (t < 0)
      throw std::invalid_argument("override '" + std::string(item) + "': type must be one of q4_0, q8_0, bf16, f16, f32");
    out.emplace_back(std::string(item.substr(0, eq)), t);
    pos = comma + 1;
  }
  return out;
}

std::string json_escape(std::string_view s) {
  static const char* hex = "0123456789abcdef";
  std::string out;
  for (const char ch : s) {
    const auto c = static_cast<unsigned char>(ch);
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c < 0x20) {
          out += "\\u00";
          out += hex[c >> 4];
          out += hex[c & 0xF];
        } else {
          out += ch;
        }
    }
  }
  return out;
}

// Twelve characters for any statistic, so the final header has the placeholder's length.
std::string fixed_num(double v) {
  if (!(v >= 0.0) || !std::isfinite(v)) v = 0.0;
  if (v >= 9.999999e99) v = 9.999999e99;
  if (v != 0.0 && v < 1e-99) v = 0.0;
  char b[64];
  std::snprintf(b, sizeof b, "%.6e", v);
  return b;
}

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

struct OutTensor {
  std::string name, rule;
  int type = 0;
  std::vector<uint64_t> shape;
  uint64_t bytes = 0, offset = 0;
  double rel_rmse = 0.0, max_abs_err = 0.0;
  uint64_t rows() const { return shape.size() == 2 ? shape[0] : 1; }
  uint64_t cols() const { return shape.empty() ? 1 : shape.back(); }
};

struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  int ensure(size_t n) {
    if (n <= cap) return EFG_OK;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    EFG_TRY_CUDA(cudaMalloc(&p, n ? n : 16), "writer buffer");
    cap = n;
    return EFG_OK;
  }
};

struct Stream {
  cudaStream_t s = nullptr;
  ~Stream() {
    if (s) cudaStreamDestroy(s);
  }
};

// Quantizes one tensor into `out` (q.bytes) and fills its statistics.
int quantize_tensor(const SrcTensor& src, OutTensor& q, std::vector<uint8_t>& out, DevBuf& draw, DevBuf& df32,
                    DevBuf& dq, DevBuf& dstats, cudaStream_t s) {
  const uint64_t rows = q.rows(), cols = q.cols(), n = rows * cols;
  out.assign(q.bytes, 0);
  if (q.type == 3 || q.type == 4) {
    if (int st = draw.ensure(src.bytes)) return st;
    if (int st = df32.ensure(n * sizeof(float))) return st;
    if (int st = dq.ensure(q.bytes)) return st;
    if (int st = dstats.ensure(3 * rows * sizeof(double))) return st;
    EFG_TRY_CUDA(cudaMemcpyAsync(draw.p, src.data, src.bytes, cudaMemcpyHostToDevice, s), "source upload");
    const float* f32 = static_cast<const float*>(draw.p);
    if (src.dtype != 0) {
      if (int st = launch_dequantize(src.dtype, draw.p, n, static_cast<float*>(df32.p), s)) return st;
      f32 = static_cast<const float*>(df32.p);
    }
    if (int st = launch_quantize(q.type, f32, n, dq.p, true, s)) return st;
    auto* sse = static_cast<double*>(dstats.p);
    if (int st = launch_quant_stats(q.type, f32, static_cast<const uint8_t*>(dq.p), rows, cols, sse, sse + rows,
                                    sse + 2 * rows, s))
      return st;
    std::vector<double> stats(3 * rows);
    EFG_TRY_CUDA(cudaMemcpyAsync(out.data(), dq.p, q.bytes, cudaMemcpyDeviceToHost, s), "download");
    EFG_TRY_CUDA(cudaMemcpyAsync(stats.data(), dstats.p, stats.size() * sizeof(double), cudaMemcpyDeviceToHost, s),
                 "download");
    EFG_TRY_CUDA(cudaStreamSynchronize(s), "stream synchronize");
    double tsse = 0.0, tref = 0.0, tmax = 0.0;
    for (uint64_t r = 0; r < rows; ++r) {  // fixed row order, as the reference sums them
      tsse += stats[r];
      tref += stats[rows + r];
      tmax = std::max(tmax, stats[2 * rows + r]);
    }
    q.rel_rmse = tref > 0.0 ? std::sqrt(tsse / tref) : 0.0;
    q.max_abs_err = tmax;
    return EFG_OK;
  }
  // F32 / F16 / BF16 targets on the host.
  auto src_at = [&](uint64_t i) -> float {
    if (src.dtype == 0) {
      float f;
      std::memcpy(&f, src.data + 4 * i, 4);
      return f;
    }
    const uint16_t h = static_cast<uint16_t>(src.data[2 * i] | (src.data[2 * i + 1] << 8));
    return src.dtype == 1 ? half_to_float(h) : from_bits(static_cast<uint32_t>(h) << 16);
  };
  if (q.type == 2 && src.dtype == 2) {  // exact copy (src/quantizer.cpp:127-128)
    std::memcpy(out.data(), src.data, q.bytes);
    return EFG_OK;
  }
  double tsse = 0.0, tref = 0.0, tmax = 0.0;
  for (uint64_t r = 0; r < rows; ++r) {
    double sse = 0.0, ref = 0.0, mx = 0.0;
    for (uint64_t c = 0; c < cols; ++c) {
      const uint64_t i = r * cols + c;
      const float v = src_at(i);
      float back;
      if (q.type == 0) {
        std::memcpy(out.data() + 4 * i, &v, 4);
        back = v;
      } else if (q.type == 1) {
        const uint16_t h = float_to_half(v);
        out[2 * i] = static_cast<uint8_t>(h & 0xFF);
        out[2 * i + 1] = static_cast<uint8_t>(h >> 8);
        back = half_to_float(h);
      } else {
        const uint16_t h = float_to_bf16(v);
        out[2 * i] = static_cast<uint8_t>(h & 0xFF);
        out[2 * i + 1] = static_cast<uint8_t>(h >> 8);
        back = from_bits(static_cast<uint32_t>(h) << 16);
      }
      const double e = static_cast<double>(v) - static_cast<double>(back);
      sse += e * e;
      ref += static_cast<double>(v) * static_cast<double>(v);
      mx = std::max(mx, std::fabs(e));
    }
    tsse += sse;
    tref += ref;
    tmax = std::max(tmax, mx);
  }
  q.rel_rmse = tref > 0.0 ? std::sqrt(tsse / tref) : 0.0;
  q.max_abs_err = tmax;
  return EFG_OK;
}

std::string read_text(const std::string& p) {
  std::ifstream in(p, std::ios::binary);
  if (!in) throw FormatError("cannot open '" + p + "'");
  return std::string((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
}

int run(const char* model_dir, const char* out_file, const char* policy_arg, const char* overrides_arg,
        efg_quantize_report* rep) {
  const auto t0 = std::chrono::steady_clock::now();
  const std::string dir = model_dir;
  std::string config_text;
  efq::Config cfg;
  Safetensors st;
  try {
    config_text = read_text(dir + "/config.json");
    cfg = efq::parse_config(efq::parse_json(config_text));
    open_safetensors(dir + "/model.safetensors", st);
  } catch (const FormatError& e) {
    return fail(EFG_EFORMAT, "%s", e.what());
  }
  const auto expected = efq::expected_tensors(cfg);
  {  // check_checkpoint (src/model_config.cpp:179-224): the first problem found
    std::map<std::string, bool> wanted;
    for (const auto& e : expected) {
      wanted[e.first] = true;
      auto it = st.tensors.find(e.first);
      if (it == st.tensors.end())
        return fail(EFG_EFORMAT, "checkpoint does not match config.json: missing tensor '%s'", e.first.c_str());
      if (it->second.shape != e.second)
        return fail(EFG_EFORMAT, "checkpoint does not match config.json: tensor '%s' has shape %s, expected %s",
                    e.first.c_str(), shape_str(it->second.shape).c_str(), shape_str(e.second).c_str());
      if (it->second.dtype < 0)
        return fail(EFG_EFORMAT, "checkpoint does not match config.json: tensor '%s' has a non-float dtype",
                    e.first.c_str());
    }
    for (const auto& name : st.order) {
      if (wanted.count(name)) continue;
      const std::string suffix = "rotary_emb.inv_freq";
      const bool rope_buf = name.size() >= suffix.size() && name.compare(name.size() - suffix.size(), suffix.size(), suffix) == 0;
      if (!rope_buf && !(cfg.tie_embeddings && name == "lm_head.weight"))
        return fail(EFG_EFORMAT, "checkpoint does not match config.json: unexpected tensor '%s'", name.c_str());
    }
  }
  // the policy: explicit overrides, else a named policy (select_policy, src/quantizer.cpp:92-115)
  efq::Policy pol;  // layers Q4_0, lm_head Q8_0, embed BF16
  try {
    if (overrides_arg && *overrides_arg) {
      pol.overrides = parse_overrides(overrides_arg);
      pol.name = pol.overrides.empty() ? "uniform" : "custom";
    } else {
      const std::string p = policy_arg && *policy_arg ? policy_arg : "auto";
      const NamedPolicy* chosen = nullptr;
      if (p == "auto") {
        for (const auto& np : named_policies())
          if (np.hidden != 0 && policy_matches(np, cfg)) chosen = &np;
        if (!chosen) chosen = &named_policies()[0];
      } else {
        for (const auto& np : named_policies())
          if (p == np.name) chosen = &np;
        if (!chosen) throw std::invalid_argument("unknown policy '" + p + "' (auto, uniform, tinyllama-1.1b-chat-v1.0)");
        if (!policy_matches(*chosen, cfg))
          throw std::invalid_argument("policy '" + p +
                                      "' was measured on another architecture; this model's config differs (use "
                                      "--policy uniform)");
      }
      pol.overrides = chosen->overrides;
      pol.name = chosen->name;
    }
  } catch (const std::invalid_argument& e) {
    return fail(EFG_EINVAL, "%s", e.what());
  }
  for (const auto& o : pol.overrides) {  // check_overrides (src/qfile.cpp:79-92)
    if (o.first.empty()) return fail(EFG_EINVAL, "override with an empty tensor pattern");
    size_t hits = 0;
    for (const auto& e : expected) {
      if (!efq::glob_match(o.first, e.first)) continue;
      if (e.first.find("norm") != std::string::npos)
        return fail(EFG_EINVAL, "override '%s' matches norm tensor '%s' (norms are always F32)", o.first.c_str(),
                    e.first.c_str());
      ++hits;
    }
    if (hits == 0) return fail(EFG_EINVAL, "override '%s' matches no tensor of this model", o.first.c_str());
  }

  // layout (forward-pass order)
  std::vector<OutTensor> ts;
  uint64_t bpt = 0, src_bytes = 0;
  int64_t extra = 0;
  try {
    for (const auto& e : expected) {
      OutTensor q;
      q.name = e.first;
      q.shape = e.second;
      const auto ch = efq::policy_choice(pol, q.name, q.cols());
      q.type = ch.first;
      q.rule = ch.second;
      q.bytes = efq::row_bytes(q.type, q.cols()) * q.rows();
      if (q.rule == "override") {
        const auto base = efq::policy_choice(pol, q.name, q.cols(), false);
        extra += static_cast<int64_t>(q.bytes) - static_cast<int64_t>(efq::row_bytes(base.first, q.cols()) * q.rows());
      }
      src_bytes += st.tensors.at(q.name).bytes;
      if (q.name != "model.embed_tokens.weight" || cfg.tie_embeddings) bpt += q.bytes;
      ts.push_back(std::move(q));
    }
  } catch (const FormatError& e) {
    return fail(EFG_EFORMAT, "%s", e.what());
  }
  std::string trimmed = config_text;
  while (!trimmed.empty() && std::isspace(static_cast<unsigned char>(trimmed.back()))) trimmed.pop_back();
  std::string ov = "[";
  for (const auto& o : pol.overrides)
    ov += (ov.size() > 1 ? "," : "") + std::string("{\"pattern\":\"") + json_escape(o.first) + "\",\"type\":\"" +
          efq::type_name(o.second) + "\"}";
  ov += "]";
  auto header = [&](uint64_t data_start, bool stats) {
    std::string h = std::string("{\"format\":\"edgeforge-quant\",\"version\":1,\n\"quant\":{\"layers\":\"") +
                    efq::type_name(pol.layers) + "\",\"lm_head\":\"" + efq::type_name(pol.lm_head) + "\",\"embed\":\"" +
                    efq::type_name(pol.embed) + "\",\"norms\":\"F32\",\"block\":32,\"scale\":\"mse-search\",\n\"policy\":\"" +
                    json_escape(pol.name) + "\",\"overrides\":" + ov +
                    "},\n\"source\":{\"file\":\"model.safetensors\",\"bytes\":" + std::to_string(st.size) +
                    "},\n\"config\":" + trimmed + ",\n\"tensors\":[\n";
    uint64_t off = data_start;
    for (size_t i = 0; i < ts.size(); ++i) {
      const OutTensor& q = ts[i];
      off = align_up(off, 64);
      h += "{\"name\":\"" + json_escape(q.name) + "\",\"type\":\"" + efq::type_name(q.type) + "\",\"rule\":\"" + q.rule +
           "\",\"shape\":" + shape_str(q.shape) + ",\"offset\":" + std::to_string(off) +
           ",\"bytes\":" + std::to_string(q.bytes) + ",\"rel_rmse\":" + fixed_num(stats ? q.rel_rmse : 0.0) +
           ",\"max_abs_err\":" + fixed_num(stats ? q.max_abs_err : 0.0) + "}" + (i + 1 < ts.size() ? ",\n" : "\n");
      off += q.bytes;
    }
    return h + "]}";
  };
  uint64_t data_start = 64;
  std::string hdr;
  for (int it = 0; it < 16; ++it) {
    hdr = header(data_start, false);
    const uint64_t need = align_up(16 + hdr.size(), 64);
    if (need <= data_start) break;
    data_start = need;
  }
  hdr.resize(data_start - 16, ' ');
  uint64_t off = data_start;
  for (auto& q : ts) {
    off = align_up(off, 64);
    q.offset = off;
    off += q.bytes;
  }
  const uint64_t file_bytes = off;

  FILE* f = std::fopen(out_file, "wb");
  if (!f) return fail(EFG_EINVAL, "cannot create '%s'", out_file);
  std::unique_ptr<FILE, int (*)(FILE*)> guard(f, std::fclose);
  uint8_t pre[16] = {'E', 'F', 'Q', '1', 1, 0, 0, 0};
  for (int i = 0; i < 8; ++i) pre[8 + i] = static_cast<uint8_t>(((data_start - 16) >> (8 * i)) & 0xFF);
  if (std::fwrite(pre, 1, 16, f) != 16 || std::fwrite(hdr.data(), 1, hdr.size(), f) != hdr.size())
    return fail(EFG_EINVAL, "write failed for '%s'", out_file);
  Stream stream;
  EFG_TRY_CUDA(cudaStreamCreateWithFlags(&stream.s, cudaStreamNonBlocking), "stream create");
  DevBuf draw, df32, dq, dstats;
  std::vector<uint8_t> buf;
  static const uint8_t zeros[64] = {};
  uint64_t pos = data_start;
  for (auto& q : ts) {
    if (q.offset - pos > 64) return fail(EFG_EINVAL, "internal: layout overrun at '%s'", q.name.c_str());
    if (q.offset > pos && std::fwrite(zeros, 1, q.offset - pos, f) != q.offset - pos)
      return fail(EFG_EINVAL, "write failed for '%s'", out_file);
    if (int s = quantize_tensor(st.tensors.at(q.name), q, buf, draw, df32, dq, dstats, stream.s)) return s;
    if (std::fwrite(buf.data(), 1, buf.size(), f) != buf.size())
      return fail(EFG_EINVAL, "write failed for '%s' (disk full?)", out_file);
    pos = q.offset + q.bytes;
  }
  std::string fin = header(data_start, true);
  fin.resize(data_start - 16, ' ');
  if (fin.size() != hdr.size()) return fail(EFG_EINVAL, "internal: header size changed");
  if (std::fseek(f, 16, SEEK_SET) != 0 || std::fwrite(fin.data(), 1, fin.size(), f) != fin.size())
    return fail(EFG_EINVAL, "write failed for '%s'", out_file);
  if (std::fclose(guard.release()) != 0) return fail(EFG_EINVAL, "could not finish writing '%s'", out_file);
  if (rep) {
    rep->file_bytes = file_bytes;
    rep->bytes_per_token = bpt;
    rep->source_tensor_bytes = src_bytes;
    rep->override_extra_bytes = extra;
    rep->n_tensors = static_cast<int32_t>(ts.size());
    rep->seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  }
  return EFG_OK;
}

}  // namespace
}  // namespace efg::writer

extern "C" int efg_quantize_model(const char* model_dir, const char* out_file, const char* policy,
                                  const char* overrides, efg_quantize_report* report) {
  if (!model_dir || !out_file) return efg::fail(EFG_EINVAL, "quantize_model: null path");
  try {
    return efg::writer::run(model_dir, out_file, policy, overrides, report);
  } catch (const efg::efq::FormatError& e) {
    return efg::fail(EFG_EFORMAT, "%s", e.what());
  } catch (const std::exception& e) {
    return efg::fail(EFG_EINVAL, "quantize_model: %s", e.what());
  }
}
