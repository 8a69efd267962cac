// efg_efq.h - host-side reader of the .efq model file (the reference's on-disk format,
// include/ef/qfile.h:1-21), with the reference's validation (src/qfile.cpp:125-223).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace efg::efq {

// A malformed file; what() carries the reference's message for the same fault.
struct FormatError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// Minimal strict JSON value (objects keep document order; duplicate keys are rejected).
struct Json {
  enum class T { Null, Bool, Num, Str, Arr, Obj };
  T t = T::Null;
  bool b = false;
  bool is_int = false;
  int64_t i = 0;
  double d = 0.0;
  std::string s;  // string payload, or the literal text of a number
  std::vector<Json> items;
  std::vector<std::string> keys;

  const Json* find(std::string_view key) const;
  const Json& at(std::string_view key) const;  // throws FormatError if missing
  const std::string& str() const;
  uint64_t u64() const;
  double num() const;
};
Json parse_json(std::string_view text);

// config.json fields the engine uses (src/model_config.cpp:parse_model_config).
struct Config {
  int64_t hidden = 0, intermediate = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0,
          max_position = 2048;
  double rms_eps = 0.0, rope_theta = 10000.0;
  bool tie_embeddings = false;
  int64_t kv_dim() const { return kv_heads * head_dim; }
};
Config parse_config(const Json& root);

struct Tensor {
  std::string name;
  int type = 0;  // ef::QType numbering: 0 F32, 1 F16, 2 BF16, 3 Q8_0, 4 Q4_0
  std::string rule;
  std::vector<uint64_t> shape;
  uint64_t offset = 0, bytes = 0;
  uint64_t rows() const { return shape.size() == 2 ? shape[0] : 1; }
  uint64_t cols() const { return shape.empty() ? 0 : shape.back(); }
};

struct Policy {
  int layers = 4, lm_head = 3, embed = 2;
  std::vector<std::pair<std::string, int>> overrides;  // (pattern, type)
  std::string name;
};

struct Layout {
  uint64_t header_len = 0, data_start = 0;
  Config cfg;
  Policy policy;
  std::vector<Tensor> tensors;
  const Tensor* find(std::string_view name) const;
  const Tensor& at(std::string_view name) const;  // throws FormatError
};

// Parses and validates a whole file image (src/qfile.cpp:125-223). Throws FormatError.
Layout parse(const uint8_t* file, uint64_t size);

// Storage type and rule of one tensor under a policy (src/qfile.cpp:45-77).
bool glob_match(std::string_view pattern, std::string_view text);
std::pair<int, std::string> policy_choice(const Policy& p, const std::string& name, uint64_t cols,
                                          bool use_overrides = true);

// The tensors a config requires, in forward-pass order (src/model_config.cpp:expected_tensors).
std::vector<std::pair<std::string, std::vector<uint64_t>>> expected_tensors(const Config& c);

const char* type_name(int t);
int type_from_string(std::string_view s);  // -1 if unknown
uint64_t row_bytes(int type, uint64_t cols);  // throws FormatError for a block type with cols % 32

}  // namespace efg::efq
