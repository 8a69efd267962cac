// efg_ref_shim.hpp - the reference's C++ API for the packed matrix-product path, with
// the reference's exact signatures (include/ef/quant.h, include/ef/qkernels.h), running
// on a B200 through the C ABI of include/efg.h. Header-only; link with libefg.so.
//
// A program written against the reference's kernel API compiles against this header
// unchanged and runs on the GPU: pointers are host pointers and calls are synchronous.
// Weights are uploaded on every call unless they lie inside a range registered with
// efg_host_register_weights(); an integration registers the memory-mapped .efq data once
// at load (the reference passes read-only views of it, src/model.cpp:71-74), after which
// each call moves only x and y.
//
// Error behaviour follows the reference: calls that throw ef::Error there
// (qtype_row_bytes, quantize_row, dequantize_row, backend_from_string) throw ef::Error here
// with the same message; the noexcept kernels (matvec, dot) print the library's message and
// call std::abort() if the device fails, since they cannot report errors.
// The reference's CPU ThreadPool argument is accepted and ignored: the GPU grid does the
// row split. Its kernel backends (scalar / avx2) are names only here: both select the one
// sm_100a path.
//
// Inside the reference's own source tree, include/shim/ef/quant.h and include/shim/ef/
// qkernels.h stand in for the reference's headers of the same name (put include/shim before
// the reference's include directory), so its engine (src/model.cpp, src/qfile.cpp, ...)
// compiles unchanged with src/quant.cpp and src/qkernels.cpp left out.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <optional>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

#include "efg.h"

#if __has_include("ef/error.h")
#include "ef/error.h"  // the reference's own ef::Error, when its headers are on the path
#else
namespace ef {
// include/ef/error.h:11-13
struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};
}  // namespace ef
#endif

namespace ef {

// include/ef/quant.h:22-42
inline constexpr std::size_t kQK = 32;
struct BlockQ4_0 {
  std::uint16_t d;
  std::uint8_t qs[16];
};
struct BlockQ8_0 {
  std::uint16_t d;
  std::int8_t qs[32];
};
static_assert(sizeof(BlockQ4_0) == 18, "BlockQ4_0 must be packed to 18 bytes");
static_assert(sizeof(BlockQ8_0) == 34, "BlockQ8_0 must be packed to 34 bytes");
enum class QType : std::uint8_t { F32 = EFG_F32, F16 = EFG_F16, BF16 = EFG_BF16, Q8_0 = EFG_Q8_0, Q4_0 = EFG_Q4_0 };

namespace shim_detail {
inline void throw_if(int status) {
  if (status != EFG_OK) throw Error(efg_last_error());
}
inline void abort_if(int status, const char* what) noexcept {
  if (status != EFG_OK) {
    std::fprintf(stderr, "edgeforge-b200: %s failed: %s: %s\n", what, efg_status_string(status), efg_last_error());
    std::abort();
  }
}
}  // namespace shim_detail

// include/ef/quant.h:37-42: the type table
inline const char* qtype_name(QType t) noexcept {
  switch (t) {
    case QType::F32: return "F32";
    case QType::F16: return "F16";
    case QType::BF16: return "BF16";
    case QType::Q8_0: return "Q8_0";
    case QType::Q4_0: return "Q4_0";
  }
  return "?";
}
// The upper-case name or its lower-case spelling.
inline std::optional<QType> qtype_from_string(std::string_view s) noexcept {
  for (QType t : {QType::F32, QType::F16, QType::BF16, QType::Q8_0, QType::Q4_0}) {
    const std::string_view name = qtype_name(t);
    if (s.size() != name.size()) continue;
    bool upper = true, lower = true;
    for (std::size_t i = 0; i < s.size(); ++i) {
      const char c = name[i];
      const char lc = (c >= 'A' && c <= 'Z') ? static_cast<char>(c - 'A' + 'a') : c;
      upper = upper && s[i] == c;
      lower = lower && s[i] == lc;
    }
    if (upper || lower) return t;
  }
  return std::nullopt;
}
inline bool qtype_is_block(QType t) noexcept { return t == QType::Q8_0 || t == QType::Q4_0; }
inline double qtype_bits_per_weight(QType t) noexcept {
  switch (t) {
    case QType::F32: return 32.0;
    case QType::F16:
    case QType::BF16: return 16.0;
    case QType::Q8_0: return 8.0 * sizeof(BlockQ8_0) / kQK;
    case QType::Q4_0: return 8.0 * sizeof(BlockQ4_0) / kQK;
  }
  return 0.0;
}

inline std::uint64_t qtype_row_bytes(QType t, std::uint64_t cols) {
  const std::uint64_t n = efg_row_bytes(static_cast<int>(t), cols);
  if (n == 0 && cols != 0) throw Error(efg_last_error());
  return n;
}

// include/ef/quant.h:45-53 (blocks and rows); every type, on the device
inline void quantize_row(QType t, const float* x, std::size_t n, void* out, bool search = true) {
  shim_detail::throw_if(efg_host_quantize_row(static_cast<int>(t), x, n, out, search ? 1 : 0));
}
inline void dequantize_row(QType t, const void* in, std::size_t n, float* out) {
  shim_detail::throw_if(efg_host_dequantize_row(static_cast<int>(t), in, n, out));
}
inline void quantize_block_q4_0(const float* x, BlockQ4_0& out, bool search = true) noexcept {
  shim_detail::abort_if(efg_host_quantize_row(EFG_Q4_0, x, kQK, &out, search ? 1 : 0), "quantize_block_q4_0");
}
inline void quantize_block_q8_0(const float* x, BlockQ8_0& out) noexcept {
  shim_detail::abort_if(efg_host_quantize_row(EFG_Q8_0, x, kQK, &out, 1), "quantize_block_q8_0");
}
inline void dequantize_block_q4_0(const BlockQ4_0& b, float* out) noexcept {
  shim_detail::abort_if(efg_host_dequantize_row(EFG_Q4_0, &b, kQK, out), "dequantize_block_q4_0");
}
inline void dequantize_block_q8_0(const BlockQ8_0& b, float* out) noexcept {
  shim_detail::abort_if(efg_host_dequantize_row(EFG_Q8_0, &b, kQK, out), "dequantize_block_q8_0");
}

// include/ef/quant.h:58
inline void fake_quant_q4_group(const float* x, std::size_t n, float* out, bool search) noexcept {
  shim_detail::abort_if(efg_host_fake_quant_q4_group(x, n, out, search ? 1 : 0), "fake_quant_q4_group");
}

// include/ef/qkernels.h:28-34
struct WeightView {
  QType type = QType::BF16;
  const std::uint8_t* data = nullptr;
  std::size_t rows = 0, cols = 0;
  std::size_t row_bytes() const { return static_cast<std::size_t>(qtype_row_bytes(type, cols)); }
  std::uint64_t bytes() const { return static_cast<std::uint64_t>(row_bytes()) * rows; }
};

class ThreadPool;  // the reference's CPU pool; accepted and ignored here

namespace kern {

// include/ef/qkernels.h:38-44: the backend switch. The names are kept so callers compile and
// behave; every backend is the same GPU path, so no choice can fail.
enum class Backend { Scalar, Avx2 };
namespace shim_detail_backend {
inline Backend& current() noexcept {
  static Backend b = Backend::Scalar;
  return b;
}
}  // namespace shim_detail_backend
inline bool avx2_compiled() noexcept { return false; }  // no CPU SIMD kernels in this build
inline Backend default_backend() noexcept { return Backend::Scalar; }
inline Backend backend() noexcept { return shim_detail_backend::current(); }
inline void set_backend(Backend b) { shim_detail_backend::current() = b; }
inline const char* backend_name(Backend b) noexcept { return b == Backend::Avx2 ? "avx2" : "scalar"; }
inline Backend backend_from_string(const std::string& s) {
  if (s == "auto") return default_backend();
  if (s == "scalar") return Backend::Scalar;
  if (s == "avx2") return Backend::Avx2;
  throw Error("--kernels expects scalar, avx2 or auto; got '" + s + "'");
}

// include/ef/qkernels.h:47-51
inline void matvec_q4_0(float* y, const std::uint8_t* W, const float* x, std::size_t rows, std::size_t cols) noexcept {
  shim_detail::abort_if(efg_host_matvec(EFG_Q4_0, y, W, x, rows, cols), "matvec_q4_0");
}
inline void matvec_q8_0(float* y, const std::uint8_t* W, const float* x, std::size_t rows, std::size_t cols) noexcept {
  shim_detail::abort_if(efg_host_matvec(EFG_Q8_0, y, W, x, rows, cols), "matvec_q8_0");
}
inline float dot_q4_0(const std::uint8_t* row, const float* x, std::size_t n) noexcept {
  float y = 0.0f;
  matvec_q4_0(&y, row, x, 1, n);
  return y;
}
inline float dot_q8_0(const std::uint8_t* row, const float* x, std::size_t n) noexcept {
  float y = 0.0f;
  matvec_q8_0(&y, row, x, 1, n);
  return y;
}

// include/ef/qkernels.h:63: rows [begin, end) of y = W x (y indexed by row), any type
inline void matvec_rows(float* y, const WeightView& W, const float* x, std::size_t begin, std::size_t end) noexcept {
  if (begin >= end) return;
  const std::size_t rb = static_cast<std::size_t>(efg_row_bytes(static_cast<int>(W.type), W.cols));
  shim_detail::abort_if(efg_host_matvec(static_cast<int>(W.type), y + begin, W.data + begin * rb, x, end - begin, W.cols),
                        "matvec_rows");
}

// include/ef/qkernels.h:66 (every storage type; the pool argument is ignored)
inline void matvec(float* y, const WeightView& W, const float* x, ThreadPool* = nullptr) noexcept {
  shim_detail::abort_if(efg_host_matvec(static_cast<int>(W.type), y, W.data, x, W.rows, W.cols), "matvec");
}

// include/ef/qkernels.h:70-75
struct MatvecJob {
  float* y;
  const WeightView* W;
  const float* x;
};
inline void matvec_jobs(const MatvecJob* jobs, std::size_t n_jobs, ThreadPool* pool) noexcept {
  for (std::size_t j = 0; j < n_jobs; ++j) matvec(jobs[j].y, *jobs[j].W, jobs[j].x, pool);
}

// include/ef/qkernels.h:78: row r of W as FP32 (exact widening or dequantization)
inline void row_f32(float* out, const WeightView& W, std::size_t r) noexcept {
  const std::size_t rb = W.row_bytes();
  shim_detail::abort_if(efg_host_dequantize_row(static_cast<int>(W.type), W.data + r * rb, W.cols, out), "row_f32");
}

}  // namespace kern
}  // namespace ef
