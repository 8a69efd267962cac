// ref_bridge.cpp - TEST INFRASTRUCTURE ONLY.
//
// extern "C" entry points over the reference implementation (MG782469/EdgeForge),
// so Python tests and bench.py's CPU legs can drive the reference's own code via
// ctypes. oracle/Makefile compiles this file together with the reference's
// sources, read in place, into oracle/_ref/libefref.so. Nothing here re-implements
// reference logic: every function forwards to the reference symbol it names.
#include <cstdint>
#include <cstring>
#include <exception>
#include <filesystem>
#include <memory>
#include <string>
#include <vector>

#include "ef/fp16.h"
#include "ef/kernels.h"
#include "ef/model.h"
#include "ef/qkernels.h"
#include "ef/quant.h"
#include "ef/quantizer.h"
#include "ef/threadpool.h"

namespace {

thread_local std::string g_err;

ef::QType qt(int t) { return static_cast<ef::QType>(t); }

template <class F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

struct Decoder {
  ef::Model model;
  std::unique_ptr<ef::ThreadPool> pool;
  std::unique_ptr<ef::Transformer> tr;
};

}  // namespace

extern "C" {

const char* efr_last_error() { return g_err.c_str(); }
int efr_avx2_compiled() { return ef::kern::avx2_compiled() ? 1 : 0; }

// include/ef/fp16.h:28-92
float efr_fp16_to_f32(std::uint16_t h) { return ef::fp16_to_f32(h); }
std::uint16_t efr_f32_to_fp16(float f) { return ef::f32_to_fp16(f); }
float efr_bf16_to_f32(std::uint16_t h) { return ef::bf16_to_f32(h); }
std::uint16_t efr_f32_to_bf16(float f) { return ef::f32_to_bf16(f); }

// include/ef/quant.h:42-53
std::uint64_t efr_row_bytes(int t, std::uint64_t cols) {
  std::uint64_t r = 0;
  if (guarded([&] { r = ef::qtype_row_bytes(qt(t), cols); }) != 0) return 0;
  return r;
}
int efr_quantize_row(int t, const float* x, std::size_t n, void* out, int search) {
  return guarded([&] { ef::quantize_row(qt(t), x, n, out, search != 0); });
}
int efr_dequantize_row(int t, const void* in, std::size_t n, float* out) {
  return guarded([&] { ef::dequantize_row(qt(t), in, n, out); });
}
void efr_fake_quant_q4_group(const float* x, std::size_t n, float* out, int search) {
  ef::fake_quant_q4_group(x, n, out, search != 0);
}
void efr_quantize_block_q4_0(const float* x, std::uint8_t* out, int search) {
  ef::BlockQ4_0 b;
  ef::quantize_block_q4_0(x, b, search != 0);
  std::memcpy(out, &b, sizeof b);
}
void efr_quantize_block_q8_0(const float* x, std::uint8_t* out) {
  ef::BlockQ8_0 b;
  ef::quantize_block_q8_0(x, b);
  std::memcpy(out, &b, sizeof b);
}

// Row-parallel quantize/dequantize of a [rows][cols] matrix on the reference's
// ThreadPool (the split quantizer.cpp:37-51 uses: contiguous row chunks).
void* efr_pool_new(unsigned threads) { return new ef::ThreadPool(threads); }
void efr_pool_free(void* p) { delete static_cast<ef::ThreadPool*>(p); }
unsigned efr_pool_size(void* p) { return static_cast<ef::ThreadPool*>(p)->size(); }

int efr_quantize_rows(void* pool, int t, const float* x, std::size_t rows, std::size_t cols, void* out, int search) {
  return guarded([&] {
    const std::size_t rb = static_cast<std::size_t>(ef::qtype_row_bytes(qt(t), cols));
    auto* o = static_cast<std::uint8_t*>(out);
    auto body = [&](std::size_t, std::size_t b, std::size_t e) {
      for (std::size_t r = b; r < e; ++r) ef::quantize_row(qt(t), x + r * cols, cols, o + r * rb, search != 0);
    };
    if (pool) static_cast<ef::ThreadPool*>(pool)->parallel_for(rows, body, 1);
    else body(0, 0, rows);
  });
}

int efr_dequantize_rows(void* pool, int t, const void* in, std::size_t rows, std::size_t cols, float* out) {
  return guarded([&] {
    const std::size_t rb = static_cast<std::size_t>(ef::qtype_row_bytes(qt(t), cols));
    const auto* p = static_cast<const std::uint8_t*>(in);
    auto body = [&](std::size_t, std::size_t b, std::size_t e) {
      for (std::size_t r = b; r < e; ++r) ef::dequantize_row(qt(t), p + r * rb, cols, out + r * cols);
    };
    if (pool) static_cast<ef::ThreadPool*>(pool)->parallel_for(rows, body, 1);
    else body(0, 0, rows);
  });
}

// src/qkernels.cpp:39-75 (scalar backend) and :131-180 (AVX2 backend)
float efr_dot_q4_0(const std::uint8_t* row, const float* x, std::size_t n) { return ef::kern::dot_q4_0(row, x, n); }
float efr_dot_q8_0(const std::uint8_t* row, const float* x, std::size_t n) { return ef::kern::dot_q8_0(row, x, n); }
void efr_matvec_q4_0(float* y, const std::uint8_t* W, const float* x, std::size_t rows, std::size_t cols) {
  ef::kern::matvec_q4_0(y, W, x, rows, cols);
}
void efr_matvec_q8_0(float* y, const std::uint8_t* W, const float* x, std::size_t rows, std::size_t cols) {
  ef::kern::matvec_q8_0(y, W, x, rows, cols);
}

// kern::matvec (qkernels.cpp:275-297) with an explicit backend (0 scalar, 1 avx2)
// and an optional pool. The backend is process-wide in the reference, so this
// sets it for the call.
int efr_matvec(int backend, void* pool, int t, float* y, const std::uint8_t* W, const float* x, std::size_t rows,
               std::size_t cols) {
  return guarded([&] {
    ef::kern::set_backend(backend ? ef::kern::Backend::Avx2 : ef::kern::Backend::Scalar);
    const ef::WeightView v{qt(t), W, rows, cols};
    ef::kern::matvec(y, v, x, static_cast<ef::ThreadPool*>(pool));
  });
}

// src/kernels.cpp
void efr_rmsnorm(float* out, const float* x, const float* w, std::size_t n, float eps) {
  ef::kern::rmsnorm(out, x, w, n, eps);
}
void efr_swiglu(float* out, const float* g, const float* u, std::size_t n) { ef::kern::swiglu(out, g, u, n); }
std::size_t efr_argmax(const float* x, std::size_t n) { return ef::kern::argmax(x, n); }
void efr_softmax(float* x, std::size_t n) { ef::kern::softmax_inplace(x, n); }
void efr_rope_table(float* c, float* s, std::size_t max_pos, std::size_t hd, float theta) {
  const ef::kern::RopeTable t(max_pos, hd, theta);
  for (std::size_t p = 0; p < max_pos; ++p) {
    std::memcpy(c + p * (hd / 2), t.cos_row(p), hd / 2 * sizeof(float));
    std::memcpy(s + p * (hd / 2), t.sin_row(p), hd / 2 * sizeof(float));
  }
}
void efr_rope_apply(float* x, std::size_t nh, std::size_t hd, const float* c, const float* s) {
  ef::kern::rope_apply(x, nh, hd, c, s);
}
void efr_attention(float* out, const float* q, const float* k, const float* v, std::size_t n_pos, std::size_t H,
                   std::size_t KV, std::size_t hd, float* scores) {
  ef::kern::attention(out, q, k, v, n_pos, H, KV, hd, scores);
}

// src/quantizer.cpp:92-115,151-290: quantize a model directory (config.json +
// model.safetensors) into an .efq with the named policy ("auto", "uniform", ...).
int efr_quantize_model(const char* model_dir, const char* out_file, const char* policy, const char* overrides,
                       unsigned threads) {
  return guarded([&] {
    const ef::ModelConfig cfg = ef::load_model_config(std::filesystem::path(model_dir) / "config.json");
    ef::QuantizeOptions o;
    if (overrides && *overrides) {  // explicit per-tensor overrides (ef::parse_overrides)
      o.overrides = ef::parse_overrides(overrides);
    } else {
      const ef::PolicySelection sel = ef::select_policy(policy, cfg);
      o.overrides = sel.overrides;
      o.policy_name = sel.name;
    }
    o.threads = threads;
    ef::quantize_model(model_dir, out_file, o);
  });
}

// Model::load_efq + Transformer (src/model.cpp:66-111,153-276). backend: 0 scalar, 1 avx2.
void* efr_decoder_new(const char* efq_file, std::size_t max_seq, unsigned threads) {
  auto* d = new Decoder;
  if (guarded([&] {
        d->model = ef::Model::load_efq(efq_file);
        if (threads > 1) d->pool = std::make_unique<ef::ThreadPool>(threads);
        d->tr = std::make_unique<ef::Transformer>(d->model, max_seq, d->pool.get());
      }) != 0) {
    delete d;
    return nullptr;
  }
  return d;
}
void efr_decoder_free(void* d) { delete static_cast<Decoder*>(d); }
void efr_decoder_reset(void* d) { static_cast<Decoder*>(d)->tr->reset(); }
int efr_decoder_forward(void* h, int backend, std::int32_t token, std::size_t pos, float* logits) {
  return guarded([&] {
    ef::kern::set_backend(backend ? ef::kern::Backend::Avx2 : ef::kern::Backend::Scalar);
    auto* d = static_cast<Decoder*>(h);
    const float* lg = d->tr->forward(token, pos, logits != nullptr);
    if (logits) std::memcpy(logits, lg, static_cast<std::size_t>(d->model.config().vocab_size) * sizeof(float));
  });
}
std::uint64_t efr_decoder_bytes_per_token(void* h) {
  return static_cast<Decoder*>(h)->model.weight_bytes_per_token();
}

}  // extern "C"
