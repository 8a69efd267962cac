// Reference test cases, written against the reference's C++ API (include/ef/quant.h,
// include/ef/qkernels.h) and compiled here against include/efg_ref_shim.hpp, so they run
// on the B200 through libefg.so. Each case names the reference test it restates.
// Build: g++ -std=c++20 -O2 -Iinclude tests/shim/shim_test.cpp -Ledgeforge_b200 -lefg
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "efg_ref_shim.hpp"

using namespace ef;

static int g_checks = 0, g_failures = 0;
#define CHECK(cond)                                                        \
  do {                                                                     \
    ++g_checks;                                                            \
    if (!(cond)) {                                                         \
      ++g_failures;                                                        \
      std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #cond); \
    }                                                                      \
  } while (0)

static std::uint16_t f16(float f) {
  // 1.0 and 0.0 only: exact half bit patterns
  return f == 1.0f ? 0x3C00 : 0x0000;
}

// test_quant.cpp:52-69
static void quant_q4_exact_on_grid_and_nibble_layout() {
  float x[kQK], y[kQK];
  for (std::size_t j = 0; j < kQK; ++j) x[j] = static_cast<float>(static_cast<int>(j % 16) - 8) * 0.25f;
  BlockQ4_0 b;
  quantize_block_q4_0(x, b);
  dequantize_block_q4_0(b, y);
  CHECK(std::memcmp(x, y, sizeof x) == 0);
  BlockQ4_0 m{};
  m.d = f16(1.0f);
  m.qs[0] = 0x2F;
  dequantize_block_q4_0(m, y);
  CHECK(y[0] == 7.0f && y[16] == -6.0f && y[1] == -8.0f);
  const float zeros[kQK] = {};
  quantize_block_q4_0(zeros, b);
  CHECK(b.d == 0 && b.qs[0] == 0x88);
}

// test_quant.cpp:125-130
static void quant_rows_types() {
  CHECK(qtype_row_bytes(QType::Q4_0, 2048) == 64 * 18);
  CHECK(qtype_row_bytes(QType::Q8_0, 2048) == 64 * 34);
  CHECK(qtype_row_bytes(QType::BF16, 2048) == 4096);
  bool threw = false;
  try {
    qtype_row_bytes(QType::Q4_0, 30);
  } catch (const Error& e) {
    threw = std::strstr(e.what(), "divisible by 32") != nullptr;
  }
  CHECK(threw);
  std::mt19937 rng(13);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  std::vector<float> x(256), y(256);
  for (auto& v : x) v = nd(rng);
  for (QType t : {QType::Q8_0, QType::Q4_0}) {
    std::vector<std::uint8_t> buf(static_cast<std::size_t>(qtype_row_bytes(t, 256)));
    quantize_row(t, x.data(), 256, buf.data());
    dequantize_row(t, buf.data(), 256, y.data());
    double e = 0;
    for (std::size_t i = 0; i < 256; ++i) e = std::max(e, double(std::fabs(x[i] - y[i])));
    CHECK(e < 0.6);
  }
}

// test_qinfer.cpp:100-122
static void qinfer_packed_dot_layout_and_edge_codes() {
  std::uint8_t blk[18] = {};
  const std::uint16_t one = f16(1.0f);
  std::memcpy(blk, &one, 2);
  for (std::size_t j = 0; j < 16; ++j) blk[2 + j] = 0x88;
  blk[2 + 3] = 0x0F;
  float x[32] = {};
  x[3] = 2.0f;
  x[19] = 0.5f;
  CHECK(kern::dot_q4_0(blk, x, 32) == 7.0f * 2.0f + -8.0f * 0.5f);
  const std::uint16_t zero = 0;
  std::memcpy(blk, &zero, 2);
  CHECK(kern::dot_q4_0(blk, x, 32) == 0.0f);
  std::uint8_t b8[34] = {};
  std::memcpy(b8, &one, 2);
  b8[2 + 0] = static_cast<std::uint8_t>(-127);
  b8[2 + 31] = 127;
  for (auto& v : x) v = 1.0f;
  CHECK(kern::dot_q8_0(b8, x, 32) == 0.0f);
  b8[2 + 5] = 3;
  CHECK(kern::dot_q8_0(b8, x, 32) == 3.0f);
}

// test_qinfer.cpp:71-98: matvec == row dots, error <= 1e-5 of sum |w x| vs the
// dequantized weights (rel_dot_error, test_qinfer.cpp:58-67)
static void qinfer_packed_dots_match_dequantized_weights() {
  std::mt19937 rng(61);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  std::uniform_int_distribution<int> byte(0, 255);
  std::uniform_real_distribution<float> scale(-0.05f, 0.05f);
  double worst = 0.0;
  for (std::size_t n : {std::size_t{32}, std::size_t{64}, std::size_t{2048}, std::size_t{5632}}) {
    std::vector<float> x(n);
    for (auto& v : x) v = nd(rng) * (nd(rng) > 2.0f ? 30.0f : 1.0f);
    for (QType t : {QType::Q4_0, QType::Q8_0}) {
      const std::size_t rows = 24, rb = static_cast<std::size_t>(qtype_row_bytes(t, n));
      const std::size_t bsz = t == QType::Q4_0 ? sizeof(BlockQ4_0) : sizeof(BlockQ8_0);
      std::vector<std::uint8_t> W(rows * rb);
      for (auto& v : W) v = static_cast<std::uint8_t>(byte(rng));
      for (std::size_t off = 0; off < W.size(); off += bsz) {
        const float s = scale(rng);
        // fp16 of a value in (-0.05, 0.05): build it through the library's quantizer of a
        // block whose max is s * 127 (Q8_0 gives d = s exactly rounded to fp16)
        float blk[kQK] = {};
        blk[0] = s * 127.0f;
        BlockQ8_0 q;
        quantize_block_q8_0(blk, q);
        std::memcpy(W.data() + off, &q.d, 2);
      }
      std::vector<float> y(rows);
      if (t == QType::Q4_0) kern::matvec_q4_0(y.data(), W.data(), x.data(), rows, n);
      else kern::matvec_q8_0(y.data(), W.data(), x.data(), rows, n);
      std::vector<float> w(n);
      for (std::size_t r = 0; r < rows; ++r) {
        const float d = t == QType::Q4_0 ? kern::dot_q4_0(W.data() + r * rb, x.data(), n)
                                         : kern::dot_q8_0(W.data() + r * rb, x.data(), n);
        CHECK(d == y[r]);
        dequantize_row(t, W.data() + r * rb, n, w.data());
        double exact = 0.0, mag = 0.0;
        for (std::size_t i = 0; i < n; ++i) {
          exact += static_cast<double>(w[i]) * x[i];
          mag += std::fabs(static_cast<double>(w[i]) * x[i]);
        }
        worst = std::max(worst, std::fabs(y[r] - exact) / std::max(mag, 1e-30));
      }
    }
  }
  CHECK(worst < 1e-5);
  std::printf("    packed vs dequantized-then-dot (relative to sum|w*x|): worst %.2e\n", worst);
}

int main() {
  quant_q4_exact_on_grid_and_nibble_layout();
  quant_rows_types();
  qinfer_packed_dot_layout_and_edge_codes();
  qinfer_packed_dots_match_dequantized_weights();
  std::printf("%d checks, %d failures\n", g_checks, g_failures);
  return g_failures == 0 ? 0 : 1;
}
