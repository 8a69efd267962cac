// efg_dot.cuh - the per-lane packed dot products of the matvec kernels: a lane owns a
// 64-column slot of a row (two Q4_0 or Q8_0 blocks) and keeps the matching 64 values of
// x in registers; codes become floats through exponent tricks (no integer->float
// conversion instructions) and are accumulated with packed FP32 FMAs. Shared by the
// standalone matvec kernel and the persistent decode kernel.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

#include "efg_device.cuh"
#include "efg_matvec.cuh"

namespace efg {

// ------------------------------------------------------------------ code -> float
// float whose value is 2^(23-p) + field, for the 4-bit field at bit p (p <= 16).
template <int P>
__device__ __forceinline__ float q4_field(uint32_t w) {
  return __uint_as_float((w & (0xFu << P)) | (uint32_t(150 - P) << 23));
}
template <int P>
__device__ __forceinline__ constexpr float q4_bias() {
  return float((1u << (23 - P)) + 8u);  // exact: offset of the field plus the code bias 8
}

// float 2^(23-p) + (int8 code + 128) for the byte at bit p (p = 0 or 8): the sign bit
// of the byte is flipped inside the same LOP3 (a ^ c) & b | c & ~b.
template <int P>
__device__ __forceinline__ float q8_field(uint32_t w) {
  constexpr uint32_t K1 = 0xFFu << P;
  constexpr uint32_t K2 = (uint32_t(150 - P) << 23) | (0x80u << P);
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(w), "r"(K1), "r"(K2));
  return __uint_as_float(r);
}
template <int P>
__device__ __forceinline__ constexpr float q8_bias() {
  return float((1u << (23 - P)) + 128u);
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// Q4_0: a word holding 4 code bytes m..m+3 of one block; byte j carries column j (low
// nibble) and j + 16 (high nibble). xp[k] = (x[k], x[k + 16]).
__device__ __forceinline__ void q4_word(uint32_t w, float2 x0, float2 x1, float2 x2, float2 x3, float2& a,
                                        float2& b) {
  const uint32_t ws = w >> 12;  // high nibble of byte 2 and both nibbles of byte 3
  a = __ffma2_rn(__fadd2_rn(f2(q4_field<0>(w), q4_field<4>(w)), f2(-q4_bias<0>(), -q4_bias<4>())), x0, a);
  b = __ffma2_rn(__fadd2_rn(f2(q4_field<8>(w), q4_field<12>(w)), f2(-q4_bias<8>(), -q4_bias<12>())), x1, b);
  a = __ffma2_rn(__fadd2_rn(f2(q4_field<16>(w), q4_field<8>(ws)), f2(-q4_bias<16>(), -q4_bias<8>())), x2, a);
  b = __ffma2_rn(__fadd2_rn(f2(q4_field<12>(ws), q4_field<16>(ws)), f2(-q4_bias<12>(), -q4_bias<16>())), x3, b);
}

// Two code bytes in bits 0..15.
__device__ __forceinline__ void q4_half(uint32_t w, float2 x0, float2 x1, float2& a, float2& b) {
  a = __ffma2_rn(__fadd2_rn(f2(q4_field<0>(w), q4_field<4>(w)), f2(-q4_bias<0>(), -q4_bias<4>())), x0, a);
  b = __ffma2_rn(__fadd2_rn(f2(q4_field<8>(w), q4_field<12>(w)), f2(-q4_bias<8>(), -q4_bias<12>())), x1, b);
}

// Q8_0: two int8 codes in bits 0..15, columns c, c + 1; xp = (x[c], x[c + 1]).
__device__ __forceinline__ void q8_half(uint32_t w, float2 xp, float2& a) {
  a = __ffma2_rn(__fadd2_rn(f2(q8_field<0>(w), q8_field<8>(w)), f2(-q8_bias<0>(), -q8_bias<8>())), xp, a);
}

// fp16 bits -> float on the FMA pipe (mixed-precision add of -0.0, exact for every
// input; the plain conversion goes through the slower XU pipe).
__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
  float r;
  asm("add.rn.f32.f16 %0, %1, 0f80000000;" : "=f"(r) : "h"(static_cast<unsigned short>(h)));
  return r;
}

// Column offset (within the 64-column slot) of x pair k: Q4 pairs (c, c + 16) for the
// first 16 pairs of each block, Q8 pairs (2k, 2k + 1).
template <Fmt F>
__device__ __forceinline__ int pair_col(int k) {
  if constexpr (F == Fmt::Q4) return k < 16 ? k : 32 + (k - 16);
  else return 2 * k;
}
template <Fmt F>
__device__ __forceinline__ int pair_step() {
  return F == Fmt::Q4 ? 16 : 1;
}

template <Fmt F>
constexpr int slot_words() {
  return F == Fmt::Q4 ? 9 : 17;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// Word K of a slot (compile-time) for one row: which x pairs it multiplies and which
// block accumulators it feeds. Q4_0 slot: word 0 = d_b, codes 0-1 | words 1-3 = codes
// 2-13 | word 4 = codes 14-15, d_b+1 | words 5-8 = the 16 code bytes of block b+1.
// Q8_0 slot: word 0 = d_b, codes 0-1 | words 1-7 = codes 2-29 | word 8 = codes 30-31,
// d_b+1 | words 9-16 = the 32 codes of block b+1.
template <Fmt F, int K>
__device__ __forceinline__ void slot_word(uint32_t w, const float2 (&xp)[32], float2& a0, float2& b0, float2& a1,
                                          float2& b1) {
  if constexpr (F == Fmt::Q4) {
    if constexpr (K == 0) q4_half(w >> 16, xp[0], xp[1], a0, b0);
    else if constexpr (K <= 3) q4_word(w, xp[4 * K - 2], xp[4 * K - 1], xp[4 * K], xp[4 * K + 1], a0, b0);
    else if constexpr (K == 4) q4_half(w, xp[14], xp[15], a0, b0);
    else q4_word(w, xp[16 + 4 * (K - 5)], xp[17 + 4 * (K - 5)], xp[18 + 4 * (K - 5)], xp[19 + 4 * (K - 5)], a1, b1);
  } else {
    if constexpr (K == 0) {
      q8_half(w >> 16, xp[0], a0);
    } else if constexpr (K <= 7) {
      q8_half(w, xp[2 * K - 1], b0);
      q8_half(w >> 16, xp[2 * K], a0);
    } else if constexpr (K == 8) {
      q8_half(w, xp[15], b0);
    } else {
      q8_half(w, xp[16 + 2 * (K - 9)], a1);
      q8_half(w >> 16, xp[17 + 2 * (K - 9)], b1);
    }
  }
}

template <Fmt F, int RB, int K>
__device__ __forceinline__ void rows_word(const uint32_t (&w)[RB][slot_words<F>()], const float2 (&xp)[32],
                                          float2 (&a0)[RB], float2 (&b0)[RB], float2 (&a1)[RB], float2 (&b1)[RB]) {
  if constexpr (K < slot_words<F>()) {
#pragma unroll
    for (int r = 0; r < RB; ++r) slot_word<F, K>(w[r][K], xp, a0[r], b0[r], a1[r], b1[r]);
    rows_word<F, RB, K + 1>(w, xp, a0, b0, a1, b1);
  }
}

// Dots of RB rows' slots (64 columns, two blocks each) with the lane's x registers,
// computed word by word across the rows so their independent FMA chains interleave.
// addr[r]: shared-memory address of row r's slot; rows with valid[r] false give 0.
template <Fmt F, int RB>
__device__ __forceinline__ void slot_dots(const uint32_t (&addr)[RB], const bool (&valid)[RB], const float2 (&xp)[32],
                                          float (&out)[RB]) {
  constexpr int NW = slot_words<F>();
  uint32_t w[RB][NW];
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int i = 0; i < NW; ++i) w[r][i] = valid[r] ? lds32(addr[r] + 4u * i) : 0u;
  const float2 z = f2(0.f, 0.f);
  float2 a0[RB], b0[RB], a1[RB], b1[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) a0[r] = b0[r] = a1[r] = b1[r] = z;
  rows_word<F, RB, 0>(w, xp, a0, b0, a1, b1);
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    const float d0 = half_bits_to_float(w[r][0] & 0xFFFFu);
    const float d1 = half_bits_to_float(w[r][F == Fmt::Q4 ? 4 : 8] >> 16);
    const float s0 = (a0[r].x + a0[r].y) + (b0[r].x + b0[r].y);
    const float s1 = (a1[r].x + a1[r].y) + (b1[r].x + b1[r].y);
    out[r] = valid[r] ? d0 * s0 + d1 * s1 : 0.f;
  }
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

}  // namespace efg
