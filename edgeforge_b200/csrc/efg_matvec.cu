// efg_matvec.cu - packed Q4_0 / Q8_0 matvec for B200 (sm_100a).
//
// The reference computes y = W x row by row on CPU threads, one 18/34-byte block at a
// time (src/qkernels.cpp:39-75, 213-297). Here the whole matrix streams from HBM once:
//
//  * One persistent CTA per SM. A producer warp copies row tiles (TR whole rows, a
//    contiguous byte range of the packed matrix) into a ring of NS shared-memory stages
//    with 1-D bulk async copies (cp.async.bulk, completion counted on an mbarrier), so
//    no thread spends instructions moving weights and every byte of HBM is read once.
//  * Each consumer lane owns one 64-column "slot" of a row: a pair of blocks, which is
//    9 (Q4_0) or 17 (Q8_0) aligned 32-bit words whatever the row's offset, read from
//    shared memory without bank conflicts (stride 9 or 17 words). The lane keeps the 64
//    x values of its slot in registers for the whole kernel, so x is read from global
//    memory once per CTA.
//  * A code becomes an exact float with one LOP3: the nibble (or byte) stays where it is
//    in the word and the OR-ed exponent makes the field the units digit,
//    float(2^(23-p) + code), for a field at bit p. One packed f32x2 add removes the
//    offset (exact), one packed f32x2 FMA multiplies by x. The block sum is scaled by
//    the fp16 d once per block.
//  * Rows are summed across lanes with a reduce-scatter shuffle butterfly (RB rows at a
//    time), and across the G warps that cover a long row through shared memory.
//
// Optional fusions used by the decode step: an RMSNorm prologue (x <- rmsnorm(x) * w,
// src/kernels.cpp:69-75), a residual epilogue (y += W x, model.cpp:249/262) and a SwiGLU
// epilogue over a gate/up pair (src/kernels.cpp:94-99, model.cpp:255-258).
#include <algorithm>
#include <cstdio>

#include <cuda_fp16.h>

#include "efg_device.cuh"
#include "efg_host.h"
#include "efg_matvec.cuh"

namespace efg {

namespace {

constexpr int kMaxThreads = 384;  // 1 producer warp + up to 11 consumer warps
constexpr int kMaxConsumerWarps = kMaxThreads / 32 - 1;
constexpr int kNormBarrier = 15;  // named barrier id for the RMSNorm reduction

struct KParams {
  const float* x;
  const float* norm_w;
  float norm_eps;
  int* err;
  const int32_t* pos;
  uint32_t cols, rb_words, S, G, RG, TR, NS, stage_bytes, n_jobs, tiles_total;
  uint32_t job_tile_start[kMaxJobs + 1];
  MatvecJobDev jobs[kMaxJobs];
};

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

__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
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

// Dot of one slot (64 columns, two blocks) with the lane's x registers.
template <Fmt F>
__device__ __forceinline__ float slot_dot(const uint32_t* __restrict__ wp, const float2 (&xp)[32]) {
  uint32_t w[slot_words<F>()];
#pragma unroll
  for (int i = 0; i < slot_words<F>(); ++i) w[i] = wp[i];
  const float2 z = f2(0.f, 0.f);
  float2 a0 = z, b0 = z, a1 = z, b1 = z;
  float d0, d1;
  if constexpr (F == Fmt::Q4) {
    // word 0: d_b, codes 0-1 | words 1-3: codes 2-13 | word 4: codes 14-15, d_b+1 |
    // words 5-8: the 16 code bytes of block b+1.
    d0 = half_bits_to_float(w[0] & 0xFFFFu);
    d1 = half_bits_to_float(w[4] >> 16);
    q4_half(w[0] >> 16, xp[0], xp[1], a0, b0);
    q4_word(w[1], xp[2], xp[3], xp[4], xp[5], a0, b0);
    q4_word(w[2], xp[6], xp[7], xp[8], xp[9], a0, b0);
    q4_word(w[3], xp[10], xp[11], xp[12], xp[13], a0, b0);
    q4_half(w[4], xp[14], xp[15], a0, b0);
    q4_word(w[5], xp[16], xp[17], xp[18], xp[19], a1, b1);
    q4_word(w[6], xp[20], xp[21], xp[22], xp[23], a1, b1);
    q4_word(w[7], xp[24], xp[25], xp[26], xp[27], a1, b1);
    q4_word(w[8], xp[28], xp[29], xp[30], xp[31], a1, b1);
  } else {
    // word 0: d_b, codes 0-1 | words 1-7: codes 2-29 | word 8: codes 30-31, d_b+1 |
    // words 9-16: the 32 codes of block b+1.
    d0 = half_bits_to_float(w[0] & 0xFFFFu);
    d1 = half_bits_to_float(w[8] >> 16);
    q8_half(w[0] >> 16, xp[0], a0);
#pragma unroll
    for (int k = 1; k < 8; ++k) {
      q8_half(w[k], xp[2 * k - 1], b0);
      q8_half(w[k] >> 16, xp[2 * k], a0);
    }
    q8_half(w[8], xp[15], b0);
#pragma unroll
    for (int k = 9; k < 17; ++k) {
      q8_half(w[k], xp[16 + 2 * (k - 9)], a1);
      q8_half(w[k] >> 16, xp[17 + 2 * (k - 9)], b1);
    }
  }
  const float s0 = (a0.x + a0.y) + (b0.x + b0.y);
  const float s1 = (a1.x + a1.y) + (b1.x + b1.y);
  return d0 * s0 + d1 * s1;
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// Which job a tile belongs to, and its first row.
__device__ __forceinline__ void locate_tile(const KParams& p, uint32_t tile, uint32_t& j, uint32_t& r0,
                                            uint32_t& nrows) {
  j = 0;
  while (j + 1 < p.n_jobs && tile >= p.job_tile_start[j + 1]) ++j;
  r0 = (tile - p.job_tile_start[j]) * p.TR;
  nrows = min(p.TR, p.jobs[j].rows - r0);
}

template <Fmt F, int RB, Epi E, bool NORM>
__global__ void __launch_bounds__(kMaxThreads, 1) matvec_fast_kernel(const __grid_constant__ KParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t nc = p.G * p.RG;  // consumer warps
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.NS * p.stage_bytes);
  uint64_t* empty = full + p.NS;
  float* red = reinterpret_cast<float*>(empty + p.NS);  // [2][RG][RB][G]
  double* norm_red = reinterpret_cast<double*>(red + 2 * p.RG * RB * p.G + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < p.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], nc);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // Dependents may start as soon as they find room; they only touch data this kernel
  // writes after their own pdl_wait().
  pdl_launch_dependents();

  if (warp == static_cast<int>(nc)) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    const uint64_t pol = l2_evict_first_policy();
    uint32_t it = 0;
    bool ok = true;
    for (uint32_t tile = blockIdx.x; tile < p.tiles_total; tile += gridDim.x, ++it) {
      const uint32_t s = it % p.NS;
      if (it >= p.NS && !mbar_wait(&empty[s], ((it / p.NS) & 1u) ^ 1u, p.err)) {
        ok = false;
        break;
      }
      uint32_t j, r0, nrows;
      locate_tile(p, tile, j, r0, nrows);
      const uint32_t rb = p.rb_words * 4u;
      const uint32_t bytes = nrows * rb;
      const uint32_t bulk = bytes & ~15u;
      uint8_t* dst = stages + s * p.stage_bytes;
      const int n_mat = E == Epi::SwiGLU ? 2 : 1;
      // The ragged end of the last tile (bytes % 16) is copied by this thread; the
      // release of the arrive below orders it before the consumers' acquire.
      for (int m = 0; m < n_mat; ++m) {
        const uint8_t* src = p.jobs[E == Epi::SwiGLU ? m : j].W + static_cast<size_t>(r0) * rb;
        uint8_t* d = dst + m * (p.TR * rb);
        for (uint32_t b = bulk; b < bytes; ++b) d[b] = src[b];
      }
      mbar_arrive_expect_tx(&full[s], bulk * n_mat);
      for (int m = 0; m < n_mat; ++m) {
        const uint8_t* src = p.jobs[E == Epi::SwiGLU ? m : j].W + static_cast<size_t>(r0) * rb;
        if (bulk) bulk_g2s(dst + m * (p.TR * rb), src, bulk, &full[s], pol);
      }
    }
    if (!ok) {
      // Let copies already issued land before the CTA can exit (bounded as well).
      const uint32_t first = it > p.NS ? it - p.NS : 0;
      for (uint32_t k = first; k < it; ++k) mbar_wait(&full[k % p.NS], (k / p.NS) & 1u, nullptr);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const uint32_t g = warp % p.G, rg = warp / p.G;
  const uint32_t slot = g * 32 + lane;
  const bool active = slot < p.S;
  pdl_wait();  // x, norm weights and y belong to the previous kernel in the stream

  float inv = 1.0f;
  if constexpr (NORM) {
    // rmsnorm scale from the whole x (src/kernels.cpp:69-73): double sum of squares.
    double ss = 0.0;
    for (uint32_t i = threadIdx.x; i < p.cols; i += nc * 32) {
      const double v = static_cast<double>(p.x[i]);
      ss += v * v;
    }
    ss = warp_sum_d(ss);
    if (lane == 0) norm_red[warp] = ss;
    named_barrier(kNormBarrier, nc * 32);
    double tot = 0.0;
    for (uint32_t w = 0; w < nc; ++w) tot += norm_red[w];
    const double mean = p.cols ? tot / static_cast<double>(p.cols) : 0.0;
    inv = static_cast<float>(1.0 / sqrt(mean + static_cast<double>(p.norm_eps)));
  }
  float2 xp[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    float lo = 0.f, hi = 0.f;
    if (active) {
      const uint32_t c = slot * 64 + pair_col<F>(k);
      lo = p.x[c];
      hi = p.x[c + pair_step<F>()];
      if constexpr (NORM) {
        lo = p.norm_w[c] * (lo * inv);
        hi = p.norm_w[c + pair_step<F>()] * (hi * inv);
      }
    }
    xp[k] = f2(lo, hi);
  }

  constexpr int RBH = E == Epi::SwiGLU ? RB / 2 : RB;  // logical rows per warp per tile
  // After a failed (timed-out) wait a warp stops reading and writing but keeps walking
  // the tile loop, so the named barriers of its row group still see every warp.
  bool alive = true;
  uint32_t it = 0, buf = 0;
  for (uint32_t tile = blockIdx.x; tile < p.tiles_total; tile += gridDim.x, ++it) {
    const uint32_t s = it % p.NS;
    if (alive && !mbar_wait(&full[s], (it / p.NS) & 1u, p.err)) alive = false;
    uint32_t j, r0, nrows;
    locate_tile(p, tile, j, r0, nrows);
    if (!alive) nrows = 0;
    const uint32_t* stage = reinterpret_cast<const uint32_t*>(stages + s * p.stage_bytes);
    float acc[RB];
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      // SwiGLU: the first RB/2 entries are gate rows, the rest the matching up rows
      // (stored TR rows further on in the stage).
      const uint32_t lr = rg * RBH + (i % RBH);
      const uint32_t srow = (E == Epi::SwiGLU && i >= RBH) ? lr + p.TR : lr;
      acc[i] = (active && lr < nrows) ? slot_dot<F>(stage + srow * p.rb_words + slot * slot_words<F>(), xp) : 0.f;
    }
    __syncwarp();
    if (alive && lane == 0) mbar_arrive(&empty[s]);

    const float v = warp_reduce_rows<RB>(acc, lane);
    const float mine = __shfl_sync(0xFFFFFFFFu, v, (lane % RB) * (32 / RB));  // lane i < RB: row i
    float total = mine;
    bool writer = lane < RB;
    if (p.G > 1) {
      float* rbuf = red + buf * p.RG * RB * p.G;
      if (lane < RB) rbuf[(rg * RB + lane) * p.G + g] = mine;
      named_barrier(1 + rg, p.G * 32);
      writer = writer && g == 0;
      if (writer) {
        total = 0.f;
        for (uint32_t q = 0; q < p.G; ++q) total += rbuf[(rg * RB + lane) * p.G + q];
      }
      buf ^= 1u;
    }
    if constexpr (E == Epi::SwiGLU) {
      const float up = __shfl_down_sync(0xFFFFFFFFu, total, RBH);
      const uint32_t lr = rg * RBH + lane;
      if (writer && lane < RBH && lr < nrows) {
        float* y = p.jobs[0].y + (p.pos ? *p.pos * p.jobs[0].y_pos_stride : 0);
        y[r0 + lr] = silu(total) * up;
      }
    } else {
      const uint32_t lr = rg * RB + lane;
      if (writer && lr < nrows) {
        float* y = p.jobs[j].y + (p.pos ? *p.pos * p.jobs[j].y_pos_stride : 0);
        if constexpr (E == Epi::Add) y[r0 + lr] += total;
        else y[r0 + lr] = total;
      }
    }
  }
}

// ------------------------------------------------------------------ generic path
// Any cols % 32 == 0 and any pointer alignment: one warp per row, lanes stride over
// blocks, bytes read one at a time. Used only for shapes the fast path rejects.
template <Fmt F, Epi E>
__global__ void matvec_generic_kernel(const __grid_constant__ KParams p) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr uint32_t BB = F == Fmt::Q4 ? 18 : 34;
  const uint32_t nb = p.cols / 32;
  const int lane = threadIdx.x & 31;
  const uint32_t warps = gridDim.x * (blockDim.x / 32);
  // Work items are single rows here: job_tile_start holds row offsets.
  for (uint32_t t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); t < p.tiles_total; t += warps) {
    uint32_t j = 0;
    while (j + 1 < p.n_jobs && t >= p.job_tile_start[j + 1]) ++j;
    const uint32_t r = t - p.job_tile_start[j];
    float sums[2] = {0.f, 0.f};
    const int n_mat = E == Epi::SwiGLU ? 2 : 1;
    for (int m = 0; m < n_mat; ++m) {
      const uint8_t* row = p.jobs[E == Epi::SwiGLU ? m : j].W + static_cast<size_t>(r) * nb * BB;
      float acc = 0.f;
      for (uint32_t b = lane; b < nb; b += 32) {
        const uint8_t* blk = row + static_cast<size_t>(b) * BB;
        const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
        const float* xb = p.x + b * 32;
        float s = 0.f;
        for (int k = 0; k < 32; ++k) {
          const float xv = xb[k];
          int code;
          if constexpr (F == Fmt::Q4) code = (k < 16 ? (blk[2 + k] & 15) : (blk[2 + k - 16] >> 4)) - 8;
          else code = static_cast<int8_t>(blk[2 + k]);
          s += static_cast<float>(code) * xv;
        }
        acc += d * s;
      }
      sums[m] = warp_sum(acc);
    }
    if (lane == 0) {
      float* y = p.jobs[j].y + (p.pos ? *p.pos * p.jobs[j].y_pos_stride : 0);
      if constexpr (E == Epi::SwiGLU) y[r] = silu(sums[0]) * sums[1];
      else if constexpr (E == Epi::Add) y[r] += sums[0];
      else y[r] = sums[0];
    }
  }
}

// cols == 0: every dot is over zero blocks, which the reference returns as 0.
__global__ void zero_rows_kernel(float* y, uint32_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] = 0.f;
}

using FastFn = void (*)(KParams);

template <Fmt F, int RB, Epi E>
FastFn pick_norm(bool norm) {
  return norm ? matvec_fast_kernel<F, RB, E, true> : matvec_fast_kernel<F, RB, E, false>;
}

template <Fmt F, int RB>
FastFn pick_epi(Epi e, bool norm) {
  switch (e) {
    case Epi::Store: return pick_norm<F, RB, Epi::Store>(norm);
    case Epi::Add: return pick_norm<F, RB, Epi::Add>(norm);
    case Epi::SwiGLU:
      if constexpr (RB >= 2) return pick_norm<F, RB, Epi::SwiGLU>(norm);
      else return nullptr;
  }
  return nullptr;
}

template <Fmt F>
FastFn pick_rb(int rb, Epi e, bool norm) {
  switch (rb) {
    case 1: return pick_epi<F, 1>(e, norm);
    case 2: return pick_epi<F, 2>(e, norm);
    default: return pick_epi<F, 4>(e, norm);
  }
}

FastFn pick_fast(Fmt f, int rb, Epi e, bool norm) {
  return f == Fmt::Q4 ? pick_rb<Fmt::Q4>(rb, e, norm) : pick_rb<Fmt::Q8>(rb, e, norm);
}

using GenFn = void (*)(KParams);
GenFn pick_generic(Fmt f, Epi e) {
  if (f == Fmt::Q4) {
    return e == Epi::Store ? matvec_generic_kernel<Fmt::Q4, Epi::Store>
           : e == Epi::Add ? matvec_generic_kernel<Fmt::Q4, Epi::Add>
                           : matvec_generic_kernel<Fmt::Q4, Epi::SwiGLU>;
  }
  return e == Epi::Store ? matvec_generic_kernel<Fmt::Q8, Epi::Store>
         : e == Epi::Add ? matvec_generic_kernel<Fmt::Q8, Epi::Add>
                         : matvec_generic_kernel<Fmt::Q8, Epi::SwiGLU>;
}

struct Plan {
  uint32_t S, G, RG, RB, TR, NS, stage_bytes, tiles;
  size_t smem;
  bool ok;
};

constexpr size_t kSmemBudget = 200 * 1024;

Plan plan_fast(const MatvecArgs& a, const DeviceInfo& dev) {
  Plan pl{};
  const uint32_t bb = a.fmt == Fmt::Q4 ? 18u : 34u;
  const uint32_t rb = static_cast<uint32_t>(a.cols / 32 * bb);
  pl.S = static_cast<uint32_t>(a.cols / 64);
  pl.G = (pl.S + 31) / 32;
  pl.ok = a.cols % 64 == 0 && pl.G >= 1 && pl.G <= static_cast<uint32_t>(kMaxConsumerWarps);
  if (!pl.ok) return pl;
  pl.RG = std::max<uint32_t>(1, 8 / pl.G);
  if (pl.G * pl.RG > static_cast<uint32_t>(kMaxConsumerWarps)) pl.RG = kMaxConsumerWarps / pl.G;
  const int n_mat = a.epi == Epi::SwiGLU ? 2 : 1;
  auto tiles_for = [&](uint32_t TR) {
    uint32_t t = 0;
    const int nj = a.epi == Epi::SwiGLU ? 1 : a.n_jobs;
    for (int j = 0; j < nj; ++j) t += (a.jobs[j].rows + TR - 1) / TR;
    return t;
  };
  // Largest row batch that still leaves >= 2 tiles per SM (load balance); if none
  // does, the smallest one. The tile byte size must be a multiple of 16 so every tile
  // starts 16-byte aligned for the bulk copy.
  pl.RB = 0;
  for (uint32_t rbv : {4u, 2u, 1u}) {
    if (a.epi == Epi::SwiGLU && rbv < 2) continue;
    const uint32_t TR = pl.RG * (a.epi == Epi::SwiGLU ? rbv / 2 : rbv);
    if ((static_cast<uint64_t>(TR) * rb) % 16 != 0) continue;
    pl.RB = rbv;
    if (tiles_for(TR) >= 2u * static_cast<uint32_t>(dev.sm_count)) break;
  }
  if (pl.RB == 0) {
    pl.ok = false;
    return pl;
  }
  pl.TR = pl.RG * (a.epi == Epi::SwiGLU ? pl.RB / 2 : pl.RB);
  pl.tiles = tiles_for(pl.TR);
  pl.stage_bytes = static_cast<uint32_t>((static_cast<uint64_t>(pl.TR) * rb * n_mat + 127) / 128 * 128);
  const size_t tail = 2 * 8 * 16 /* barriers */ + (2 * pl.RG * pl.RB * pl.G + 2) * 4 + 16 * 8 + 128;
  const size_t budget = std::min(kSmemBudget, dev.smem_optin > tail ? dev.smem_optin - tail : 0);
  pl.NS = static_cast<uint32_t>(std::min<size_t>(8, budget / std::max<uint32_t>(pl.stage_bytes, 1)));
  if (pl.NS < 2) {
    pl.ok = false;
    return pl;
  }
  pl.smem = pl.NS * static_cast<size_t>(pl.stage_bytes) + 2 * pl.NS * 8 + (2 * pl.RG * pl.RB * pl.G + 2) * 4 +
            16 * 8;
  return pl;
}

}  // namespace

bool matvec_fast_path_ok(const MatvecArgs& a) {
  DeviceInfo* dev = current_device();
  if (!dev) return false;
  for (int j = 0; j < (a.epi == Epi::SwiGLU ? 2 : a.n_jobs); ++j)
    if (reinterpret_cast<uintptr_t>(a.jobs[j].W) % 16 != 0) return false;
  return plan_fast(a, *dev).ok;
}

int launch_matvec(const MatvecArgs& a, int* d_err, cudaStream_t stream) {
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  if (a.fmt != Fmt::Q4 && a.fmt != Fmt::Q8) return fail(EFG_EINVAL, "matvec: type must be Q4_0 or Q8_0");
  if (a.cols % 32 != 0) {
    return fail(EFG_EINVAL, "%s needs a row length divisible by 32, got %zu", a.fmt == Fmt::Q4 ? "Q4_0" : "Q8_0",
                a.cols);
  }
  const int n_mat = a.epi == Epi::SwiGLU ? 2 : a.n_jobs;
  if (a.n_jobs < 1 || a.n_jobs > kMaxJobs || (a.epi == Epi::SwiGLU && a.n_jobs != 2))
    return fail(EFG_EINVAL, "matvec: bad job count %d", a.n_jobs);
  if (a.epi == Epi::SwiGLU && a.jobs[0].rows != a.jobs[1].rows)
    return fail(EFG_EINVAL, "matvec: gate and up must have the same rows");
  uint64_t total_rows = 0;
  for (int j = 0; j < n_mat; ++j) {
    if (a.jobs[j].rows && (!a.jobs[j].y || (!a.jobs[j].W && a.cols))) return fail(EFG_EINVAL, "matvec: null pointer");
    total_rows += a.jobs[j].rows;
  }
  if (total_rows == 0) return EFG_OK;
  if (!a.x && a.cols) return fail(EFG_EINVAL, "matvec: null x");
  if (a.cols >= (1ull << 31) || total_rows >= (1ull << 31)) return fail(EFG_EINVAL, "matvec: shape too large");

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;

  KParams k{};
  k.x = a.x;
  k.norm_w = a.norm_w;
  k.norm_eps = a.norm_eps;
  k.err = d_err;
  k.pos = a.pos;
  k.cols = static_cast<uint32_t>(a.cols);
  k.n_jobs = static_cast<uint32_t>(a.epi == Epi::SwiGLU ? 1 : a.n_jobs);
  for (int j = 0; j < n_mat; ++j) k.jobs[j] = a.jobs[j];

  if (a.cols == 0) {  // every dot is over zero blocks: y = 0 (sum32 of zero lanes)
    for (int j = 0; j < (a.epi == Epi::SwiGLU ? 1 : a.n_jobs); ++j) {
      if (!a.jobs[j].rows) continue;
      float* y = a.jobs[j].y;
      if (a.pos) return fail(EFG_EINVAL, "matvec: cols == 0 with a device position");
      if (a.epi == Epi::Add) continue;  // adds zero
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(std::max(1u, std::min(1024u, (a.jobs[j].rows + 255) / 256)));
      cfg.blockDim = dim3(256);
      cfg.stream = stream;
      cfg.attrs = attr;
      cfg.numAttrs = a.pdl ? 1 : 0;
      EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, zero_rows_kernel, y, a.jobs[j].rows), "matvec launch");
    }
    return EFG_OK;
  }

  bool fast = true;
  for (int j = 0; j < n_mat; ++j)
    if (reinterpret_cast<uintptr_t>(a.jobs[j].W) % 16 != 0) fast = false;
  Plan pl = plan_fast(a, *dev);
  fast = fast && pl.ok;

  if (fast) {
    k.S = pl.S;
    k.G = pl.G;
    k.RG = pl.RG;
    k.TR = pl.TR;
    k.NS = pl.NS;
    k.stage_bytes = pl.stage_bytes;
    k.rb_words = static_cast<uint32_t>(a.cols / 32 * (a.fmt == Fmt::Q4 ? 18 : 34) / 4);
    uint32_t t = 0;
    for (uint32_t j = 0; j < k.n_jobs; ++j) {
      k.job_tile_start[j] = t;
      t += (k.jobs[j].rows + pl.TR - 1) / pl.TR;
    }
    k.job_tile_start[k.n_jobs] = t;
    k.tiles_total = t;
    FastFn fn = pick_fast(a.fmt, static_cast<int>(pl.RB), a.epi, a.norm_w != nullptr);
    if (!fn) return fail(EFG_EINVAL, "matvec: no kernel for this configuration");
    if (int st = ensure_smem_attr(reinterpret_cast<const void*>(fn), pl.smem)) return st;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(std::min<uint32_t>(k.tiles_total, static_cast<uint32_t>(dev->sm_count)));
    cfg.blockDim = dim3(32 * (pl.G * pl.RG + 1));
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = a.pdl ? 1 : 0;
    EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, fn, k), "matvec launch");
    return EFG_OK;
  }

  // Generic path. The RMSNorm prologue is not fused there.
  if (a.norm_w) return fail(EFG_EINVAL, "matvec: fused RMSNorm needs cols %% 64 == 0 and 16-byte aligned weights");
  uint32_t t = 0;
  for (uint32_t j = 0; j < k.n_jobs; ++j) {
    k.job_tile_start[j] = t;
    t += k.jobs[j].rows;
  }
  k.job_tile_start[k.n_jobs] = t;
  k.tiles_total = t;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(std::max(1u, std::min<uint32_t>((t + 7) / 8, 8u * dev->sm_count)));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, pick_generic(a.fmt, a.epi), k), "matvec launch");
  return EFG_OK;
}

}  // namespace efg
