// efg_matvec.cu - packed Q4_0 / Q8_0 matvec for B200 (sm_100a).
//
// The reference computes y = W x row by row on CPU threads, one 18/34-byte block at a
// time (src/qkernels.cpp:39-75, 213-297). Here the whole matrix streams from HBM once:
//
//  * One persistent CTA per SM. A producer warp copies row tiles (RB whole rows, a
//    contiguous byte range of the packed matrix, a few KB) into a ring of up to 32
//    shared-memory stages with 1-D bulk async copies (cp.async.bulk, completion counted
//    on an mbarrier), so >100 KB per SM stays in flight, no thread spends instructions
//    moving weights and every byte of HBM is read once. Tile k of a CTA belongs to row
//    group k % RG (the G warps that together cover one row).
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
#include "efg_dot.cuh"
#include "efg_gather.cuh"
#include "efg_host.h"
#include "efg_matvec.cuh"

namespace efg {

namespace {

constexpr int kMaxThreads = 512;  // 1 producer warp + up to 15 consumer warps (4 warps per SMSP: 128 registers)
constexpr int kMaxConsumerWarps = kMaxThreads / 32 - 1;
constexpr int kNormBarrier = 15;  // named barrier id for the RMSNorm reduction

struct KParams {
  const float* x;
  const float* norm_w;
  float norm_eps;
  int* err;
  const int32_t* pos;
  uint32_t cols, rb_words, S, G, H, RG, TR, BPS, NS, stage_bytes, n_jobs, tiles_total;
  uint32_t x_vec4;  // x and norm_w are 16-byte aligned: staged with float4 loads
  uint32_t job_tile_start[kMaxJobs + 1];
  MatvecJobDev jobs[kMaxJobs];
  GatherDev g;  // the in-kernel all-gather of the row-sharded matvec (GATHER kernels only)
};

// Which job a tile belongs to, and its first row.
__device__ __forceinline__ void locate_tile(const KParams& p, uint32_t tile, uint32_t& j, uint32_t& r0,
                                            uint32_t& nrows) {
  j = 0;
  while (j + 1 < p.n_jobs && tile >= p.job_tile_start[j + 1]) ++j;
  r0 = (tile - p.job_tile_start[j]) * p.TR;
  nrows = min(p.TR, p.jobs[j].rows - r0);
}

template <Fmt F, int RB, Epi E, bool NORM, bool GATHER>
__global__ void __launch_bounds__(kMaxThreads, 1) matvec_fast_kernel(const __grid_constant__ KParams p) {
  // A tile (one stage) holds TR = BPS * H * RB/n_mat rows of each matrix and is consumed
  // by one row group: G x H warps, G warps covering the 64-column slots of a row and H
  // warps taking different rows. It is read in BPS batches; in each batch warp (g, h)
  // handles RB rows (for SwiGLU RB/2 gate rows and the same RB/2 up rows, the up rows
  // being stored TR rows on). The CTA's k-th tile (tile = blockIdx.x + k * gridDim.x)
  // goes to stage k % NS and row group k % RG. NS is a multiple of RG, so stage s belongs
  // to row group s % RG alone and its phases are consumed in order.
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t nc = p.G * p.H * p.RG;  // consumer warps
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.NS * p.stage_bytes);
  uint64_t* empty = full + p.NS;
  uint64_t* xready = empty + p.NS;                                                   // x staged
  float* red = reinterpret_cast<float*>(xready + 1);                                 // [RG*H][2][RB][G]
  double* norm_red = reinterpret_cast<double*>(red + 2 * p.RG * p.H * RB * p.G + 2);  // [16]
  float* xs = reinterpret_cast<float*>(norm_red + 16);                          // [S][65]
  constexpr int n_mat = E == Epi::SwiGLU ? 2 : 1;
  constexpr uint32_t RBH = E == Epi::SwiGLU ? RB / 2 : RB;  // rows of each matrix per batch

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < p.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], p.G * p.H);
    }
    mbar_init(xready, 1);
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
    const uint32_t rb = p.rb_words * 4u;
    // Weight tiles requested for this SM return in order, so a deep prefetch would hold
    // back the consumers' read of x by microseconds. Prefetch ~32 KB (it lands while the
    // previous kernel finishes), then wait until x is staged before filling the ring.
    const uint32_t prefetch = std::max(1u, std::min(p.NS, (32768u + p.stage_bytes - 1) / p.stage_bytes));
    uint32_t k = 0, s = 0, round = 0;
    bool ok = true;
    for (uint32_t tile = blockIdx.x; tile < p.tiles_total; tile += gridDim.x, ++k) {
      if (k == prefetch && !mbar_wait(xready, 0, p.err)) {
        ok = false;
        break;
      }
      if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1u, p.err)) {
        ok = false;
        break;
      }
      uint32_t j, r0, nrows;
      locate_tile(p, tile, j, r0, nrows);
      const uint32_t bytes = nrows * rb;
      const uint32_t bulk = bytes & ~15u;
      uint8_t* dst = stages + s * p.stage_bytes;
      // The ragged end of the last tile (bytes % 16) is copied by this thread; the
      // release of the arrive below orders it before the consumers' acquire.
      for (int m = 0; m < n_mat; ++m) {
        const uint8_t* src = p.jobs[E == Epi::SwiGLU ? m : j].W + static_cast<size_t>(r0) * rb;
        uint8_t* d = dst + m * (p.TR * rb);
        for (uint32_t b = bulk; b < bytes; ++b) d[b] = src[b];
      }
      mbar_arrive_expect_tx(&full[s], bulk * n_mat);
      if (bulk) {
        for (int m = 0; m < n_mat; ++m) {
          const uint8_t* src = p.jobs[E == Epi::SwiGLU ? m : j].W + static_cast<size_t>(r0) * rb;
          bulk_g2s(dst + m * (p.TR * rb), src, bulk, &full[s], pol);
        }
      }
      if (++s == p.NS) {
        s = 0;
        ++round;
      }
    }
    if (!ok) {
      // Let copies already issued land before the CTA can exit (bounded as well).
      const uint32_t first = k > p.NS ? k - p.NS : 0;
      for (uint32_t q = first; q < k; ++q) mbar_wait(&full[q % p.NS], (q / p.NS) & 1u, nullptr);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const uint32_t g = warp % p.G, h = (warp / p.G) % p.H, rg = warp / (p.G * p.H);
  const uint32_t slot = g * 32 + lane;
  const bool active = slot < p.S;

  // x is read once per CTA with coalesced loads into a padded shared array (65 floats
  // per 64-column slot, so the per-lane reads below hit 32 different banks), with the
  // RMSNorm folded in: h = w * (x * inv) exactly as src/kernels.cpp:74. Each thread
  // issues up to kXv float4 loads before it uses any (one memory latency, not one per
  // element). The norm weights are model constants: when x fits in one pass they are
  // loaded before waiting for the previous kernel, which wrote x (and y).
  const uint32_t tid = threadIdx.x, nthr = nc * 32;  // consumers are threads [0, nthr)
  constexpr uint32_t kXv = 4;
  const uint32_t n4 = p.cols / 4;
  const bool one_pass = p.x_vec4 && n4 <= kXv * nthr;
  float4 wv[kXv];
  if (NORM && one_pass) {
    const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
#pragma unroll
    for (uint32_t u = 0; u < kXv; ++u) {
      const uint32_t i = tid + u * nthr;
      wv[u] = i < n4 ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  pdl_wait();  // x and y belong to the previous kernel in the stream
  uint32_t epoch = 0;
  if constexpr (GATHER) {
    epoch = gather_epoch(p.g);
    if (blockIdx.x == 0 && tid < 32) gather_announce(p.g, epoch);
  }
  double ss = 0.0;
  if (p.x_vec4) {
    const float4* x4 = reinterpret_cast<const float4*>(p.x);
    for (uint32_t base = tid; base < n4; base += kXv * nthr) {
      float4 v[kXv];
#pragma unroll
      for (uint32_t u = 0; u < kXv; ++u) {
        const uint32_t i = base + u * nthr;
        v[u] = i < n4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (uint32_t u = 0; u < kXv; ++u) {
        const uint32_t i = base + u * nthr;
        if (i < n4) {
          float* d = xs + ((4 * i) >> 6) * 65 + ((4 * i) & 63);
          d[0] = v[u].x;
          d[1] = v[u].y;
          d[2] = v[u].z;
          d[3] = v[u].w;
          if constexpr (NORM) {
            ss += static_cast<double>(v[u].x) * static_cast<double>(v[u].x);
            ss += static_cast<double>(v[u].y) * static_cast<double>(v[u].y);
            ss += static_cast<double>(v[u].z) * static_cast<double>(v[u].z);
            ss += static_cast<double>(v[u].w) * static_cast<double>(v[u].w);
          }
        }
      }
    }
  } else {
    for (uint32_t i = tid; i < p.cols; i += nthr) {
      const float v = p.x[i];
      xs[(i >> 6) * 65 + (i & 63)] = v;
      if constexpr (NORM) ss += static_cast<double>(v) * static_cast<double>(v);
    }
  }
  if constexpr (NORM) {
    // rmsnorm scale from the whole x (src/kernels.cpp:69-73): double sum of squares.
    ss = warp_sum_d(ss);
    if (lane == 0) norm_red[warp] = ss;
    named_barrier(kNormBarrier, nthr);
    double tot = 0.0;
    for (uint32_t w = 0; w < nc; ++w) tot += norm_red[w];
    const double mean = p.cols ? tot / static_cast<double>(p.cols) : 0.0;
    const float inv = static_cast<float>(1.0 / sqrt(mean + static_cast<double>(p.norm_eps)));
    if (p.x_vec4) {
      const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
      for (uint32_t base = tid; base < n4; base += kXv * nthr) {
        float4 w[kXv];
#pragma unroll
        for (uint32_t u = 0; u < kXv; ++u) {
          const uint32_t i = base + u * nthr;
          w[u] = one_pass ? wv[u] : (i < n4 ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f));
        }
#pragma unroll
        for (uint32_t u = 0; u < kXv; ++u) {
          const uint32_t i = base + u * nthr;
          if (i < n4) {
            float* d = xs + ((4 * i) >> 6) * 65 + ((4 * i) & 63);
            d[0] = w[u].x * (d[0] * inv);
            d[1] = w[u].y * (d[1] * inv);
            d[2] = w[u].z * (d[2] * inv);
            d[3] = w[u].w * (d[3] * inv);
          }
        }
      }
    } else {
      for (uint32_t i = tid; i < p.cols; i += nthr) {
        float& h = xs[(i >> 6) * 65 + (i & 63)];
        h = p.norm_w[i] * (h * inv);
      }
    }
  }
  named_barrier(kNormBarrier, nc * 32);
  if (threadIdx.x == 0) mbar_arrive(xready);  // the producer may now fill the whole ring
  float2 xp[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    float lo = 0.f, hi = 0.f;
    if (active) {
      const float* xr = xs + slot * 65 + pair_col<F>(k);
      lo = xr[0];
      hi = xr[pair_step<F>()];
    }
    xp[k] = f2(lo, hi);
  }

  const uint32_t lane_base = smem_addr(stages) + slot * slot_words<F>() * 4u;
  const uint32_t row_bytes = p.rb_words * 4u;
  float* rbase = red + (rg * p.H + h) * 2 * RB * p.G;
  const uint32_t batch_rows = p.H * RBH;  // rows of each matrix per batch
  // After a failed (timed-out) wait a warp stops reading and writing but keeps walking
  // its tiles, so the named barriers of its row group still see every warp.
  bool alive = true;
  uint32_t ready = 0;  // gather: 0 = peers not checked yet, 1 = every peer ready, 2 = gave up
  uint32_t buf = 0, s = rg, phase = 0;
  for (uint32_t tile = blockIdx.x + rg * gridDim.x; tile < p.tiles_total; tile += p.RG * gridDim.x) {
    if (alive && !mbar_wait(&full[s], phase, p.err)) alive = false;
    uint32_t j, r0, nrows;
    locate_tile(p, tile, j, r0, nrows);
    if (!alive) nrows = 0;
    const uint32_t sbase = lane_base + s * p.stage_bytes;
    float* y = p.jobs[j].y + (p.pos ? *p.pos * p.jobs[j].y_pos_stride : 0);
    for (uint32_t b = 0; b < p.BPS; ++b) {
      float acc[RB];
      uint32_t addr[RB];
      bool valid[RB];
#pragma unroll
      for (int i = 0; i < static_cast<int>(RB); ++i) {
        const uint32_t lr = b * batch_rows + h * RBH + i % RBH;  // row within the tile, per matrix
        const uint32_t srow = (E == Epi::SwiGLU && i >= static_cast<int>(RBH)) ? lr + p.TR : lr;
        addr[i] = sbase + srow * row_bytes;
        valid[i] = active && lr < nrows;
      }
      slot_dots<F, static_cast<int>(RB)>(addr, valid, xp, acc);
      if (b + 1 == p.BPS) {
        __syncwarp();
        if (alive && lane == 0) mbar_arrive(&empty[s]);  // all reads of this stage are done
      }
      const float v = warp_reduce_rows<RB>(acc, lane);
      const float mine = __shfl_sync(0xFFFFFFFFu, v, (lane % RB) * (32 / RB));  // lane i < RB: row i
      float total = mine;
      bool writer = lane < static_cast<int>(RB);
      if (p.G > 1) {
        float* rbuf = rbase + buf * RB * p.G;
        if (lane < static_cast<int>(RB)) rbuf[lane * p.G + g] = mine;
        named_barrier(1 + rg * p.H + h, p.G * 32);
        writer = writer && g == 0;
        if (writer) {
          total = 0.f;
          for (uint32_t q = 0; q < p.G; ++q) total += rbuf[lane * p.G + q];
        }
        buf ^= 1u;
      }
      const uint32_t lr = b * batch_rows + h * RBH + lane;
      if constexpr (GATHER) {
        if (g == 0 && ready == 0) ready = gather_wait_ready(p.g, epoch, p.err) ? 1u : 2u;  // warp-uniform
        if (writer && lr < nrows && alive && ready == 1) gather_store(p.g, r0 + lr, total);
      }
      if constexpr (E == Epi::SwiGLU) {
        const float up = __shfl_down_sync(0xFFFFFFFFu, total, RBH);
        if (writer && lane < static_cast<int>(RBH) && lr < nrows) y[r0 + lr] = silu(total) * up;
      } else {
        if (writer && lr < nrows) {
          if constexpr (E == Epi::Add) y[r0 + lr] += total;
          else y[r0 + lr] = total;
        }
      }
    }
    s += p.RG;
    if (s >= p.NS) {
      s -= p.NS;
      phase ^= 1u;
    }
  }
  if constexpr (GATHER) {
    named_barrier(kNormBarrier, nc * 32);  // every store of the CTA into the peers' y is issued
    if (warp == 0) gather_finish(p.g, epoch, p.err);
  }
}

// ------------------------------------------------------------------ generic path
// Any cols % 32 == 0 and any pointer alignment: one warp per row, lanes stride over
// blocks, bytes read one at a time. Used only for shapes the fast path rejects.
template <Fmt F, Epi E, bool GATHER>
__global__ void matvec_generic_kernel(const __grid_constant__ KParams p) {
  pdl_wait();
  pdl_launch_dependents();
  uint32_t epoch = 0;
  if constexpr (GATHER) {
    epoch = gather_epoch(p.g);
    if (blockIdx.x == 0 && threadIdx.x < 32) gather_announce(p.g, epoch);
  }
  bool ready = true;
  constexpr uint32_t BB = F == Fmt::Q4 ? 18 : 34;
  const uint32_t nb = p.cols / 32;
  const int lane = threadIdx.x & 31;
  const uint32_t warps = gridDim.x * (blockDim.x / 32);
  // Work items are single rows here: job_tile_start holds row offsets.
  if constexpr (GATHER) {
    if (blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5) < p.tiles_total)
      ready = gather_wait_ready(p.g, epoch, p.err);  // warps with rows, before their first store
  }
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
      if constexpr (GATHER) {
        if (ready) gather_store(p.g, r, sums[0]);
      }
    }
  }
  if constexpr (GATHER) {
    __syncthreads();  // every store of the CTA into the peers' y is issued
    if (threadIdx.x < 32) gather_finish(p.g, epoch, p.err);
  }
}

// ------------------------------------------------------------------ F32 / F16 / BF16 weights
// y = W x for the plain storage types (src/qkernels.cpp:237-269; the reference's BF16 and F32
// rows are its Stage 2 dot kernels, F16 widens per element): one warp per row, FP32
// accumulation, 16-byte loads of W and x when both are 16-byte aligned (row bytes too).
struct DenseParams {
  const uint8_t* W;
  float* y;
  const float* x;
  uint32_t rows, cols;
  uint64_t row_bytes;
  int vec;
};

template <int QT>
__device__ __forceinline__ float dense_elem(const uint8_t* row, uint32_t c) {
  if constexpr (QT == 0) {
    return __uint_as_float(row[4 * c] | (row[4 * c + 1] << 8) | (row[4 * c + 2] << 16) |
                           (static_cast<uint32_t>(row[4 * c + 3]) << 24));
  } else {
    const uint32_t h = row[2 * c] | (row[2 * c + 1] << 8);
    return QT == 1 ? fp16_to_f32(h) : bf16_to_f32(h);
  }
}

template <int QT>
__global__ void __launch_bounds__(256) dense_matvec_kernel(const __grid_constant__ DenseParams p) {
  pdl_wait();  // x and y belong to the previous kernel in the stream
  pdl_launch_dependents();
  constexpr uint32_t E = QT == 0 ? 4 : 8;  // weights per 16 bytes
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t warps = gridDim.x * (blockDim.x / 32);
  const uint32_t n16 = p.vec ? p.cols / E : 0;
  for (uint32_t r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); r < p.rows; r += warps) {
    const uint8_t* row = p.W + static_cast<uint64_t>(r) * p.row_bytes;
    float acc0 = 0.f, acc1 = 0.f;
    for (uint32_t c = lane; c < n16; c += 32) {
      const uint4 w = __ldcs(reinterpret_cast<const uint4*>(row) + c);  // streamed once
      const float4* xv = reinterpret_cast<const float4*>(p.x) + c * (E / 4);
      if constexpr (QT == 0) {
        const float4 a = __ldg(xv);
        acc0 = fmaf(__uint_as_float(w.x), a.x, acc0);
        acc1 = fmaf(__uint_as_float(w.y), a.y, acc1);
        acc0 = fmaf(__uint_as_float(w.z), a.z, acc0);
        acc1 = fmaf(__uint_as_float(w.w), a.w, acc1);
      } else {
        const float4 a = __ldg(xv), b = __ldg(xv + 1);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        const float xs[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float lo = QT == 1 ? fp16_to_f32(ws[k] & 0xFFFFu) : __uint_as_float(ws[k] << 16);
          const float hi = QT == 1 ? fp16_to_f32(ws[k] >> 16) : __uint_as_float(ws[k] & 0xFFFF0000u);
          acc0 = fmaf(lo, xs[2 * k], acc0);
          acc1 = fmaf(hi, xs[2 * k + 1], acc1);
        }
      }
    }
    for (uint32_t c = n16 * E + lane; c < p.cols; c += 32) acc0 = fmaf(dense_elem<QT>(row, c), p.x[c], acc0);
    const float v = warp_sum(acc0 + acc1);
    if (lane == 0) p.y[r] = v;
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
  return norm ? matvec_fast_kernel<F, RB, E, true, false> : matvec_fast_kernel<F, RB, E, false, false>;
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

// The gather kernels: one plain product (Store, no norm), any RB.
template <Fmt F>
FastFn pick_gather(int rb) {
  switch (rb) {
    case 1: return matvec_fast_kernel<F, 1, Epi::Store, false, true>;
    case 2: return matvec_fast_kernel<F, 2, Epi::Store, false, true>;
    default: return matvec_fast_kernel<F, 4, Epi::Store, false, true>;
  }
}

FastFn pick_fast(Fmt f, int rb, Epi e, bool norm, bool gather) {
  if (gather) {
    if (e != Epi::Store || norm) return nullptr;
    return f == Fmt::Q4 ? pick_gather<Fmt::Q4>(rb) : pick_gather<Fmt::Q8>(rb);
  }
  return f == Fmt::Q4 ? pick_rb<Fmt::Q4>(rb, e, norm) : pick_rb<Fmt::Q8>(rb, e, norm);
}

using GenFn = void (*)(KParams);
GenFn pick_generic(Fmt f, Epi e, bool gather) {
  if (gather) {
    if (e != Epi::Store) return nullptr;
    return f == Fmt::Q4 ? matvec_generic_kernel<Fmt::Q4, Epi::Store, true> : matvec_generic_kernel<Fmt::Q8, Epi::Store, true>;
  }
  if (f == Fmt::Q4) {
    return e == Epi::Store ? matvec_generic_kernel<Fmt::Q4, Epi::Store, false>
           : e == Epi::Add ? matvec_generic_kernel<Fmt::Q4, Epi::Add, false>
                           : matvec_generic_kernel<Fmt::Q4, Epi::SwiGLU, false>;
  }
  return e == Epi::Store ? matvec_generic_kernel<Fmt::Q8, Epi::Store, false>
         : e == Epi::Add ? matvec_generic_kernel<Fmt::Q8, Epi::Add, false>
                         : matvec_generic_kernel<Fmt::Q8, Epi::SwiGLU, false>;
}

struct Plan {
  uint32_t S, G, H, RG, RB, BPS, TR, NS, stage_bytes, tiles;
  size_t smem;
  bool ok;
};

constexpr size_t kSmemBudget = 212 * 1024;
constexpr uint32_t kMaxStages = 48;

// Chooses the shape of the pipeline for one launch. Measured on B200: a CTA's bulk-copy
// ring streams at full rate with stages of >= 16 KB and ~200 KB in flight per SM (4-5 KB
// stages stall at under half rate), and 16 consumer warps hide the arithmetic. The
// candidates are (H warps per stage splitting rows, RB rows per warp per batch, BPS
// batches per stage); each must keep every row group busy when the matrix is large
// enough, with NS a multiple of the row-group count.
Plan plan_fast(const MatvecArgs& a, const DeviceInfo& dev) {
  Plan best{};
  best.ok = false;
  const uint32_t bb = a.fmt == Fmt::Q4 ? 18u : 34u;
  const uint32_t rb = static_cast<uint32_t>(a.cols / 32 * bb);
  const uint32_t S = static_cast<uint32_t>(a.cols / 64);
  const uint32_t G = (S + 31) / 32;
  if (a.cols % 64 != 0 || G < 1 || G > static_cast<uint32_t>(kMaxConsumerWarps)) return best;
  const int n_mat = a.epi == Epi::SwiGLU ? 2 : 1;
  const int nj = a.epi == Epi::SwiGLU ? 1 : a.n_jobs;
  auto tiles_for = [&](uint32_t TR) {
    uint32_t t = 0;
    for (int j = 0; j < nj; ++j) t += (a.jobs[j].rows + TR - 1) / TR;
    return t;
  };
  const size_t xs_bytes = static_cast<size_t>(S) * 65 * 4;
  long best_score = -1;
  for (uint32_t H : {1u, 2u, 4u}) {
    const uint32_t RG = static_cast<uint32_t>(kMaxConsumerWarps) / (G * H);
    if (RG < 1) continue;
    for (uint32_t rbv : {4u, 2u, 1u}) {
      if (a.epi == Epi::SwiGLU && rbv < 2) continue;
      const uint32_t rbh = a.epi == Epi::SwiGLU ? rbv / 2 : rbv;
      for (uint32_t bps : {1u, 2u, 4u}) {
        const uint32_t TR = bps * H * rbh;
        if ((static_cast<uint64_t>(TR) * rb) % 16 != 0) continue;
        const uint64_t stage = (static_cast<uint64_t>(TR) * rb * n_mat + 15) / 16 * 16;
        const size_t tail = 2 * 8 * kMaxStages + 8 + (2 * RG * H * rbv * G + 2) * 4 + 16 * 8 + xs_bytes + 128;
        const size_t budget = std::min(kSmemBudget, dev.smem_optin > tail ? dev.smem_optin - tail : 0);
        uint32_t NS = static_cast<uint32_t>(std::min<uint64_t>(kMaxStages, budget / stage));
        NS = NS / RG * RG;
        if (NS < RG || NS < 2) continue;
        const uint32_t tiles = tiles_for(TR);
        const bool busy = tiles >= static_cast<uint32_t>(dev.sm_count) * RG;
        const long stage_kb = static_cast<long>(std::min<uint64_t>(stage, 16384) / 1024);
        const long flight_kb = static_cast<long>(std::min<uint64_t>(NS * stage, 160 * 1024) / 1024);
        const long warps = static_cast<long>(G * H * RG);
        // busy first (else the most tiles), then stage size, bytes in flight, warps, RB
        const long score = busy ? (1L << 40) + (stage_kb << 28) + (flight_kb << 16) + (warps << 8) + (rbv << 4)
                                : static_cast<long>(tiles) * 64 + rbv;
        if (score > best_score) {
          best_score = score;
          best.S = S;
          best.G = G;
          best.H = H;
          best.RG = RG;
          best.RB = rbv;
          best.BPS = bps;
          best.TR = TR;
          best.NS = NS;
          best.stage_bytes = static_cast<uint32_t>(stage);
          best.tiles = tiles;
          best.smem = NS * stage + 2 * NS * 8 + 8 + (2 * RG * H * rbv * G + 2) * 4 + 16 * 8 + xs_bytes;
          best.ok = true;
        }
      }
    }
  }
  return best;
}

}  // namespace

int launch_dense_matvec(int qtype, float* y, const uint8_t* W, const float* x, size_t rows, size_t cols,
                        cudaStream_t stream, bool pdl) {
  if (qtype < 0 || qtype > 2) return fail(EFG_EINVAL, "matvec: type %d is not F32, F16 or BF16", qtype);
  if (rows == 0) return EFG_OK;
  if (rows >= (1ull << 31) || cols >= (1ull << 31)) return fail(EFG_EINVAL, "matvec: shape too large");
  if (!y || (cols && (!W || !x))) return fail(EFG_EINVAL, "matvec: null pointer");
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  DenseParams p{};
  p.W = W;
  p.y = y;
  p.x = x;
  p.rows = static_cast<uint32_t>(rows);
  p.cols = static_cast<uint32_t>(cols);
  p.row_bytes = static_cast<uint64_t>(cols) * (qtype == 0 ? 4 : 2);
  p.vec = reinterpret_cast<uintptr_t>(W) % 16 == 0 && p.row_bytes % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(std::max<uint64_t>(1, std::min<uint64_t>((rows + 7) / 8, 16ull * dev->sm_count))));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  auto fn = qtype == 0 ? dense_matvec_kernel<0> : qtype == 1 ? dense_matvec_kernel<1> : dense_matvec_kernel<2>;
  EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, fn, p), "matvec launch");
  return EFG_OK;
}

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
  return launch_matvec_on(a, *dev, d_err, stream, false);
}

int launch_matvec_on(const MatvecArgs& a, const DeviceInfo& devinfo, int* d_err, cudaStream_t stream,
                     bool direct_smem_attr) {
  const DeviceInfo* dev = &devinfo;
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
  k.x_vec4 = reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && reinterpret_cast<uintptr_t>(a.norm_w) % 16 == 0 ? 1u : 0u;
  k.norm_eps = a.norm_eps;
  k.err = d_err;
  k.pos = a.pos;
  k.cols = static_cast<uint32_t>(a.cols);
  k.n_jobs = static_cast<uint32_t>(a.epi == Epi::SwiGLU ? 1 : a.n_jobs);
  for (int j = 0; j < n_mat; ++j) k.jobs[j] = a.jobs[j];
  k.g = a.gather;
  if (a.gather.nranks > 0) {
    if (a.gather.nranks > kMaxGatherRanks || a.epi != Epi::Store || a.norm_w || a.pos || a.n_jobs != 1 ||
        a.cols == 0 || a.gather.rank < 0 || a.gather.rank >= a.gather.nranks)
      return fail(EFG_EINVAL, "matvec: the in-kernel gather takes one plain product of cols > 0 rows");
  }

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

  if (q4_mma_flag() && a.small_kernel && matvec_small_ok(a, *dev))
    return launch_matvec_q4_small(a, *dev, d_err, stream, direct_smem_attr);
  if (q4_mma_flag() && matvec_mma_ok(a, *dev)) return launch_matvec_q4_mma(a, *dev, d_err, stream, direct_smem_attr);

  bool fast = true;
  for (int j = 0; j < n_mat; ++j)
    if (reinterpret_cast<uintptr_t>(a.jobs[j].W) % 16 != 0) fast = false;
  Plan pl = plan_fast(a, *dev);
  fast = fast && pl.ok;

  if (fast) {
    k.S = pl.S;
    k.G = pl.G;
    k.H = pl.H;
    k.RG = pl.RG;
    k.TR = pl.TR;
    k.BPS = pl.BPS;
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
    FastFn fn = pick_fast(a.fmt, static_cast<int>(pl.RB), a.epi, a.norm_w != nullptr, k.g.nranks > 0);
    if (!fn) return fail(EFG_EINVAL, "matvec: no kernel for this configuration");
    if (direct_smem_attr) {
      EFG_TRY_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(pl.smem)),
                   "kernel shared-memory attribute");
    } else if (int st = ensure_smem_attr(reinterpret_cast<const void*>(fn), pl.smem)) {
      return st;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(std::min<uint32_t>(k.tiles_total, static_cast<uint32_t>(dev->sm_count)));
    cfg.blockDim = dim3(32 * (pl.G * pl.H * pl.RG + 1));
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
  GenFn gfn = pick_generic(a.fmt, a.epi, k.g.nranks > 0);
  if (!gfn) return fail(EFG_EINVAL, "matvec: the in-kernel gather takes one plain product (no norm, no add)");
  EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, gfn, k), "matvec launch");
  return EFG_OK;
}

}  // namespace efg
