// efg_matvec_mma.cu - Q4_0 matvec with the integer tensor-core MMA (sm_100a).
//
// The CUDA-core kernel (efg_matvec.cu) spends ~2 lane-instructions per Q4_0 weight turning
// codes into floats and multiplying; at ~25 weights per clock per SM that caps it near
// 3 TB/s. Here the arithmetic moves to `mma.sync.m16n8k32.s8.s8.s32`, exactly:
//
//  * A (16 x 32): a code c becomes the int8 (c - 8) * 16 with one LOP3 per 4 codes:
//    (w ^ 0x80808080) & 0xF0F0F0F0 for the high nibbles, the same on w << 4 for the low
//    ones. Byte j of a block's 16 code bytes holds columns j and j + 16, which is the
//    m16n8k32 fragment's split of K.
//  * B (32 x 8): x of a block as a fixed-point integer X = round(x * 2^s), |X| < 2^30,
//    written as four balanced int8 digits (X = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3). The
//    block's s makes its largest |x| use the full range, so each x is kept to 2^-31 of
//    its block's largest |x|.
//  * One MMA covers 8 rows and a block pair: A rows 0..7 are the even block of 8 tile
//    rows, A rows 8..15 the odd block of the same rows; B columns 0..3 are the even
//    block's digits, 4..7 the odd block's. The int32 products are exact; each lane keeps
//    one useful pair of digit sums, c_lo + 256 c_hi, which becomes a float scaled by
//    d * 2^-s / 16 (or 2^(16-s) / 16 for digits 2, 3) and accumulates in FP32 with one
//    FMA. The error against the exact dot is below 2^-31 * sum over blocks of
//    max|x| * sum|w| plus FP32 accumulation rounding, far inside the 1e-5 of sum |w x|
//    the reference's tests allow for realistic activations.
//
// Streaming: one 2-D TMA tensor copy per stage. W is seen as [rows][row bytes / 8] of
// 8-byte elements and a stage is the box {146 elements, 16 rows} at the K segment's
// start (segments of 64 blocks, 1152 bytes, so x is a multiple of 16 bytes): it lands as
// 16 rows of 1168 bytes, 16 bytes (mod 128) apart, so the 8 rows a fragment load touches
// fall in 8 different bank quads. The 16 bytes past the segment are the next segment's
// (or zero fill past the row end) and are not read; rows past the matrix are zero fill.
// One instruction per 18.7 KB stage keeps the copy engine ahead of HBM; 16 separate 1-D
// copies per stage held the producer warp in the copy instruction half of the time.
//
// Work: a row tile is taken by a group of Wk * nseg consumer warps, Wk per K segment,
// each with a fixed share of the segment's block pairs, so the stages of a tile are
// consumed at once and the ring drains in order; the group adds its 16 row sums in warp
// order after one named barrier per tile, so results do not depend on timing. Groups
// take every Gs-th tile of the CTA. The producer issues two stages, then waits until
// every consumer warp has issued its x loads, so those reach the memory system ahead of
// the ring's fill. A CTA whose x holds a non-finite value, or a block maximum outside
// [2^-69, 2^100), computes its rows with plain FP32 dots instead.
#include <algorithm>
#include <cstdint>

#include <cuda.h>

#include "../../include/efg.h"
#include "efg_device.cuh"
#include "efg_dot.cuh"
#include "efg_gather.cuh"
#include "efg_gemm.cuh"
#include "efg_host.h"
#include "efg_matvec.cuh"

#ifndef EFG_MMA_MIN_BYTES
#define EFG_MMA_MIN_BYTES (48ull << 20)  // matrices from this size take the MMA kernel
#endif

namespace efg {
namespace {

constexpr int kMmaConsumers = 12;
constexpr int kMmaThreads = (kMmaConsumers + 1) * 32;
constexpr uint32_t kTileRows = 16;
constexpr uint32_t kMinBlk = 64;          // cols >= 2048
constexpr uint32_t kMaxBlk = 256;         // cols <= 8192
constexpr uint32_t kSegBlk = 64;          // K segment: 64 blocks, 1152 bytes of a row
constexpr uint32_t kBoxElems = 146;       // box row: 1168 bytes = 1152 + 16 (8-byte elements)
constexpr uint32_t kRowStride = kBoxElems * 8;
constexpr uint32_t kStageBytes = kTileRows * kRowStride;  // 18688 = 146 * 128
constexpr uint32_t kMaxStages = 16;
constexpr uint32_t kGroupBarrier0 = 2;    // named barriers 2 .. 2 + Gs - 1 <= 15 (1: all consumers)
constexpr uint32_t kPrefetchStages = 2;   // stages the producer issues before the x loads

// Shared memory, fixed part first: full[S] | empty[S] | xready | tile_id[S] | bad_x |
// dred[C] (f64) | red[C][2][16] (f32) | xsc[2 nblk] | xdig[nblk * 128] | ring (128-aligned).
constexpr uint32_t kDredOffset = (2 * kMaxStages * 8 + 8 + kMaxStages * 4 + 4 + 7) / 8 * 8;
constexpr uint32_t kRedOffset = kDredOffset + kMmaConsumers * 8;
constexpr uint32_t kXscOffset = kRedOffset + kMmaConsumers * 2 * kTileRows * 4;

struct MmaParams {
  CUtensorMap maps[kMaxJobs];  // one per job: W as [rows][rb / 8] u64, box {146, 16}
  const float* x;
  const float* norm_w;
  float norm_eps;
  int* err;
  const int32_t* pos;
  uint32_t cols, nblk, rb, nseg;
  uint32_t NS, ring_offset;
  uint32_t Wk, Gs;  // warps per K segment, tile groups (of Wk * nseg warps)
  uint32_t rt_total, n_jobs;
  uint32_t job_rt_start[kMaxJobs + 1];
  MatvecJobDev jobs[kMaxJobs];
  GatherDev g;  // the in-kernel all-gather of the row-sharded matvec (GATHER kernels only)
};

__device__ __forceinline__ uint32_t a_lo(uint32_t w) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x28;" : "=r"(r) : "r"(w << 4), "r"(0x80808080u), "r"(0xF0F0F0F0u));
  return r;  // ((w << 4) ^ 0x80808080) & 0xF0F0F0F0
}
__device__ __forceinline__ uint32_t a_hi(uint32_t w) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x28;" : "=r"(r) : "r"(w), "r"(0x80808080u), "r"(0xF0F0F0F0u));
  return r;
}

// No side effects and no memory operands: the compiler may schedule it freely among the
// shared-memory loads of neighbouring block pairs.
__device__ __forceinline__ void mma_s8(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int (&c)[4]) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// x -> fixed-point digits of one 32-column block for the B fragments. Lane (q = lane >> 3,
// c = lane & 7) holds columns 4c..4c+3 of block b (h, after any RMSNorm); the 8 lanes of the
// block find its largest |x| and write its four int8 digit planes and two scales (2^(-4-s),
// 2^(12-s)). For an odd block, columns 4c..4c+3 are B-fragment columns k = 16 v2 + 4 t + v0
// with v2 = c / 4, t = c % 4, so digit g of the four is one 32-bit word at [t][g][v2]; even
// blocks use the K order in which the consumers read their codes (two half-words). Returns
// false (the same on every lane of the warp) when one of the warp's four blocks holds a
// non-finite value or a maximum outside [2^-69, 2^100): the caller then uses plain FP32 dots,
// so that d * 2^-s / 16 stays a normal float for every FP16 d. The 8 lanes of a block past the
// caller's range pass write = false (and h = 0): they take part in the warp's vote and store
// nothing.
__device__ __forceinline__ bool x_block_digits(const float (&h)[4], uint32_t b, uint32_t c, uint8_t* xdig,
                                               float* xsc, bool write = true) {
  float amax = fmaxf(fmaxf(fabsf(h[0]), fabsf(h[1])), fmaxf(fabsf(h[2]), fabsf(h[3])));
  const bool fin = isfinite(h[0]) && isfinite(h[1]) && isfinite(h[2]) && isfinite(h[3]);
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  const int e = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu) - 127;
  if (__any_sync(0xFFFFFFFFu, !fin || (amax != 0.f && (e < -69 || e >= 100)))) return false;
  if (!write) return true;
  const int s = amax == 0.f ? 0 : 29 - e;  // |x| * 2^s < 2^30; -70 <= s <= 98
  // 2^s, 2^(-4-s) and 2^(12-s) are normal floats for these s: built from their bits.
  // x * 2^s is exact wherever rint can see it (|x * 2^s| >= 2^-126 or it rounds to 0).
  const float p2s = __uint_as_float(static_cast<uint32_t>(s + 127) << 23);
  uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int v0 = 0; v0 < 4; ++v0) {
    int X = __float2int_rn(h[v0] * p2s);
    const int d0 = static_cast<int8_t>(X & 0xFF);
    X = (X - d0) >> 8;
    const int d1 = static_cast<int8_t>(X & 0xFF);
    X = (X - d1) >> 8;
    const int d2 = static_cast<int8_t>(X & 0xFF);
    const int d3 = (X - d2) >> 8;
    words[0] |= (static_cast<uint32_t>(d0) & 0xFFu) << (8 * v0);
    words[1] |= (static_cast<uint32_t>(d1) & 0xFFu) << (8 * v0);
    words[2] |= (static_cast<uint32_t>(d2) & 0xFFu) << (8 * v0);
    words[3] |= (static_cast<uint32_t>(d3) & 0xFFu) << (8 * v0);
  }
  const uint32_t c3 = c & 3u, v2 = c >> 2;
  if (b & 1u) {  // odd block: natural order, lane t holds code bytes 4t..4t+3
    uint32_t* base = reinterpret_cast<uint32_t*>(xdig + b * 128 + c3 * 32 + v2 * 4);
#pragma unroll
    for (int gd = 0; gd < 4; ++gd) base[gd * 2] = words[gd];
  } else {
    // even block: lane t holds code bytes 2+4t..5+4t (t < 3) and 0, 1, 14, 15 (t = 3),
    // so columns (4 c3, 4 c3 + 1) and (4 c3 + 2, 4 c3 + 3) land in two half-words
    const uint32_t tA = c3 == 0 ? 3u : c3 - 1, vA = c3 == 0 ? 0u : 2u;
    const uint32_t tB = c3 == 3 ? 3u : c3, vB = c3 == 3 ? 2u : 0u;
    uint8_t* base = xdig + b * 128 + v2 * 4;
#pragma unroll
    for (int gd = 0; gd < 4; ++gd) {
      *reinterpret_cast<uint16_t*>(base + tA * 32 + gd * 8 + vA) = static_cast<uint16_t>(words[gd]);
      *reinterpret_cast<uint16_t*>(base + tB * 32 + gd * 8 + vB) = static_cast<uint16_t>(words[gd] >> 16);
    }
  }
  if (c == 0) {
    xsc[2 * b] = __uint_as_float(static_cast<uint32_t>(123 - s) << 23);      // digits 0, 1: 2^(-4-s)
    xsc[2 * b + 1] = __uint_as_float(static_cast<uint32_t>(139 - s) << 23);  // digits 2, 3: 2^(12-s)
  }
  return true;
}

// Which job a row tile belongs to and its first row.
__device__ __forceinline__ void locate_rt(const MmaParams& p, uint32_t rt, uint32_t& j, uint32_t& r0, uint32_t& nrows) {
  j = 0;
  while (j + 1 < p.n_jobs && rt >= p.job_rt_start[j + 1]) ++j;
  r0 = (rt - p.job_rt_start[j]) * kTileRows;
  nrows = min(kTileRows, p.jobs[j].rows - r0);
}

template <Epi E, bool NORM, bool GATHER>
__global__ void __launch_bounds__(kMmaThreads, 1) matvec_q4_mma_kernel(const __grid_constant__ MmaParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* xready = empty + kMaxStages;
  volatile uint32_t* tile_id = reinterpret_cast<volatile uint32_t*>(xready + 1);
  volatile int* bad_x = reinterpret_cast<volatile int*>(tile_id + kMaxStages);
  double* dred = reinterpret_cast<double*>(smem + kDredOffset);   // [consumer warps]
  float* red = reinterpret_cast<float*>(smem + kRedOffset);       // [consumer warp][2][16]
  float* xsc = reinterpret_cast<float*>(smem + kXscOffset);       // [nblk][2]
  uint8_t* xdig = reinterpret_cast<uint8_t*>(xsc + 2 * p.nblk);   // [nblk][4 t][4 g][8 bytes]
  uint8_t* ring = smem + p.ring_offset;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < p.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], p.Wk);
      tile_id[s] = 0xFFFFFFFFu;
    }
    mbar_init(xready, kMmaConsumers);
    *bad_x = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  const uint32_t rt_b = static_cast<uint32_t>(static_cast<uint64_t>(p.rt_total) * blockIdx.x / gridDim.x);
  const uint32_t rt_e = static_cast<uint32_t>(static_cast<uint64_t>(p.rt_total) * (blockIdx.x + 1) / gridDim.x);
  const uint32_t R = rt_e - rt_b;

  if (warp == kMmaConsumers) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    const uint64_t pol = l2_evict_first_policy();
    uint32_t gt = 0;
    bool ok = true;
    for (uint32_t tl = 0; tl < R && ok; ++tl) {
      uint32_t j, r0, nrows;
      locate_rt(p, rt_b + tl, j, r0, nrows);
      for (uint32_t ks = 0; ks < p.nseg; ++ks, ++gt) {
        const uint32_t s = gt % p.NS, gen = gt / p.NS;
        if (gt == kPrefetchStages && !mbar_wait(xready, 0, p.err)) {
          ok = false;
          break;
        }
        if (gen > 0 && !mbar_wait(&empty[s], (gen - 1) & 1u, p.err)) {
          ok = false;
          break;
        }
        tile_id[s] = gt;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_2d(ring + s * kStageBytes, &p.maps[j], static_cast<int32_t>(ks * kSegBlk * 18 / 8),
                    static_cast<int32_t>(r0), &full[s], pol);
      }
    }
    // copies issued into the ring land before the CTA may exit (bounded)
    for (uint32_t q = gt > p.NS ? gt - p.NS : 0; q < gt; ++q) mbar_wait(&full[q % p.NS], (q / p.NS) & 1u, nullptr);
    return;
  }

  // -------------------------------------------------------------- consumers
  const uint32_t tid = threadIdx.x, nthr = kMmaConsumers * 32;
  pdl_wait();  // x, norm weights and y belong to the previous kernel in the stream
  uint32_t epoch = 0;
  if constexpr (GATHER) {
    epoch = gather_epoch(p.g);
    if (blockIdx.x == 0 && tid < 32) gather_announce(p.g, epoch);
  }
  float inv = 1.f;
  if constexpr (NORM) {  // rmsnorm scale (src/kernels.cpp:69-73): double sum of squares
    double ss = 0.0;
    for (uint32_t i = tid; i < p.cols; i += nthr) {
      const double v = static_cast<double>(__ldg(p.x + i));
      ss += v * v;
    }
    ss = warp_sum_d(ss);
    if (lane == 0) dred[warp] = ss;
    named_barrier(1, nthr);
    double tot = 0.0;
    for (int w = 0; w < kMmaConsumers; ++w) tot += dred[w];
    const double mean = p.cols ? tot / static_cast<double>(p.cols) : 0.0;
    inv = static_cast<float>(1.0 / sqrt(mean + static_cast<double>(p.norm_eps)));
  }
  // x -> per-block fixed-point digits (x_block_digits). 8 lanes per block, 4 consecutive
  // columns per lane (one float4), 4 blocks per warp step; a warp's loads are all issued first.
  {
    const uint32_t q = lane >> 3, c = lane & 7;
    constexpr uint32_t kSteps = kMaxBlk / (4 * kMmaConsumers) + 1;
    float4 hv[kSteps];
#pragma unroll
    for (uint32_t i = 0; i < kSteps; ++i) {
      const uint32_t b = (warp + i * kMmaConsumers) * 4 + q;
      hv[i] = b < p.nblk ? __ldg(reinterpret_cast<const float4*>(p.x) + b * 8 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // the loads above are issued; the arrive (an asm with a memory clobber) stays after them
    __syncwarp();
    if (lane == 0) mbar_arrive(xready);
#pragma unroll
    for (uint32_t i = 0; i < kSteps; ++i) {
      const uint32_t b = (warp + i * kMmaConsumers) * 4 + q;
      if ((warp + i * kMmaConsumers) * 4 >= p.nblk) break;  // uniform per warp (nblk % 4 == 0)
      float h[4] = {hv[i].x, hv[i].y, hv[i].z, hv[i].w};
      if constexpr (NORM) {  // w * (x * inv), src/kernels.cpp:74
        const float4 nw = __ldg(reinterpret_cast<const float4*>(p.norm_w) + b * 8 + c);
        h[0] = nw.x * (h[0] * inv);
        h[1] = nw.y * (h[1] * inv);
        h[2] = nw.z * (h[2] * inv);
        h[3] = nw.w * (h[3] * inv);
      }
      if (!x_block_digits(h, b, c, xdig, xsc)) {  // warp-uniform
        if (lane == 0) *bad_x = 1;
        continue;
      }
    }
  }
  named_barrier(1, nthr);
  const bool fallback = *bad_x != 0;
  const uint32_t SG = p.Wk * p.nseg;  // warps per tile
  const uint32_t gi = warp / SG, u = warp % SG, ks = u / p.Wk, kidx = u % p.Wk;
  // Consumer warps beyond Gs * SG have no tiles (with the gather they still meet the others
  // at the closing barrier).
  if (!GATHER && gi >= p.Gs) return;
  // this warp's share of its segment: block pairs [p0, p1)
  const uint32_t kb = min(kSegBlk, p.nblk - ks * kSegBlk);
  const uint32_t p0 = (kb / 2) * kidx / p.Wk, p1 = (kb / 2) * (kidx + 1) / p.Wk;
  const uint32_t g = lane >> 2, t = lane & 3;
  // Lane (g, t) holds one useful sum per MMA: t < 2 its C row g, columns 2t, 2t+1 (even
  // block, digits 2t, 2t+1); t >= 2 its C row g + 8, columns 2t, 2t+1 (odd block, digits
  // 2t-4, 2t-3). Its scale is xsc[2 blk_e + t] either way.
  //
  // Words of a 36-byte pair (w = 9 pr): w holds d_e and even codes 0, 1; w+1..w+3 even
  // codes 2..13; w+4 even codes 14, 15 and d_o; w+5..w+8 odd codes. Lane t takes
  // X1 = word w+1+t and X2 = word w (t = 2: w+4): even codes = X1 (t < 3) or bytes
  // {X2.2, X2.3, X1.0, X1.1} (t = 3), its d = d_e (t < 2) or d_o; the x digits of even
  // blocks are stored in this order. Odd codes = word w+5+t.
  const uint32_t x1_off = 1 + t, x2_off = t == 2 ? 4u : 0u;
  const uint32_t sel_code = t == 3 ? 0x1076u : 0x3210u;
  const uint32_t sel_d = t < 2 ? 0x5454u : (t == 2 ? 0x7676u : 0x3232u);
  const bool c_hi = t >= 2;
  // B fragment of lane (g, t): column g, i.e. digit g & 3 of the even (g < 4) or odd block
  const uint2* xd = reinterpret_cast<const uint2*>(xdig + (g >> 2) * 128 + (t * 4 + (g & 3u)) * 8);  // + 16 / block
  const float* xs_l = xsc + t;                                                                          // + 2 / block
  const uint32_t off_g = g * kRowStride, off_g8 = (g + 8) * kRowStride;
  bool ok = true;
  uint32_t ready = 0;  // gather: 0 = peers not checked yet, 1 = every peer ready, 2 = gave up
  uint32_t m = 0;      // tiles this group has finished
  for (uint32_t tl = gi; gi < p.Gs && tl < R; tl += p.Gs, ++m) {
    uint32_t j, r0, nrows;
    locate_rt(p, rt_b + tl, j, r0, nrows);
    float acc_g = 0.f, acc_g8 = 0.f;  // MMA path: rows g, g + 8
    float facc[kTileRows];            // fallback path: every row, this lane's columns
#pragma unroll
    for (int r = 0; r < static_cast<int>(kTileRows); ++r) facc[r] = 0.f;
    const uint32_t gt = tl * p.nseg + ks;
    const uint32_t s = gt % p.NS;
    // the slot must carry this stage (its sequence number), then its bytes
    if (ok && tile_id[s] != gt) {
      const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
      for (uint32_t i = 0; tile_id[s] != gt; ++i) {
        __nanosleep(32);  // leave the issue slots to the warps that compute
        if ((i & 63u) == 63u && (error_raised(p.err) || globaltimer_ns() - t0 > kWaitTimeoutNs)) {
          record_error(p.err, EFG_ETIMEOUT);
          ok = false;
          break;
        }
      }
    }
    ok = ok && mbar_wait(&full[s], (gt / p.NS) & 1u, p.err);
    if (ok && !fallback) {
      // Plain shared loads: the mbarrier wait above (an asm with a memory clobber) keeps
      // them after the stage's bytes have landed.
      const uint32_t* rw = reinterpret_cast<const uint32_t*>(ring + s * kStageBytes + off_g);
      const uint32_t* rw8 = reinterpret_cast<const uint32_t*>(ring + s * kStageBytes + off_g8);
#pragma unroll 4
      for (uint32_t pr = p0; pr < p1; ++pr) {
        const uint32_t w = pr * 9;  // a block pair is 36 bytes
        const uint32_t X1 = rw[w + x1_off], X2 = rw[w + x2_off], Y = rw[w + 5 + t];
        const uint32_t X18 = rw8[w + x1_off], X28 = rw8[w + x2_off], Y8 = rw8[w + 5 + t];
        const uint32_t ce = __byte_perm(X1, X2, sel_code), ce8 = __byte_perm(X18, X28, sel_code);
        const uint32_t db = __byte_perm(X1, X2, sel_d), db8 = __byte_perm(X18, X28, sel_d);
        const uint32_t blk = ks * kSegBlk + 2 * pr;
        const uint2 bf = xd[blk * 16];
        const float sc = xs_l[2 * blk];
        const uint32_t a[4] = {a_lo(ce), a_lo(Y), a_hi(ce), a_hi(Y)};
        const uint32_t a8[4] = {a_lo(ce8), a_lo(Y8), a_hi(ce8), a_hi(Y8)};
        int c[4], c8[4];
        mma_s8(a, bf.x, bf.y, c);
        mma_s8(a8, bf.x, bf.y, c8);
        const int v = (c_hi ? c[2] : c[0]) + ((c_hi ? c[3] : c[1]) << 8);
        const int v8 = (c_hi ? c8[2] : c8[0]) + ((c_hi ? c8[3] : c8[1]) << 8);
        acc_g = fmaf(static_cast<float>(v), half_bits_to_float(db) * sc, acc_g);
        acc_g8 = fmaf(static_cast<float>(v8), half_bits_to_float(db8) * sc, acc_g8);
      }
    } else if (ok) {
      // plain FP32 dots (non-finite or out-of-range x): this warp's blocks, lane-strided
      const uint8_t* st = ring + s * kStageBytes;
      for (uint32_t r = 0; r < nrows; ++r)
        for (uint32_t bb = 2 * p0 + lane; bb < 2 * p1; bb += 32) {
          const uint8_t* blkp = st + r * kRowStride + bb * 18;
          const float d = fp16_to_f32(blkp[0] | (blkp[1] << 8));
          const uint32_t col0 = (ks * kSegBlk + bb) * 32;
          float sacc = 0.f;
          for (int k = 0; k < 32; ++k) {
            const int cd = (k < 16 ? (blkp[2 + k] & 15) : (blkp[2 + k - 16] >> 4)) - 8;
            float xv = __ldg(p.x + col0 + k);
            if constexpr (NORM) xv = __ldg(p.norm_w + col0 + k) * (xv * inv);
            sacc += static_cast<float>(cd) * xv;
          }
#pragma unroll
          for (int qq = 0; qq < static_cast<int>(kTileRows); ++qq)
            if (qq == static_cast<int>(r)) facc[qq] += d * sacc;
        }
    }
    __syncwarp();
    if (ok && lane == 0) mbar_arrive(&empty[s]);  // every read of this stage is done
    // this warp's 16 row sums -> red[warp][m & 1], then the group adds them in warp order
    float* mine = red + (warp * 2 + (m & 1u)) * kTileRows;
    if (!fallback) {
      acc_g += __shfl_xor_sync(0xFFFFFFFFu, acc_g, 1);
      acc_g += __shfl_xor_sync(0xFFFFFFFFu, acc_g, 2);
      acc_g8 += __shfl_xor_sync(0xFFFFFFFFu, acc_g8, 1);
      acc_g8 += __shfl_xor_sync(0xFFFFFFFFu, acc_g8, 2);
      if (t == 0) {
        mine[g] = acc_g;
        mine[g + 8] = acc_g8;
      }
    } else {
#pragma unroll
      for (int qq = 0; qq < static_cast<int>(kTileRows); ++qq) {
        const float v = warp_sum(facc[qq]);
        if (lane == 0) mine[qq] = v;
      }
    }
    // Two buffers per warp: buffer m & 1 is rewritten two tiles later, after the group
    // barrier of tile m + 1, which the group's first warp passes only once it has read
    // tile m's sums.
    if (SG > 1)
      named_barrier(kGroupBarrier0 + gi, SG * 32);
    else
      __syncwarp();
    if (u == 0) {
      if constexpr (GATHER) {
        if (ready == 0) ready = gather_wait_ready(p.g, epoch, p.err) ? 1u : 2u;  // the whole warp
      }
      if (lane < nrows) {
        float v = 0.f;
        for (uint32_t k = 0; k < SG; ++k) v += red[((gi * SG + k) * 2 + (m & 1u)) * kTileRows + lane];
        float* y = p.jobs[j].y + (p.pos ? *p.pos * p.jobs[j].y_pos_stride : 0);
        if (ok) y[r0 + lane] = E == Epi::Add ? y[r0 + lane] + v : v;
        if constexpr (GATHER) {
          if (ok && ready == 1) gather_store(p.g, r0 + lane, v);
        }
      }
    }
  }
  if constexpr (GATHER) {
    named_barrier(1, nthr);  // every store of the CTA into the peers' y is issued
    if (warp == 0) gather_finish(p.g, epoch, p.err);
  }
}

using MmaFn = void (*)(MmaParams);

MmaFn pick_mma(Epi e, bool norm, bool gather) {
  if (gather) return e == Epi::Store && !norm ? matvec_q4_mma_kernel<Epi::Store, false, true> : nullptr;
  if (e == Epi::Add)
    return norm ? matvec_q4_mma_kernel<Epi::Add, true, false> : matvec_q4_mma_kernel<Epi::Add, false, false>;
  return norm ? matvec_q4_mma_kernel<Epi::Store, true, false> : matvec_q4_mma_kernel<Epi::Store, false, false>;
}

struct MmaPlan {
  uint32_t nseg, NS, ring_offset, Wk, Gs;
  size_t smem;
};

bool plan_mma(uint32_t nblk, const DeviceInfo& dev, MmaPlan& pl) {
  if (nblk < kMinBlk || nblk > kMaxBlk || nblk % 8 != 0) return false;
  pl.nseg = (nblk + kSegBlk - 1) / kSegBlk;
  pl.ring_offset = (kXscOffset + nblk * 8 + nblk * 128 + 127) / 128 * 128;
  const size_t optin = static_cast<size_t>(dev.smem_optin);
  if (optin <= pl.ring_offset) return false;
  pl.NS = static_cast<uint32_t>(std::min<size_t>(kMaxStages, (optin - pl.ring_offset) / kStageBytes));
  if (pl.NS < 2) return false;
  // 32 block pairs per stage, Wk warps on each: the Wk in 2..4 that leaves the fewest of
  // the consumer warps idle (groups of Wk * nseg warps), the smaller Wk on ties
  pl.Wk = 0;
  uint32_t best_idle = kMmaConsumers + 1;
  for (uint32_t wk = 2; wk <= 4; ++wk) {
    const uint32_t sg = wk * pl.nseg;
    if (sg > static_cast<uint32_t>(kMmaConsumers)) break;
    const uint32_t idle = kMmaConsumers % sg;
    if (idle < best_idle) {
      best_idle = idle;
      pl.Wk = wk;
    }
  }
  if (pl.Wk == 0) return false;
  pl.Gs = kMmaConsumers / (pl.Wk * pl.nseg);
  pl.smem = pl.ring_offset + static_cast<size_t>(pl.NS) * kStageBytes;
  return true;
}

// W (rows x rb bytes, 16-byte aligned) as [rows][rb / 8] u64 with the box {146, 16}; the
// box may reach past the row (zero fill) and past the last row (zero fill).
bool encode_w_map(CUtensorMap* m, const uint8_t* W, uint32_t rows, uint32_t rb) {
  return encode_u64_rows_map(m, W, rows, rb, kBoxElems, kTileRows);
}

// ------------------------------------------------------------------ small matrices
// Q4_0 matrices of a few MB (every decode-step matrix of a TinyLlama-sized model) are bound by
// the chain of dependent launches, not by HBM: a matvec can only start on x once the kernel
// that wrote x has finished. This kernel is shaped for that chain:
//  * Each CTA owns a few 8-row units (8 rows of every K segment) and fetches all of their
//    bytes with 2-D TMA copies the moment it starts, before waiting for the previous kernel
//    (the weights are static: weight prefetch). It needs at most ~100 KB of shared memory and
//    256 threads, so the next launch's CTA fits beside it on the same SM and fetches its own
//    weights while this one computes: the weight stream of launch i + 1 overlaps launch i.
//  * After the grid-dependency wait, each of the 8 warps reads only its own K range of x
//    (one round of float4 loads), turns it into fixed-point digits (x_block_digits) in its
//    own piece of shared memory, and multiplies it against every unit of the CTA with the
//    exact integer MMA of the large kernel: one m16n8k32 per 8 rows and block pair.
//  * The warps' row partials meet once in shared memory and are added in warp order (one
//    CTA barrier), so results are deterministic. RMSNorm, residual-add, SwiGLU (gate and up
//    units side by side) and a device-side output position are fused as in the other kernels.
constexpr int kSmallWarps = 8;
constexpr int kSmallThreads = kSmallWarps * 32;
constexpr uint32_t kUnitRows = 8;
constexpr uint32_t kSlotBytes = kUnitRows * kRowStride;  // one 8-row box of one K segment: 9344
constexpr uint32_t kSmallMaxSlots = 10;                  // units x matrices x segments per CTA
constexpr uint32_t kSmallMaxUnits = 10;
constexpr size_t kSmallSmemCap = 108 * 1024;             // two CTAs (two launches) per SM

struct SmallParams {
  CUtensorMap maps[kMaxJobs];  // W as [rows][rb / 8] u64, box {146, 8}
  const float* x;
  const float* norm_w;
  float norm_eps;
  int* err;
  const int32_t* pos;
  uint32_t cols, nblk, nseg, npairs;
  uint32_t units_total, n_jobs;  // SwiGLU: one unit space (gate's), two matrices per unit
  uint32_t job_unit_start[kMaxJobs + 1];
  MatvecJobDev jobs[kMaxJobs];
  uint32_t xsc_offset, xdig_offset, red_offset, w_offset;
};

__device__ __forceinline__ void locate_unit(const SmallParams& p, uint32_t u, uint32_t& j, uint32_t& r0,
                                            uint32_t& nrows) {
  j = 0;
  while (j + 1 < p.n_jobs && u >= p.job_unit_start[j + 1]) ++j;
  r0 = (u - p.job_unit_start[j]) * kUnitRows;
  nrows = min(kUnitRows, p.jobs[j].rows - r0);
}

template <Epi E, bool NORM>
__global__ void __launch_bounds__(kSmallThreads, 2) matvec_q4_small_kernel(const __grid_constant__ SmallParams p) {
  constexpr uint32_t NM = E == Epi::SwiGLU ? 2 : 1;  // matrices per unit
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);            // [kSmallMaxUnits]
  double* dred = reinterpret_cast<double*>(smem + 128);         // [kSmallWarps]
  float* xsc = reinterpret_cast<float*>(smem + p.xsc_offset);   // [nblk][2]
  uint8_t* xdig = smem + p.xdig_offset;                         // [nblk][128]
  float* red = reinterpret_cast<float*>(smem + p.red_offset);   // [warp][unit][NM][8]
  uint8_t* wbuf = smem + p.w_offset;                            // [unit][NM][seg] slots
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t u_b = static_cast<uint32_t>(static_cast<uint64_t>(p.units_total) * blockIdx.x / gridDim.x);
  const uint32_t u_e = static_cast<uint32_t>(static_cast<uint64_t>(p.units_total) * (blockIdx.x + 1) / gridDim.x);
  const uint32_t nu = u_e - u_b;
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < nu; ++i) mbar_init(&bar[i], 1);
    fence_barrier_init();
    const uint64_t pol = l2_evict_first_policy();
    for (uint32_t i = 0; i < nu; ++i) {
      uint32_t j, r0, nrows;
      locate_unit(p, u_b + i, j, r0, nrows);
      mbar_arrive_expect_tx(&bar[i], NM * p.nseg * kSlotBytes);
      for (uint32_t m = 0; m < NM; ++m)
        for (uint32_t ks = 0; ks < p.nseg; ++ks)
          tma_load_2d(wbuf + ((i * NM + m) * p.nseg + ks) * kSlotBytes, &p.maps[E == Epi::SwiGLU ? m : j],
                      static_cast<int32_t>(ks * kSegBlk * 18 / 8), static_cast<int32_t>(r0), &bar[i], pol);
    }
  }
  __syncthreads();  // the barriers are initialised before anyone waits on them
  pdl_launch_dependents();

  // this warp's K range: block pairs [p0, p1) of every row, blocks [2 p0, 2 p1)
  const uint32_t p0 = p.npairs * warp / kSmallWarps, p1 = p.npairs * (warp + 1) / kSmallWarps;
  const uint32_t b0 = 2 * p0, nb = 2 * (p1 - p0);
  constexpr uint32_t kSteps = kMaxBlk / kSmallWarps / 4 + 1;  // float4 loads per lane, at most
  const uint32_t q = lane >> 3, c = lane & 7;
  float4 nwv[kSteps];
  if constexpr (NORM) {  // model constants: fetched before the wait
#pragma unroll
    for (uint32_t i = 0; i < kSteps; ++i) {
      const uint32_t k = i * 4 + q;
      nwv[i] = k < nb ? __ldg(reinterpret_cast<const float4*>(p.norm_w) + (b0 + k) * 8 + c)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  pdl_wait();  // x (and y for the add epilogue) belong to the previous kernel in the stream
  float4 hv[kSteps];
#pragma unroll
  for (uint32_t i = 0; i < kSteps; ++i) {
    const uint32_t k = i * 4 + q;
    hv[i] = k < nb ? __ldg(reinterpret_cast<const float4*>(p.x) + (b0 + k) * 8 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float inv = 1.f;
  if constexpr (NORM) {  // rmsnorm scale (src/kernels.cpp:69-73): double sum of squares of all x
    double ss = 0.0;
#pragma unroll
    for (uint32_t i = 0; i < kSteps; ++i) {
      ss += static_cast<double>(hv[i].x) * static_cast<double>(hv[i].x);
      ss += static_cast<double>(hv[i].y) * static_cast<double>(hv[i].y);
      ss += static_cast<double>(hv[i].z) * static_cast<double>(hv[i].z);
      ss += static_cast<double>(hv[i].w) * static_cast<double>(hv[i].w);
    }
    ss = warp_sum_d(ss);
    if (lane == 0) dred[warp] = ss;
    __syncthreads();
    double tot = 0.0;
    for (int w = 0; w < kSmallWarps; ++w) tot += dred[w];
    const double mean = p.cols ? tot / static_cast<double>(p.cols) : 0.0;
    inv = static_cast<float>(1.0 / sqrt(mean + static_cast<double>(p.norm_eps)));
  }
  bool fast = true;
#pragma unroll
  for (uint32_t i = 0; i < kSteps; ++i) {
    if (i * 4 >= nb) break;  // uniform per warp
    const uint32_t k = i * 4 + q;
    float h[4] = {hv[i].x, hv[i].y, hv[i].z, hv[i].w};
    if constexpr (NORM) {  // w * (x * inv), src/kernels.cpp:74
      h[0] = nwv[i].x * (h[0] * inv);
      h[1] = nwv[i].y * (h[1] * inv);
      h[2] = nwv[i].z * (h[2] * inv);
      h[3] = nwv[i].w * (h[3] * inv);
    }
    // lanes past this warp's range (k >= nb) carry zeros, vote, and store nothing
    fast = x_block_digits(h, b0 + (k < nb ? k : 0u), c, xdig, xsc, k < nb) && fast;
  }
  __syncwarp();

  // Lane (g, t): row g of the unit, as in the large kernel (one useful digit-pair sum per MMA).
  const uint32_t g = lane >> 2, t = lane & 3;
  const uint32_t x1_off = 1 + t, x2_off = t == 2 ? 4u : 0u;
  const uint32_t sel_code = t == 3 ? 0x1076u : 0x3210u;
  const uint32_t sel_d = t < 2 ? 0x5454u : (t == 2 ? 0x7676u : 0x3232u);
  const bool c_hi = t >= 2;
  const uint2* xd = reinterpret_cast<const uint2*>(xdig + (g >> 2) * 128 + (t * 4 + (g & 3u)) * 8);
  const float* xs_l = xsc + t;
  bool ok = true;
  for (uint32_t i = 0; i < nu; ++i) ok = mbar_wait(&bar[i], 0, p.err) && ok;  // fetched at the start
  // Block pairs outer, units inner: the units' MMA chains are independent, so their latencies
  // overlap, and the x fragment and scale of a pair are read once for all units.
  float acc[kSmallMaxUnits][NM];
#pragma unroll
  for (uint32_t i = 0; i < kSmallMaxUnits; ++i)
#pragma unroll
    for (uint32_t m = 0; m < NM; ++m) acc[i][m] = 0.f;
  if (ok && fast) {
#pragma unroll 1
    for (uint32_t pr = p0; pr < p1; ++pr) {
      const uint32_t ks = pr / (kSegBlk / 2), w = (pr % (kSegBlk / 2)) * 9;
      const uint2 bf = xd[2 * pr * 16];
      const float sc = xs_l[4 * pr];
#pragma unroll
      for (uint32_t i = 0; i < kSmallMaxUnits; ++i) {
        if (i >= nu) break;
#pragma unroll
        for (uint32_t m = 0; m < NM; ++m) {
          const uint32_t* rw = reinterpret_cast<const uint32_t*>(wbuf + ((i * NM + m) * p.nseg + ks) * kSlotBytes +
                                                                 g * kRowStride);
          const uint32_t X1 = rw[w + x1_off], X2 = rw[w + x2_off], Y = rw[w + 5 + t];
          const uint32_t ce = __byte_perm(X1, X2, sel_code), db = __byte_perm(X1, X2, sel_d);
          const uint32_t a[4] = {a_lo(ce), a_lo(Y), a_hi(ce), a_hi(Y)};
          int cc[4];
          mma_s8(a, bf.x, bf.y, cc);
          const int v = (c_hi ? cc[2] : cc[0]) + ((c_hi ? cc[3] : cc[1]) << 8);
          acc[i][m] = fmaf(static_cast<float>(v), half_bits_to_float(db) * sc, acc[i][m]);
        }
      }
    }
#pragma unroll
    for (uint32_t i = 0; i < kSmallMaxUnits; ++i) {
      if (i >= nu) break;
#pragma unroll
      for (uint32_t m = 0; m < NM; ++m) {
        acc[i][m] += __shfl_xor_sync(0xFFFFFFFFu, acc[i][m], 1);
        acc[i][m] += __shfl_xor_sync(0xFFFFFFFFu, acc[i][m], 2);
        if (t == 0) red[((warp * kSmallMaxUnits + i) * NM + m) * kUnitRows + g] = acc[i][m];
      }
    }
  } else if (ok) {
    // plain FP32 dots of this warp's blocks (non-finite or out-of-range x): row r's sum lands
    // in lane 4 r, where the MMA path leaves it
    for (uint32_t i = 0; i < nu; ++i)
      for (uint32_t m = 0; m < NM; ++m) {
        const uint8_t* slot0 = wbuf + (i * NM + m) * p.nseg * kSlotBytes;
        float accf = 0.f;
        for (uint32_t r = 0; r < kUnitRows; ++r) {
          float part = 0.f;
          for (uint32_t bb = b0 + lane; bb < b0 + nb; bb += 32) {
            const uint8_t* blkp = slot0 + (bb / kSegBlk) * kSlotBytes + r * kRowStride + (bb % kSegBlk) * 18;
            const float d = fp16_to_f32(blkp[0] | (blkp[1] << 8));
            float sacc = 0.f;
            for (int k = 0; k < 32; ++k) {
              const int cd = (k < 16 ? (blkp[2 + k] & 15) : (blkp[2 + k - 16] >> 4)) - 8;
              float xv = __ldg(p.x + bb * 32 + k);
              if constexpr (NORM) xv = __ldg(p.norm_w + bb * 32 + k) * (xv * inv);
              sacc += static_cast<float>(cd) * xv;
            }
            part += d * sacc;
          }
          part = warp_sum(part);
          if (g == r) accf = part;
        }
        if (t == 0) red[((warp * kSmallMaxUnits + i) * NM + m) * kUnitRows + g] = accf;
      }
  }
  __syncthreads();
  // one thread per (unit, row): the warps' partials in warp order, then the epilogue
  const uint32_t tid = threadIdx.x;
  if (ok && tid < nu * kUnitRows) {
    const uint32_t i = tid / kUnitRows, r = tid % kUnitRows;
    uint32_t j, r0, nrows;
    locate_unit(p, u_b + i, j, r0, nrows);
    if (r < nrows) {
      float v[NM];
#pragma unroll
      for (uint32_t m = 0; m < NM; ++m) {
        float s = 0.f;
        for (int w = 0; w < kSmallWarps; ++w) s += red[((w * kSmallMaxUnits + i) * NM + m) * kUnitRows + r];
        v[m] = s;
      }
      float* y = p.jobs[j].y + (p.pos ? *p.pos * p.jobs[j].y_pos_stride : 0);
      if constexpr (E == Epi::SwiGLU) y[r0 + r] = silu(v[0]) * v[NM - 1];
      else if constexpr (E == Epi::Add) y[r0 + r] += v[0];
      else y[r0 + r] = v[0];
    }
  }
}

using SmallFn = void (*)(SmallParams);

SmallFn pick_small(Epi e, bool norm) {
  switch (e) {
    case Epi::Store: return norm ? matvec_q4_small_kernel<Epi::Store, true> : matvec_q4_small_kernel<Epi::Store, false>;
    case Epi::Add: return norm ? matvec_q4_small_kernel<Epi::Add, true> : matvec_q4_small_kernel<Epi::Add, false>;
    case Epi::SwiGLU:
      return norm ? matvec_q4_small_kernel<Epi::SwiGLU, true> : matvec_q4_small_kernel<Epi::SwiGLU, false>;
  }
  return nullptr;
}

struct SmallPlan {
  uint32_t nblk, nseg, units, grid;
  uint32_t xsc_offset, xdig_offset, red_offset, w_offset;
  size_t smem;
};

// The small kernel's plan, or false when the call does not fit it (then the other kernels run).
bool plan_small(const MatvecArgs& a, const DeviceInfo& dev, SmallPlan& pl) {
  if (a.fmt != Fmt::Q4 || a.gather.nranks > 0) return false;
  if (a.cols == 0 || a.cols % 256 != 0 || a.cols / 32 < kMinBlk || a.cols / 32 > kMaxBlk) return false;
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0 || reinterpret_cast<uintptr_t>(a.norm_w) % 16 != 0) return false;
  const int n_mat = a.epi == Epi::SwiGLU ? 2 : a.n_jobs;
  const uint32_t NM = a.epi == Epi::SwiGLU ? 2 : 1;
  uint64_t units = 0;
  for (int j = 0; j < n_mat; ++j)
    if (reinterpret_cast<uintptr_t>(a.jobs[j].W) % 16 != 0) return false;
  for (int j = 0; j < (a.epi == Epi::SwiGLU ? 1 : a.n_jobs); ++j) units += (a.jobs[j].rows + kUnitRows - 1) / kUnitRows;
  if (units == 0) return false;
  pl.nblk = static_cast<uint32_t>(a.cols / 32);
  pl.nseg = (pl.nblk + kSegBlk - 1) / kSegBlk;
  pl.units = static_cast<uint32_t>(units);
  pl.grid = static_cast<uint32_t>(std::min<uint64_t>(units, static_cast<uint64_t>(dev.sm_count)));
  const uint32_t upc = (pl.units + pl.grid - 1) / pl.grid;
  if (upc > kSmallMaxUnits || upc * NM * pl.nseg > kSmallMaxSlots) return false;
  pl.xsc_offset = 256;
  pl.xdig_offset = (pl.xsc_offset + pl.nblk * 8 + 127) / 128 * 128;
  pl.red_offset = pl.xdig_offset + pl.nblk * 128;
  pl.w_offset = (pl.red_offset + kSmallWarps * kSmallMaxUnits * NM * kUnitRows * 4 + 127) / 128 * 128;
  pl.smem = pl.w_offset + static_cast<size_t>(upc) * NM * pl.nseg * kSlotBytes;
  return pl.smem <= kSmallSmemCap && pl.smem <= dev.smem_optin;
}

// ------------------------------------------------------------------ small-batch GEMM
// Y[b][m] = sum_k W[m][k] X[b][k] for B <= 64 columns of X (a short prompt, a few decoded
// sequences): the reference's per-column matvec loop (src/qkernels.cpp:275-297) in one launch
// on the same exact integer MMA, with the roles turned around so that no output is wasted:
//  * A (16 x 32): 16 columns of X, one int8 digit plane of their fixed-point form per MMA
//    (digit g of round(x 2^s), s per column and block), K in natural column order;
//  * B (32 x 8): the codes of 8 weight rows of one block, (c - 8) * 16 as int8, taken from
//    one code word per lane (bytes 4t..4t+3 hold columns 4t..4t+3 and 16+4t..19+4t, exactly
//    the fragment's K split);
//  * four MMAs (the digit planes) give 16 x 8 exact int32 dot products of the block; digits
//    0, 1 and 2, 3 are combined in integers, and each pair becomes a float scaled by
//    d * 2^-s / 16 (2^(16-s) / 16) and accumulates in FP32, as in the matvec kernels.
// A CTA owns a few 8-row units, fetched whole with 2-D TMA copies at its start (before the
// grid-dependency wait: static weights). X is turned into digits in chunks of 8 blocks by all
// threads into a double-buffered shared area (one barrier per chunk); warp w multiplies block
// w of each chunk against every unit, so each warp's sums cover the blocks w mod 8 and the 8
// partial sums are added in warp order at the end (deterministic). A column whose X holds a
// non-finite value or a block maximum outside [2^-69, 2^100) is computed afterwards with
// plain FP32 dots, so every column equals what the FP32 matvec arithmetic gives.
constexpr int kSgWarps = 8;
constexpr int kSgThreads = kSgWarps * 32;
constexpr uint32_t kSgCols = 16;                      // columns of X per MMA tile
constexpr uint32_t kSgChunk = 8;                      // blocks per staged chunk (one per warp)
constexpr uint32_t kSgColStride = 48;                 // bytes per column and digit plane (32 + pad)
constexpr uint32_t kSgPlaneBytes = kSgCols * kSgColStride;              // 768
constexpr uint32_t kSgBlockBytes = 4 * kSgPlaneBytes;                   // 3072
constexpr uint32_t kSgBufBytes = kSgChunk * kSgBlockBytes;              // 24 KB
constexpr uint32_t kSgMaxUnits = 10;
constexpr uint32_t kSgMaxSlots = 18;
constexpr uint32_t kSgMaxB = 64;
constexpr uint32_t kSgMaxJobs = 3;

struct SmallGemmParams {
  CUtensorMap maps[kSgMaxJobs];  // W as [rows][rb / 8] u64, box {146, 8}
  const float* X;                // [B][K]
  float* Y[kSgMaxJobs];          // [B][M_j]
  uint32_t M[kSgMaxJobs];
  uint32_t K, nblk, nseg, B, n_jobs, units_total, accumulate;
  uint32_t job_unit_start[kSgMaxJobs + 1];
  int* err;
  uint32_t xs_offset, xd_offset, w_offset;
};

__device__ __forceinline__ void sg_locate(const SmallGemmParams& p, uint32_t u, uint32_t& j, uint32_t& r0) {
  j = 0;
  while (j + 1 < p.n_jobs && u >= p.job_unit_start[j + 1]) ++j;
  r0 = (u - p.job_unit_start[j]) * kUnitRows;
}

__global__ void __launch_bounds__(kSgThreads, 1) gemm_q4_small_kernel(const __grid_constant__ SmallGemmParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);         // [kSgMaxUnits]
  uint32_t* badcol = reinterpret_cast<uint32_t*>(smem + 96);  // one bit per column (B <= 64)
  float* xs = reinterpret_cast<float*>(smem + p.xs_offset);   // [2 buf][kSgChunk][kSgCols][2]
  uint8_t* xd = smem + p.xd_offset;                           // [2 buf][kSgChunk][4 plane][16 col][48 B]
  uint8_t* wbuf = smem + p.w_offset;                          // [unit][seg] slots
  float* red = reinterpret_cast<float*>(xd);                  // after the MMAs: [warp][unit][128]
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const uint32_t u_b = static_cast<uint32_t>(static_cast<uint64_t>(p.units_total) * blockIdx.x / gridDim.x);
  const uint32_t u_e = static_cast<uint32_t>(static_cast<uint64_t>(p.units_total) * (blockIdx.x + 1) / gridDim.x);
  const uint32_t nu = u_e - u_b;
  if (tid == 0) {
    for (uint32_t i = 0; i < nu; ++i) mbar_init(&bar[i], 1);
    badcol[0] = 0u;
    badcol[1] = 0u;
    fence_barrier_init();
    const uint64_t pol = l2_evict_first_policy();
    for (uint32_t i = 0; i < nu; ++i) {
      uint32_t j, r0;
      sg_locate(p, u_b + i, j, r0);
      mbar_arrive_expect_tx(&bar[i], p.nseg * kSlotBytes);
      for (uint32_t ks = 0; ks < p.nseg; ++ks)
        tma_load_2d(wbuf + (i * p.nseg + ks) * kSlotBytes, &p.maps[j], static_cast<int32_t>(ks * kSegBlk * 18 / 8),
                    static_cast<int32_t>(r0), &bar[i], pol);
    }
  }
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();  // X (and Y when adding) belong to the previous kernel in the stream

  const uint32_t gq = lane >> 2, t = lane & 3;  // A rows (columns of X) gq, gq + 8; B column (row) gq
  const uint32_t n_chunks = p.nblk / kSgChunk;
  const uint32_t n_ct = (p.B + kSgCols - 1) / kSgCols;
  bool ok = true, waited = false;
  for (uint32_t ct = 0; ct < n_ct; ++ct) {
    const uint32_t col0 = ct * kSgCols;
    float acc[kSgMaxUnits][4];
#pragma unroll
    for (uint32_t i = 0; i < kSgMaxUnits; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    for (uint32_t kc = 0; kc < n_chunks; ++kc) {
      const uint32_t buf = (ct * n_chunks + kc) & 1u;
      // ---- X chunk -> digits: item = (column, block, 4-value group); 8 lanes share a block
      {
        uint8_t* xdb = xd + buf * kSgBufBytes;
        float* xsb = xs + buf * kSgChunk * kSgCols * 2;
        const uint32_t c8 = lane & 7;
#pragma unroll
        for (uint32_t it = 0; it < (kSgCols * kSgChunk * 8) / kSgThreads; ++it) {
          const uint32_t item = (it * kSgThreads + tid) >> 3;   // (column, block) pair of these 8 lanes
          const uint32_t col = item / kSgChunk, bi = item % kSgChunk;
          const uint32_t gcol = col0 + col, blk = kc * kSgChunk + bi;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (gcol < p.B) v = __ldg(reinterpret_cast<const float4*>(p.X + static_cast<size_t>(gcol) * p.K + blk * 32) + c8);
          float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
          const bool fin = isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
#pragma unroll
          for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
          const int e = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu) - 127;
          const bool bad = !fin || (amax != 0.f && (e < -69 || e >= 100));
          if (bad && gcol < p.B) atomicOr(&badcol[gcol >> 5], 1u << (gcol & 31));
          const int s = (amax == 0.f || bad) ? 0 : 29 - e;
          const float p2s = __uint_as_float(static_cast<uint32_t>(s + 127) << 23);
          const float h[4] = {v.x, v.y, v.z, v.w};
          uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int v0 = 0; v0 < 4; ++v0) {
            int X = bad ? 0 : __float2int_rn(h[v0] * p2s);
            const int d0 = static_cast<int8_t>(X & 0xFF);
            X = (X - d0) >> 8;
            const int d1 = static_cast<int8_t>(X & 0xFF);
            X = (X - d1) >> 8;
            const int d2 = static_cast<int8_t>(X & 0xFF);
            const int d3 = (X - d2) >> 8;
            words[0] |= (static_cast<uint32_t>(d0) & 0xFFu) << (8 * v0);
            words[1] |= (static_cast<uint32_t>(d1) & 0xFFu) << (8 * v0);
            words[2] |= (static_cast<uint32_t>(d2) & 0xFFu) << (8 * v0);
            words[3] |= (static_cast<uint32_t>(d3) & 0xFFu) << (8 * v0);
          }
          uint8_t* dst = xdb + bi * kSgBlockBytes + col * kSgColStride + c8 * 4;
#pragma unroll
          for (int g = 0; g < 4; ++g) *reinterpret_cast<uint32_t*>(dst + g * kSgPlaneBytes) = words[g];
          if (c8 == 0) {
            xsb[(bi * kSgCols + col) * 2] = __uint_as_float(static_cast<uint32_t>(123 - s) << 23);      // 2^(-4-s)
            xsb[(bi * kSgCols + col) * 2 + 1] = __uint_as_float(static_cast<uint32_t>(139 - s) << 23);  // 2^(12-s)
          }
        }
      }
      __syncthreads();  // the chunk's digits are in place; the other buffer is free again
      if (!waited) {    // the weights arrive once
        for (uint32_t i = 0; i < nu; ++i) ok = mbar_wait(&bar[i], 0, p.err) && ok;
        waited = true;
      }
      if (!ok) continue;
      // ---- MMAs: warp w takes block w of the chunk, against every unit
      const uint32_t blk = kc * kSgChunk + warp;
      const uint8_t* xdb = xd + buf * kSgBufBytes + warp * kSgBlockBytes;
      const float* xsb = xs + (buf * kSgChunk + warp) * kSgCols * 2;
      uint32_t a[4][4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const uint8_t* pl = xdb + g * kSgPlaneBytes;
        a[g][0] = *reinterpret_cast<const uint32_t*>(pl + gq * kSgColStride + 4 * t);
        a[g][1] = *reinterpret_cast<const uint32_t*>(pl + (gq + 8) * kSgColStride + 4 * t);
        a[g][2] = *reinterpret_cast<const uint32_t*>(pl + gq * kSgColStride + 16 + 4 * t);
        a[g][3] = *reinterpret_cast<const uint32_t*>(pl + (gq + 8) * kSgColStride + 16 + 4 * t);
      }
      const float s01_a = xsb[gq * 2], s23_a = xsb[gq * 2 + 1];                // column gq
      const float s01_b = xsb[(gq + 8) * 2], s23_b = xsb[(gq + 8) * 2 + 1];    // column gq + 8
      const uint32_t seg = blk / kSegBlk, jb = (blk % kSegBlk) * 18;
#pragma unroll
      for (uint32_t i = 0; i < kSgMaxUnits; ++i) {  // unrolled: acc stays in registers
        if (i >= nu) break;
        const uint8_t* slot = wbuf + (i * p.nseg + seg) * kSlotBytes + jb;
        // this lane's code word: bytes 4t..4t+3 of row gq's 16 code bytes (2 bytes into the block)
        const uint8_t* cp = slot + gq * kRowStride + 2 + 4 * t;
        uint32_t cw;
        if (blk & 1u) {
          cw = *reinterpret_cast<const uint32_t*>(cp);
        } else {
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(cp - 2), w1 = *reinterpret_cast<const uint32_t*>(cp + 2);
          cw = __byte_perm(w0, w1, 0x5432);
        }
        const uint32_t b0 = a_lo(cw), b1 = a_hi(cw);
        // the fp16 scales of rows 2t and 2t + 1 (this lane's two output rows)
        const float d0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(slot + (2 * t) * kRowStride));
        const float d1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(slot + (2 * t + 1) * kRowStride));
        int c[4][4];
#pragma unroll
        for (int g = 0; g < 4; ++g) mma_s8(a[g], b0, b1, c[g]);
        // c[g][0..3]: (column gq, row 2t), (gq, 2t + 1), (gq + 8, 2t), (gq + 8, 2t + 1)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int v01 = c[0][q] + (c[1][q] << 8), v23 = c[2][q] + (c[3][q] << 8);
          const float d = (q & 1) ? d1 : d0;
          const float s01 = q < 2 ? s01_a : s01_b, s23 = q < 2 ? s23_a : s23_b;
          acc[i][q] = fmaf(static_cast<float>(v01), d * s01, acc[i][q]);
          acc[i][q] = fmaf(static_cast<float>(v23), d * s23, acc[i][q]);
        }
      }
    }
    // ---- the warps' sums over their blocks, added in warp order
    __syncthreads();  // every MMA of this column tile has read its digits
#pragma unroll
    for (uint32_t i = 0; i < kSgMaxUnits; ++i) {
      if (i >= nu) break;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t col = gq + (q >> 1) * 8, row = 2 * t + (q & 1);
        red[(warp * kSgMaxUnits + i) * 128 + col * 8 + row] = acc[i][q];
      }
    }
    __syncthreads();
    const uint32_t bad_lo = badcol[0], bad_hi = badcol[1];
    for (uint32_t e = tid; e < nu * 128; e += kSgThreads) {
      const uint32_t i = e / 128, col = (e % 128) / 8, row = e % 8;
      const uint32_t gcol = col0 + col;
      uint32_t j, r0;
      sg_locate(p, u_b + i, j, r0);
      if (!ok || gcol >= p.B || r0 + row >= p.M[j]) continue;
      if (((gcol < 32 ? bad_lo >> gcol : bad_hi >> (gcol - 32)) & 1u) != 0u) continue;  // FP32 path below
      float v = 0.f;
      for (int w = 0; w < kSgWarps; ++w) v += red[(w * kSgMaxUnits + i) * 128 + col * 8 + row];
      float* y = p.Y[j] + static_cast<size_t>(gcol) * p.M[j] + r0 + row;
      *y = p.accumulate ? *y + v : v;
    }
    __syncthreads();  // red (the digit area) is rewritten by the next column tile
  }
  // ---- columns with non-finite or out-of-range x: plain FP32 dots, one warp per (row, column)
  const uint32_t bad_lo = badcol[0], bad_hi = badcol[1];
  if (ok && (bad_lo | bad_hi) != 0u) {
    for (uint32_t e = warp; e < nu * kUnitRows * p.B; e += kSgWarps) {
      const uint32_t gcol = e % p.B, rr = e / p.B, i = rr / kUnitRows, row = rr % kUnitRows;
      if (((gcol < 32 ? bad_lo >> gcol : bad_hi >> (gcol - 32)) & 1u) == 0u) continue;
      uint32_t j, r0;
      sg_locate(p, u_b + i, j, r0);
      if (r0 + row >= p.M[j]) continue;
      const float* xr = p.X + static_cast<size_t>(gcol) * p.K;
      float part = 0.f;
      for (uint32_t bb = lane; bb < p.nblk; bb += 32) {
        const uint8_t* blkp = wbuf + (i * p.nseg + bb / kSegBlk) * kSlotBytes + row * kRowStride + (bb % kSegBlk) * 18;
        const float d = fp16_to_f32(blkp[0] | (blkp[1] << 8));
        float sacc = 0.f;
        for (int k = 0; k < 32; ++k) {
          const int cd = (k < 16 ? (blkp[2 + k] & 15) : (blkp[2 + k - 16] >> 4)) - 8;
          sacc += static_cast<float>(cd) * __ldg(xr + bb * 32 + k);
        }
        part += d * sacc;
      }
      part = warp_sum(part);
      if (lane == 0) {
        float* y = p.Y[j] + static_cast<size_t>(gcol) * p.M[j] + r0 + row;
        *y = p.accumulate ? *y + part : part;
      }
    }
  }
}

struct SmallGemmPlan {
  uint32_t nblk, nseg, units, grid;
  uint32_t xs_offset, xd_offset, w_offset;
  size_t smem;
};

bool plan_small_gemm(const GemmCall& c, const DeviceInfo& dev, SmallGemmPlan& pl) {
  if (c.qtype != 4 || c.B == 0 || c.B > kSgMaxB || c.n_jobs < 1 || c.n_jobs > static_cast<int>(kSgMaxJobs))
    return false;
  if (c.K == 0 || c.K % 256 != 0 || c.K / 32 < kMinBlk || c.K / 32 > kMaxBlk) return false;
  if (reinterpret_cast<uintptr_t>(c.X) % 16 != 0) return false;
  uint64_t units = 0;
  for (int j = 0; j < c.n_jobs; ++j) {
    if (reinterpret_cast<uintptr_t>(c.jobs[j].W) % 16 != 0 || c.jobs[j].M == 0) return false;
    units += (c.jobs[j].M + kUnitRows - 1) / kUnitRows;
  }
  pl.nblk = static_cast<uint32_t>(c.K / 32);
  pl.nseg = (pl.nblk + kSegBlk - 1) / kSegBlk;
  pl.units = static_cast<uint32_t>(units);
  pl.grid = static_cast<uint32_t>(std::min<uint64_t>(units, static_cast<uint64_t>(dev.sm_count)));
  const uint32_t upc = (pl.units + pl.grid - 1) / pl.grid;
  if (upc > kSgMaxUnits || upc * pl.nseg > kSgMaxSlots) return false;
  pl.xs_offset = 128;
  pl.xd_offset = (pl.xs_offset + 2 * kSgChunk * kSgCols * 8 + 127) / 128 * 128;
  const uint32_t xd_bytes = std::max<uint32_t>(2 * kSgBufBytes, kSgWarps * kSgMaxUnits * 128 * 4);
  pl.w_offset = (pl.xd_offset + xd_bytes + 127) / 128 * 128;
  pl.smem = pl.w_offset + static_cast<size_t>(upc) * pl.nseg * kSlotBytes;
  return pl.smem <= dev.smem_optin;
}

}  // namespace

bool matvec_mma_ok(const MatvecArgs& a, const DeviceInfo& dev) {
  if (a.fmt != Fmt::Q4 || a.epi == Epi::SwiGLU) return false;
  if (a.cols == 0 || a.cols % 256 != 0 || a.cols / 32 < kMinBlk || a.cols / 32 > kMaxBlk) return false;
  // x and the norm weights are read as float4
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0 || reinterpret_cast<uintptr_t>(a.norm_w) % 16 != 0) return false;
  uint64_t bytes = 0;
  for (int j = 0; j < a.n_jobs; ++j) {
    if (reinterpret_cast<uintptr_t>(a.jobs[j].W) % 16 != 0) return false;
    bytes += static_cast<uint64_t>(a.jobs[j].rows) * (a.cols / 32) * 18;
  }
  MmaPlan pl;
  if (bytes < EFG_MMA_MIN_BYTES || !plan_mma(static_cast<uint32_t>(a.cols / 32), dev, pl)) return false;
  CUtensorMap m;  // the driver must accept every job's map (else the CUDA-core kernel runs)
  for (int j = 0; j < a.n_jobs; ++j)
    if (a.jobs[j].rows && !encode_w_map(&m, a.jobs[j].W, a.jobs[j].rows, static_cast<uint32_t>(a.cols / 32 * 18)))
      return false;
  return true;
}

int launch_matvec_q4_mma(const MatvecArgs& a, const DeviceInfo& dev, int* d_err, cudaStream_t stream,
                         bool direct_smem_attr) {
  MmaParams p{};
  p.x = a.x;
  p.norm_w = a.norm_w;
  p.norm_eps = a.norm_eps;
  p.err = d_err;
  p.pos = a.pos;
  p.cols = static_cast<uint32_t>(a.cols);
  p.nblk = p.cols / 32;
  p.rb = p.nblk * 18;
  MmaPlan pl;
  if (!plan_mma(p.nblk, dev, pl)) return fail(EFG_EINVAL, "matvec: no MMA plan for %u columns", p.cols);
  p.nseg = pl.nseg;
  p.NS = pl.NS;
  p.ring_offset = pl.ring_offset;
  p.Wk = pl.Wk;
  p.Gs = pl.Gs;
  p.n_jobs = static_cast<uint32_t>(a.n_jobs);
  uint32_t rt = 0;
  for (int j = 0; j < a.n_jobs; ++j) {
    p.jobs[j] = a.jobs[j];
    if (a.jobs[j].rows && !encode_w_map(&p.maps[j], a.jobs[j].W, a.jobs[j].rows, p.rb))
      return fail(EFG_ECUDA, "matvec: tensor map for a %u x %u Q4_0 matrix", a.jobs[j].rows, p.cols);
    p.job_rt_start[j] = rt;
    rt += (a.jobs[j].rows + kTileRows - 1) / kTileRows;
  }
  p.job_rt_start[a.n_jobs] = rt;
  p.rt_total = rt;
  if (rt == 0) return EFG_OK;
  p.g = a.gather;
  MmaFn fn = pick_mma(a.epi, a.norm_w != nullptr, a.gather.nranks > 0);
  if (!fn) return fail(EFG_EINVAL, "matvec: the in-kernel gather takes one plain product (no norm, no add)");
  if (direct_smem_attr) {
    EFG_TRY_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pl.smem)),
                 "kernel shared-memory attribute");
  } else if (int st = ensure_smem_attr(reinterpret_cast<const void*>(fn), pl.smem)) {
    return st;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(std::min<uint32_t>(rt, static_cast<uint32_t>(dev.sm_count)));
  cfg.blockDim = dim3(kMmaThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, fn, p), "matvec launch");
  return EFG_OK;
}

bool matvec_small_ok(const MatvecArgs& a, const DeviceInfo& dev) {
  SmallPlan pl;
  if (!plan_small(a, dev, pl)) return false;
  CUtensorMap m;  // the driver must accept every matrix's map
  const int n_mat = a.epi == Epi::SwiGLU ? 2 : a.n_jobs;
  for (int j = 0; j < n_mat; ++j)
    if (a.jobs[j].rows && !encode_u64_rows_map(&m, a.jobs[j].W, a.jobs[j].rows, a.cols / 32 * 18, kBoxElems, kUnitRows))
      return false;
  return true;
}

int launch_matvec_q4_small(const MatvecArgs& a, const DeviceInfo& dev, int* d_err, cudaStream_t stream,
                           bool direct_smem_attr) {
  SmallPlan pl;
  if (!plan_small(a, dev, pl)) return fail(EFG_EINVAL, "matvec: no small-matrix plan for this call");
  SmallParams p{};
  p.x = a.x;
  p.norm_w = a.norm_w;
  p.norm_eps = a.norm_eps;
  p.err = d_err;
  p.pos = a.pos;
  p.cols = static_cast<uint32_t>(a.cols);
  p.nblk = pl.nblk;
  p.nseg = pl.nseg;
  p.npairs = pl.nblk / 2;
  p.units_total = pl.units;
  p.xsc_offset = pl.xsc_offset;
  p.xdig_offset = pl.xdig_offset;
  p.red_offset = pl.red_offset;
  p.w_offset = pl.w_offset;
  const int n_mat = a.epi == Epi::SwiGLU ? 2 : a.n_jobs;
  p.n_jobs = static_cast<uint32_t>(a.epi == Epi::SwiGLU ? 1 : a.n_jobs);
  const uint32_t rb = pl.nblk * 18;
  for (int j = 0; j < n_mat; ++j) {
    p.jobs[j] = a.jobs[j];
    if (a.jobs[j].rows && !encode_u64_rows_map(&p.maps[j], a.jobs[j].W, a.jobs[j].rows, rb, kBoxElems, kUnitRows))
      return fail(EFG_ECUDA, "matvec: tensor map for a %u x %u Q4_0 matrix", a.jobs[j].rows, p.cols);
  }
  uint32_t u = 0;
  for (uint32_t j = 0; j < p.n_jobs; ++j) {
    p.job_unit_start[j] = u;
    u += (a.jobs[j].rows + kUnitRows - 1) / kUnitRows;
  }
  p.job_unit_start[p.n_jobs] = u;
  SmallFn fn = pick_small(a.epi, a.norm_w != nullptr);
  if (direct_smem_attr) {
    EFG_TRY_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pl.smem)),
                 "kernel shared-memory attribute");
  } else if (int st = ensure_smem_attr(reinterpret_cast<const void*>(fn), pl.smem)) {
    return st;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kSmallThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, fn, p), "matvec launch");
  return EFG_OK;
}

bool gemm_q4_small_ok(const GemmCall& c, const DeviceInfo& dev) {
  SmallGemmPlan pl;
  if (!plan_small_gemm(c, dev, pl)) return false;
  CUtensorMap m;
  for (int j = 0; j < c.n_jobs; ++j)
    if (!encode_u64_rows_map(&m, c.jobs[j].W, c.jobs[j].M, c.K / 32 * 18, kBoxElems, kUnitRows)) return false;
  return true;
}

int launch_gemm_q4_small(const GemmCall& c, const DeviceInfo& dev, int* d_err, cudaStream_t s) {
  SmallGemmPlan pl;
  if (!plan_small_gemm(c, dev, pl)) return fail(EFG_EINVAL, "gemm: no small-batch plan for this call");
  SmallGemmParams p{};
  p.X = c.X;
  p.K = static_cast<uint32_t>(c.K);
  p.nblk = pl.nblk;
  p.nseg = pl.nseg;
  p.B = static_cast<uint32_t>(c.B);
  p.n_jobs = static_cast<uint32_t>(c.n_jobs);
  p.units_total = pl.units;
  p.accumulate = c.accumulate ? 1u : 0u;
  p.err = d_err;
  p.xs_offset = pl.xs_offset;
  p.xd_offset = pl.xd_offset;
  p.w_offset = pl.w_offset;
  uint32_t u = 0;
  for (int j = 0; j < c.n_jobs; ++j) {
    if (!encode_u64_rows_map(&p.maps[j], c.jobs[j].W, c.jobs[j].M, pl.nblk * 18, kBoxElems, kUnitRows))
      return fail(EFG_ECUDA, "gemm: tensor map for a %zu x %zu Q4_0 matrix", c.jobs[j].M, c.K);
    p.Y[j] = c.jobs[j].Y;
    p.M[j] = static_cast<uint32_t>(c.jobs[j].M);
    p.job_unit_start[j] = u;
    u += static_cast<uint32_t>((c.jobs[j].M + kUnitRows - 1) / kUnitRows);
  }
  p.job_unit_start[c.n_jobs] = u;
  if (int st = ensure_smem_attr(reinterpret_cast<const void*>(gemm_q4_small_kernel), pl.smem)) return st;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kSgThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = weight_prefetch_flag() ? 1 : 0;
  EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, gemm_q4_small_kernel, p), "gemm launch");
  return EFG_OK;
}

}  // namespace efg
