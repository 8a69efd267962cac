// efg_gemm.cu - batched Q4_0 / Q8_0 x activation GEMM on the 5th-generation tensor cores.
//
//   Y[b][m] = sum_k W[m][k] X[b][k]      W: Q4_0 or Q8_0 rows [M][K/32 blocks], X: FP32
//                                         [B][K], Y: FP32 [B][M]
//
// The reference has no GEMM: its prompt and multi-sequence work is one ef::kern::matvec per
// column (src/qkernels.cpp:275-297), which is the oracle here. The tensor-core formulation
// keeps that FP32 result within 1e-5 of sum |w x| per output:
//   * a Q4_0 weight w = (c - 8) * d (4-bit code, FP16 scale) has at most 14 significant
//     bits, so w = w_hi + w_lo with w_hi = bf16(w) and w_lo = bf16(w - w_hi) is EXACT; a
//     Q8_0 weight q * d has at most 18, and three BF16 terms represent it exactly;
//   * x = x1 + x2 with x1 = bf16(x), x2 = bf16(x - x1) keeps 16 significant bits;
//   * products of BF16 operands (tcgen05.mma kind::f16) are exact in FP32; the only error
//     is the dropped residual of x, at most 2^-16 of each |w x| and of random sign.
//
// Two kernels. gemm_ws_kernel (K % 256 == 0, every shape the decoder uses) is warp-
// specialised, with the dequantised weights in TMEM, X stacked along N and split-K over a
// thread-block cluster; its role notes are above it. gemm_q4_0_kernel handles Q4_0 with
// K % 256 != 0: one CTA computes a 128-row x N_TILE tile (N_TILE = B rounded up to 16, at
// most 256), K advances in 64-wide chunks through two shared-memory stages: all 256 threads
// dequantize the chunk's W rows into W_hi / W_lo tiles and split X into X1 / X2 (K-major,
// 128-byte swizzled, the canonical UMMA layout), then one thread issues the 12 MMAs of the
// chunk (W_hi X1 + W_hi X2 + W_lo X1 over 4 K-steps) and commits them to the stage's
// mbarrier, which the threads wait on before they refill that stage two chunks later. The
// epilogue reads TMEM with tcgen05.ld (warp w sees lanes 32 (w % 4) ..) and writes Y with
// coalesced stores.
#include <algorithm>
#include <cstdint>
#include <mutex>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/efg.h"
#include "efg_device.cuh"
#include "efg_dot.cuh"
#include "efg_gemm.cuh"
#include "efg_host.h"

namespace efg {
namespace {

constexpr int kGemmThreads = 256;
constexpr int kTileM = 128;
constexpr int kChunkK = 64;   // bf16 elements per 128-byte swizzle row
constexpr int kMaxTileN = 256;
constexpr uint32_t kATileBytes = kTileM * 128;  // 16 KB

// ---------------------------------------------------------------- tcgen05 wrappers

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory operand written by threads -> visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D (TMEM) [+]= A (smem) * B (smem)^T, BF16 operands, FP32 accumulator.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// 32 lanes x 8 consecutive FP32 columns of TMEM -> 8 registers per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Instruction descriptor of kind::f16: BF16 A and B (K-major), FP32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t M, uint32_t N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Shared-memory descriptor of a K-major, 128-byte-swizzled operand tile whose rows are 128
// bytes and whose 8-row groups are 1024 bytes apart (the tile base is 1024-byte aligned).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// Byte offset of the 16-byte chunk `c` (0..7) of row `r` in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // .x = a (low half), .y = b
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float bf16_lo_f(uint32_t p) { return __uint_as_float(p << 16); }
__device__ __forceinline__ float bf16_hi_f(uint32_t p) { return __uint_as_float(p & 0xFFFF0000u); }

// Splits 2 floats into packed (hi, lo) bf16 pairs with v = hi + lo (+ residual).
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16(a, b);
  lo = pack_bf16(__fsub_rn(a, bf16_lo_f(hi)), __fsub_rn(b, bf16_hi_f(hi)));
}

// Bounded wait that ignores other CTAs' errors: used to drain this CTA's own MMAs before
// TMEM is released, so it only gives up on its own timeout.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity, int* err) {
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u && globaltimer_ns() - t0 > kWaitTimeoutNs) {
      record_error(err, EFG_ETIMEOUT);
      return false;
    }
  }
}

struct GemmParams {
  const uint8_t* W;
  const float* X;
  float* Y;
  uint32_t M, K, B, rb, n_tile;
  int* err;
};

__global__ void __launch_bounds__(kGemmThreads, 1) gemm_q4_0_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t mma_done[2];
  __shared__ uint32_t tmem_slot;
  pdl_wait();
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t m0 = blockIdx.x * kTileM, n0 = blockIdx.y * p.n_tile, N = p.n_tile;
  const uint32_t b_tile_bytes = N * 128u;
  const uint32_t stage_bytes = 2 * kATileBytes + 2 * b_tile_bytes;
  // 1024-byte aligned operand area (the swizzle pattern repeats every 8 rows of 128 B)
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  uint32_t ncols = 32;
  while (ncols < N) ncols <<= 1;

  if (tid == 0) {
    mbar_init(&mma_done[0], 1);
    mbar_init(&mma_done[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_slot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  const uint32_t nchunks = (p.K + kChunkK - 1) / kChunkK;
  const uint32_t idesc = idesc_bf16(kTileM, N);
  bool ok = true;
  uint32_t issued = 0;  // chunks whose MMAs have been committed
  for (uint32_t i = 0; i < nchunks; ++i) {
    const uint32_t s = i & 1u;
    if (i >= 2) ok = mbar_wait(&mma_done[s], ((i >> 1) - 1) & 1u, p.err) && ok;
    if (!__syncthreads_and(ok)) break;
    uint8_t* st = gbase + s * stage_bytes;
    uint8_t* a_hi = st;
    uint8_t* a_lo = st + kATileBytes;
    uint8_t* b1 = st + 2 * kATileBytes;
    uint8_t* b2 = b1 + b_tile_bytes;
    // ---- W: thread -> (row, block) of this chunk: 32 weights -> 4 chunks of hi and of lo
    {
      const uint32_t r = tid >> 1, blk = tid & 1u;
      const uint32_t kb = i * 2 + blk;  // global block index along the row
      uint4 hi4[4], lo4[4];
      if (m0 + r < p.M && kb * 32 < p.K) {
        const uint16_t* q = reinterpret_cast<const uint16_t*>(p.W + static_cast<uint64_t>(m0 + r) * p.rb + kb * 18u);
        const float d = fp16_to_f32(__ldg(q));
        uint32_t qs[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) qs[t] = __ldg(q + 1 + 2 * t) | (static_cast<uint32_t>(__ldg(q + 2 + 2 * t)) << 16);
        // weights j = 0..15: low nibbles of bytes 0..15; j = 16..31: high nibbles
        float w[32];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const uint32_t byte = (qs[j >> 2] >> (8 * (j & 3))) & 0xFFu;
          w[j] = __fmul_rn(static_cast<float>(static_cast<int>(byte & 15u) - 8), d);
          w[j + 16] = __fmul_rn(static_cast<float>(static_cast<int>(byte >> 4) - 8), d);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t h[4], l[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) split2(w[8 * c + 2 * e], w[8 * c + 2 * e + 1], h[e], l[e]);
          hi4[c] = make_uint4(h[0], h[1], h[2], h[3]);
          lo4[c] = make_uint4(l[0], l[1], l[2], l[3]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) hi4[c] = lo4[c] = make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t off = sw128(r, blk * 4 + c);
        *reinterpret_cast<uint4*>(a_hi + off) = hi4[c];
        *reinterpret_cast<uint4*>(a_lo + off) = lo4[c];
      }
    }
    // ---- X: 16 threads per batch row, 4 floats each -> X1 / X2 (8 bytes each)
    for (uint32_t n = tid >> 4; n < N; n += kGemmThreads / 16) {
      const uint32_t k4 = (tid & 15u) * 4;
      const uint32_t k = i * kChunkK + k4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (n0 + n < p.B && k < p.K)
        v = __ldg(reinterpret_cast<const float4*>(p.X + static_cast<uint64_t>(n0 + n) * p.K + k));
      uint32_t h0, l0, h1, l1;
      split2(v.x, v.y, h0, l0);
      split2(v.z, v.w, h1, l1);
      const uint32_t off = sw128(n, k4 >> 3) + (k4 & 7u) * 2;
      *reinterpret_cast<uint2*>(b1 + off) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(b2 + off) = make_uint2(l0, l1);
    }
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint64_t dah = smem_desc_sw128(smem_addr(a_hi)), dal = smem_desc_sw128(smem_addr(a_lo));
      const uint64_t db1 = smem_desc_sw128(smem_addr(b1)), db2 = smem_desc_sw128(smem_addr(b2));
#pragma unroll
      for (uint32_t ks = 0; ks < kChunkK / 16; ++ks) {
        const uint64_t adv = 2ull * ks;  // 32 bytes further along K, in 16-byte units
        mma_bf16(tmem, dah + adv, db1 + adv, idesc, (i | ks) != 0);
        mma_bf16(tmem, dah + adv, db2 + adv, idesc, 1);
        mma_bf16(tmem, dal + adv, db1 + adv, idesc, 1);
      }
      mma_commit(&mma_done[s]);
    }
    issued = i + 1;
  }
  // drain: the last committed chunk's MMAs (commits complete in order, so all are done)
  if (issued > 0) {
    const uint32_t last = issued - 1;
    ok = mbar_drain(&mma_done[last & 1u], (last >> 1) & 1u, p.err) && ok && issued == nchunks;
  }
  ok = __syncthreads_and(ok);
  tc_fence_after();
  pdl_launch_dependents();
  if (ok) {
    const uint32_t q = warp & 3u, half = warp >> 2;
    const uint32_t row = m0 + 32 * q + lane;
    for (uint32_t c0 = half * (N / 2); c0 < (half + 1) * (N / 2); c0 += 8) {
      float v[8];
      tmem_ld8(tmem + ((32 * q) << 16) + c0, v);
      if (row < p.M) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (n0 + c0 + e < p.B) p.Y[static_cast<uint64_t>(n0 + c0 + e) * p.M + row] = v[e];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

// ================================================================ warp-specialised kernel
//
// For K a multiple of 256 (every config-3 shape), Q4_0 or Q8_0 (template argument kQ), one
// to three matrices sharing X per launch (each CTA finds its matrix from blockIdx.x), and
// optionally Y += product (the residual add). The dequantised W operand lives in TMEM,
// not shared memory: the MMAs read A from tensor memory ("A in TMEM" form of tcgen05.mma),
// so the dequantising threads write their rows with tcgen05.st (one lane per row, no
// swizzle, no generic->async proxy fence) and the tensor core reads no A bytes from shared
// memory. Roles per CTA (22 warps):
//   warp 0      streams the CTA's raw W rows, 256 columns (144 bytes for Q4_0, 272 for Q8_0)
//               per row and chunk, into a 4-stage (Q8_0: 3-stage) ring with one 2-D tensor
//               copy per chunk;
//   warps 18..21 fill the B operand stages, hi rows then lo rows of the swizzled UMMA layout,
//               so one stage is one MMA operand of 2 N rows. For N <= 64 they build the tiles
//               from X (read the tile's N rows of FP32, split every value into BF16 hi / lo
//               parts): no separate kernel and no workspace. For wider tiles that work would be
//               repeated by every row tile, so X is split once per call by split_x_kernel into
//               a per-device scratch laid out tile by tile, and each warp bulk-copies a quarter
//               of the stage;
//   warps 2..17 dequantize the 64-column sub-chunks in two groups of 8 (warps 2..9 the even
//               sub-chunks, 10..17 the odd ones, so one group's waits overlap the other's
//               arithmetic): warp w owns TMEM lanes 32 (w % 4) .. +31 (one row each) and half
//               of the sub-chunk's columns (one block), writing the weight's exact BF16 terms
//               (two for Q4_0, three for Q8_0) as packed pairs; warps 2..9 then run the
//               epilogue;
//   warp 1      allocates TMEM and issues the MMAs (one thread): per 16-wide K step and
//               weight term t, D[:, 0:2N] += W_t [X_hi | X_lo], so D[:, n] collects the X_hi
//               products and D[:, N + n] the X_lo products (their sum is the FP32 result;
//               the W_lo X_lo parts are below 2^-16 of |w x| and add nothing harmful). Each
//               sub-chunk is committed to its stage's "empty" barrier, the last one to
//               "acc_full".
// TMEM: the accumulator at columns [0, 2N), then the A stages (32 columns per term) from
// column 128 (N <= 64) or 256 (N <= 128), as many as fit (six / four for Q4_0).
// Split-K: a cluster of S CTAs along z shares an output tile and splits its 64-column
// sub-chunks evenly (a raw chunk at a split boundary is streamed by both CTAs, each using its
// own sub-chunks); each CTA writes its partial tile into shared memory, and after a cluster
// barrier CTA z sums its share of the valid columns over all S partials through distributed
// shared memory in rank order (fixed order: the result does not depend on timing).
constexpr int kWsWarps = 22;
constexpr uint32_t kDequantWarps = 16, kBWarp0 = 18, kBWarps = 4;
constexpr int kWsThreads = kWsWarps * 32;
constexpr uint32_t kMaxGemmJobs = 3;
constexpr uint32_t kRawK = 256, kMaxRawStages = 4, kMaxAStages = 6, kMaxTileN2 = 128, kMaxSplit = 8;

// Per weight format: bytes of one 32-column block, of one raw chunk row (256 columns), the
// raw ring depth, and how many exact BF16 terms a dequantised weight needs (Q4_0: (c - 8) d
// has at most 14 significant bits, two terms; Q8_0: q d has at most 18, three terms).
template <int kQ>
struct WsFormat;
template <>
struct WsFormat<4> {
  static constexpr uint32_t kBlock = 18, kRawRow = 144, kRawStages = 4, kTerms = 2;
};
template <>
struct WsFormat<8> {
  static constexpr uint32_t kBlock = 34, kRawRow = 272, kRawStages = 3, kTerms = 3;
};
constexpr uint32_t kTmemCols = 512;
constexpr size_t kWsMinSmem = 120 * 1024;  // keeps one CTA per SM (it holds all 512 TMEM columns)

// One matrix of a launch: the CTAs with blockIdx.x in [tile0, next job's tile0) compute its
// 128-row tiles; every job shares K and the B operand.
struct alignas(64) GemmJobDev {
  CUtensorMap wmap;  // W as [M][row bytes / 8] u64, box {raw chunk row / 8, 128}: one raw chunk of a row tile
  float* Y;          // [B][M]
  uint32_t M, tile0;
};

struct GemmWsParams {
  GemmJobDev jobs[kMaxGemmJobs];
  const float* X;     // [B][K], 16-byte aligned
  const uint8_t* Xs;  // null, or the B operand split by split_x_kernel: [n_tiles][K/64][2][n_tile][128 B]
  uint32_t n_jobs, K, B, n_tile, S, a_stages, accumulate;  // accumulate: Y += product
  int* err;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_map(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  return remote;
}
__device__ __forceinline__ float ld_dsmem(uint32_t remote_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote_addr) : "memory");
  return v;
}

// D (TMEM) [+]= A (TMEM, one row per lane, K pairs packed per 32-bit column) * B (smem)^T.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 consecutive 32-bit TMEM columns of this thread's lane <- 16 registers.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// X [B][K] FP32 -> the B operand tiles: for every n-tile and 64-column chunk, n_tile rows of
// 128 bytes (8 chunks of 8 BF16), swizzled as the MMA reads them; hi part then lo part.
__global__ void split_x_kernel(const float* __restrict__ X, uint32_t B, uint32_t K, uint32_t n_tile,
                               uint8_t* __restrict__ out, uint32_t n_tiles) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t kc_n = K / kChunkK;
  const uint64_t items = static_cast<uint64_t>(n_tiles) * kc_n * n_tile * 8;  // 16-byte chunks per part
  for (uint64_t it = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < items;
       it += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t c = it % 8, n = (it / 8) % n_tile;
    const uint32_t kc = (it / (8ull * n_tile)) % kc_n, nt = static_cast<uint32_t>(it / (8ull * n_tile * kc_n));
    const uint32_t b = nt * n_tile + n, k = kc * kChunkK + c * 8;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (b < B) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(X + static_cast<uint64_t>(b) * K + k));
      const float4 d = __ldg(reinterpret_cast<const float4*>(X + static_cast<uint64_t>(b) * K + k + 4));
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = d.x, v[5] = d.y, v[6] = d.z, v[7] = d.w;
    }
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) split2(v[2 * e], v[2 * e + 1], hi[e], lo[e]);
    const uint64_t tile = (static_cast<uint64_t>(nt) * kc_n + kc) * 2 * n_tile * 128;
    const uint32_t off = sw128(n, c);
    *reinterpret_cast<uint4*>(out + tile + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(out + tile + n_tile * 128 + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// One Q4_0 block (18 bytes at `blk_ptr - 2 * odd`, `odd` = the block starts 2 bytes into a
// 32-bit word) -> 16 packed BF16 pairs of W_hi and of W_lo, pair j = columns 2j, 2j + 1.
// Each code becomes the exact float c - 8 through its exponent field, (c - 8) * d is exact in
// binary32, w_hi = bf16(w) and w_lo = bf16(w - w_hi) (exact: w has at most 14 significant bits).
__device__ __forceinline__ void dequant_block_bf16x2(const uint32_t* q, uint32_t odd, uint32_t (&hi)[16],
                                                     uint32_t (&lo)[16]) {
  uint32_t wv[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) wv[i] = q[i];
  const uint32_t sh = odd * 16;
  const float d = fp16_to_f32(wv[0] >> sh);
  const float2 dd = make_float2(d, d);
  const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t qs = __funnelshift_rc(wv[i], wv[i + 1], sh + 16);  // code bytes 4i .. 4i+3
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // bytes 2h, 2h+1: low nibbles are columns 4i+2h, 4i+2h+1, high nibbles those + 16
      const uint32_t v = h ? (qs >> 16) : qs;
      const float2 lo_c = __fadd2_rn(make_float2(q4_field<0>(v), q4_field<8>(v)), make_float2(-q4_bias<0>(), -q4_bias<8>()));
      const float2 hi_c = __fadd2_rn(make_float2(q4_field<4>(v), q4_field<12>(v)), make_float2(-q4_bias<4>(), -q4_bias<12>()));
      const float2 wl = __fmul2_rn(lo_c, dd), wh = __fmul2_rn(hi_c, dd);
      const uint32_t hl = pack_bf16(wl.x, wl.y), hh = pack_bf16(wh.x, wh.y);
      const float2 rl = __ffma2_rn(make_float2(bf16_lo_f(hl), bf16_hi_f(hl)), neg1, wl);
      const float2 rh = __ffma2_rn(make_float2(bf16_lo_f(hh), bf16_hi_f(hh)), neg1, wh);
      hi[2 * i + h] = hl;
      lo[2 * i + h] = pack_bf16(rl.x, rl.y);
      hi[8 + 2 * i + h] = hh;
      lo[8 + 2 * i + h] = pack_bf16(rh.x, rh.y);
    }
  }
}

// One Q8_0 block (34 bytes, same addressing as dequant_block_bf16x2) -> 16 packed BF16 pairs
// of each of three terms t0 + t1 + t2 = w exactly: q becomes the exact float through its
// exponent field, w = q d is exact in binary32 (at most 18 significant bits), t0 = bf16(w),
// t1 = bf16(w - t0) and t2 = w - t0 - t1 (at most 3 significant bits left, exact in BF16).
__device__ __forceinline__ void dequant_q8_block_bf16x3(const uint32_t* q, uint32_t odd, uint32_t (&t0)[16],
                                                        uint32_t (&t1)[16], uint32_t (&t2)[16]) {
  uint32_t wv[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) wv[i] = q[i];
  const uint32_t sh = odd * 16;
  const float d = fp16_to_f32(wv[0] >> sh);
  const float2 dd = make_float2(d, d);
  const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t qs = __funnelshift_rc(wv[i], wv[i + 1], sh + 16);  // code bytes 4i .. 4i+3
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t v = h ? (qs >> 16) : qs;  // columns 4i+2h, 4i+2h+1
      const float2 c = __fadd2_rn(make_float2(q8_field<0>(v), q8_field<8>(v)), make_float2(-q8_bias<0>(), -q8_bias<8>()));
      const float2 w = __fmul2_rn(c, dd);
      const uint32_t a = pack_bf16(w.x, w.y);
      const float2 r1 = __ffma2_rn(make_float2(bf16_lo_f(a), bf16_hi_f(a)), neg1, w);
      const uint32_t b = pack_bf16(r1.x, r1.y);
      const float2 r2 = __ffma2_rn(make_float2(bf16_lo_f(b), bf16_hi_f(b)), neg1, r1);
      t0[2 * i + h] = a;
      t1[2 * i + h] = b;
      t2[2 * i + h] = pack_bf16(r2.x, r2.y);
    }
  }
}

template <int kQ>
__global__ void __launch_bounds__(kWsThreads, 1) gemm_ws_kernel(const __grid_constant__ GemmWsParams p) {
  using F = WsFormat<kQ>;
  constexpr uint32_t kRawRow = F::kRawRow, kRawBytes = kTileM * F::kRawRow, kRawStages = F::kRawStages;
  constexpr uint32_t kStageCols = 32 * F::kTerms;  // TMEM columns of one A stage
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t raw_full[kMaxRawStages], raw_empty[kMaxRawStages], a_full[kMaxAStages], b_full[kMaxAStages],
      op_empty[kMaxAStages], acc_full;
  __shared__ uint32_t tmem_slot;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t j = 0;
  while (j + 1 < p.n_jobs && blockIdx.x >= p.jobs[j + 1].tile0) ++j;
  const GemmJobDev& job = p.jobs[j];
  const uint32_t N = p.n_tile, m0 = (blockIdx.x - job.tile0) * kTileM, n0 = blockIdx.y * N, M = job.M;
  float* const Y = job.Y;
  const uint32_t z = p.S > 1 ? cluster_rank() : 0;
  const uint32_t n_stage = p.a_stages;
  // this CTA's 64-column sub-chunks [g0, g1) and the raw chunks that hold them
  const uint32_t sub_total = p.K / kChunkK;
  const uint32_t g0 = static_cast<uint32_t>(static_cast<uint64_t>(sub_total) * z / p.S);
  const uint32_t g1 = static_cast<uint32_t>(static_cast<uint64_t>(sub_total) * (z + 1) / p.S);
  const uint32_t n_sub = g1 - g0;
  const uint32_t rc_first = g0 / (kRawK / kChunkK);
  const uint32_t n_raw = n_sub ? (g1 - 1) / (kRawK / kChunkK) - rc_first + 1 : 0;
  const uint32_t b_bytes = 2 * N * 128;  // X_hi rows then X_lo rows
  // 1024-byte aligned: the B stages, then the raw ring
  const uint32_t raw_base_addr = smem_addr(smem_raw);
  uint8_t* bst = smem_raw + (((raw_base_addr + 1023u) & ~1023u) - raw_base_addr);
  uint8_t* raw = bst + n_stage * b_bytes;

  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&job.wmap)) : "memory");
    for (uint32_t i = 0; i < kRawStages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kDequantWarps);
    }
    for (uint32_t i = 0; i < n_stage; ++i) {
      mbar_init(&a_full[i], 8);
      mbar_init(&b_full[i], kBWarps);
      mbar_init(&op_empty[i], 1);
    }
    mbar_init(&acc_full, 1);
    fence_barrier_init();
    // the first raw chunks go out now, before the CTA-wide barrier and the TMEM allocation
    const uint64_t pol = l2_evict_first_policy();
    for (uint32_t rc = 0; rc < min(n_raw, kRawStages); ++rc) {
      mbar_arrive_expect_tx(&raw_full[rc], kRawBytes);
      tma_load_2d(raw + rc * kRawBytes, &job.wmap, static_cast<int32_t>((rc_first + rc) * (kRawRow / 8)),
                  static_cast<int32_t>(m0), &raw_full[rc], pol);
    }
  }
  if (warp == 1) tmem_alloc(&tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // W is constant: the raw W producer, the dequantising warps and the MMA issuer start while
  // the previous kernel (the X split) finishes. Only the B producer reads that kernel's
  // output, so only it waits for the grid dependency; every MMA waits for its B tile and the
  // epilogue for every MMA, so Y is written after all earlier kernels (which may read Y)
  // have completed.
  if (warp >= kBWarp0) pdl_wait();
  // The next kernel may be scheduled now (it only starts once every CTA of this grid has
  // run this, and waits for this grid's completion before reading what it writes): its
  // launch overlaps this kernel instead of following it.
  pdl_launch_dependents();
  const uint32_t tmem = tmem_slot;
  const uint32_t a_col0 = 2 * N <= 128 ? 128u : 256u;
  bool ok = true;

  if (warp == 0) {
    // ---------------------------------------------------------- raw W producer
    const uint64_t pol = l2_evict_first_policy();
    uint32_t issued_raw = min(n_raw, kRawStages);  // issued by thread 0 in the prologue
    for (uint32_t rc = issued_raw; rc < n_raw && ok; ++rc) {
      const uint32_t rs = rc % kRawStages;
      if (rc >= kRawStages) ok = mbar_wait_idle(&raw_empty[rs], ((rc / kRawStages) - 1) & 1u, p.err);
      if (!__all_sync(0xFFFFFFFFu, ok)) {
        ok = false;
        break;
      }
      // one 2-D tensor copy per raw chunk: 128 rows x 144 bytes, rows past M zero-filled
      if (lane == 0) {
        mbar_arrive_expect_tx(&raw_full[rs], kRawBytes);
        tma_load_2d(raw + rs * kRawBytes, &job.wmap, static_cast<int32_t>((rc_first + rc) * (kRawRow / 8)),
                    static_cast<int32_t>(m0), &raw_full[rs], pol);
      }
      __syncwarp();
      issued_raw = rc + 1;
    }
    // copies issued into the ring land before the CTA may exit (bounded; immediate when done)
    if (lane == 0)
      for (uint32_t q = issued_raw > kRawStages ? issued_raw - kRawStages : 0; q < issued_raw; ++q)
        mbar_drain(&raw_full[q % kRawStages], (q / kRawStages) & 1u, p.err);
    __syncwarp();
  } else if (warp >= kBWarp0) {
    // ---------------------------------------------------------- B tile builders (X split)
    // item i of a sub-chunk: row n = i / 8 of the n-tile, 8 columns starting at 8 (i % 8);
    // eight consecutive threads cover one row (32-byte loads, conflict-free 16-byte stores)
    const uint32_t bt = tid - kBWarp0 * 32, n_items = N * 8, quarter = b_bytes / kBWarps;
    const uint64_t keep = l2_evict_last_policy();  // the split X is read by every row tile
    uint32_t issued = 0;
    for (uint32_t s = 0; s < n_sub && ok; ++s) {
      const uint32_t os = s % n_stage;
      if (s >= n_stage) ok = mbar_wait_idle(&op_empty[os], ((s / n_stage) - 1) & 1u, p.err);
      if (!__all_sync(0xFFFFFFFFu, ok)) {
        ok = false;
        break;
      }
      uint8_t* st = bst + os * b_bytes;
      if (p.Xs) {
        if (lane == 0) {
          const uint32_t part = warp - kBWarp0;
          const uint8_t* src = p.Xs + (static_cast<uint64_t>(blockIdx.y) * sub_total + g0 + s) * b_bytes;
          mbar_arrive_expect_tx(&b_full[os], quarter);
          bulk_g2s(st + part * quarter, src + part * quarter, quarter, &b_full[os], keep);
        }
        __syncwarp();
        issued = s + 1;
        continue;
      }
      const uint32_t k0 = (g0 + s) * kChunkK;
      if (N == 64) {
        // four items per thread: every load goes out before the first split (one load
        // latency per sub-chunk instead of four; measured faster only at this width)
        constexpr uint32_t kItems = 64 * 8 / (kBWarps * 32);
        float4 va[kItems], vb[kItems];
#pragma unroll
        for (uint32_t u = 0; u < kItems; ++u) {
          const uint32_t i = bt + u * kBWarps * 32, n = i >> 3, c = i & 7u;
          va[u] = vb[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (n0 + n < p.B) {
            const uint64_t o = static_cast<uint64_t>(n0 + n) * p.K + k0 + 8 * c;
            va[u] = __ldg(reinterpret_cast<const float4*>(p.X + o));
            vb[u] = __ldg(reinterpret_cast<const float4*>(p.X + o) + 1);
          }
        }
#pragma unroll
        for (uint32_t u = 0; u < kItems; ++u) {
          const uint32_t i = bt + u * kBWarps * 32, n = i >> 3, c = i & 7u;
          uint32_t h[4], l[4];
          split2(va[u].x, va[u].y, h[0], l[0]);
          split2(va[u].z, va[u].w, h[1], l[1]);
          split2(vb[u].x, vb[u].y, h[2], l[2]);
          split2(vb[u].z, vb[u].w, h[3], l[3]);
          *reinterpret_cast<uint4*>(st + sw128(n, c)) = make_uint4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<uint4*>(st + sw128(N + n, c)) = make_uint4(l[0], l[1], l[2], l[3]);
        }
      } else {
        for (uint32_t i = bt; i < n_items; i += kBWarps * 32) {
          const uint32_t n = i >> 3, c = i & 7u;
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
          if (n0 + n < p.B) {
            const uint64_t o = static_cast<uint64_t>(n0 + n) * p.K + k0 + 8 * c;
            a = __ldg(reinterpret_cast<const float4*>(p.X + o));
            b = __ldg(reinterpret_cast<const float4*>(p.X + o) + 1);
          }
          uint32_t h[4], l[4];
          split2(a.x, a.y, h[0], l[0]);
          split2(a.z, a.w, h[1], l[1]);
          split2(b.x, b.y, h[2], l[2]);
          split2(b.z, b.w, h[3], l[3]);
          *reinterpret_cast<uint4*>(st + sw128(n, c)) = make_uint4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<uint4*>(st + sw128(N + n, c)) = make_uint4(l[0], l[1], l[2], l[3]);
        }
      }
      fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&b_full[os]);
    }
    // bulk copies issued into the stages land before the CTA may exit (bounded)
    if (p.Xs && lane == 0)
      for (uint32_t q = issued > n_stage ? issued - n_stage : 0; q < issued; ++q)
        mbar_drain(&b_full[q % n_stage], (q / n_stage) & 1u, p.err);
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kTileM, 2 * N);
      for (uint32_t s = 0; s < n_sub && ok; ++s) {
        const uint32_t os = s % n_stage, par = (s / n_stage) & 1u;
        ok = mbar_wait_idle(&a_full[os], par, p.err) && mbar_wait_idle(&b_full[os], par, p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a0 = tmem + a_col0 + os * kStageCols;
        const uint64_t db = smem_desc_sw128(smem_addr(bst + os * b_bytes));
#pragma unroll
        for (uint32_t ks = 0; ks < kChunkK / 16; ++ks)
#pragma unroll
          for (uint32_t t = 0; t < F::kTerms; ++t)
            mma_bf16_ts(tmem, a0 + 32 * t + 8 * ks, db + 2ull * ks, idesc, (s | ks | t) != 0);
        mma_commit(&op_empty[os]);
      }
      mma_commit(&acc_full);  // after every MMA issued (or none)
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- dequant (warps 2..17)
    // Every warp walks every sub-chunk so that each raw chunk is waited for and released by
    // all 16 warps in order; a warp dequantizes only its group's sub-chunks.
    const uint32_t grp = (warp - 2) >> 3, q = warp & 3u, blk = ((warp - 2) >> 2) & 1u, r = 32 * q + lane;
    const uint32_t lane_addr = tmem + ((32 * q) << 16) + a_col0 + blk * 16;
    for (uint32_t s = 0; s < n_sub && ok; ++s) {
      const uint32_t g = g0 + s, rc = g / (kRawK / kChunkK) - rc_first, sub = g % (kRawK / kChunkK);
      const uint32_t rs = rc % kRawStages, os = s % n_stage;
      const bool mine = (s & 1u) == grp;
      if (s == 0 || sub == 0) ok = mbar_wait_idle(&raw_full[rs], (rc / kRawStages) & 1u, p.err);
      if (mine && ok && s >= n_stage) ok = mbar_wait_idle(&op_empty[os], ((s / n_stage) - 1) & 1u, p.err);
      if (!__all_sync(0xFFFFFFFFu, ok)) {
        ok = false;
        break;
      }
      if (mine) {
        tc_fence_after();
        // the block starts 2 bytes into a 32-bit word when blk is odd (18- and 34-byte
        // blocks in rows of a multiple of 4 bytes): read from the aligned word below it
        const uint32_t* src = reinterpret_cast<const uint32_t*>(raw + rs * kRawBytes + r * kRawRow +
                                                                (sub * 2 + blk) * F::kBlock - blk * 2);
        const uint32_t ta = lane_addr + os * kStageCols;
        if constexpr (kQ == 4) {
          uint32_t hi[16], lo[16];
          dequant_block_bf16x2(src, blk, hi, lo);
          tmem_st16(ta, hi);
          tmem_st16(ta + 32, lo);
        } else {
          uint32_t t0[16], t1[16], t2[16];
          dequant_q8_block_bf16x3(src, blk, t0, t1, t2);
          tmem_st16(ta, t0);
          tmem_st16(ta + 32, t1);
          tmem_st16(ta + 64, t2);
        }
        tmem_wait_st();
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) {
        if (mine) mbar_arrive(&a_full[os]);
        if (sub == 3 || s + 1 == n_sub) mbar_arrive(&raw_empty[rs]);  // this warp is done with the chunk
      }
    }
  }

  // ------------------------------------------------------------ epilogue (warps 2..9)
  // every warp, on every path, reaches the same barriers below
  if (warp >= 2 && warp < 10) ok = mbar_drain(&acc_full, 0, p.err) && ok;
  const int all_ok = __syncthreads_and(ok);
  tc_fence_after();
  const uint32_t n_valid = min(N, p.B - n0);
  float* part = reinterpret_cast<float*>(bst);  // [N][128] partial tile, reusing the B stages
  if (warp >= 2 && warp < 10) {
    const uint32_t q = warp & 3u, half = (warp - 2) >> 2, row = 32 * q + lane;
    for (uint32_t c0 = half * (N / 2); c0 < (half + 1) * (N / 2) && c0 < n_valid; c0 += 8) {
      float v[8], u[8];
      tmem_ld8(tmem + ((32 * q) << 16) + c0, v);
      tmem_ld8(tmem + ((32 * q) << 16) + N + c0, u);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += u[e];
      if (p.S == 1) {
        if (all_ok && m0 + row < M)
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (c0 + e < n_valid) {
              float* y = Y + static_cast<uint64_t>(n0 + c0 + e) * M + m0 + row;
              *y = p.accumulate ? __fadd_rn(*y, v[e]) : v[e];
            }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) part[(c0 + e) * kTileM + row] = v[e];
      }
    }
  }
  if (p.S > 1) {
    cluster_sync();  // every partial tile of the cluster is in shared memory
    const uint32_t c_lo = static_cast<uint32_t>(static_cast<uint64_t>(n_valid) * z / p.S);
    const uint32_t c_hi = static_cast<uint32_t>(static_cast<uint64_t>(n_valid) * (z + 1) / p.S);
    const uint32_t base_addr = smem_addr(part);
    for (uint32_t i = tid; i < (c_hi - c_lo) * kTileM; i += kWsThreads) {
      const uint32_t c = c_lo + i / kTileM, row = i % kTileM;
      const uint32_t a = base_addr + (c * kTileM + row) * 4u;
      float v[kMaxSplit];
#pragma unroll
      for (uint32_t rk = 0; rk < kMaxSplit; ++rk)
        if (rk < p.S) v[rk] = ld_dsmem(dsmem_map(a, rk));  // all loads in flight, then a fixed-order sum
      float acc = v[0];
#pragma unroll
      for (uint32_t rk = 1; rk < kMaxSplit; ++rk)
        if (rk < p.S) acc += v[rk];
      if (all_ok && m0 + row < M) {
        float* y = Y + static_cast<uint64_t>(n0 + c) * M + m0 + row;
        *y = p.accumulate ? __fadd_rn(*y, acc) : acc;
      }
    }
    cluster_sync();  // peers keep their shared memory until every read is done
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// Per-device grow-only scratch for the split X of wide tiles (N > 64).
struct GemmScratch {
  std::mutex mu;
  void* p = nullptr;
  size_t cap = 0;
};
GemmScratch g_gemm_scratch[64];

// Largest number of S-CTA clusters the device keeps resident at once, per (device, S, smem):
// the split is chosen so that every cluster of a call is resident in one wave.
struct ClusterFit {
  std::mutex mu;
  size_t smem[kMaxSplit + 1] = {};
  int clusters[kMaxSplit + 1] = {};
};
ClusterFit g_cluster_fit[64][2];  // [device][Q4_0, Q8_0]

}  // namespace

// The warp-specialised path (K % 256 == 0): one kernel, split-K over a cluster of S CTAs
// sized so that one wave covers the SMs.
template <int kQ>
int launch_gemm_ws(const GemmCall& c, int* d_err, cudaStream_t s) {
  using F = WsFormat<kQ>;
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  const size_t K = c.K, B = c.B;
  const uint32_t n_tile = static_cast<uint32_t>(std::min<size_t>(kMaxTileN2, (B + 15) / 16 * 16));
  const uint32_t n_tiles = static_cast<uint32_t>((B + n_tile - 1) / n_tile);
  GemmWsParams p{};
  uint32_t m_tiles = 0;
  for (int j = 0; j < c.n_jobs; ++j) {
    const GemmJob& jb = c.jobs[j];
    GemmJobDev& jd = p.jobs[j];
    if (!encode_u64_rows_map(&jd.wmap, jb.W, jb.M, K / 32 * F::kBlock, F::kRawRow / 8, kTileM))
      return fail(EFG_ECUDA, "gemm: tensor map for a %zu x %zu Q%d_0 matrix", jb.M, K, kQ);
    jd.Y = jb.Y;
    jd.M = static_cast<uint32_t>(jb.M);
    jd.tile0 = m_tiles;
    m_tiles += static_cast<uint32_t>((jb.M + kTileM - 1) / kTileM);
  }
  const uint8_t* Xs = nullptr;
  std::unique_lock<std::mutex> lk;
  if (n_tile > 64) {  // split X once per call (see the kernel's role notes)
    GemmScratch& gs = g_gemm_scratch[dev->device];
    lk = std::unique_lock<std::mutex>(gs.mu);
    const size_t ws_bytes = static_cast<size_t>(n_tiles) * (K / kChunkK) * 2 * n_tile * 128;
    if (ws_bytes > gs.cap) {
      if (gs.p) cudaFree(gs.p);
      gs.p = nullptr;
      gs.cap = 0;
      EFG_TRY_CUDA(cudaMalloc(&gs.p, ws_bytes), "gemm workspace");
      gs.cap = ws_bytes;
    }
    const uint64_t items = static_cast<uint64_t>(n_tiles) * (K / kChunkK) * n_tile * 8;
    const unsigned grid = static_cast<unsigned>(std::min<uint64_t>((items + 255) / 256, 8ull * dev->sm_count));
    split_x_kernel<<<grid, 256, 0, s>>>(c.X, static_cast<uint32_t>(B), static_cast<uint32_t>(K), n_tile,
                                        static_cast<uint8_t*>(gs.p), n_tiles);
    EFG_TRY_CUDA(cudaGetLastError(), "gemm split launch");
    Xs = static_cast<const uint8_t*>(gs.p);
  }
  // TMEM: the accumulator below column 128 or 256, then as many A stages as fit
  const uint32_t a_col0 = 2 * n_tile <= 128 ? 128u : 256u;
  const uint32_t a_stages = std::min<uint32_t>(kMaxAStages, (kTmemCols - a_col0) / (32 * F::kTerms));
  const size_t smem = std::max(kWsMinSmem, 1024 + a_stages * 2 * static_cast<size_t>(n_tile) * 128 +
                                               static_cast<size_t>(F::kRawStages) * kTileM * F::kRawRow);
  auto* kernel = gemm_ws_kernel<kQ>;
  if (int st = ensure_smem_attr(reinterpret_cast<const void*>(kernel), smem)) return st;
  const uint32_t sub_total = static_cast<uint32_t>(K / kChunkK);
  uint32_t S = std::max<uint32_t>(1, static_cast<uint32_t>(dev->sm_count) / (m_tiles * n_tiles));
  S = std::min<uint32_t>({S, kMaxSplit, std::max<uint32_t>(1, sub_total / 4)});
  p.n_jobs = static_cast<uint32_t>(c.n_jobs);
  p.X = c.X;
  p.Xs = Xs;
  p.accumulate = c.accumulate ? 1u : 0u;
  p.K = static_cast<uint32_t>(K);
  p.B = static_cast<uint32_t>(B);
  p.n_tile = n_tile;
  p.a_stages = a_stages;
  p.err = d_err;
  ClusterFit& fit = g_cluster_fit[dev->device][kQ == 8];
  for (;; --S) {  // the largest split whose clusters are all resident at once
    p.S = std::max(S, 1u);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(m_tiles, n_tiles, p.S);
    cfg.blockDim = dim3(kWsThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = p.S;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (p.S > 1) {
      int clusters = 0;
      {
        std::lock_guard<std::mutex> g(fit.mu);
        if (fit.smem[p.S] == smem) {
          clusters = fit.clusters[p.S];
        } else {
          if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
            cudaGetLastError();
            clusters = 0;
          }
          fit.smem[p.S] = smem;
          fit.clusters[p.S] = clusters;
        }
      }
      if (clusters < static_cast<int>(m_tiles * n_tiles)) continue;
    }
    EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, kernel, p), "gemm launch");
    return EFG_OK;
  }
}

int launch_gemm_q4_0(float* Y, const uint8_t* W, const float* X, size_t M, size_t K, size_t B, int* d_err,
                     cudaStream_t s) {
  if (K % 32 != 0) return fail(EFG_EINVAL, "Q4_0 needs a row length divisible by 32, got %zu", K);
  if (M == 0 || B == 0) return EFG_OK;
  if (!Y || (K && (!W || !X))) return fail(EFG_EINVAL, "gemm: null pointer");
  if (M >= (1u << 31) || K >= (1u << 30) || B >= (1u << 20)) return fail(EFG_EINVAL, "gemm: shape too large");
  if (K == 0) {
    EFG_TRY_CUDA(cudaMemsetAsync(Y, 0, M * B * sizeof(float), s), "gemm zero fill");
    return EFG_OK;
  }
  if (reinterpret_cast<uintptr_t>(X) % 16 != 0 || reinterpret_cast<uintptr_t>(W) % 2 != 0 ||
      reinterpret_cast<uintptr_t>(Y) % 4 != 0)
    return fail(EFG_EINVAL, "gemm: X must be 16-byte aligned, W 2-byte aligned and Y 4-byte aligned");
  if (K % kRawK == 0 && reinterpret_cast<uintptr_t>(W) % 16 == 0) {
    GemmCall c;
    c.qtype = 4;
    c.jobs[0] = GemmJob{W, Y, M};
    c.n_jobs = 1;
    c.X = X;
    c.K = K;
    c.B = B;
    if (DeviceInfo* dev = current_device(); dev && small_gemm_flag() && gemm_q4_small_ok(c, *dev))
      return launch_gemm_q4_small(c, *dev, d_err, s);
    return launch_gemm_ws<4>(c, d_err, s);
  }
  const uint32_t n_tile = static_cast<uint32_t>(std::min<size_t>(kMaxTileN, (B + 15) / 16 * 16));
  GemmParams p{W, X, Y, static_cast<uint32_t>(M), static_cast<uint32_t>(K), static_cast<uint32_t>(B),
               static_cast<uint32_t>(K / 32 * 18), n_tile, d_err};
  const size_t smem = 1024 + 2 * (2 * kATileBytes + 2 * static_cast<size_t>(n_tile) * 128);
  if (int st = ensure_smem_attr(reinterpret_cast<const void*>(gemm_q4_0_kernel), smem)) return st;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>((M + kTileM - 1) / kTileM), static_cast<unsigned>((B + n_tile - 1) / n_tile));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = weight_prefetch_flag() ? 1 : 0;
  EFG_TRY_CUDA(cudaLaunchKernelEx(&cfg, gemm_q4_0_kernel, p), "gemm launch");
  return EFG_OK;
}

int launch_gemm_q8_0(float* Y, const uint8_t* W, const float* X, size_t M, size_t K, size_t B, int* d_err,
                     cudaStream_t s) {
  if (K % kRawK != 0)
    return fail(EFG_EINVAL, "the Q8_0 GEMM needs a row length divisible by %u, got %zu", kRawK, K);
  if (M == 0 || B == 0) return EFG_OK;
  if (!Y || (K && (!W || !X))) return fail(EFG_EINVAL, "gemm: null pointer");
  if (M >= (1u << 31) || K >= (1u << 30) || B >= (1u << 20)) return fail(EFG_EINVAL, "gemm: shape too large");
  if (K == 0) {
    EFG_TRY_CUDA(cudaMemsetAsync(Y, 0, M * B * sizeof(float), s), "gemm zero fill");
    return EFG_OK;
  }
  if (reinterpret_cast<uintptr_t>(X) % 16 != 0 || reinterpret_cast<uintptr_t>(W) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(Y) % 4 != 0)
    return fail(EFG_EINVAL, "gemm: X and W must be 16-byte aligned and Y 4-byte aligned");
  GemmCall c;
  c.qtype = 8;
  c.jobs[0] = GemmJob{W, Y, M};
  c.n_jobs = 1;
  c.X = X;
  c.K = K;
  c.B = B;
  return launch_gemm_ws<8>(c, d_err, s);
}

int launch_gemm(const GemmCall& call, int* d_err, cudaStream_t s) {
  if ((call.qtype != 4 && call.qtype != 8) || call.n_jobs < 1 || call.n_jobs > static_cast<int>(kMaxGemmJobs))
    return fail(EFG_EINVAL, "gemm: %d jobs of type %d", call.n_jobs, call.qtype);
  if (call.K % kRawK != 0 || call.K >= (1u << 30) || call.B >= (1u << 20))
    return fail(EFG_EINVAL, "gemm: K = %zu, B = %zu", call.K, call.B);
  GemmCall c = call;  // the jobs with rows
  c.n_jobs = 0;
  size_t tiles = 0;
  for (int j = 0; j < call.n_jobs; ++j) {
    const GemmJob& jb = call.jobs[j];
    if (jb.M == 0) continue;
    if (!jb.Y || (call.K && !jb.W) || jb.M >= (1u << 31) || reinterpret_cast<uintptr_t>(jb.W) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(jb.Y) % 4 != 0)
      return fail(EFG_EINVAL, "gemm: job %d (M = %zu) needs 16-byte aligned weights and an output", j, jb.M);
    c.jobs[c.n_jobs++] = jb;
    tiles += (jb.M + kTileM - 1) / kTileM;
  }
  if (c.n_jobs == 0 || c.B == 0) return EFG_OK;
  if (c.K == 0) {  // every dot is empty: Y = 0, or Y unchanged when adding
    if (!c.accumulate)
      for (int j = 0; j < c.n_jobs; ++j)
        EFG_TRY_CUDA(cudaMemsetAsync(c.jobs[j].Y, 0, c.jobs[j].M * c.B * sizeof(float), s), "gemm zero fill");
    return EFG_OK;
  }
  if (!c.X || reinterpret_cast<uintptr_t>(c.X) % 16 != 0)
    return fail(EFG_EINVAL, "gemm: the B operand must be 16-byte aligned");
  if (tiles >= (1u << 31)) return fail(EFG_EINVAL, "gemm: too many row tiles");
  if (c.qtype == 4)
    if (DeviceInfo* dev = current_device(); dev && small_gemm_flag() && gemm_q4_small_ok(c, *dev))
      return launch_gemm_q4_small(c, *dev, d_err, s);
  return c.qtype == 4 ? launch_gemm_ws<4>(c, d_err, s) : launch_gemm_ws<8>(c, d_err, s);
}

}  // namespace efg

extern "C" int efg_gemm_q4_0(float* d_Y, const uint8_t* d_W, const float* d_X, size_t M, size_t K, size_t B,
                             void* stream) {
  efg::DeviceInfo* dev = efg::current_device();
  if (!dev) return EFG_ECUDA;
  return efg::launch_gemm_q4_0(d_Y, d_W, d_X, M, K, B, dev->d_err, static_cast<cudaStream_t>(stream));
}

extern "C" int efg_gemm_q8_0(float* d_Y, const uint8_t* d_W, const float* d_X, size_t M, size_t K, size_t B,
                             void* stream) {
  efg::DeviceInfo* dev = efg::current_device();
  if (!dev) return EFG_ECUDA;
  return efg::launch_gemm_q8_0(d_Y, d_W, d_X, M, K, B, dev->d_err, static_cast<cudaStream_t>(stream));
}

extern "C" int efg_gemm_jobs(int qtype, int n_jobs, const uint8_t* const* d_W, float* const* d_Y, const size_t* M,
                             const float* d_X, size_t K, size_t B, int accumulate, void* stream) {
  efg::DeviceInfo* dev = efg::current_device();
  if (!dev) return EFG_ECUDA;
  if ((qtype != EFG_Q4_0 && qtype != EFG_Q8_0) || n_jobs < 1 || n_jobs > 3 || !d_W || !d_Y || !M)
    return efg::fail(EFG_EINVAL, "gemm jobs: type %d with %d jobs (1 to 3 of Q4_0 or Q8_0)", qtype, n_jobs);
  efg::GemmCall c;
  c.qtype = qtype == EFG_Q4_0 ? 4 : 8;
  for (int j = 0; j < n_jobs; ++j) c.jobs[j] = efg::GemmJob{d_W[j], d_Y[j], M[j]};
  c.n_jobs = n_jobs;
  c.X = d_X;
  c.K = K;
  c.B = B;
  c.accumulate = accumulate != 0;
  return efg::launch_gemm(c, dev->d_err, static_cast<cudaStream_t>(stream));
}
