// efg_gemm.cu - batched Q4_0 x activation GEMM on the 5th-generation tensor cores.
//
//   Y[b][m] = sum_k W[m][k] X[b][k]      W: Q4_0 rows [M][K/32 blocks], X: FP32 [B][K],
//                                         Y: FP32 [B][M]
//
// The reference has no GEMM: its prompt and multi-sequence work is one ef::kern::matvec per
// column (src/qkernels.cpp:275-297), which is the oracle here. The tensor-core formulation
// keeps that FP32 result within 1e-5 of sum |w x| per output:
//   * a Q4_0 weight w = (c - 8) * d (4-bit code, FP16 scale) has at most 14 significant
//     bits, so w = w_hi + w_lo with w_hi = bf16(w) and w_lo = bf16(w - w_hi) is EXACT;
//   * x = x1 + x2 with x1 = bf16(x), x2 = bf16(x - x1) keeps 16 significant bits;
//   * D = W_hi X1 + W_hi X2 + W_lo X1 in FP32 (tcgen05.mma kind::f16, BF16 operands): every
//     product is exact in FP32, the dropped terms (W_lo X2 and the residual of x) are at most
//     2^-16 of each |w x| and of random sign.
//
// One CTA computes a 128-row x N_TILE tile (N_TILE = B rounded up to 16, at most 256), the
// accumulator in TMEM (128 lanes x N_TILE FP32 columns). K advances in 64-wide chunks
// through two shared-memory stages: all 256 threads dequantize the chunk's W rows into the
// W_hi / W_lo tiles and split X into X1 / X2 (K-major, 128-byte swizzled, the canonical
// UMMA layout), then one thread issues the 12 MMAs of the chunk (3 products x 4 K-steps)
// and commits them to the stage's mbarrier, which the threads wait on before they refill
// that stage two chunks later. The epilogue reads TMEM with tcgen05.ld (warp w sees lanes
// 32 (w % 4) ..) and writes Y with coalesced stores.
#include <algorithm>
#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/efg.h"
#include "efg_device.cuh"
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

}  // namespace

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

}  // namespace efg

extern "C" int efg_gemm_q4_0(float* d_Y, const uint8_t* d_W, const float* d_X, size_t M, size_t K, size_t B,
                             void* stream) {
  efg::DeviceInfo* dev = efg::current_device();
  if (!dev) return EFG_ECUDA;
  return efg::launch_gemm_q4_0(d_Y, d_W, d_X, M, K, B, dev->d_err, static_cast<cudaStream_t>(stream));
}
