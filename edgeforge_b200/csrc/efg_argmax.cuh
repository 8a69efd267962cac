// efg_argmax.cuh - kern::argmax (src/kernels.cpp:105-111) on the device: the block-level
// scan shared by the decode step's argmax and the standalone / row-sharded entry points.
//
// The reference starts from index 0 and takes strictly greater values, so its result is
// the largest non-NaN value with the lowest index among ties -- unless element 0 is NaN,
// which no comparison replaces (result 0). That rule distributes: each shard reports its
// largest non-NaN value and lowest index, and the shards are combined in index order.
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace efg {

// One shard's candidate: i >= 0 its global index and value; i = -1 no non-NaN element;
// i = -2 the shard starts the vector and its element 0 is NaN (the result is 0).
struct ArgmaxPair {
  float v;
  int32_t i;
};

#ifdef __CUDACC__
// Largest non-NaN element of x[0..n) with the lowest index among ties, by one CTA (any
// blockDim that is a multiple of 32, <= 1024). Valid in thread 0: idx = 0xFFFFFFFF when
// there is none. Loads are float4 (up to 8 in flight per thread) when x is 16-byte aligned.
__device__ __forceinline__ void block_argmax(const float* __restrict__ x, uint32_t n, float& best_out,
                                             uint32_t& idx_out) {
  __shared__ float bv[32];
  __shared__ uint32_t bi[32];
  float best = -INFINITY;
  uint32_t idx = 0xFFFFFFFFu;
  // each thread scans its elements in increasing index order: the first non-NaN value,
  // then strictly greater ones
  auto take = [&](float v, uint32_t i) {
    if (idx == 0xFFFFFFFFu ? !(v != v) : v > best) {
      best = v;
      idx = i;
    }
  };
  const uint32_t n4 = reinterpret_cast<uintptr_t>(x) % 16 == 0 ? n / 4 : 0;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (uint32_t base = threadIdx.x; base < n4; base += 8 * blockDim.x) {
    float4 v[8];
#pragma unroll
    for (uint32_t u = 0; u < 8; ++u) {
      const uint32_t c = base + u * blockDim.x;
      v[u] = c < n4 ? x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (uint32_t u = 0; u < 8; ++u) {
      const uint32_t c = base + u * blockDim.x;
      if (c < n4) {
        take(v[u].x, 4 * c);
        take(v[u].y, 4 * c + 1);
        take(v[u].z, 4 * c + 2);
        take(v[u].w, 4 * c + 3);
      }
    }
  }
  for (uint32_t i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) take(x[i], i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
    if (oi != 0xFFFFFFFFu && (idx == 0xFFFFFFFFu || ov > best || (ov == best && oi < idx))) {
      best = ov;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = best;
    bi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    best = bv[0];
    idx = bi[0];
    for (uint32_t w = 1; w < blockDim.x / 32; ++w)
      if (bi[w] != 0xFFFFFFFFu && (idx == 0xFFFFFFFFu || bv[w] > best || (bv[w] == best && bi[w] < idx))) {
        best = bv[w];
        idx = bi[w];
      }
    best_out = best;
    idx_out = idx;
  }
}
#endif  // __CUDACC__

// *index = kern::argmax(x, n) (0 for n = 0).
int launch_argmax_index(const float* x, size_t n, int32_t* index, cudaStream_t s);
// out = this shard's ArgmaxPair (x = logits [offset, offset + n) of the whole vector).
int launch_argmax_local(const float* x, size_t n, size_t offset, ArgmaxPair* out, cudaStream_t s);
// *index = the whole vector's argmax from every shard's pair, shards in index order.
int launch_argmax_combine(const ArgmaxPair* pairs, int count, int32_t* index, cudaStream_t s);
// The row-sharded argmax in one launch: this shard's pair (logits [offset, offset + n)) stored
// into every rank's flag area by peer stores, the peers' pairs awaited (bounded: EFG_ETIMEOUT
// in *err) and combined; every rank's flag area must be mapped (efg_comm_register).
struct GatherDev;
int launch_argmax_exchange(const float* x, size_t n, size_t offset, const GatherDev& g, int32_t* index, int* err,
                           cudaStream_t s);

}  // namespace efg
