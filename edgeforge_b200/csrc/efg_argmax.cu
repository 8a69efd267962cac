// efg_argmax.cu - kern::argmax (src/kernels.cpp:105-111) as a device entry point, and its
// row-sharded form for an lm_head split over the GPUs of one node (efg_shard.cpp).
#include "../../include/efg.h"
#include "efg_argmax.cuh"
#include "efg_device.cuh"
#include "efg_gather.cuh"
#include "efg_host.h"

namespace efg {
namespace {

__device__ __forceinline__ ArgmaxPair shard_pair(const float* x, uint32_t n, uint64_t offset, float best, uint32_t idx) {
  if (offset == 0 && n > 0 && x[0] != x[0]) return ArgmaxPair{0.f, -2};
  if (idx == 0xFFFFFFFFu) return ArgmaxPair{0.f, -1};
  return ArgmaxPair{best, static_cast<int32_t>(offset + idx)};
}

// The pairs in rank (= index) order -> the whole vector's argmax (kern::argmax's rule).
__device__ __forceinline__ int32_t combine_pair(int32_t& idx, float& best, const ArgmaxPair p) {
  if (idx == -3) return idx;     // decided: element 0 of the whole vector is NaN
  if (p.i == -2) return idx = -3;
  if (p.i >= 0 && (idx < 0 || p.v > best)) {  // shards in index order: ties keep the lower index
    best = p.v;
    idx = p.i;
  }
  return idx;
}

__global__ void __launch_bounds__(1024) argmax_index_kernel(const float* __restrict__ x, uint32_t n,
                                                            int32_t* __restrict__ index) {
  float best;
  uint32_t idx;
  block_argmax(x, n, best, idx);
  if (threadIdx.x == 0) *index = n == 0 || x[0] != x[0] || idx == 0xFFFFFFFFu ? 0 : static_cast<int32_t>(idx);
}

__global__ void __launch_bounds__(1024) argmax_local_kernel(const float* __restrict__ x, uint32_t n, uint64_t offset,
                                                            ArgmaxPair* __restrict__ out) {
  float best;
  uint32_t idx;
  block_argmax(x, n, best, idx);
  if (threadIdx.x == 0) *out = shard_pair(x, n, offset, best, idx);
}

// This shard's argmax, its pair stored into every rank's flag area over NVLink (one lane per
// rank, the pair then a release flag carrying the call number), a bounded wait for every
// peer's pair of the same call, and the combination in rank order: one launch instead of a
// local argmax, a collective and a combine. Pairs alternate between two slots by call
// parity: a rank can be at most one call ahead of another (call e + 1 waits for every rank's
// pair of call e + 1, which a rank sends only after its call e has read its slots).
__global__ void __launch_bounds__(1024) argmax_exchange_kernel(const float* __restrict__ x, uint32_t n,
                                                               uint64_t offset, const GatherDev g,
                                                               int32_t* __restrict__ index, int* err) {
  __shared__ ArgmaxPair mine_s;
  __shared__ uint32_t epoch_s;
  float best;
  uint32_t idx;
  block_argmax(x, n, best, idx);
  if (threadIdx.x == 0) {
    mine_s = shard_pair(x, n, offset, best, idx);
    epoch_s = *reinterpret_cast<const volatile uint32_t*>(g.flags + kPairEpochOff) + 1u;
  }
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  const uint32_t epoch = epoch_s, par = epoch & 1u;
  const ArgmaxPair mine = mine_s;
  if (lane < g.nranks) {  // lane == rank: this rank's own slot (peer_flags[rank] is flags)
    uint32_t* f = g.peer_flags[lane];
    f[kPairOff + (par * kMaxGatherRanks + g.rank) * 2] = __float_as_uint(mine.v);
    f[kPairOff + (par * kMaxGatherRanks + g.rank) * 2 + 1] = static_cast<uint32_t>(mine.i);
    st_release_sys(f + kPairFlagOff + par * kMaxGatherRanks + g.rank, epoch);
  }
  const bool ok = gather_wait_flags(g, kPairFlagOff + par * kMaxGatherRanks, epoch, err);
  // lane q reads rank q's pair after its own acquire of that rank's flag (or its own store)
  ArgmaxPair p{0.f, -1};
  if (lane < g.nranks) {
    const volatile uint32_t* slot = g.flags + kPairOff + (par * kMaxGatherRanks + lane) * 2;
    p = lane == g.rank ? mine : ArgmaxPair{__uint_as_float(slot[0]), static_cast<int32_t>(slot[1])};
  }
  int32_t r = -1;
  float b = 0.f;
  for (int q = 0; q < g.nranks; ++q) {
    const float v = __shfl_sync(0xFFFFFFFFu, p.v, q);
    const int32_t i = __shfl_sync(0xFFFFFFFFu, p.i, q);
    combine_pair(r, b, ArgmaxPair{v, i});
  }
  if (lane == 0) {
    *index = !ok ? 0 : (r < 0 ? 0 : r);
    *reinterpret_cast<volatile uint32_t*>(g.flags + kPairEpochOff) = epoch;
  }
}

__global__ void argmax_combine_kernel(const ArgmaxPair* __restrict__ pairs, int count, int32_t* __restrict__ index) {
  if (threadIdx.x != 0) return;
  int32_t idx = -1;
  float best = 0.f;
  for (int r = 0; r < count; ++r) combine_pair(idx, best, pairs[r]);
  *index = idx < 0 ? 0 : idx;
}

}  // namespace

int launch_argmax_index(const float* x, size_t n, int32_t* index, cudaStream_t s) {
  if (n >= (1ull << 31)) return fail(EFG_EINVAL, "argmax: n too large");
  argmax_index_kernel<<<1, 1024, 0, s>>>(x, static_cast<uint32_t>(n), index);
  EFG_TRY_CUDA(cudaGetLastError(), "argmax launch");
  return EFG_OK;
}

int launch_argmax_local(const float* x, size_t n, size_t offset, ArgmaxPair* out, cudaStream_t s) {
  if (n >= (1ull << 31)) return fail(EFG_EINVAL, "argmax: n too large");
  argmax_local_kernel<<<1, 1024, 0, s>>>(x, static_cast<uint32_t>(n), offset, out);
  EFG_TRY_CUDA(cudaGetLastError(), "argmax launch");
  return EFG_OK;
}

int launch_argmax_exchange(const float* x, size_t n, size_t offset, const GatherDev& g, int32_t* index, int* err,
                           cudaStream_t s) {
  if (n >= (1ull << 31)) return fail(EFG_EINVAL, "argmax: n too large");
  if (g.nranks < 1 || g.nranks > kMaxGatherRanks || g.rank < 0 || g.rank >= g.nranks || !g.flags)
    return fail(EFG_EINVAL, "argmax exchange: bad ranks");
  for (int q = 0; q < g.nranks; ++q)
    if (!g.peer_flags[q]) return fail(EFG_EINVAL, "argmax exchange: rank %d's flag area is not mapped", q);
  argmax_exchange_kernel<<<1, 1024, 0, s>>>(x, static_cast<uint32_t>(n), offset, g, index, err);
  EFG_TRY_CUDA(cudaGetLastError(), "argmax launch");
  return EFG_OK;
}

int launch_argmax_combine(const ArgmaxPair* pairs, int count, int32_t* index, cudaStream_t s) {
  argmax_combine_kernel<<<1, 32, 0, s>>>(pairs, count, index);
  EFG_TRY_CUDA(cudaGetLastError(), "argmax launch");
  return EFG_OK;
}

}  // namespace efg

extern "C" int efg_argmax(const float* d_x, size_t n, int32_t* d_index, void* stream) {
  if (!d_index || (!d_x && n)) return efg::fail(EFG_EINVAL, "argmax: null pointer");
  return efg::launch_argmax_index(d_x, n, d_index, static_cast<cudaStream_t>(stream));
}
