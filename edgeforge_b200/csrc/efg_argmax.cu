// efg_argmax.cu - kern::argmax (src/kernels.cpp:105-111) as a device entry point, and its
// row-sharded form for an lm_head split over the GPUs of one node (efg_shard.cpp).
#include "../../include/efg.h"
#include "efg_argmax.cuh"
#include "efg_device.cuh"
#include "efg_host.h"

namespace efg {
namespace {

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
  if (threadIdx.x == 0) {
    ArgmaxPair p;
    if (offset == 0 && n > 0 && x[0] != x[0]) {
      p = ArgmaxPair{0.f, -2};
    } else if (idx == 0xFFFFFFFFu) {
      p = ArgmaxPair{0.f, -1};
    } else {
      p = ArgmaxPair{best, static_cast<int32_t>(offset + idx)};
    }
    *out = p;
  }
}

__global__ void argmax_combine_kernel(const ArgmaxPair* __restrict__ pairs, int count, int32_t* __restrict__ index) {
  if (threadIdx.x != 0) return;
  int32_t idx = -1;
  float best = 0.f;
  for (int r = 0; r < count; ++r) {
    const ArgmaxPair p = pairs[r];
    if (p.i == -2) {  // element 0 of the whole vector is NaN
      idx = 0;
      break;
    }
    if (p.i >= 0 && (idx < 0 || p.v > best)) {  // shards in index order: ties keep the lower index
      best = p.v;
      idx = p.i;
    }
  }
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
