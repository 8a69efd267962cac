// efg_gemm.cuh - the batched Q4_0 GEMM (efg_gemm.cu) for other library code.
#pragma once
#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace efg {

// Y[b][m] = sum_k W[m][k] * X[b][k] for b < B (W Q4_0 M x K, X [B][K] FP32 16-byte aligned,
// Y [B][M]); the tcgen05 kernels of efg_gemm.cu. For B <= 64 (and K % 256 == 0) one kernel
// launch and no scratch memory, safe to record in a CUDA graph; wider calls first split X into
// a per-device scratch that grows with the largest call (do not record those in a graph that
// may outlive a larger call, and do not let wide calls on different streams overlap: they
// share the scratch). Returns an EFG_* status.
int launch_gemm_q4_0(float* Y, const uint8_t* W, const float* X, size_t M, size_t K, size_t B, int* d_err,
                     cudaStream_t s);
// The same product for Q8_0 weights (K a multiple of 256, W and X 16-byte aligned).
int launch_gemm_q8_0(float* Y, const uint8_t* W, const float* X, size_t M, size_t K, size_t B, int* d_err,
                     cudaStream_t s);

// Several matrices of one weight format that share K and the B operand X, in one launch;
// the product may be added into Y (the decoder's residual add, Y = fl(Y + product) as an
// elementwise add after the product would give). K a multiple of 256, weights and X 16-byte
// aligned.
struct GemmJob {
  const uint8_t* W = nullptr;
  float* Y = nullptr;  // [B][M]
  size_t M = 0;
};
struct GemmCall {
  int qtype = 4;  // 4: Q4_0, 8: Q8_0
  GemmJob jobs[3];
  int n_jobs = 0;
  const float* X = nullptr;  // [B][K]
  size_t K = 0, B = 0;
  bool accumulate = false;  // Y += product (the residual add)
};
int launch_gemm(const GemmCall& c, int* d_err, cudaStream_t s);

struct DeviceInfo;
// The Q4_0 GEMM for small batches (B <= 64) on the exact integer MMA (efg_matvec_mma.cu): the
// X columns as the A operand in int8 digit planes, the codes as B; each CTA fetches its 8-row
// units whole at its start. Taken for Q4_0 calls with 2048 <= K <= 8192, K % 256 == 0, 16-byte
// aligned weights and X, and a per-CTA share that fits in shared memory; columns with
// non-finite x come out as the FP32 matvec computes them. One launch, no scratch.
bool gemm_q4_small_ok(const GemmCall& c, const DeviceInfo& dev);
int launch_gemm_q4_small(const GemmCall& c, const DeviceInfo& dev, int* d_err, cudaStream_t s);

}  // namespace efg
