// efg_gemm.cuh - the batched Q4_0 GEMM (efg_gemm.cu) for other library code.
#pragma once
#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace efg {

// Y[b][m] = sum_k W[m][k] * X[b][k] for b < B (W Q4_0 M x K, X [B][K] FP32 16-byte aligned,
// Y [B][M]); the tcgen05 kernels of efg_gemm.cu. The split copy of X goes to `ws` (at least
// gemm_ws_bytes(K, B) bytes) when given, else to a per-device scratch shared by every caller
// that does not pass one (reallocated when it grows). Returns an EFG_* status.
int launch_gemm_q4_0(float* Y, const uint8_t* W, const float* X, size_t M, size_t K, size_t B, int* d_err,
                     cudaStream_t s, void* ws = nullptr, size_t ws_cap = 0);
// Workspace bytes launch_gemm_q4_0 needs for a K-column, B-row product (0: none).
size_t gemm_ws_bytes(size_t K, size_t B);

}  // namespace efg
