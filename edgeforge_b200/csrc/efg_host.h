// efg_host.h - host-side helpers shared by the C-ABI implementation: the thread-local
// error message, status helpers and per-device state (SM count, the device error word).
#pragma once

#include <cstdarg>
#include <cstdint>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>

#include "efg_status.h"

namespace efg {

// Sets the thread-local message returned by efg_last_error() and returns `status`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();
const char* last_error();

// Checks a CUDA runtime result; on failure records "<what>: <cuda message>".
int cuda_check(cudaError_t e, const char* what);

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  size_t smem_optin = 0;  // max dynamic shared memory per block (opt-in)
  int* d_err = nullptr;   // device error word written by bounded waits
};

// Thread-local default for MatvecArgs::pdl in the C-ABI calls (efg_set_weight_prefetch).
bool& weight_prefetch_flag();

// Thread-local switch for the tensor-core Q4_0 matvec on large matrices (efg_set_q4_mma).
bool& q4_mma_flag();

// Thread-local switch for the small-batch Q4_0 GEMM on the integer MMA (efg_set_small_gemm;
// off by default: measured slower than the tcgen05 GEMM at every config-3 shape).
bool& small_gemm_flag();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (device, kernel, size);
// later calls are free, so launches can be captured into CUDA graphs.
int ensure_smem_attr(const void* fn, size_t bytes);

// A 2-D TMA tensor map over `rows` rows of `row_bytes` bytes (16-byte aligned base and row
// stride) seen as 8-byte elements, with a box of box_elems x box_rows; the box may reach past
// a row's end or past the last row (zero fill). cuTensorMapEncodeTiled from the driver, looked
// up once. False when the driver rejects the map.
bool encode_u64_rows_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_elems,
                         uint32_t box_rows);

// State of the current device, created on first use (allocates the error word).
// Returns nullptr and records an error if the device cannot be queried.
DeviceInfo* current_device();

}  // namespace efg

#define EFG_TRY_CUDA(expr, what)                      \
  do {                                                \
    const cudaError_t efg_e_ = (expr);                \
    if (efg_e_ != cudaSuccess) return ::efg::cuda_check(efg_e_, what); \
  } while (0)
