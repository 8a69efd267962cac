// efg_quant.cuh - launchers of the quantize / dequantize kernels (efg_quant.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace efg {

// n_values floats (a multiple of 32) -> n_values / 32 blocks of type qtype (3 = Q8_0,
// 4 = Q4_0), or the plain conversions to 0 = F32, 1 = F16, 2 = BF16 (any n_values).
// Bit-exact with ef::quantize_row.
int launch_quantize(int qtype, const float* x, uint64_t n_values, void* out, bool search, cudaStream_t s,
                    bool pdl = false);
// Inverse, also for 0 = F32, 1 = F16, 2 = BF16 (exact widening).
int launch_dequantize(int qtype, const void* in, uint64_t n_values, float* out, cudaStream_t s, bool pdl = false);
// ef::fake_quant_q4_group on the first min(n, 256) values: the Q4 quantize of one group of
// any size with its FP16 scale, written back as floats. Bit-exact.
int launch_fake_quant_q4_group(const float* x, uint64_t n, float* out, bool search, cudaStream_t s);
// Per-row reconstruction statistics of a quantized [rows][cols] matrix against its FP32
// source (the writer's rel_rmse / max_abs_err, src/quantizer.cpp:131-147).
int launch_quant_stats(int qtype, const float* src, const uint8_t* q, uint64_t rows, uint64_t cols, double* sse,
                       double* ref, double* mx, cudaStream_t s);
// Row lookup (embedding): row *d_r (or r_host when d_r is null) of W as FP32.
int launch_row_f32(int qtype, const uint8_t* W, uint64_t rows, uint64_t cols, const int32_t* d_r, uint64_t r_host,
                   float* out, cudaStream_t s, bool pdl = false);

}  // namespace efg
