// efg_quant.cu - Q4_0 / Q8_0 quantize and dequantize on B200, bit-exact with the
// reference (src/quant.cpp:26-249).
//
// A packed matrix is a flat sequence of blocks (rows are back to back and cols % 32 ==
// 0), so both directions work on block indices. Quantize: one warp takes 32 consecutive
// blocks, loads their 4 KB of floats with coalesced 16-byte loads into shared memory
// (padded rows, no bank conflicts), each lane quantizes one block with exactly the
// reference's operation sequence, and the warp writes the 576 / 1088 packed bytes back
// contiguously. Every floating-point step is an explicit round-to-nearest intrinsic so
// nothing is contracted into an FMA (the reference builds with -ffp-contract=off).
// Dequantize: 8 lanes per block, each writing 4 consecutive floats.
#include <algorithm>

#include "efg_device.cuh"
#include "efg_host.h"
#include "efg_quant.cuh"

namespace efg {

namespace {

constexpr float kFp16Max = 65504.0f;

// static_cast<int>(std::nearbyint(v)) as the reference build executes it on x86-64:
// round half to even, then a truncating conversion that yields INT_MIN for NaN and for
// values outside int range (cvttss2si's "integer indefinite").
__device__ __forceinline__ int round_to_int(float v) {
  const float r = rintf(v);
  if (!(r >= -2147483648.0f && r < 2147483648.0f)) return INT_MIN;
  return static_cast<int>(r);
}

// float(code) * d with the NaN results of the reference's x86-64 build (SSE mulss):
// a NaN operand comes back quieted with its payload, and 0 * inf gives the "real
// indefinite" NaN 0xFFC00000. For every other input this is the IEEE product.
__device__ __forceinline__ float dequant_mul(int code, float d) {
  const uint32_t db = __float_as_uint(d);
  if ((db & 0x7FFFFFFFu) > 0x7F800000u) return __uint_as_float(db | 0x00400000u);
  if ((db & 0x7FFFFFFFu) == 0x7F800000u && code == 0) return __uint_as_float(0xFFC00000u);
  return __fmul_rn(static_cast<float>(code), d);
}

__device__ __forceinline__ int clamp_i(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
__device__ __forceinline__ float clamp_f(float v, float lo, float hi) { return v < lo ? lo : (hi < v ? hi : v); }
__device__ __forceinline__ double clamp_d(double v, double lo, double hi) { return v < lo ? lo : (hi < v ? hi : v); }

__device__ __forceinline__ int q4_code(float x, float inv) { return clamp_i(round_to_int(__fmul_rn(x, inv)) + 8, 0, 15); }

// Squared error of the scale d (src/quant.cpp:52-58, 79-85): codes from x * (1/d), the
// reconstruction float(code - 8) * d, double error summed in j order.
__device__ __forceinline__ double q4_error(const float* x, float d) {
  const float inv = __fdiv_rn(1.0f, d);
  double err = 0.0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int c = q4_code(x[j], inv);
    const float w = __fmul_rn(static_cast<float>(c - 8), d);
    const double e = __dsub_rn(static_cast<double>(x[j]), static_cast<double>(w));
    err = __dadd_rn(err, __dmul_rn(e, e));
  }
  return err;
}

// The Q4_0 scale of one block (q4_group, src/quant.cpp:26-99). Codes are a pure
// function of (x, d), so only the winning scale is carried and codes are recomputed.
__device__ float q4_scale(const float* x, bool search) {
  float amax = 0.0f, smax = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float a = fabsf(x[j]);
    if (a > amax) {
      amax = a;
      smax = x[j];
    }
  }
  if (!(amax > 0.0f) || !isfinite(amax)) return 0.0f;
  float best_d = 0.0f;
  double best = -1.0;
  const int n_cand = search ? 6 : 1;
  for (int c = 0; c < n_cand; ++c) {
    float cand;
    switch (c) {  // llama.cpp's max/-8 first, then the symmetric divisors
      case 0: cand = __fdiv_rn(smax, -8.0f); break;
      case 1: cand = __fdiv_rn(amax, 7.0f); break;
      case 2: cand = __fdiv_rn(amax, 7.25f); break;
      case 3: cand = __fdiv_rn(amax, 7.5f); break;
      case 4: cand = __fdiv_rn(amax, 7.75f); break;
      default: cand = __fdiv_rn(amax, 8.0f); break;
    }
    const float d = fp16_round(clamp_f(cand, -kFp16Max, kFp16Max));
    if (d == 0.0f) continue;
    const double err = q4_error(x, d);
    if (best < 0.0 || err < best) {
      best = err;
      best_d = d;
    }
  }
  if (best < 0.0) return 0.0f;
  if (search) {
    for (int round = 0; round < 2; ++round) {
      const float inv = __fdiv_rn(1.0f, best_d);
      double sxc = 0.0, scc = 0.0;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const double c = static_cast<double>(q4_code(x[j], inv) - 8);
        sxc = __dadd_rn(sxc, __dmul_rn(static_cast<double>(x[j]), c));
        scc = __dadd_rn(scc, __dmul_rn(c, c));
      }
      if (scc == 0.0) break;
      const float d = fp16_round(__double2float_rn(clamp_d(__ddiv_rn(sxc, scc), -65504.0, 65504.0)));
      if (d == 0.0f || d == best_d) break;
      const double err = q4_error(x, d);
      if (!(err < best)) break;
      best = err;
      best_d = d;
    }
  }
  return best_d;
}

// Writes one block: fp16 scale, then byte j = code j | code (j+16) << 4.
__device__ __forceinline__ void q4_pack(const float* x, float d, uint8_t* out) {
  const uint32_t h = f32_to_fp16(d);
  out[0] = static_cast<uint8_t>(h & 0xFF);
  out[1] = static_cast<uint8_t>(h >> 8);
  if (d == 0.0f) {  // zero / non-finite / underflowed block: every code is 8
#pragma unroll
    for (int j = 0; j < 16; ++j) out[2 + j] = 0x88;
    return;
  }
  const float inv = __fdiv_rn(1.0f, d);
#pragma unroll
  for (int j = 0; j < 16; ++j)
    out[2 + j] = static_cast<uint8_t>(q4_code(x[j], inv) | (q4_code(x[j + 16], inv) << 4));
}

// src/quant.cpp:166-175
__device__ __forceinline__ void q8_block(const float* x, uint8_t* out) {
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float a = fabsf(x[j]);
    amax = amax < a ? a : amax;  // std::max(amax, a)
  }
  float d = 0.0f;
  if (amax > 0.0f && isfinite(amax)) {
    const float s = __fdiv_rn(amax, 127.0f);
    d = fp16_round(kFp16Max < s ? kFp16Max : s);
  }
  const uint32_t h = f32_to_fp16(d);
  out[0] = static_cast<uint8_t>(h & 0xFF);
  out[1] = static_cast<uint8_t>(h >> 8);
  const float inv = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    out[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(clamp_i(round_to_int(__fmul_rn(x[j], inv)), -127, 127)));
}

constexpr int kWarpsPerBlock = 4;
constexpr int kPad = 33;  // floats per staged block row (32 + 1: conflict-free column reads)

template <int QT>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) quantize_kernel(const float* __restrict__ x,
                                                                        uint8_t* __restrict__ out, uint64_t n_blocks,
                                                                        int search) {
  constexpr int BB = QT == 4 ? 18 : 34;
  __shared__ float sx[kWarpsPerBlock][32 * kPad];
  __shared__ __align__(16) uint8_t sout[kWarpsPerBlock][32 * BB];
  pdl_wait();
  pdl_launch_dependents();
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t n_groups = (n_blocks + 31) / 32;
  const bool x_vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const bool o_vec = (reinterpret_cast<uintptr_t>(out) & 3) == 0;
  for (uint64_t g = static_cast<uint64_t>(blockIdx.x) * kWarpsPerBlock + w; g < n_groups;
       g += static_cast<uint64_t>(gridDim.x) * kWarpsPerBlock) {
    const uint64_t b0 = g * 32;
    const int nb = n_blocks - b0 < 32 ? static_cast<int>(n_blocks - b0) : 32;
    const float* src = x + b0 * 32;
    // Stage nb * 32 floats: element e of the group lands at row e / 32, column e % 32.
    if (x_vec) {
      for (int q = lane; q < nb * 8; q += 32) {
        const float4 v = reinterpret_cast<const float4*>(src)[q];
        float* d = &sx[w][(q >> 3) * kPad + (q & 7) * 4];
        d[0] = v.x;
        d[1] = v.y;
        d[2] = v.z;
        d[3] = v.w;
      }
    } else {
      for (int e = lane; e < nb * 32; e += 32) sx[w][(e >> 5) * kPad + (e & 31)] = src[e];
    }
    __syncwarp();
    if (lane < nb) {
      float xv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) xv[j] = sx[w][lane * kPad + j];
      uint8_t* o = &sout[w][lane * BB];
      if constexpr (QT == 4) {
        q4_pack(xv, q4_scale(xv, search != 0), o);
      } else {
        q8_block(xv, o);
      }
    }
    __syncwarp();
    uint8_t* dst = out + b0 * BB;
    const int bytes = nb * BB;
    if (o_vec && (bytes & 3) == 0) {
      for (int q = lane; q < bytes / 4; q += 32)
        reinterpret_cast<uint32_t*>(dst)[q] = reinterpret_cast<const uint32_t*>(sout[w])[q];
    } else {
      for (int q = lane; q < bytes; q += 32) dst[q] = sout[w][q];
    }
    __syncwarp();
  }
}

// 8 lanes per block; lane q writes floats 4q .. 4q+3 of the block (src/quant.cpp:158-164,
// 177-180: w = float(code) * d, one exact product).
template <int QT>
__global__ void dequantize_kernel(const uint8_t* __restrict__ in, float* __restrict__ out, uint64_t n_blocks) {
  constexpr int BB = QT == 4 ? 18 : 34;
  pdl_wait();
  pdl_launch_dependents();
  const bool o_vec = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  const uint64_t n_items = n_blocks * 8;
  for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n_items;
       t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t b = t >> 3;
    const int q = static_cast<int>(t & 7);
    const uint8_t* blk = in + b * BB;
    const float d = fp16_to_f32(blk[0] | (blk[1] << 8));
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * q + k;
      int code;
      if constexpr (QT == 4) code = (j < 16 ? (blk[2 + j] & 0x0F) : (blk[2 + j - 16] >> 4)) - 8;
      else code = static_cast<int8_t>(blk[2 + j]);
      v[k] = dequant_mul(code, d);
    }
    float* o = out + b * 32 + 4 * q;
    if (o_vec) {
      *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = v[k];
    }
  }
}

// F32 / F16 / BF16 rows: exact widening (src/quant.cpp:224-234).
__global__ void widen_kernel(int qtype, const uint8_t* __restrict__ in, float* __restrict__ out, uint64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    if (qtype == 0) {
      uint32_t u = in[4 * i] | (in[4 * i + 1] << 8) | (in[4 * i + 2] << 16) | (static_cast<uint32_t>(in[4 * i + 3]) << 24);
      out[i] = __uint_as_float(u);
    } else {
      const uint32_t h = in[2 * i] | (in[2 * i + 1] << 8);
      out[i] = qtype == 1 ? fp16_to_f32(h) : bf16_to_f32(h);
    }
  }
}

// binary32 -> bfloat16 of include/ef/fp16.h:34-42: NaN keeps its top bits with the quiet bit
// forced; everything else rounds to nearest even (overflow becomes inf).
__device__ __forceinline__ uint32_t f32_to_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return ((u >> 16) | 0x0040u) & 0xFFFFu;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return u >> 16;
}

// F32 / F16 / BF16 rows from floats (src/quant.cpp:186-200): an exact copy of the bits, or
// the reference's round-to-nearest-even narrowing, little-endian at any byte offset.
__global__ void narrow_kernel(int qtype, const float* __restrict__ x, uint8_t* __restrict__ out, uint64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t u = __float_as_uint(x[i]);
    if (qtype == 0) {
      out[4 * i] = static_cast<uint8_t>(u);
      out[4 * i + 1] = static_cast<uint8_t>(u >> 8);
      out[4 * i + 2] = static_cast<uint8_t>(u >> 16);
      out[4 * i + 3] = static_cast<uint8_t>(u >> 24);
    } else {
      const uint32_t h = qtype == 1 ? f32_to_fp16(x[i]) : f32_to_bf16(x[i]);
      out[2 * i] = static_cast<uint8_t>(h);
      out[2 * i + 1] = static_cast<uint8_t>(h >> 8);
    }
  }
}

// fake_quant_q4_group (src/quant.cpp:243-248): q4_group over the first min(n, 256) values of
// one group of any size, written back as float(code - 8) * d. One thread runs the whole group
// in the reference's order (analysis tooling, not a hot path).
__global__ void fake_quant_q4_group_kernel(const float* __restrict__ x, uint32_t n, float* __restrict__ out,
                                           int search) {
  pdl_wait();
  pdl_launch_dependents();
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  float amax = 0.0f, smax = 0.0f;
  for (uint32_t j = 0; j < n; ++j) {
    const float a = fabsf(x[j]);
    if (a > amax) {
      amax = a;
      smax = x[j];
    }
  }
  auto error_of = [&](float d) {
    const float inv = __fdiv_rn(1.0f, d);
    double err = 0.0;
    for (uint32_t j = 0; j < n; ++j) {
      const int c = q4_code(x[j], inv);
      const double e = __dsub_rn(static_cast<double>(x[j]), static_cast<double>(__fmul_rn(static_cast<float>(c - 8), d)));
      err = __dadd_rn(err, __dmul_rn(e, e));
    }
    return err;
  };
  float best_d = 0.0f;
  if (amax > 0.0f && isfinite(amax)) {
    double best = -1.0;
    const int n_cand = search ? 6 : 1;
    for (int c = 0; c < n_cand; ++c) {
      const float div = c == 1 ? 7.0f : c == 2 ? 7.25f : c == 3 ? 7.5f : c == 4 ? 7.75f : 8.0f;
      const float cand = c == 0 ? __fdiv_rn(smax, -8.0f) : __fdiv_rn(amax, div);
      const float d = fp16_round(clamp_f(cand, -kFp16Max, kFp16Max));
      if (d == 0.0f) continue;
      const double err = error_of(d);
      if (best < 0.0 || err < best) {
        best = err;
        best_d = d;
      }
    }
    if (best >= 0.0 && search) {
      for (int round = 0; round < 2; ++round) {
        const float inv = __fdiv_rn(1.0f, best_d);
        double sxc = 0.0, scc = 0.0;
        for (uint32_t j = 0; j < n; ++j) {
          const double c = static_cast<double>(q4_code(x[j], inv) - 8);
          sxc = __dadd_rn(sxc, __dmul_rn(static_cast<double>(x[j]), c));
          scc = __dadd_rn(scc, __dmul_rn(c, c));
        }
        if (scc == 0.0) break;
        const float d = fp16_round(__double2float_rn(clamp_d(__ddiv_rn(sxc, scc), -65504.0, 65504.0)));
        if (d == 0.0f || d == best_d) break;
        const double err = error_of(d);
        if (!(err < best)) break;
        best = err;
        best_d = d;
      }
    }
  }
  const float inv = best_d != 0.0f ? __fdiv_rn(1.0f, best_d) : 0.0f;
  for (uint32_t j = 0; j < n; ++j) {
    const int c = best_d != 0.0f ? q4_code(x[j], inv) : 8;
    out[j] = __fmul_rn(static_cast<float>(c - 8), best_d);
  }
}

// Reconstruction statistics of one quantized row per thread (src/quantizer.cpp:131-147):
// e = double(src) - double(dequantized), sse += e * e, ref += src^2 (double, column order,
// no contraction) and the largest |e|, so the totals the writer forms from them are the
// reference's to the last bit.
__global__ void quant_stats_kernel(int qtype, const float* __restrict__ src, const uint8_t* __restrict__ q,
                                   uint64_t rows, uint64_t cols, double* __restrict__ sse, double* __restrict__ ref,
                                   double* __restrict__ mx) {
  const uint64_t r = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const uint32_t bb = qtype == 4 ? 18 : 34;
  const float* x = src + r * cols;
  const uint8_t* row = q + r * (cols / 32) * bb;
  double s = 0.0, rs = 0.0, m = 0.0;
  for (uint64_t b = 0; b < cols / 32; ++b) {
    const uint8_t* blk = row + b * bb;
    const float d = fp16_to_f32(blk[0] | (blk[1] << 8));
    for (int j = 0; j < 32; ++j) {
      int code;
      if (qtype == 4) code = (j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4)) - 8;
      else code = static_cast<int8_t>(blk[2 + j]);
      const double xv = static_cast<double>(__ldg(x + b * 32 + j));
      const double e = __dsub_rn(xv, static_cast<double>(dequant_mul(code, d)));
      s = __dadd_rn(s, __dmul_rn(e, e));
      rs = __dadd_rn(rs, __dmul_rn(xv, xv));
      const double ae = fabs(e);
      m = m < ae ? ae : m;
    }
  }
  sse[r] = s;
  ref[r] = rs;
  mx[r] = m;
}

// Row r of a [rows][cols] matrix as FP32 (src/qkernels.cpp:299-305): exact for
// F32/F16/BF16, dequantized for Q8_0/Q4_0. r comes from *d_r when given (a token id
// produced on the device); an out-of-range id records EFG_EINVAL in *err and writes
// nothing.
__global__ void row_f32_kernel(int qtype, const uint8_t* __restrict__ W, uint64_t rows, uint64_t cols,
                               const int32_t* d_r, uint64_t r_host, float* __restrict__ out, int* err) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t r = d_r ? static_cast<int64_t>(*d_r) : static_cast<int64_t>(r_host);
  if (r < 0 || static_cast<uint64_t>(r) >= rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) record_error(err, EFG_EINVAL);
    return;
  }
  const uint64_t bb = qtype == 4 ? 18 : qtype == 3 ? 34 : (qtype == 0 ? 4 : 2);
  const uint8_t* row = W + static_cast<uint64_t>(r) * (qtype >= 3 ? cols / 32 * bb : cols * bb);
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < cols;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    float v;
    if (qtype == 4 || qtype == 3) {
      const uint8_t* blk = row + (i / 32) * bb;
      const int j = static_cast<int>(i % 32);
      const float d = fp16_to_f32(blk[0] | (blk[1] << 8));
      const int code = qtype == 4 ? (j < 16 ? (blk[2 + j] & 0x0F) : (blk[2 + j - 16] >> 4)) - 8
                                  : static_cast<int8_t>(blk[2 + j]);
      v = dequant_mul(code, d);
    } else if (qtype == 0) {
      v = __uint_as_float(row[4 * i] | (row[4 * i + 1] << 8) | (row[4 * i + 2] << 16) |
                          (static_cast<uint32_t>(row[4 * i + 3]) << 24));
    } else {
      const uint32_t h = row[2 * i] | (row[2 * i + 1] << 8);
      v = qtype == 1 ? fp16_to_f32(h) : bf16_to_f32(h);
    }
    out[i] = v;
  }
}

cudaLaunchConfig_t config(unsigned grid, unsigned block, cudaStream_t s, cudaLaunchAttribute* attr, bool pdl) {
  cudaLaunchConfig_t c{};
  c.gridDim = dim3(grid);
  c.blockDim = dim3(block);
  c.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return c;
}

}  // namespace

int launch_quantize(int qtype, const float* x, uint64_t n_values, void* out, bool search, cudaStream_t s, bool pdl) {
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  if (qtype >= 0 && qtype <= 2) {  // F32 / F16 / BF16: plain conversions, any length
    if (n_values == 0) return EFG_OK;
    if (!x || !out) return fail(EFG_EINVAL, "quantize: null pointer");
    const unsigned grid = static_cast<unsigned>(
        std::max<uint64_t>(1, std::min<uint64_t>((n_values + 255) / 256, 32ull * dev->sm_count)));
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t c = config(grid, 256, s, attr, pdl);
    EFG_TRY_CUDA(cudaLaunchKernelEx(&c, narrow_kernel, qtype, x, static_cast<uint8_t*>(out), n_values),
                 "quantize launch");
    return EFG_OK;
  }
  if (qtype != 4 && qtype != 3) return fail(EFG_EINVAL, "quantize: unknown type %d", qtype);
  if (n_values % 32 != 0) {
    return fail(EFG_EINVAL, "%s needs a row length divisible by 32, got %llu", qtype == 4 ? "Q4_0" : "Q8_0",
                static_cast<unsigned long long>(n_values));
  }
  const uint64_t nb = n_values / 32;
  if (nb == 0) return EFG_OK;
  if (!x || !out) return fail(EFG_EINVAL, "quantize: null pointer");
  const uint64_t groups = (nb + 31) / 32;
  const unsigned grid = static_cast<unsigned>(
      std::max<uint64_t>(1, std::min<uint64_t>((groups + kWarpsPerBlock - 1) / kWarpsPerBlock, 16ull * dev->sm_count)));
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = config(grid, kWarpsPerBlock * 32, s, attr, pdl);
  const int srch = search ? 1 : 0;
  auto* o = static_cast<uint8_t*>(out);
  EFG_TRY_CUDA(qtype == 4 ? cudaLaunchKernelEx(&c, quantize_kernel<4>, x, o, nb, srch)
                          : cudaLaunchKernelEx(&c, quantize_kernel<3>, x, o, nb, srch),
               "quantize launch");
  return EFG_OK;
}

int launch_dequantize(int qtype, const void* in, uint64_t n_values, float* out, cudaStream_t s, bool pdl) {
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  if (qtype < 0 || qtype > 4) return fail(EFG_EINVAL, "dequantize: unknown type %d", qtype);
  if ((qtype == 3 || qtype == 4) && n_values % 32 != 0) {
    return fail(EFG_EINVAL, "%s needs a row length divisible by 32, got %llu", qtype == 4 ? "Q4_0" : "Q8_0",
                static_cast<unsigned long long>(n_values));
  }
  if (n_values == 0) return EFG_OK;
  if (!in || !out) return fail(EFG_EINVAL, "dequantize: null pointer");
  cudaLaunchAttribute attr[1];
  const auto* p = static_cast<const uint8_t*>(in);
  if (qtype == 3 || qtype == 4) {
    const uint64_t items = n_values / 32 * 8;
    const unsigned grid = static_cast<unsigned>(std::max<uint64_t>(1, std::min<uint64_t>((items + 255) / 256, 32ull * dev->sm_count)));
    cudaLaunchConfig_t c = config(grid, 256, s, attr, pdl);
    EFG_TRY_CUDA(qtype == 4 ? cudaLaunchKernelEx(&c, dequantize_kernel<4>, p, out, n_values / 32)
                            : cudaLaunchKernelEx(&c, dequantize_kernel<3>, p, out, n_values / 32),
                 "dequantize launch");
  } else {
    const unsigned grid = static_cast<unsigned>(std::max<uint64_t>(1, std::min<uint64_t>((n_values + 255) / 256, 32ull * dev->sm_count)));
    cudaLaunchConfig_t c = config(grid, 256, s, attr, pdl);
    EFG_TRY_CUDA(cudaLaunchKernelEx(&c, widen_kernel, qtype, p, out, n_values), "dequantize launch");
  }
  return EFG_OK;
}

int launch_fake_quant_q4_group(const float* x, uint64_t n, float* out, bool search, cudaStream_t s) {
  if (n > 256) n = 256;  // the reference quantizes the first 256 values only
  if (n == 0) return EFG_OK;
  if (!x || !out) return fail(EFG_EINVAL, "fake_quant_q4_group: null pointer");
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = config(1, 32, s, attr, false);
  EFG_TRY_CUDA(cudaLaunchKernelEx(&c, fake_quant_q4_group_kernel, x, static_cast<uint32_t>(n), out, search ? 1 : 0),
               "fake_quant_q4_group launch");
  return EFG_OK;
}

int launch_quant_stats(int qtype, const float* src, const uint8_t* q, uint64_t rows, uint64_t cols, double* sse,
                       double* ref, double* mx, cudaStream_t s) {
  if (qtype != 3 && qtype != 4) return fail(EFG_EINVAL, "quant_stats: type must be Q8_0 or Q4_0");
  if (cols % 32 != 0) return fail(EFG_EINVAL, "quant_stats: cols %% 32 != 0");
  if (rows == 0) return EFG_OK;
  quant_stats_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0, s>>>(qtype, src, q, rows, cols, sse, ref, mx);
  EFG_TRY_CUDA(cudaGetLastError(), "quant_stats launch");
  return EFG_OK;
}

int launch_row_f32(int qtype, const uint8_t* W, uint64_t rows, uint64_t cols, const int32_t* d_r, uint64_t r_host,
                   float* out, cudaStream_t s, bool pdl) {
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  if (qtype < 0 || qtype > 4) return fail(EFG_EINVAL, "row_f32: unknown type %d", qtype);
  if ((qtype == 3 || qtype == 4) && cols % 32 != 0)
    return fail(EFG_EINVAL, "%s needs a row length divisible by 32, got %llu", qtype == 4 ? "Q4_0" : "Q8_0",
                static_cast<unsigned long long>(cols));
  if (!d_r && r_host >= rows) return fail(EFG_EINVAL, "row_f32: row %llu out of range", static_cast<unsigned long long>(r_host));
  if (cols == 0) return EFG_OK;
  if (!W || !out) return fail(EFG_EINVAL, "row_f32: null pointer");
  cudaLaunchAttribute attr[1];
  const unsigned grid = static_cast<unsigned>(std::min<uint64_t>(64, (cols + 255) / 256));
  cudaLaunchConfig_t c = config(grid, 256, s, attr, pdl);
  EFG_TRY_CUDA(cudaLaunchKernelEx(&c, row_f32_kernel, qtype, W, rows, cols, d_r, r_host, out, dev->d_err),
               "row_f32 launch");
  return EFG_OK;
}

}  // namespace efg
