// efg_decode.cu - the TinyLlama decode step of the reference (src/model.cpp:184-304) on a
// B200: Model::load_efq, Transformer::forward and generate_greedy.
//
// The .efq data region is uploaded once; every weight is a device pointer into it. One
// decode step is a fixed sequence of launches that reads the position and the token from
// device memory, so it is captured once into a CUDA graph and replayed for every token:
//
//   embed (BF16 row of tokens[pos])
//   per layer: q/k/v matvec with the RMSNorm prologue (v written straight into the KV
//              cache at pos) -> attention (RoPE of q and the new k, k-cache write, GQA
//              softmax over pos+1 positions) -> o_proj matvec with residual add ->
//              gate/up matvec with the RMSNorm prologue and SwiGLU epilogue -> down matvec
//              with residual add
//   lm_head matvec with the final RMSNorm prologue -> argmax (next token, pos + 1)
//
// All launches use programmatic dependent launch: the matvecs start streaming their
// weights while the previous kernel finishes, and wait for it before touching
// activations. Norm, residual and SwiGLU follow the reference's float operation order
// (src/kernels.cpp:69-111); matvec sums differ in order only (<= 1e-5 of sum|w x|).
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/efg.h"
#include "efg_argmax.cuh"
#include "efg_device.cuh"
#include "efg_efq.h"
#include "efg_gemm.cuh"
#include "efg_host.h"
#include "efg_matvec.cuh"
#include "efg_decode_mk.cuh"

namespace efg {
namespace {

constexpr int kAttnThreads = 128;

cudaLaunchConfig_t cfg_of(dim3 grid, dim3 block, size_t smem, cudaStream_t s, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t c{};
  c.gridDim = grid;
  c.blockDim = block;
  c.dynamicSmemBytes = smem;
  c.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = 1;
  return c;
}

// Bytes of one embedding row and element i of it as float (src/qkernels.cpp:299-305).
__device__ __forceinline__ uint64_t embed_row_bytes(int type, uint32_t dim) {
  return type == 0 ? 4ull * dim : type <= 2 ? 2ull * dim : dim / 32ull * (type == 3 ? 34 : 18);
}
__device__ __forceinline__ float embed_value(const uint8_t* __restrict__ row, int type, uint32_t i) {
  if (type == 2) return bf16_to_f32(row[2 * i] | (row[2 * i + 1] << 8));
  if (type == 1) return fp16_to_f32(row[2 * i] | (row[2 * i + 1] << 8));
  if (type == 0)
    return __uint_as_float(row[4 * i] | (row[4 * i + 1] << 8) | (row[4 * i + 2] << 16) |
                           (static_cast<uint32_t>(row[4 * i + 3]) << 24));
  const uint8_t* blk = row + (i / 32) * (type == 3 ? 34 : 18);
  const int j = i % 32;
  const float d = fp16_to_f32(blk[0] | (blk[1] << 8));
  const int code = type == 4 ? (j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4)) - 8
                             : static_cast<int8_t>(blk[2 + j]);
  return __fmul_rn(static_cast<float>(code), d);
}

// x = row tokens[*pos] of the embedding table.
__global__ void embed_kernel(const uint8_t* __restrict__ table, int type, uint32_t vocab, uint32_t dim,
                             const int32_t* __restrict__ tokens, const int32_t* __restrict__ pos,
                             float* __restrict__ x, int* err) {
  pdl_wait();
  pdl_launch_dependents();
  const int32_t tok = tokens[*pos];
  if (tok < 0 || static_cast<uint32_t>(tok) >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_error(err, EFG_EINVAL);
    return;
  }
  const uint8_t* row = table + static_cast<uint64_t>(tok) * embed_row_bytes(type, dim);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    x[i] = embed_value(row, type, i);
}

// Batched prefill: row b of xb = embedding row of tokens[b], b < n (grid.y = n).
__global__ void embed_rows_kernel(const uint8_t* __restrict__ table, int type, uint32_t vocab, uint32_t dim,
                                  const int32_t* __restrict__ tokens, float* __restrict__ xb, int* err) {
  pdl_wait();
  pdl_launch_dependents();
  const int32_t tok = tokens[blockIdx.y];
  if (tok < 0 || static_cast<uint32_t>(tok) >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_error(err, EFG_EINVAL);
    return;
  }
  const uint8_t* row = table + static_cast<uint64_t>(tok) * embed_row_bytes(type, dim);
  float* x = xb + static_cast<size_t>(blockIdx.y) * dim;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    x[i] = embed_value(row, type, i);
}

// q_h and k_h rotated by RoPE at position pos (half-split rotation, HF order a*c - b*s,
// b*c + a*s; src/kernels.cpp:133-147).
__device__ __forceinline__ void rope_pair(float a, float b, float c, float s, float& ra, float& rb) {
  ra = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  rb = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

// Positions staged per round in shared memory by attend_head (keys padded to hd + 1 floats).
constexpr int kAttnChunkPos = 64;
__host__ __device__ constexpr size_t attn_stage_floats(int hd) {
  return static_cast<size_t>(kAttnChunkPos) * (hd + 1) + static_cast<size_t>(kAttnChunkPos) * hd;
}

// Softmax attention of one rotated query head qh (shared memory) over the cached keys and
// values of positions 0..n_pos-1 of KV head kv (src/kernels.cpp:148-174): scores scaled by
// 1/sqrt(hd), softmax with a double sum, then the probability-weighted sum of the values in
// position order into out[0..hd). The key of position n_pos-1 is read from k_last. Keys
// and values come through `stage` (attn_stage_floats(hd) floats) in rounds of
// kAttnChunkPos positions, each round one set of coalesced float4 loads; hd % 4 == 0,
// hd <= 2 * blockDim.x. With `staged` (n_pos <= kAttnChunkPos only) the caller has already
// put every key and value row in `stage` and attend_head loads nothing.
__device__ void attend_head(const float* __restrict__ qh, const float* __restrict__ k_layer,
                            const float* __restrict__ v_layer, const float* __restrict__ k_last, int kv, int hd,
                            int kvd, int n_pos, float* __restrict__ sc, float* __restrict__ stage, float* red_f,
                            double* red_d, float* __restrict__ out, bool staged = false) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, h4 = hd / 4;
  float* kch = stage;                                // [kAttnChunkPos][hd + 1]
  float* vch = stage + kAttnChunkPos * (hd + 1);     // [kAttnChunkPos][hd]
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(hd)));
  float mx = -INFINITY;
  // up to kAttnChunkPos positions: the values are staged with the keys, in one round of loads
  const bool one_round = n_pos <= kAttnChunkPos;
  for (int c0 = 0; c0 < n_pos; c0 += kAttnChunkPos) {
    const int cn = min(kAttnChunkPos, n_pos - c0);
    for (int e = tid; e < (staged ? 0 : cn * h4); e += blockDim.x) {
      const int t = e / h4, i4 = e % h4;
      const float* src = c0 + t == n_pos - 1 ? k_last : k_layer + static_cast<size_t>(c0 + t) * kvd + kv * hd;
      const float4 v = reinterpret_cast<const float4*>(src)[i4];
      float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
      if (one_round) w = reinterpret_cast<const float4*>(v_layer + static_cast<size_t>(t) * kvd + kv * hd)[i4];
      float* d = kch + t * (hd + 1) + 4 * i4;
      d[0] = v.x;
      d[1] = v.y;
      d[2] = v.z;
      d[3] = v.w;
      if (one_round) reinterpret_cast<float4*>(vch + t * hd)[i4] = w;
    }
    if (!staged) __syncthreads();  // (a caller that staged the rows synchronised after it)
    for (int t = tid; t < cn; t += blockDim.x) {
      const float* kt = kch + t * (hd + 1);
      // dot with 8 partial sums combined pairwise (src/kernels.cpp:28-43)
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      int i = 0;
      for (; i + 8 <= hd; i += 8)
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = __fadd_rn(a[k], __fmul_rn(qh[i + k], kt[i + k]));
      for (; i < hd; ++i) a[0] = __fadd_rn(a[0], __fmul_rn(qh[i], kt[i]));
      const float dot = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                                  __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
      sc[c0 + t] = __fmul_rn(dot, scale);
      mx = fmaxf(mx, sc[c0 + t]);
    }
    // kch is rewritten by the next round; after the last one, the barrier of the max
    // reduction below orders the scores for the threads that read them
    if (c0 + kAttnChunkPos < n_pos) __syncthreads();
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  if (lane == 0) red_f[wid] = mx;
  __syncthreads();
  mx = red_f[0];
  for (int w = 1; w < static_cast<int>(blockDim.x / 32); ++w) mx = fmaxf(mx, red_f[w]);
  // softmax (src/kernels.cpp:77-92): exp(x - max), sum in double, scale by float(1/sum)
  double sum = 0.0;
  for (int t = tid; t < n_pos; t += blockDim.x) {
    const float e = expf(__fsub_rn(sc[t], mx));
    sc[t] = e;
    sum += static_cast<double>(e);
  }
  sum = warp_sum_d(sum);
  if (lane == 0) red_d[wid] = sum;
  __syncthreads();
  double tot = 0.0;
  for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) tot += red_d[w];
  const float inv = static_cast<float>(1.0 / tot);
  for (int t = tid; t < n_pos; t += blockDim.x) sc[t] = __fmul_rn(sc[t], inv);
  // weighted sum of the values in position order; thread tid owns d = tid and tid + blockDim
  float acc0 = 0.f, acc1 = 0.f;
  const int d0 = tid, d1 = tid + static_cast<int>(blockDim.x);
  for (int c0 = 0; c0 < n_pos; c0 += kAttnChunkPos) {
    const int cn = min(kAttnChunkPos, n_pos - c0);
    __syncthreads();  // sc is final; vch is free (or, in one round, already staged)
    if (!one_round) {
      for (int e = tid; e < cn * h4; e += blockDim.x) {
        const int t = e / h4, i4 = e % h4;
        reinterpret_cast<float4*>(vch + t * hd)[i4] =
            reinterpret_cast<const float4*>(v_layer + static_cast<size_t>(c0 + t) * kvd + kv * hd)[i4];
      }
      __syncthreads();
    }
    if (d0 < hd)
      for (int t = 0; t < cn; ++t) acc0 = __fadd_rn(acc0, __fmul_rn(sc[c0 + t], vch[t * hd + d0]));
    if (d1 < hd)
      for (int t = 0; t < cn; ++t) acc1 = __fadd_rn(acc1, __fmul_rn(sc[c0 + t], vch[t * hd + d1]));
  }
  if (d0 < hd) out[d0] = acc0;
  if (d1 < hd) out[d1] = acc1;
}

// One query head per CTA: RoPE of q and of the new key, the key written to the cache at pos
// by the first head of each KV group, then attend_head over pos + 1 positions.
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(
    const float* __restrict__ q, const float* __restrict__ knew, float* __restrict__ k_layer,
    const float* __restrict__ v_layer, float* __restrict__ ctx, const float* __restrict__ rope_cos,
    const float* __restrict__ rope_sin, const int32_t* __restrict__ pos_p, int H, int KV, int hd, int max_seq,
    int* err) {
  extern __shared__ float sm[];
  float* qh = sm;            // [hd]
  float* kn = qh + hd;       // [hd]
  float* stage = kn + hd;    // [attn_stage_floats(hd)]
  float* sc = stage + attn_stage_floats(hd);  // [max_seq]
  __shared__ float red_f[kAttnThreads / 32];
  __shared__ double red_d[kAttnThreads / 32];
  // The position, the RoPE tables and the cached keys and values of earlier positions
  // were written before this step began (graph launches are stream-ordered), so they
  // are read before waiting for the q/k/v projection; only q, the new key and the new
  // value are read after.
  const int pos = *pos_p;
  if (pos < 0 || pos >= max_seq) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) record_error(err, EFG_ESTATE);
    return;
  }
  const int h = blockIdx.x, group = H / KV, kv = h / group, half = hd / 2, kvd = KV * hd, h4 = hd / 4;
  const int tid = threadIdx.x;
  const bool staged = pos + 1 <= kAttnChunkPos;
  float* kch = stage;
  float* vch = stage + kAttnChunkPos * (hd + 1);
  if (staged)
    for (int e = tid; e < pos * h4; e += blockDim.x) {
      const int t = e / h4, i4 = e % h4;
      const size_t row = static_cast<size_t>(t) * kvd + kv * hd;
      const float4 kv4 = reinterpret_cast<const float4*>(k_layer + row)[i4];
      reinterpret_cast<float4*>(vch + t * hd)[i4] = reinterpret_cast<const float4*>(v_layer + row)[i4];
      float* d = kch + t * (hd + 1) + 4 * i4;
      d[0] = kv4.x;
      d[1] = kv4.y;
      d[2] = kv4.z;
      d[3] = kv4.w;
    }
  float cs = 0.f, sn = 0.f;
  if (tid < half) {
    cs = rope_cos[static_cast<size_t>(pos) * half + tid];
    sn = rope_sin[static_cast<size_t>(pos) * half + tid];
  }
  pdl_wait();
  pdl_launch_dependents();
  for (int i = tid; i < half; i += blockDim.x) {
    const float c = i == tid ? cs : rope_cos[static_cast<size_t>(pos) * half + i];
    const float sv = i == tid ? sn : rope_sin[static_cast<size_t>(pos) * half + i];
    rope_pair(q[h * hd + i], q[h * hd + i + half], c, sv, qh[i], qh[i + half]);
    rope_pair(knew[kv * hd + i], knew[kv * hd + i + half], c, sv, kn[i], kn[i + half]);
  }
  if (staged)
    for (int i4 = tid; i4 < h4; i4 += blockDim.x)  // the new value row (written by the projection)
      reinterpret_cast<float4*>(vch + pos * hd)[i4] =
          reinterpret_cast<const float4*>(v_layer + static_cast<size_t>(pos) * kvd + kv * hd)[i4];
  __syncthreads();
  if (h % group == 0)
    for (int i = tid; i < hd; i += blockDim.x) k_layer[static_cast<size_t>(pos) * kvd + kv * hd + i] = kn[i];
  if (staged)
    for (int i = tid; i < hd; i += blockDim.x) kch[pos * (hd + 1) + i] = kn[i];
  __syncthreads();
  attend_head(qh, k_layer, v_layer, kn, kv, hd, kvd, pos + 1, sc, stage, red_f, red_d, ctx + h * hd, staged);
}

// The same attention step for head_dim 64 and at most kWarpAttnMaxPos cached positions, one
// warp per query head: lane i holds dims i and i + 32 (exactly the RoPE pairs), scores are one
// position per lane, and the max, the softmax sum and every hand-over stay inside the warp (no
// CTA barrier after the grid-dependency wait). The arithmetic per element is attend_head's:
// the score dot in 8 partial sums combined pairwise, times 1/sqrt(hd); exp(x - max) summed in
// double; each probability times float(1 / sum); values summed in position order.
constexpr int kWarpAttnMaxPos = 128;
// Shared floats for max_seq positions: the position count is padded to a multiple of 4, so the
// values array (after n_pad * 65 key floats) starts 16-byte aligned for its float4 stores.
__host__ __device__ constexpr size_t warp_attn_smem_floats(size_t max_seq) {
  return ((max_seq + 3) / 4 * 4) * (65 + 64 + 1) + 64;
}

__global__ void __launch_bounds__(32) attention_warp_kernel(
    const float* __restrict__ q, const float* __restrict__ knew, float* __restrict__ k_layer,
    const float* __restrict__ v_layer, float* __restrict__ ctx, const float* __restrict__ rope_cos,
    const float* __restrict__ rope_sin, const int32_t* __restrict__ pos_p, int H, int KV, int max_seq, int* err) {
  extern __shared__ float sm[];
  constexpr int hd = 64, half = 32;
  const int n_cap = min(max_seq, kWarpAttnMaxPos);
  const int n_pad = (n_cap + 3) / 4 * 4;
  float* kc = sm;                   // [n_pad][65] keys (padded rows: lane t reads row t conflict-free)
  float* vc = kc + n_pad * 65;      // [n_pad][64] values, 16-byte aligned (n_pad % 4 == 0)
  float* sc = vc + n_pad * 64;      // [n_pad] scores, then probabilities
  float* qh = sc + n_pad;           // [64] rotated query
  const int lane = threadIdx.x;
  const int pos = *pos_p;
  if (pos < 0 || pos >= n_cap) {
    pdl_wait();
    pdl_launch_dependents();
    if (lane == 0) record_error(err, EFG_ESTATE);
    return;
  }
  const int h = blockIdx.x, group = H / KV, kv = h / group, kvd = KV * hd;
  // the cached history (written by earlier steps) and the RoPE row, before the wait
  for (int e = lane; e < pos * 16; e += 32) {
    const int t = e >> 4, i4 = e & 15;
    const size_t row = static_cast<size_t>(t) * kvd + kv * hd;
    const float4 k4 = reinterpret_cast<const float4*>(k_layer + row)[i4];
    reinterpret_cast<float4*>(vc + t * hd)[i4] = reinterpret_cast<const float4*>(v_layer + row)[i4];
    float* d = kc + t * 65 + 4 * i4;
    d[0] = k4.x;
    d[1] = k4.y;
    d[2] = k4.z;
    d[3] = k4.w;
  }
  const float cs = rope_cos[static_cast<size_t>(pos) * half + lane], sn = rope_sin[static_cast<size_t>(pos) * half + lane];
  pdl_wait();
  pdl_launch_dependents();
  float qa, qb, ka, kb;
  rope_pair(q[h * hd + lane], q[h * hd + lane + half], cs, sn, qa, qb);
  rope_pair(knew[kv * hd + lane], knew[kv * hd + lane + half], cs, sn, ka, kb);
  if (h % group == 0) {  // the first head of each KV group writes the rotated key to the cache
    k_layer[static_cast<size_t>(pos) * kvd + kv * hd + lane] = ka;
    k_layer[static_cast<size_t>(pos) * kvd + kv * hd + lane + half] = kb;
  }
  qh[lane] = qa;
  qh[lane + half] = qb;
  kc[pos * 65 + lane] = ka;
  kc[pos * 65 + lane + half] = kb;
  vc[pos * hd + lane] = v_layer[static_cast<size_t>(pos) * kvd + kv * hd + lane];
  vc[pos * hd + lane + half] = v_layer[static_cast<size_t>(pos) * kvd + kv * hd + lane + half];
  __syncwarp();
  const int n_pos = pos + 1;
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(hd)));
  float mx = -INFINITY;
  for (int t = lane; t < n_pos; t += 32) {
    const float* kt = kc + t * 65;
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < hd; i += 8)
#pragma unroll
      for (int k = 0; k < 8; ++k) a[k] = __fadd_rn(a[k], __fmul_rn(qh[i + k], kt[i + k]));
    const float dot = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                                __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
    sc[t] = __fmul_rn(dot, scale);
    mx = fmaxf(mx, sc[t]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  double sum = 0.0;
  for (int t = lane; t < n_pos; t += 32) {
    const float e = expf(__fsub_rn(sc[t], mx));
    sc[t] = e;
    sum += static_cast<double>(e);
  }
  sum = warp_sum_d(sum);
  const float inv = static_cast<float>(1.0 / sum);
  for (int t = lane; t < n_pos; t += 32) sc[t] = __fmul_rn(sc[t], inv);
  __syncwarp();
  float acc0 = 0.f, acc1 = 0.f;
  for (int t = 0; t < n_pos; ++t) {
    const float pr = sc[t];
    acc0 = __fadd_rn(acc0, __fmul_rn(pr, vc[t * hd + lane]));
    acc1 = __fadd_rn(acc1, __fmul_rn(pr, vc[t * hd + lane + half]));
  }
  ctx[h * hd + lane] = acc0;
  ctx[h * hd + lane + half] = acc1;
}

// Batched prefill: rotate the keys of positions p0..p0+n-1, written unrotated into the
// cache by the k projection, in place (grid.x = n, one position per CTA).
__global__ void rope_keys_kernel(float* __restrict__ k_layer, const float* __restrict__ rope_cos,
                                 const float* __restrict__ rope_sin, int p0, int KV, int hd) {
  pdl_wait();
  pdl_launch_dependents();
  const int pos = p0 + static_cast<int>(blockIdx.x), half = hd / 2, kvd = KV * hd;
  const float* c = rope_cos + static_cast<size_t>(pos) * half;
  const float* s = rope_sin + static_cast<size_t>(pos) * half;
  float* kr = k_layer + static_cast<size_t>(pos) * kvd;
  for (int e = threadIdx.x; e < KV * half; e += blockDim.x) {
    const int kv = e / half, i = e % half;
    float ra, rb;
    rope_pair(kr[kv * hd + i], kr[kv * hd + i + half], c[i], s[i], ra, rb);
    kr[kv * hd + i] = ra;
    kr[kv * hd + i + half] = rb;
  }
}

// Multi-sequence step: row b's key (rotated at row_pos[b]) and value into its slot's cache
// at that position (grid.x = rows).
__global__ void store_kv_rows_kernel(const float* __restrict__ kb, const float* __restrict__ vb,
                                     const uint64_t* __restrict__ slot_k, const uint64_t* __restrict__ slot_v,
                                     const int32_t* __restrict__ row_slot, const int32_t* __restrict__ row_pos,
                                     uint64_t layer_off, const float* __restrict__ rope_cos,
                                     const float* __restrict__ rope_sin, int KV, int hd) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x, pos = row_pos[b], half = hd / 2, kvd = KV * hd;
  float* kc = reinterpret_cast<float*>(slot_k[row_slot[b]]) + layer_off + static_cast<size_t>(pos) * kvd;
  float* vc = reinterpret_cast<float*>(slot_v[row_slot[b]]) + layer_off + static_cast<size_t>(pos) * kvd;
  const float* kr = kb + static_cast<size_t>(b) * kvd;
  const float* c = rope_cos + static_cast<size_t>(pos) * half;
  const float* s = rope_sin + static_cast<size_t>(pos) * half;
  for (int e = threadIdx.x; e < KV * half; e += blockDim.x) {
    const int kv = e / half, i = e % half;
    rope_pair(kr[kv * hd + i], kr[kv * hd + i + half], c[i], s[i], kc[kv * hd + i], kc[kv * hd + i + half]);
  }
  for (int e = threadIdx.x; e < kvd; e += blockDim.x) vc[e] = vb[static_cast<size_t>(b) * kvd + e];
}

// Multi-sequence step: next[b] = argmax of logits row b (kern::argmax's rule), one CTA per row.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* __restrict__ logits, uint32_t n,
                                                           int32_t* __restrict__ next) {
  pdl_wait();
  pdl_launch_dependents();
  const float* x = logits + static_cast<size_t>(blockIdx.x) * n;
  float best;
  uint32_t idx;
  block_argmax(x, n, best, idx);
  if (threadIdx.x == 0) next[blockIdx.x] = x[0] != x[0] || idx == 0xFFFFFFFFu ? 0 : static_cast<int32_t>(idx);
}

// Batched prefill: query head blockIdx.x of token blockIdx.y (position p0 + blockIdx.y),
// RoPE of q, then attend_head over the cache, which holds every rotated key up to its
// position (causal: later tokens of the batch are not read).
// Multi-sequence steps pass row_pos / row_slot: row b attends over its own slot's cache
// (slot_k[row_slot[b]] + layer_off) up to row_pos[b] instead.
__global__ void __launch_bounds__(kAttnThreads) attention_rows_kernel(
    const float* __restrict__ qb, const float* __restrict__ k_layer, const float* __restrict__ v_layer,
    float* __restrict__ ctxb, const float* __restrict__ rope_cos, const float* __restrict__ rope_sin, int p0, int H,
    int KV, int hd, int dim, const int32_t* __restrict__ row_pos, const int32_t* __restrict__ row_slot,
    const uint64_t* __restrict__ slot_k, const uint64_t* __restrict__ slot_v, uint64_t layer_off) {
  extern __shared__ float sm[];
  float* qh = sm;                             // [hd]
  float* stage = qh + hd;                     // [attn_stage_floats(hd)]
  float* sc = stage + attn_stage_floats(hd);  // [max_seq]
  __shared__ float red_f[kAttnThreads / 32];
  __shared__ double red_d[kAttnThreads / 32];
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.y, pos = row_pos ? row_pos[b] : p0 + b;
  if (row_pos) {
    k_layer = reinterpret_cast<const float*>(slot_k[row_slot[b]]) + layer_off;
    v_layer = reinterpret_cast<const float*>(slot_v[row_slot[b]]) + layer_off;
  }
  const int h = blockIdx.x, group = H / KV, kv = h / group, half = hd / 2, kvd = KV * hd;
  const float* q = qb + static_cast<size_t>(b) * dim;
  const float* c = rope_cos + static_cast<size_t>(pos) * half;
  const float* s = rope_sin + static_cast<size_t>(pos) * half;
  for (int i = threadIdx.x; i < half; i += blockDim.x)
    rope_pair(q[h * hd + i], q[h * hd + i + half], c[i], s[i], qh[i], qh[i + half]);
  __syncthreads();
  attend_head(qh, k_layer, v_layer, k_layer + static_cast<size_t>(pos) * kvd + kv * hd, kv, hd, kvd, pos + 1, sc,
              stage, red_f, red_d, ctxb + static_cast<size_t>(b) * dim + h * hd);
}

// out = silu(gate) * up (src/kernels.cpp:94-99), for the unfused path.
__global__ void swiglu_kernel(float* __restrict__ out, const float* __restrict__ g, const float* __restrict__ u,
                              uint32_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    out[i] = swiglu_value(g[i], u[i]);
  }
}

// h = w * (x * inv) with inv = float(1 / sqrt(mean(x^2) + eps)) (src/kernels.cpp:69-75), by
// one CTA.
__device__ __forceinline__ void rmsnorm_row(float* __restrict__ h, const float* __restrict__ x,
                                            const float* __restrict__ w, uint32_t n, float eps, double* red) {
  // Rows of up to 8 elements per thread are read into registers first (all loads in flight
  // at once instead of one load latency per element); the arithmetic and its order are the
  // same on both paths.
  constexpr uint32_t kPer = 8;
  const bool regs = n <= kPer * blockDim.x;
  float xv[kPer], wv[kPer];
  double ss = 0.0;
  if (regs) {
#pragma unroll
    for (uint32_t k = 0; k < kPer; ++k) {
      const uint32_t i = threadIdx.x + k * blockDim.x;
      xv[k] = i < n ? x[i] : 0.f;
      wv[k] = i < n ? w[i] : 0.f;
    }
#pragma unroll
    for (uint32_t k = 0; k < kPer; ++k)
      if (threadIdx.x + k * blockDim.x < n) ss += static_cast<double>(xv[k]) * static_cast<double>(xv[k]);
  } else {
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += static_cast<double>(x[i]) * static_cast<double>(x[i]);
  }
  ss = warp_sum_d(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  double tot = 0.0;
  for (uint32_t k = 0; k < blockDim.x / 32; ++k) tot += red[k];
  const float inv = static_cast<float>(1.0 / sqrt((n ? tot / n : 0.0) + static_cast<double>(eps)));
  if (regs) {
#pragma unroll
    for (uint32_t k = 0; k < kPer; ++k) {
      const uint32_t i = threadIdx.x + k * blockDim.x;
      if (i < n) h[i] = __fmul_rn(wv[k], __fmul_rn(xv[k], inv));
    }
  } else {
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) h[i] = __fmul_rn(w[i], __fmul_rn(x[i], inv));
  }
}

// RMSNorm for the unfused path; one CTA.
__global__ void rmsnorm_kernel(float* __restrict__ h, const float* __restrict__ x, const float* __restrict__ w,
                               uint32_t n, float eps) {
  __shared__ double red[32];
  pdl_wait();
  pdl_launch_dependents();
  rmsnorm_row(h, x, w, n, eps, red);
}

// Batched prefill: RMSNorm of every row of xb into hb (one CTA per row).
__global__ void rmsnorm_rows_kernel(float* __restrict__ hb, const float* __restrict__ xb,
                                    const float* __restrict__ w, uint32_t n, float eps) {
  __shared__ double red[32];
  pdl_wait();
  pdl_launch_dependents();
  const size_t o = static_cast<size_t>(blockIdx.x) * n;
  rmsnorm_row(hb + o, xb + o, w, n, eps, red);
}

// Residual add x += y (src/model.cpp:247-249, 260-262), elementwise.
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, size_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    x[i] = __fadd_rn(x[i], y[i]);
}

// Index of the first maximum of logits (src/kernels.cpp:105-111); records it, makes it the
// next token unless that token is given, and advances the position.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, uint32_t n,
                                                      int32_t* __restrict__ tokens, int32_t* __restrict__ out_tokens,
                                                      int32_t* __restrict__ pos_p, const int32_t* __restrict__ n_fixed,
                                                      int max_seq) {
  pdl_wait();
  pdl_launch_dependents();
  float best;
  uint32_t idx;
  block_argmax(logits, n, best, idx);
  if (threadIdx.x == 0) {
    // The reference starts from index 0 and takes strictly greater values, so a NaN at
    // index 0 is never replaced (all comparisons with it are false).
    const float first = logits[0];
    if (first != first) idx = 0;
    if (idx == 0xFFFFFFFFu) idx = 0;
    const int32_t pos = *pos_p;
    out_tokens[pos] = static_cast<int32_t>(idx);
    if (pos + 1 < max_seq && pos + 1 >= *n_fixed) tokens[pos + 1] = static_cast<int32_t>(idx);
    *pos_p = pos + 1;
  }
}

// A prefill step without logits only advances the position.
__global__ void advance_kernel(int32_t* pos_p) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) *pos_p += 1;
}

struct Mat {
  int type = 0;
  const uint8_t* w = nullptr;
  uint32_t rows = 0, cols = 0;
};

struct Layer {
  Mat q, k, v, o, gate, up, down;
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
};

}  // namespace

struct Decoder {
  efq::Layout L;
  efq::Config c;
  int device = 0;
  cudaStream_t stream = nullptr;
  uint8_t* d_data = nullptr;
  float *kc = nullptr, *vc = nullptr, *rcos = nullptr, *rsin = nullptr;
  float *x = nullptr, *h = nullptr, *q = nullptr, *knew = nullptr, *ctx = nullptr, *act = nullptr, *gate = nullptr,
        *up = nullptr, *logits = nullptr;
  int32_t *state = nullptr;  // [0] pos, [1] n_fixed, then tokens[max_seq], out_tokens[max_seq]
  size_t max_seq = 0;
  size_t cached = 0;
  Mat embed, lm_head;
  const float* final_norm = nullptr;
  std::vector<Layer> layers;
  uint64_t bytes_per_token = 0;
  int n_q4 = 0, n_q8 = 0;
  cudaGraphExec_t g_full = nullptr, g_prefill = nullptr;
  int* d_err = nullptr;
  // persistent decode kernel (efg_decode_mk.cuh)
  bool mk_ok = false, use_mk = false;
  std::string mk_why;  // why the persistent kernel cannot run this model (when !mk_ok)
  mk::Phase* d_phases = nullptr;  // one token's phases
  uint32_t n_phases = 0;
  unsigned* d_bar = nullptr;      // [0] barrier counter, then ctl[2] as int32
  float* d_keep = nullptr;        // per-step logits kept by generate
  size_t keep_cap = 0;
  int grid = 0;
  // batched prefill (prefill_tokens): [P][hidden] x5, [P][intermediate] x3, allocated on first use
  float* pb = nullptr;
  float *xb = nullptr, *hb = nullptr, *qb = nullptr, *cb = nullptr, *ob = nullptr, *gb = nullptr, *ub = nullptr,
        *ab = nullptr, *kt = nullptr, *vt = nullptr;
  size_t pb_rows = 0;
  // sequence slots for multi-sequence steps (efg_decoder_set_slots); slot 0 is kc / vc and
  // `cached`, the cache of forward / prefill / generate
  size_t n_slots = 1;
  std::vector<float*> slot_kc, slot_vc;  // slots 1.. (index s - 1)
  std::vector<size_t> slot_cached;        // slots 1..
  uint64_t *d_slot_k = nullptr, *d_slot_v = nullptr;  // [n_slots] cache base addresses
  int32_t* d_rows = nullptr;  // [3][pb_rows]: token, slot, position per row of a step
  float* d_lb = nullptr;      // [pb_rows][vocab] logits of a step
  int32_t* d_next = nullptr;  // [pb_rows] argmax of each row
  std::map<size_t, cudaGraphExec_t> step_graphs;  // a multi-sequence step per row count
  int32_t* pos_p() const { return state; }
  int32_t* nfix_p() const { return state + 1; }
  int32_t* tokens() const { return state + 2; }
  int32_t* out_tokens() const { return state + 2 + max_seq; }
};

namespace {

int check_mat(const Mat& m, const char* name) {
  if (m.type != 3 && m.type != 4)
    return fail(EFG_EINVAL, "matrix '%s' is stored as %s; the B200 decode step runs Q4_0 and Q8_0 matrices", name,
                efq::type_name(m.type));
  return EFG_OK;
}

// The decode step's matvecs stay on the CUDA-core and large-matrix kernels: in its chain of
// different kernels the small-matrix MMA kernel measured slower (1447-1501 tok/s against 1572
// on the TinyLlama shape, whichever subset of the step's calls it took).
MatvecArgs decode_args(MatvecArgs a) {
  a.small_kernel = false;
  return a;
}

// logits = lm_head . rmsnorm(x, final_norm) (src/model.cpp:266-270).
int enqueue_lm_head(Decoder& D, const float* x, cudaStream_t s, float* out = nullptr) {
  cudaLaunchAttribute attr[1];
  const uint32_t Dm = static_cast<uint32_t>(D.c.hidden);
  MatvecArgs a;
  a.fmt = D.lm_head.type == 4 ? Fmt::Q4 : Fmt::Q8;
  a.x = x;
  a.norm_w = D.final_norm;
  a.norm_eps = static_cast<float>(D.c.rms_eps);
  a.cols = Dm;
  a.pdl = true;
  a.n_jobs = 1;
  a.jobs[0] = MatvecJobDev{D.lm_head.w, out ? out : D.logits, D.lm_head.rows, 0};
  if (!matvec_fast_path_ok(a)) {
    cudaLaunchConfig_t cf = cfg_of(dim3(1), dim3(256), 0, s, attr);
    EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, rmsnorm_kernel, D.h, x, D.final_norm, Dm, static_cast<float>(D.c.rms_eps)),
                 "rmsnorm launch");
    a.x = D.h;
    a.norm_w = nullptr;
  }
  return launch_matvec(decode_args(a), D.d_err, s);
}

// Next token = argmax(logits) at the device-side position, which then advances.
int enqueue_argmax(Decoder& D, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cf = cfg_of(dim3(1), dim3(1024), 0, s, attr);
  EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, argmax_kernel, static_cast<const float*>(D.logits),
                                  static_cast<uint32_t>(D.c.vocab), D.tokens(), D.out_tokens(), D.pos_p(),
                                  static_cast<const int32_t*>(D.nfix_p()), static_cast<int>(D.max_seq)),
               "argmax launch");
  return EFG_OK;
}

int enqueue_step(Decoder& D, bool logits, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  const uint32_t Dm = static_cast<uint32_t>(D.c.hidden), F = static_cast<uint32_t>(D.c.intermediate),
                 kvd = static_cast<uint32_t>(D.c.kv_dim()), V = static_cast<uint32_t>(D.c.vocab);
  const int H = static_cast<int>(D.c.heads), KV = static_cast<int>(D.c.kv_heads), hd = static_cast<int>(D.c.head_dim);
  {
    cudaLaunchConfig_t cf = cfg_of(dim3(std::max(1u, std::min(16u, (Dm + 255) / 256))), dim3(256), 0, s, attr);
    EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, embed_kernel, D.embed.w, D.embed.type, V, Dm,
                                    static_cast<const int32_t*>(D.tokens()), static_cast<const int32_t*>(D.pos_p()),
                                    D.x, D.d_err),
                 "embed launch");
  }
  for (size_t l = 0; l < D.layers.size(); ++l) {
    const Layer& Ly = D.layers[l];
    float* kl = D.kc + l * D.max_seq * kvd;
    float* vl = D.vc + l * D.max_seq * kvd;
    // q/k/v: jobs grouped by type; v goes straight into the cache at pos.
    const MatvecJobDev jq{Ly.q.w, D.q, Ly.q.rows, 0}, jk{Ly.k.w, D.knew, Ly.k.rows, 0}, jv{Ly.v.w, vl, Ly.v.rows, kvd};
    const Mat* mats[3] = {&Ly.q, &Ly.k, &Ly.v};
    const MatvecJobDev js[3] = {jq, jk, jv};
    bool done[3] = {false, false, false};
    for (int i = 0; i < 3; ++i) {
      if (done[i]) continue;
      MatvecArgs a;
      a.fmt = mats[i]->type == 4 ? Fmt::Q4 : Fmt::Q8;
      a.x = D.x;
      a.norm_w = Ly.attn_norm;
      a.norm_eps = static_cast<float>(D.c.rms_eps);
      a.pos = D.pos_p();
      a.cols = Dm;
      a.pdl = true;
      for (int k = i; k < 3; ++k)
        if (!done[k] && mats[k]->type == mats[i]->type) {
          a.jobs[a.n_jobs++] = js[k];
          done[k] = true;
        }
      if (!matvec_fast_path_ok(a)) {  // explicit RMSNorm, then plain matvecs
        cudaLaunchConfig_t cf = cfg_of(dim3(1), dim3(256), 0, s, attr);
        EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, rmsnorm_kernel, D.h, static_cast<const float*>(D.x), Ly.attn_norm, Dm,
                                        static_cast<float>(D.c.rms_eps)),
                     "rmsnorm launch");
        a.x = D.h;
        a.norm_w = nullptr;
      }
      if (int st = launch_matvec(decode_args(a), D.d_err, s)) return st;
    }
    if (hd == 64 && D.max_seq <= static_cast<size_t>(kWarpAttnMaxPos)) {
      const size_t smem = warp_attn_smem_floats(D.max_seq) * sizeof(float);
      cudaLaunchConfig_t cf = cfg_of(dim3(H), dim3(32), smem, s, attr);
      EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, attention_warp_kernel, static_cast<const float*>(D.q),
                                      static_cast<const float*>(D.knew), kl, static_cast<const float*>(vl), D.ctx,
                                      static_cast<const float*>(D.rcos), static_cast<const float*>(D.rsin),
                                      static_cast<const int32_t*>(D.pos_p()), H, KV, static_cast<int>(D.max_seq),
                                      D.d_err),
                   "attention launch");
    } else {
      const size_t smem = (2 * hd + attn_stage_floats(hd) + D.max_seq) * sizeof(float);
      cudaLaunchConfig_t cf = cfg_of(dim3(H), dim3(kAttnThreads), smem, s, attr);
      EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, attention_kernel, static_cast<const float*>(D.q),
                                      static_cast<const float*>(D.knew), kl, static_cast<const float*>(vl), D.ctx,
                                      static_cast<const float*>(D.rcos), static_cast<const float*>(D.rsin),
                                      static_cast<const int32_t*>(D.pos_p()), H, KV, hd, static_cast<int>(D.max_seq),
                                      D.d_err),
                   "attention launch");
    }
    {  // o_proj, residual add into x (src/model.cpp:247-249)
      MatvecArgs a;
      a.fmt = Ly.o.type == 4 ? Fmt::Q4 : Fmt::Q8;
      a.epi = Epi::Add;
      a.x = D.ctx;
      a.cols = Dm;
      a.pdl = true;
      a.n_jobs = 1;
      a.jobs[0] = MatvecJobDev{Ly.o.w, D.x, Ly.o.rows, 0};
      if (int st = launch_matvec(decode_args(a), D.d_err, s)) return st;
    }
    {  // gate/up with the ffn RMSNorm and SwiGLU (src/model.cpp:253-258)
      MatvecArgs a;
      a.fmt = Ly.gate.type == 4 ? Fmt::Q4 : Fmt::Q8;
      a.epi = Epi::SwiGLU;
      a.x = D.x;
      a.norm_w = Ly.ffn_norm;
      a.norm_eps = static_cast<float>(D.c.rms_eps);
      a.cols = Dm;
      a.pdl = true;
      a.n_jobs = 2;
      a.jobs[0] = MatvecJobDev{Ly.gate.w, D.act, Ly.gate.rows, 0};
      a.jobs[1] = MatvecJobDev{Ly.up.w, D.act, Ly.up.rows, 0};
      if (Ly.gate.type == Ly.up.type && matvec_fast_path_ok(a)) {
        if (int st = launch_matvec(decode_args(a), D.d_err, s)) return st;
      } else {
        cudaLaunchConfig_t cf = cfg_of(dim3(1), dim3(256), 0, s, attr);
        EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, rmsnorm_kernel, D.h, static_cast<const float*>(D.x), Ly.ffn_norm, Dm,
                                        static_cast<float>(D.c.rms_eps)),
                     "rmsnorm launch");
        for (int m = 0; m < 2; ++m) {
          const Mat& M = m == 0 ? Ly.gate : Ly.up;
          MatvecArgs b;
          b.fmt = M.type == 4 ? Fmt::Q4 : Fmt::Q8;
          b.x = D.h;
          b.cols = Dm;
          b.pdl = true;
          b.n_jobs = 1;
          b.jobs[0] = MatvecJobDev{M.w, m == 0 ? D.gate : D.up, M.rows, 0};
          if (int st = launch_matvec(decode_args(b), D.d_err, s)) return st;
        }
        cudaLaunchConfig_t cg = cfg_of(dim3(std::max(1u, std::min(64u, (F + 255) / 256))), dim3(256), 0, s, attr);
        EFG_TRY_CUDA(cudaLaunchKernelEx(&cg, swiglu_kernel, D.act, static_cast<const float*>(D.gate),
                                        static_cast<const float*>(D.up), F),
                     "swiglu launch");
      }
    }
    {  // down, residual add (src/model.cpp:260-262)
      MatvecArgs a;
      a.fmt = Ly.down.type == 4 ? Fmt::Q4 : Fmt::Q8;
      a.epi = Epi::Add;
      a.x = D.act;
      a.cols = F;
      a.pdl = true;
      a.n_jobs = 1;
      a.jobs[0] = MatvecJobDev{Ly.down.w, D.x, Ly.down.rows, 0};
      if (int st = launch_matvec(decode_args(a), D.d_err, s)) return st;
    }
  }
  if (logits) {
    if (int st = enqueue_lm_head(D, D.x, s)) return st;
    if (int st = enqueue_argmax(D, s)) return st;
  } else {
    cudaLaunchConfig_t cf = cfg_of(dim3(1), dim3(32), 0, s, attr);
    EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, advance_kernel, D.pos_p()), "advance launch");
  }
  return EFG_OK;
}

int capture(Decoder& D, bool logits, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  EFG_TRY_CUDA(cudaStreamBeginCapture(D.stream, cudaStreamCaptureModeThreadLocal), "graph capture");
  const int st = enqueue_step(D, logits, D.stream);
  const cudaError_t e = cudaStreamEndCapture(D.stream, &g);
  if (st != EFG_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  EFG_TRY_CUDA(e, "graph capture end");
  const cudaError_t ie = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  EFG_TRY_CUDA(ie, "graph instantiate");
  return EFG_OK;
}

// ---------------------------------------------------------------- persistent kernel setup

// Rows per batch and per tile of one matrix in the persistent kernel: 4 rows per batch
// (2 for long Q8_0 rows), and as many batches per tile as one ring slot holds.
bool mk_job(const Mat& m, float* y, uint32_t y_pos_stride, mk::Job& J) {
  J.W = m.w;
  J.y = y;
  J.rows = m.rows;
  J.rb = m.cols / 32 * (m.type == 4 ? 18 : 34);
  J.y_pos_stride = y_pos_stride;
  J.fmt = static_cast<uint32_t>(m.type);
  if (J.rb % 16 != 0 || reinterpret_cast<uintptr_t>(m.w) % 16 != 0) return false;
  // 2 rows per batch: the unrolled per-row code of one batch is what every phase runs
  // once or twice, so it is kept small enough to stay in the instruction cache
  J.RB = 2;
  if (J.RB * J.rb > mk::kSlotBytes) return false;
  // as many batches per tile as one ring slot holds (at most kMaxBatches): large bulk copies
  // keep ~180 KB in flight per SM; the batches of a tile go to different warps
  const uint32_t max_batches = std::min<uint32_t>(mk::kMaxBatches, mk::kSlotBytes / (J.RB * J.rb));
  J.TR = J.RB * max_batches;
  return true;
}

int build_mk(Decoder& D) {
  const efq::Config& c = D.c;
  D.mk_ok = false;
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  int coop = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev->device);
  auto no = [&](const char* why) {
    D.mk_why = why;
    return EFG_OK;
  };
  if (!coop) return no("the device has no cooperative launch");
  if (dev->smem_optin < mk::smem_bytes()) return no("not enough shared memory per block");
  if ((2 + mk::kAttnChunk) * static_cast<size_t>(c.head_dim) + D.max_seq > mk::kXsFloats)
    return no("max_seq too long for the attention scratch");
  if (c.hidden % 64 != 0 || c.intermediate % 64 != 0 || c.hidden / 64 > static_cast<int64_t>(mk::kMaxSlotsX) ||
      c.intermediate / 64 > static_cast<int64_t>(mk::kMaxSlotsX))
    return no("hidden and intermediate sizes must be multiples of 64 up to 6144");
  EFG_TRY_CUDA(cudaFuncSetAttribute(mk::decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(mk::smem_bytes())),
               "decode kernel attribute");
  int per_sm = 0;
  EFG_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mk::decode_kernel, mk::kThreads, mk::smem_bytes()),
               "decode kernel occupancy");
  if (per_sm < 1) return no("the decode kernel does not fit on an SM");
  const uint32_t grid = static_cast<uint32_t>(dev->sm_count);
  D.grid = static_cast<int>(grid);
  const uint32_t Dm = static_cast<uint32_t>(c.hidden), F = static_cast<uint32_t>(c.intermediate),
                 kvd = static_cast<uint32_t>(c.kv_dim());
  auto gof = [](uint32_t cols) { return (cols / 64 + 31) / 32; };
  if (gof(Dm) > 3 || gof(F) > 3) return no("rows longer than 6144 columns");
  auto mv = [&](uint32_t epi, uint32_t in_mode, const float* x, const float* x2, const float* nw, uint32_t cols) {
    mk::Phase P{};
    P.kind = mk::kMatvec;
    P.epi = epi;
    P.in_mode = in_mode;
    P.x = x;
    P.x2 = x2;
    P.norm_w = nw;
    P.cols = cols;
    P.G = gof(cols);
    return P;
  };
  std::vector<mk::Phase> full;
  bool fit = true;
  mk::Phase e{};
  e.kind = mk::kEmbed;
  full.push_back(e);
  for (size_t l = 0; l < D.layers.size(); ++l) {
    const Layer& Ly = D.layers[l];
    float* vl = D.vc + l * D.max_seq * kvd;
    mk::Phase qkv = mv(0, mk::kInNorm, D.x, nullptr, Ly.attn_norm, Dm);
    const uint32_t rg = mk::kConsumerWarps / qkv.G;
    qkv.n_jobs = 3;
    fit = fit && mk_job(Ly.q, D.q, 0, qkv.jobs[0]) && mk_job(Ly.k, D.knew, 0, qkv.jobs[1]) &&
          mk_job(Ly.v, vl, kvd, qkv.jobs[2]);
    (void)rg;
    full.push_back(qkv);
    mk::Phase at{};
    at.kind = mk::kAttn;
    at.layer = static_cast<uint32_t>(l);
    full.push_back(at);
    mk::Phase o = mv(1, mk::kInPlain, D.ctx, nullptr, nullptr, Dm);
    o.n_jobs = 1;
    fit = fit && mk_job(Ly.o, D.x, 0, o.jobs[0]);
    full.push_back(o);
    mk::Phase gu = mv(0, mk::kInNorm, D.x, nullptr, Ly.ffn_norm, Dm);
    gu.n_jobs = 2;
    fit = fit && mk_job(Ly.gate, D.gate, 0, gu.jobs[0]) && mk_job(Ly.up, D.up, 0, gu.jobs[1]);
    full.push_back(gu);
    mk::Phase dn = mv(1, mk::kInSwiGLU, D.gate, D.up, nullptr, F);
    dn.n_jobs = 1;
    fit = fit && mk_job(Ly.down, D.x, 0, dn.jobs[0]);
    full.push_back(dn);
  }
  mk::Phase lm = mv(0, mk::kInNorm, D.x, nullptr, D.final_norm, Dm);
  lm.n_jobs = 1;
  fit = fit && mk_job(D.lm_head, nullptr, 0, lm.jobs[0]);  // y: the launch's logits
  full.push_back(lm);
  mk::Phase am{};
  am.kind = mk::kArgmax;
  full.push_back(am);
  if (!fit) return no("a matrix's rows are not 16-byte multiples");
  if (full.size() > mk::kMaxPhases) return no("too many layers for the persistent kernel's phase list");
  D.n_phases = static_cast<uint32_t>(full.size());
  EFG_TRY_CUDA(cudaMalloc(&D.d_phases, full.size() * sizeof(mk::Phase)), "phase table allocation");
  EFG_TRY_CUDA(cudaMemcpy(D.d_phases, full.data(), full.size() * sizeof(mk::Phase), cudaMemcpyHostToDevice),
               "phase table upload");
  EFG_TRY_CUDA(cudaMalloc(&D.d_bar, 16), "barrier allocation");
  D.mk_ok = true;
  return EFG_OK;
}

int32_t* mk_ctl(Decoder& D) { return reinterpret_cast<int32_t*>(D.d_bar + 1); }

// One launch of the persistent kernel: n_pre steps without logits, then n_full steps with
// logits and argmax (kept per step at `keep` when not null), stopping after `eos`.
int launch_mk(Decoder& D, uint32_t n_pre, uint32_t n_full, float* keep, int32_t eos) {
  if (n_pre + n_full == 0) return EFG_OK;
  EFG_TRY_CUDA(cudaMemsetAsync(D.d_bar, 0, 16, D.stream), "barrier reset");
  mk::Params p{};
  p.phases = D.d_phases;
  p.n_phases = D.n_phases;
  p.n_prefill_steps = n_pre;
  p.n_full_steps = n_full;
  p.embed = D.embed.w;
  p.embed_type = D.embed.type;
  p.vocab = static_cast<uint32_t>(D.c.vocab);
  p.dim = static_cast<uint32_t>(D.c.hidden);
  p.H = static_cast<uint32_t>(D.c.heads);
  p.KV = static_cast<uint32_t>(D.c.kv_heads);
  p.hd = static_cast<uint32_t>(D.c.head_dim);
  p.max_seq = static_cast<uint32_t>(D.max_seq);
  p.kc = D.kc;
  p.vc = D.vc;
  p.rcos = D.rcos;
  p.rsin = D.rsin;
  p.q = D.q;
  p.knew = D.knew;
  p.ctx = D.ctx;
  p.x = D.x;
  p.logits = keep ? keep : D.logits;
  p.logits_step_stride = keep ? static_cast<uint32_t>(D.c.vocab) : 0;
  p.eps = static_cast<float>(D.c.rms_eps);
  p.pos = D.pos_p();
  p.n_fixed = D.nfix_p();
  p.tokens = D.tokens();
  p.out_tokens = D.out_tokens();
  p.eos = eos;
  p.ctl = mk_ctl(D);
  p.bar = D.d_bar;
  p.err = D.d_err;
  cudaLaunchConfig_t cf{};
  cf.gridDim = dim3(static_cast<unsigned>(D.grid));
  cf.blockDim = dim3(mk::kThreads);
  cf.dynamicSmemBytes = mk::smem_bytes();
  cf.stream = D.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cf.attrs = attr;
  cf.numAttrs = 1;
  EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, mk::decode_kernel, p), "decode kernel launch");
  return EFG_OK;
}

int device_status(Decoder& D) {
  int e = 0;
  EFG_TRY_CUDA(cudaMemcpyAsync(&e, D.d_err, sizeof e, cudaMemcpyDeviceToHost, D.stream), "error word read");
  EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
  if (e != 0) {
    cudaMemsetAsync(D.d_err, 0, sizeof(int), D.stream);
    cudaStreamSynchronize(D.stream);
    return fail(e, "decode: the device reported %s", efg_status_string(e));
  }
  return EFG_OK;
}

void drop_step_graphs(Decoder& D) {
  for (auto& kv : D.step_graphs) cudaGraphExecDestroy(kv.second);
  D.step_graphs.clear();
}

void free_slots(Decoder& D) {
  for (float* p : D.slot_kc) cudaFree(p);
  for (float* p : D.slot_vc) cudaFree(p);
  D.slot_kc.clear();
  D.slot_vc.clear();
  D.slot_cached.clear();
  D.n_slots = 1;
}

void destroy(Decoder* D) {
  if (!D) return;
  if (D->stream) cudaStreamSynchronize(D->stream);
  if (D->g_full) cudaGraphExecDestroy(D->g_full);
  if (D->g_prefill) cudaGraphExecDestroy(D->g_prefill);
  if (D->pb) cudaFree(D->pb);
  drop_step_graphs(*D);
  free_slots(*D);
  for (void* p : {static_cast<void*>(D->d_slot_k), static_cast<void*>(D->d_slot_v), static_cast<void*>(D->d_rows),
                  static_cast<void*>(D->d_lb), static_cast<void*>(D->d_next)})
    if (p) cudaFree(p);
  for (void* p : {static_cast<void*>(D->d_data), static_cast<void*>(D->kc), static_cast<void*>(D->vc),
                  static_cast<void*>(D->rcos), static_cast<void*>(D->rsin), static_cast<void*>(D->x),
                  static_cast<void*>(D->state), static_cast<void*>(D->d_phases), static_cast<void*>(D->d_bar),
                  static_cast<void*>(D->d_keep)})
    if (p) cudaFree(p);
  if (D->stream) cudaStreamDestroy(D->stream);
  delete D;
}

int open_decoder(const char* path, size_t max_seq, Decoder** out) {
  if (!path || !out) return fail(EFG_EINVAL, "decoder_open: null argument");
  *out = nullptr;
  FILE* f = std::fopen(path, "rb");
  if (!f) return fail(EFG_EINVAL, "cannot open '%s'", path);
  std::fseek(f, 0, SEEK_END);
  const long long fsize = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  std::vector<uint8_t> file(static_cast<size_t>(fsize > 0 ? fsize : 0));
  const size_t got = file.empty() ? 0 : std::fread(file.data(), 1, file.size(), f);
  std::fclose(f);
  if (got != file.size()) return fail(EFG_EINVAL, "'%s': short read", path);
  std::unique_ptr<Decoder, void (*)(Decoder*)> D(new Decoder, destroy);
  try {
    D->L = efq::parse(file.data(), file.size());
  } catch (const efq::FormatError& e) {
    return fail(EFG_EFORMAT, "'%s': %s", path, e.what());
  }
  D->c = D->L.cfg;
  const efq::Config& c = D->c;
  if (max_seq == 0) return fail(EFG_EINVAL, "Transformer: max_seq must be > 0");
  if (max_seq > static_cast<size_t>(c.max_position))
    return fail(EFG_EINVAL, "Transformer: max_seq %zu exceeds max_position_embeddings %lld", max_seq,
                static_cast<long long>(c.max_position));
  D->max_seq = max_seq;
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  D->device = dev->device;
  D->d_err = dev->d_err;
  EFG_TRY_CUDA(cudaStreamCreateWithFlags(&D->stream, cudaStreamNonBlocking), "stream create");
  const uint64_t base = D->L.data_start;
  const uint64_t region = file.size() - base;
  EFG_TRY_CUDA(cudaMalloc(&D->d_data, region ? region : 16), "weight allocation");
  EFG_TRY_CUDA(cudaMemcpy(D->d_data, file.data() + base, region, cudaMemcpyHostToDevice), "weight upload");
  auto mat = [&](const std::string& name) {
    const efq::Tensor& t = D->L.at(name);
    Mat m;
    m.type = t.type;
    m.w = D->d_data + (t.offset - base);
    m.rows = static_cast<uint32_t>(t.rows());
    m.cols = static_cast<uint32_t>(t.cols());
    (m.type == 4 ? D->n_q4 : D->n_q8) += (m.type == 3 || m.type == 4) ? 1 : 0;
    return m;
  };
  auto vec = [&](const std::string& name) {
    const efq::Tensor& t = D->L.at(name);
    return reinterpret_cast<const float*>(D->d_data + (t.offset - base));
  };
  try {
    D->embed = mat("model.embed_tokens.weight");
    if (D->embed.type == 3 || D->embed.type == 4) (D->embed.type == 4 ? D->n_q4 : D->n_q8) -= 1;
    D->lm_head = c.tie_embeddings ? D->embed : mat("lm_head.weight");
    D->final_norm = vec("model.norm.weight");
    D->layers.resize(static_cast<size_t>(c.layers));
    for (int64_t l = 0; l < c.layers; ++l) {
      const std::string p = "model.layers." + std::to_string(l) + ".";
      Layer& Ly = D->layers[static_cast<size_t>(l)];
      Ly.q = mat(p + "self_attn.q_proj.weight");
      Ly.k = mat(p + "self_attn.k_proj.weight");
      Ly.v = mat(p + "self_attn.v_proj.weight");
      Ly.o = mat(p + "self_attn.o_proj.weight");
      Ly.gate = mat(p + "mlp.gate_proj.weight");
      Ly.up = mat(p + "mlp.up_proj.weight");
      Ly.down = mat(p + "mlp.down_proj.weight");
      Ly.attn_norm = vec(p + "input_layernorm.weight");
      Ly.ffn_norm = vec(p + "post_attention_layernorm.weight");
      for (const Mat* m : {&Ly.q, &Ly.k, &Ly.v, &Ly.o, &Ly.gate, &Ly.up, &Ly.down})
        if (int st = check_mat(*m, "layer matrix")) return st;
    }
  } catch (const efq::FormatError& e) {
    return fail(EFG_EFORMAT, "'%s': %s", path, e.what());
  }
  if (int st = check_mat(D->lm_head, "lm_head.weight")) return st;
  for (const auto& t : D->L.tensors)  // src/qfile.cpp:237-241
    if (t.name != "model.embed_tokens.weight") D->bytes_per_token += t.bytes;
  if (c.tie_embeddings) D->bytes_per_token += D->L.at("model.embed_tokens.weight").bytes;

  const size_t kvd = static_cast<size_t>(c.kv_dim()), half = static_cast<size_t>(c.head_dim / 2);
  if (c.head_dim % 4 != 0 || c.head_dim > 2 * kAttnThreads || c.heads % c.kv_heads != 0)
    return fail(EFG_EINVAL, "decoder: head_dim must be a multiple of 4 up to %d and heads a multiple of kv_heads",
                2 * kAttnThreads);
  const size_t attn_smem =
      (2 * static_cast<size_t>(c.head_dim) + attn_stage_floats(static_cast<int>(c.head_dim)) + max_seq) * sizeof(float);
  if (attn_smem > 227 * 1024)
    return fail(EFG_EINVAL, "decoder: max_seq %zu is too long for the attention kernel", max_seq);
  if (c.head_dim == 64 && max_seq <= static_cast<size_t>(kWarpAttnMaxPos)) {
    EFG_TRY_CUDA(cudaFuncSetAttribute(attention_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(warp_attn_smem_floats(max_seq) * sizeof(float))),
                 "attention smem attribute");
  }
  if (attn_smem > 48 * 1024) {
    EFG_TRY_CUDA(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(attn_smem)),
                 "attention smem attribute");
    EFG_TRY_CUDA(cudaFuncSetAttribute(attention_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(attn_smem)),
                 "attention smem attribute");
  }
  const size_t cache = static_cast<size_t>(c.layers) * max_seq * kvd;
  EFG_TRY_CUDA(cudaMalloc(&D->kc, cache * sizeof(float)), "KV cache allocation");
  EFG_TRY_CUDA(cudaMalloc(&D->vc, cache * sizeof(float)), "KV cache allocation");
  EFG_TRY_CUDA(cudaMemset(D->kc, 0, cache * sizeof(float)), "KV cache init");
  EFG_TRY_CUDA(cudaMemset(D->vc, 0, cache * sizeof(float)), "KV cache init");
  // RoPE table exactly as src/kernels.cpp:113-131 computes it (float pow/cos/sin).
  std::vector<float> cs(max_seq * half), sn(max_seq * half), inv(half);
  for (size_t i = 0; i < half; ++i)
    inv[i] = 1.0f / std::pow(static_cast<float>(c.rope_theta), static_cast<float>(2 * i) / static_cast<float>(c.head_dim));
  for (size_t p = 0; p < max_seq; ++p)
    for (size_t i = 0; i < half; ++i) {
      const float ang = static_cast<float>(p) * inv[i];
      cs[p * half + i] = std::cos(ang);
      sn[p * half + i] = std::sin(ang);
    }
  EFG_TRY_CUDA(cudaMalloc(&D->rcos, cs.size() * sizeof(float) + 16), "rope allocation");
  EFG_TRY_CUDA(cudaMalloc(&D->rsin, sn.size() * sizeof(float) + 16), "rope allocation");
  EFG_TRY_CUDA(cudaMemcpy(D->rcos, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice), "rope upload");
  EFG_TRY_CUDA(cudaMemcpy(D->rsin, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice), "rope upload");
  const size_t Dm = static_cast<size_t>(c.hidden), F = static_cast<size_t>(c.intermediate),
               V = static_cast<size_t>(c.vocab);
  // one activation arena: x, h, q, knew, ctx, act, gate, up, logits (each 256-byte aligned)
  auto al = [](size_t n) { return (n * sizeof(float) + 255) / 256 * 256; };
  const size_t arena = al(Dm) * 5 + al(kvd) + al(F) * 3 + al(V);
  EFG_TRY_CUDA(cudaMalloc(&D->x, arena), "activation allocation");
  uint8_t* a = reinterpret_cast<uint8_t*>(D->x);
  size_t o = al(Dm);
  D->h = reinterpret_cast<float*>(a + o), o += al(Dm);
  D->q = reinterpret_cast<float*>(a + o), o += al(Dm);
  D->ctx = reinterpret_cast<float*>(a + o), o += al(Dm);
  o += al(Dm);
  D->knew = reinterpret_cast<float*>(a + o), o += al(kvd);
  D->act = reinterpret_cast<float*>(a + o), o += al(F);
  D->gate = reinterpret_cast<float*>(a + o), o += al(F);
  D->up = reinterpret_cast<float*>(a + o), o += al(F);
  D->logits = reinterpret_cast<float*>(a + o);
  EFG_TRY_CUDA(cudaMalloc(&D->state, (2 + 2 * max_seq) * sizeof(int32_t)), "state allocation");
  EFG_TRY_CUDA(cudaMemset(D->state, 0, (2 + 2 * max_seq) * sizeof(int32_t)), "state init");
  if (int st = capture(*D, true, &D->g_full)) return st;
  if (int st = capture(*D, false, &D->g_prefill)) return st;
  if (int st = build_mk(*D)) return st;
  D->use_mk = false;  // the per-operation graphs are faster today; the persistent kernel is opt-in
  *out = D.release();
  return EFG_OK;
}

// ---------------------------------------------------------------- batched prefill
// The prompt through the same layers as a batch of tokens (README.md:89-90 names the
// token-by-token prompt as the reference's limit): the Q4_0 projections of every token in
// one tensor-core GEMM per matrix, Q8_0 projections one matvec per token, then batched
// RMSNorm, key RoPE, causal attention, SwiGLU and residual adds. Equivalent to forward() at
// positions p0..p0+n-1 in turn.
constexpr size_t kPrefillRows = 64;  // tokens per pass

int ensure_prefill_buffers(Decoder& D) {
  if (D.pb) return EFG_OK;
  // The pass size does not depend on max_seq: a prefill pass never exceeds the cache, but the
  // rows of a multi-sequence step are different sequences, as many as there are slots.
  const size_t P = kPrefillRows, Dm = static_cast<size_t>(D.c.hidden),
               F = static_cast<size_t>(D.c.intermediate);
  auto al = [](size_t n) { return (n * sizeof(float) + 255) / 256 * 256; };
  const size_t kvd = static_cast<size_t>(D.c.kv_dim());
  EFG_TRY_CUDA(cudaMalloc(&D.pb, al(P * Dm) * 5 + al(P * F) * 3 + al(P * kvd) * 2), "prefill buffer allocation");
  uint8_t* a = reinterpret_cast<uint8_t*>(D.pb);
  size_t o = 0;
  for (float** b : {&D.xb, &D.hb, &D.qb, &D.cb, &D.ob}) *b = reinterpret_cast<float*>(a + o), o += al(P * Dm);
  for (float** b : {&D.gb, &D.ub, &D.ab}) *b = reinterpret_cast<float*>(a + o), o += al(P * F);
  for (float** b : {&D.kt, &D.vt}) *b = reinterpret_cast<float*>(a + o), o += al(P * kvd);
  D.pb_rows = P;
  return EFG_OK;
}

// Whether the tensor-core GEMM takes a Q8_0 matrix (rows of a multiple of 256 columns,
// 16-byte aligned operands); otherwise the rows go through the matvec one by one.
bool gemm_q8_ok(const Mat& M, const float* X) {
  return M.type == 3 && M.cols % 256 == 0 && reinterpret_cast<uintptr_t>(M.w) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(X) % 16 == 0;
}

// Y[b] = M . X[b] for b < n (X [n][M.cols], Y [n][M.rows]).
int batched_proj(Decoder& D, const Mat& M, const float* X, float* Y, size_t n, cudaStream_t s) {
  if (M.type == 4) return launch_gemm_q4_0(Y, M.w, X, M.rows, M.cols, n, D.d_err, s);
  if (gemm_q8_ok(M, X)) return launch_gemm_q8_0(Y, M.w, X, M.rows, M.cols, n, D.d_err, s);
  for (size_t b = 0; b < n; ++b) {
    MatvecArgs a;
    a.fmt = Fmt::Q8;
    a.x = X + b * M.cols;
    a.cols = M.cols;
    a.pdl = true;
    a.n_jobs = 1;
    a.jobs[0] = MatvecJobDev{M.w, Y + b * M.rows, M.rows, 0};
    if (int st = launch_matvec(decode_args(a), D.d_err, s)) return st;
  }
  return EFG_OK;
}

// Whether a matrix goes through launch_gemm (fused launches): Q4_0 or Q8_0, rows of a
// multiple of 256 columns, 16-byte aligned (the batch buffers are).
bool gemm_fusable(const Mat& M) {
  return (M.type == 4 || M.type == 3) && M.cols % 256 == 0 && reinterpret_cast<uintptr_t>(M.w) % 16 == 0;
}

// Y_i = M_i . X for up to three matrices sharing X: those of one weight type that the GEMM
// takes go out as one launch per type, the others through batched_proj.
int project_group(Decoder& D, const Mat* const* mats, float* const* outs, int count, const float* X, size_t n,
                  cudaStream_t s) {
  bool done[3] = {false, false, false};
  for (int qt : {4, 3}) {
    GemmCall c;
    c.qtype = qt == 4 ? 4 : 8;
    c.X = X;
    c.K = mats[0]->cols;
    c.B = n;
    for (int i = 0; i < count; ++i)
      if (mats[i]->type == qt && mats[i]->cols == c.K && gemm_fusable(*mats[i])) {
        c.jobs[c.n_jobs++] = GemmJob{mats[i]->w, outs[i], mats[i]->rows};
        done[i] = true;
      }
    if (c.n_jobs)
      if (int st = launch_gemm(c, D.d_err, s)) return st;
  }
  for (int i = 0; i < count; ++i)
    if (!done[i])
      if (int st = batched_proj(D, *mats[i], X, outs[i], n, s)) return st;
  return EFG_OK;
}

// n <= pb_rows rows through every layer. Prefill (multi = false): tokens tokens()[p0..p0+n)
// of slot 0 at positions p0..; with `logits`, the last token's logits in D.logits.
// Multi-sequence step (multi = true): row b is d_rows' (token, slot, position); every
// row's logits into d_lb and its argmax into d_next.
int batch_pass(Decoder& D, size_t p0, size_t n, bool logits, cudaStream_t s, bool multi = false) {
  cudaLaunchAttribute attr[1];
  const uint32_t Dm = static_cast<uint32_t>(D.c.hidden), F = static_cast<uint32_t>(D.c.intermediate),
                 V = static_cast<uint32_t>(D.c.vocab);
  const size_t kvd = static_cast<size_t>(D.c.kv_dim());
  const int H = static_cast<int>(D.c.heads), KV = static_cast<int>(D.c.kv_heads), hd = static_cast<int>(D.c.head_dim);
  const float eps = static_cast<float>(D.c.rms_eps);
  const unsigned nb = static_cast<unsigned>(n);
  auto grid_for = [](size_t count) { return dim3(static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>(592, (count + 255) / 256)))); };
  {
    cudaLaunchConfig_t cf = cfg_of(dim3(std::max(1u, std::min(16u, (Dm + 255) / 256)), nb), dim3(256), 0, s, attr);
    EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, embed_rows_kernel, D.embed.w, D.embed.type, V, Dm,
                                    static_cast<const int32_t*>(multi ? D.d_rows : D.tokens() + p0), D.xb, D.d_err),
                 "embed launch");
  }
  const int32_t* row_slot = multi ? D.d_rows + D.pb_rows : nullptr;
  const int32_t* row_pos = multi ? D.d_rows + 2 * D.pb_rows : nullptr;
  for (size_t l = 0; l < D.layers.size(); ++l) {
    const Layer& Ly = D.layers[l];
    float* kl = D.kc + l * D.max_seq * kvd;
    float* vl = D.vc + l * D.max_seq * kvd;
    cudaLaunchConfig_t cn = cfg_of(dim3(nb), dim3(256), 0, s, attr);
    EFG_TRY_CUDA(cudaLaunchKernelEx(&cn, rmsnorm_rows_kernel, D.hb, static_cast<const float*>(D.xb), Ly.attn_norm, Dm,
                                    eps),
                 "rmsnorm launch");
    const uint64_t layer_off = static_cast<uint64_t>(l) * D.max_seq * kvd;
    {  // q, k and v in as few launches as the weight types allow
      const Mat* mats[3] = {&Ly.q, &Ly.k, &Ly.v};
      float* outs[3] = {D.qb, multi ? D.kt : kl + p0 * kvd, multi ? D.vt : vl + p0 * kvd};
      if (int st = project_group(D, mats, outs, 3, D.hb, n, s)) return st;
    }
    if (!multi) {  // the k projection wrote unrotated keys into the cache rows: rotate them
      cudaLaunchConfig_t cf = cfg_of(dim3(nb), dim3(128), 0, s, attr);
      EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, rope_keys_kernel, kl, static_cast<const float*>(D.rcos),
                                      static_cast<const float*>(D.rsin), static_cast<int>(p0), KV, hd),
                   "rope launch");
    } else {  // each row's key and value into its own slot's cache
      cudaLaunchConfig_t cf = cfg_of(dim3(nb), dim3(128), 0, s, attr);
      EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, store_kv_rows_kernel, static_cast<const float*>(D.kt),
                                      static_cast<const float*>(D.vt), static_cast<const uint64_t*>(D.d_slot_k),
                                      static_cast<const uint64_t*>(D.d_slot_v), row_slot, row_pos, layer_off,
                                      static_cast<const float*>(D.rcos), static_cast<const float*>(D.rsin), KV, hd),
                   "kv store launch");
    }
    {
      const size_t smem = (hd + attn_stage_floats(hd) + D.max_seq) * sizeof(float);
      cudaLaunchConfig_t cf = cfg_of(dim3(H, nb), dim3(kAttnThreads), smem, s, attr);
      EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, attention_rows_kernel, static_cast<const float*>(D.qb),
                                      static_cast<const float*>(kl), static_cast<const float*>(vl), D.cb,
                                      static_cast<const float*>(D.rcos), static_cast<const float*>(D.rsin),
                                      static_cast<int>(p0), H, KV, hd, static_cast<int>(Dm), row_pos, row_slot,
                                      static_cast<const uint64_t*>(D.d_slot_k), static_cast<const uint64_t*>(D.d_slot_v),
                                      layer_off),
                   "attention launch");
    }
    if (gemm_fusable(Ly.o)) {  // o projection with the residual add in its epilogue
      GemmCall c;
      c.qtype = Ly.o.type == 4 ? 4 : 8;
      c.jobs[0] = GemmJob{Ly.o.w, D.xb, Ly.o.rows};
      c.n_jobs = 1;
      c.X = D.cb;
      c.K = Ly.o.cols;
      c.B = n;
      c.accumulate = true;
      if (int st = launch_gemm(c, D.d_err, s)) return st;
    } else {
      if (int st = batched_proj(D, Ly.o, D.cb, D.ob, n, s)) return st;
      cudaLaunchConfig_t cf = cfg_of(grid_for(n * Dm), dim3(256), 0, s, attr);
      EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, add_kernel, D.xb, static_cast<const float*>(D.ob), n * Dm), "add launch");
    }
    EFG_TRY_CUDA(cudaLaunchKernelEx(&cn, rmsnorm_rows_kernel, D.hb, static_cast<const float*>(D.xb), Ly.ffn_norm, Dm,
                                    eps),
                 "rmsnorm launch");
    if (int st = batched_proj(D, Ly.gate, D.hb, D.gb, n, s)) return st;
    if (int st = batched_proj(D, Ly.up, D.hb, D.ub, n, s)) return st;
    {
      cudaLaunchConfig_t cf = cfg_of(grid_for(n * F), dim3(256), 0, s, attr);
      EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, swiglu_kernel, D.ab, static_cast<const float*>(D.gb),
                                      static_cast<const float*>(D.ub), static_cast<uint32_t>(n * F)),
                   "swiglu launch");
    }
    if (gemm_fusable(Ly.down)) {  // down projection with the residual add in its epilogue
      GemmCall c;
      c.qtype = Ly.down.type == 4 ? 4 : 8;
      c.jobs[0] = GemmJob{Ly.down.w, D.xb, Ly.down.rows};
      c.n_jobs = 1;
      c.X = D.ab;
      c.K = Ly.down.cols;
      c.B = n;
      c.accumulate = true;
      if (int st = launch_gemm(c, D.d_err, s)) return st;
    } else {
      if (int st = batched_proj(D, Ly.down, D.ab, D.ob, n, s)) return st;
      cudaLaunchConfig_t ca = cfg_of(grid_for(n * Dm), dim3(256), 0, s, attr);
      EFG_TRY_CUDA(cudaLaunchKernelEx(&ca, add_kernel, D.xb, static_cast<const float*>(D.ob), n * Dm), "add launch");
    }
  }
  if (multi) {
    if (D.lm_head.type == 4 || gemm_q8_ok(D.lm_head, D.hb)) {  // final norm of every row, one GEMM
      cudaLaunchConfig_t cn = cfg_of(dim3(nb), dim3(256), 0, s, attr);
      EFG_TRY_CUDA(cudaLaunchKernelEx(&cn, rmsnorm_rows_kernel, D.hb, static_cast<const float*>(D.xb), D.final_norm,
                                      Dm, eps),
                   "rmsnorm launch");
      if (int st = batched_proj(D, D.lm_head, D.hb, D.d_lb, n, s)) return st;
    } else {
      for (size_t b = 0; b < n; ++b)
        if (int st = enqueue_lm_head(D, D.xb + b * Dm, s, D.d_lb + b * V)) return st;
    }
    cudaLaunchConfig_t cf = cfg_of(dim3(nb), dim3(1024), 0, s, attr);
    EFG_TRY_CUDA(cudaLaunchKernelEx(&cf, argmax_rows_kernel, static_cast<const float*>(D.d_lb), V, D.d_next),
                 "argmax launch");
    return EFG_OK;
  }
  if (logits) return enqueue_lm_head(D, D.xb + (n - 1) * Dm, s);
  return EFG_OK;
}

// Positions p0..p0+n-1 in passes of pb_rows tokens; logits of the last token when asked.
int prefill_tokens(Decoder& D, size_t p0, size_t n, bool logits, cudaStream_t s) {
  if (int st = ensure_prefill_buffers(D)) return st;
  for (size_t c0 = 0; c0 < n; c0 += D.pb_rows) {
    const size_t cn = std::min(D.pb_rows, n - c0);
    if (int st = batch_pass(D, p0 + c0, cn, logits && c0 + cn == n, s)) return st;
  }
  return EFG_OK;
}

// Slots 1..n-1 get fresh (zeroed) caches; slot 0 keeps the decoder's own.
int set_slots(Decoder& D, size_t n) {
  if (n < 1 || n > 4096) return fail(EFG_EINVAL, "set_slots: %zu slots (1..4096)", n);
  EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
  drop_step_graphs(D);  // they hold the old slot table
  free_slots(D);
  const size_t bytes = static_cast<size_t>(D.c.layers) * D.max_seq * static_cast<size_t>(D.c.kv_dim()) * sizeof(float);
  for (size_t i = 1; i < n; ++i) {
    float *k = nullptr, *v = nullptr;
    if (cudaMalloc(&k, bytes) != cudaSuccess || cudaMalloc(&v, bytes) != cudaSuccess) {
      if (k) cudaFree(k);
      free_slots(D);
      return fail(EFG_ECUDA, "set_slots: KV-cache allocation for %zu slots", n);
    }
    D.slot_kc.push_back(k);
    D.slot_vc.push_back(v);
    D.slot_cached.push_back(0);
    EFG_TRY_CUDA(cudaMemset(k, 0, bytes), "KV cache init");
    EFG_TRY_CUDA(cudaMemset(v, 0, bytes), "KV cache init");
  }
  D.n_slots = n;
  if (D.d_slot_k) cudaFree(D.d_slot_k);
  if (D.d_slot_v) cudaFree(D.d_slot_v);
  D.d_slot_k = D.d_slot_v = nullptr;
  std::vector<uint64_t> hk(n), hv(n);
  hk[0] = reinterpret_cast<uint64_t>(D.kc);
  hv[0] = reinterpret_cast<uint64_t>(D.vc);
  for (size_t i = 1; i < n; ++i) {
    hk[i] = reinterpret_cast<uint64_t>(D.slot_kc[i - 1]);
    hv[i] = reinterpret_cast<uint64_t>(D.slot_vc[i - 1]);
  }
  EFG_TRY_CUDA(cudaMalloc(&D.d_slot_k, n * sizeof(uint64_t)), "slot table allocation");
  EFG_TRY_CUDA(cudaMalloc(&D.d_slot_v, n * sizeof(uint64_t)), "slot table allocation");
  EFG_TRY_CUDA(cudaMemcpy(D.d_slot_k, hk.data(), n * sizeof(uint64_t), cudaMemcpyHostToDevice), "slot table upload");
  EFG_TRY_CUDA(cudaMemcpy(D.d_slot_v, hv.data(), n * sizeof(uint64_t), cudaMemcpyHostToDevice), "slot table upload");
  return EFG_OK;
}

size_t& slot_cached(Decoder& D, size_t s) { return s == 0 ? D.cached : D.slot_cached[s - 1]; }

// One multi-sequence pass of cn rows (d_rows already uploaded). The first pass of a row count
// runs directly (it also allocates lazily created workspaces), then is recorded as a CUDA
// graph that later steps of the same row count replay: a step is ~20 launches per layer
// plus per-row launches, too many to issue from the host at the GPU's pace.
int step_pass(Decoder& D, size_t cn) {
  auto it = D.step_graphs.find(cn);
  if (it != D.step_graphs.end()) {
    EFG_TRY_CUDA(cudaGraphLaunch(it->second, D.stream), "graph launch");
    return EFG_OK;
  }
  if (int st = batch_pass(D, 0, cn, true, D.stream, true)) return st;
  cudaGraph_t g = nullptr;
  if (cudaStreamBeginCapture(D.stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    return EFG_OK;  // run uncaptured next time as well
  }
  const int st = batch_pass(D, 0, cn, true, D.stream, true);
  const cudaError_t e = cudaStreamEndCapture(D.stream, &g);
  if (st != EFG_OK || e != cudaSuccess || !g) {
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    return EFG_OK;
  }
  cudaGraphExec_t ge = nullptr;
  if (cudaGraphInstantiate(&ge, g, 0) == cudaSuccess) D.step_graphs[cn] = ge;
  cudaGraphDestroy(g);
  cudaGetLastError();
  return EFG_OK;
}

int set_step(Decoder& D, int32_t token, size_t pos, int32_t n_fixed) {
  const int32_t st[2] = {static_cast<int32_t>(pos), n_fixed};
  EFG_TRY_CUDA(cudaMemcpyAsync(D.state, st, sizeof st, cudaMemcpyHostToDevice, D.stream), "state upload");
  EFG_TRY_CUDA(cudaMemcpyAsync(D.tokens() + pos, &token, sizeof token, cudaMemcpyHostToDevice, D.stream),
               "token upload");
  return EFG_OK;
}

}  // namespace
}  // namespace efg

using efg::Decoder;
using efg::fail;

extern "C" {

int efg_efq_check(const void* data, uint64_t size) {
  if (!data && size) return fail(EFG_EINVAL, "efq_check: null data");
  try {
    (void)efg::efq::parse(static_cast<const uint8_t*>(data), size);
  } catch (const efg::efq::FormatError& e) {
    return fail(EFG_EFORMAT, "%s", e.what());
  }
  return EFG_OK;
}

int efg_decoder_open(const char* efq_path, size_t max_seq, efg_decoder** out) {
  Decoder* d = nullptr;
  const int st = efg::open_decoder(efq_path, max_seq, &d);
  if (out) *out = reinterpret_cast<efg_decoder*>(d);
  return st;
}

int efg_decoder_close(efg_decoder* h) {
  efg::destroy(reinterpret_cast<Decoder*>(h));
  return EFG_OK;
}

int efg_decoder_info(const efg_decoder* h, efg_model_info* info) {
  if (!h || !info) return fail(EFG_EINVAL, "decoder_info: null argument");
  const Decoder& D = *reinterpret_cast<const Decoder*>(h);
  info->hidden = static_cast<int32_t>(D.c.hidden);
  info->intermediate = static_cast<int32_t>(D.c.intermediate);
  info->layers = static_cast<int32_t>(D.c.layers);
  info->heads = static_cast<int32_t>(D.c.heads);
  info->kv_heads = static_cast<int32_t>(D.c.kv_heads);
  info->head_dim = static_cast<int32_t>(D.c.head_dim);
  info->vocab = static_cast<int32_t>(D.c.vocab);
  info->max_seq = static_cast<int32_t>(D.max_seq);
  info->n_q4 = D.n_q4;
  info->n_q8 = D.n_q8;
  info->embed_type = D.embed.type;
  info->bytes_per_token = D.bytes_per_token;
  return EFG_OK;
}

int efg_decoder_reset(efg_decoder* h) {
  if (!h) return fail(EFG_EINVAL, "decoder_reset: null handle");
  reinterpret_cast<Decoder*>(h)->cached = 0;
  return EFG_OK;
}

int efg_decoder_forward(efg_decoder* h, int32_t token, size_t pos, float* logits) {
  if (!h) return fail(EFG_EINVAL, "forward: null handle");
  Decoder& D = *reinterpret_cast<Decoder*>(h);
  if (token < 0 || token >= D.c.vocab)
    return fail(EFG_EINVAL, "forward: token id %d is outside [0, %lld)", token, static_cast<long long>(D.c.vocab));
  if (pos >= D.max_seq)
    return fail(EFG_ESTATE, "forward: position %zu exceeds the KV-cache capacity %zu", pos, D.max_seq);
  if (pos > D.cached)
    return fail(EFG_ESTATE, "forward: position %zu skips ahead of the %zu cached tokens", pos, D.cached);
  if (int st = efg::set_step(D, token, pos, static_cast<int32_t>(pos + 1))) return st;
  if (D.use_mk) {
    if (int st = efg::launch_mk(D, logits ? 0 : 1, logits ? 1 : 0, nullptr, -1)) return st;
  } else {
    EFG_TRY_CUDA(cudaGraphLaunch(logits ? D.g_full : D.g_prefill, D.stream), "graph launch");
  }
  if (logits)
    EFG_TRY_CUDA(cudaMemcpyAsync(logits, D.logits, D.c.vocab * sizeof(float), cudaMemcpyDeviceToHost, D.stream),
                 "logits download");
  EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
  if (int st = efg::device_status(D)) return st;
  D.cached = pos + 1;
  return EFG_OK;
}

int efg_decoder_prefill(efg_decoder* h, const int32_t* tokens, size_t n, size_t pos0, float* logits) {
  if (!h || (!tokens && n)) return fail(EFG_EINVAL, "prefill: null argument");
  Decoder& D = *reinterpret_cast<Decoder*>(h);
  if (n == 0) return fail(EFG_EINVAL, "prefill: no tokens");
  if (pos0 > D.cached)
    return fail(EFG_ESTATE, "prefill: position %zu skips ahead of the %zu cached tokens", pos0, D.cached);
  if (pos0 + n > D.max_seq)
    return fail(EFG_ESTATE, "prefill: positions up to %zu exceed the KV-cache capacity %zu", pos0 + n - 1, D.max_seq);
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= D.c.vocab)
      return fail(EFG_EINVAL, "prefill: token id %d is outside [0, %lld)", tokens[i], static_cast<long long>(D.c.vocab));
  EFG_TRY_CUDA(cudaMemcpyAsync(D.tokens() + pos0, tokens, n * sizeof(int32_t), cudaMemcpyHostToDevice, D.stream),
               "token upload");
  if (int st = efg::prefill_tokens(D, pos0, n, logits != nullptr, D.stream)) return st;
  if (logits)
    EFG_TRY_CUDA(cudaMemcpyAsync(logits, D.logits, D.c.vocab * sizeof(float), cudaMemcpyDeviceToHost, D.stream),
                 "logits download");
  EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
  if (int st = efg::device_status(D)) return st;
  D.cached = pos0 + n;
  return EFG_OK;
}

int efg_decoder_generate(efg_decoder* h, const int32_t* prompt, size_t n_prompt, size_t max_new, int32_t eos_id,
                         const int32_t* forced, int32_t* tokens_out, size_t* n_tokens, float* step_logits,
                         double* prefill_seconds, double* decode_seconds) {
  if (!h || !prompt || !tokens_out) return fail(EFG_EINVAL, "generate: null argument");
  Decoder& D = *reinterpret_cast<Decoder*>(h);
  if (n_prompt == 0) return fail(EFG_EINVAL, "generate: empty prompt");
  if (n_prompt + max_new > D.max_seq)
    return fail(EFG_EINVAL, "generate: prompt (%zu) + max_new (%zu) exceeds the KV-cache capacity %zu", n_prompt,
                max_new, D.max_seq);
  for (size_t i = 0; i < n_prompt; ++i)
    if (prompt[i] < 0 || prompt[i] >= D.c.vocab) return fail(EFG_EINVAL, "generate: token id %d out of range", prompt[i]);
  // tokens[]: the prompt, then (teacher forcing) the forced continuation
  const size_t n_fixed = n_prompt + (forced ? max_new : 0);
  std::vector<int32_t> seq(prompt, prompt + n_prompt);
  if (forced) seq.insert(seq.end(), forced, forced + max_new);
  const int32_t st0[2] = {0, static_cast<int32_t>(n_fixed)};
  EFG_TRY_CUDA(cudaMemcpyAsync(D.state, st0, sizeof st0, cudaMemcpyHostToDevice, D.stream), "state upload");
  EFG_TRY_CUDA(cudaMemcpyAsync(D.tokens(), seq.data(), seq.size() * sizeof(int32_t), cudaMemcpyHostToDevice, D.stream),
               "token upload");
  cudaEvent_t e0, e1, e2;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventCreate(&e2);
  if (D.use_mk) {  // two launches of the persistent kernel: the prompt, then the decode loop
    float* keep = nullptr;
    if (step_logits && max_new > 1) {
      const size_t need = (max_new - 1) * static_cast<size_t>(D.c.vocab);
      if (need > D.keep_cap) {
        if (D.d_keep) cudaFree(D.d_keep);
        D.d_keep = nullptr;
        D.keep_cap = 0;
        EFG_TRY_CUDA(cudaMalloc(&D.d_keep, need * sizeof(float)), "logits buffer");
        D.keep_cap = need;
      }
      keep = D.d_keep;
    }
    cudaEventRecord(e0, D.stream);
    if (int st = efg::launch_mk(D, static_cast<uint32_t>(n_prompt - 1), 1, nullptr, eos_id)) return st;
    cudaEventRecord(e1, D.stream);
    int32_t ctl[2] = {0, 0};
    EFG_TRY_CUDA(cudaMemcpyAsync(ctl, efg::mk_ctl(D), sizeof ctl, cudaMemcpyDeviceToHost, D.stream), "state read");
    EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
    if (int st = efg::device_status(D)) return st;
    size_t n_out = max_new ? 1 : 0;
    const bool decode = max_new > 1 && ctl[0] == 0;  // no eos straight after the prompt
    if (decode) {
      if (int st = efg::launch_mk(D, 0, static_cast<uint32_t>(max_new - 1), keep, eos_id)) return st;
      EFG_TRY_CUDA(cudaMemcpyAsync(ctl, efg::mk_ctl(D), sizeof ctl, cudaMemcpyDeviceToHost, D.stream), "state read");
    }
    cudaEventRecord(e2, D.stream);
    EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
    if (int st = efg::device_status(D)) return st;
    if (decode) n_out += static_cast<size_t>(ctl[1]);  // one token per decode step
    if (n_out)
      EFG_TRY_CUDA(cudaMemcpyAsync(tokens_out, D.out_tokens() + n_prompt - 1, n_out * sizeof(int32_t),
                                   cudaMemcpyDeviceToHost, D.stream),
                   "token download");
    if (step_logits && n_out > 1)
      EFG_TRY_CUDA(cudaMemcpyAsync(step_logits, D.d_keep, (n_out - 1) * D.c.vocab * sizeof(float),
                                   cudaMemcpyDeviceToHost, D.stream),
                   "logits download");
    EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
    float ms_pre = 0.f, ms_dec = 0.f;
    cudaEventElapsedTime(&ms_pre, e0, e1);
    cudaEventElapsedTime(&ms_dec, e1, e2);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    if (prefill_seconds) *prefill_seconds = ms_pre / 1e3;
    if (decode_seconds) *decode_seconds = ms_dec / 1e3;
    if (n_tokens) *n_tokens = n_out;
    D.cached = n_prompt + (n_out ? n_out - 1 : 0);
    return EFG_OK;
  }
  cudaEventRecord(e0, D.stream);
  // the prompt as one batch; then the last prompt token's argmax at position n_prompt - 1
  if (int st = efg::prefill_tokens(D, 0, n_prompt, true, D.stream)) return st;
  const int32_t st1[2] = {static_cast<int32_t>(n_prompt - 1), static_cast<int32_t>(n_fixed)};
  EFG_TRY_CUDA(cudaMemcpyAsync(D.state, st1, sizeof st1, cudaMemcpyHostToDevice, D.stream), "state upload");
  if (int st = efg::enqueue_argmax(D, D.stream)) return st;
  cudaEventRecord(e1, D.stream);
  size_t n_out = 0;
  bool stopped = false;
  // generate_greedy (src/model.cpp:278-304): take argmax, stop at eos or max_new, else forward.
  for (size_t step = 0; step < max_new && !stopped; ++step) {
    if (eos_id >= 0) {  // the token decides whether to go on: read it back every step
      int32_t tok = 0;
      EFG_TRY_CUDA(cudaMemcpyAsync(&tok, D.out_tokens() + n_prompt - 1 + step, sizeof tok, cudaMemcpyDeviceToHost,
                                   D.stream),
                   "token download");
      EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
      if (tok == eos_id) stopped = true;
    }
    ++n_out;
    if (stopped || step + 1 == max_new) break;
    EFG_TRY_CUDA(cudaGraphLaunch(D.g_full, D.stream), "graph launch");
    if (step_logits)
      EFG_TRY_CUDA(cudaMemcpyAsync(step_logits + step * D.c.vocab, D.logits, D.c.vocab * sizeof(float),
                                   cudaMemcpyDeviceToHost, D.stream),
                   "logits download");
  }
  cudaEventRecord(e2, D.stream);
  EFG_TRY_CUDA(cudaMemcpyAsync(tokens_out, D.out_tokens() + n_prompt - 1, n_out * sizeof(int32_t),
                               cudaMemcpyDeviceToHost, D.stream),
               "token download");
  EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
  float ms_pre = 0.f, ms_dec = 0.f;
  cudaEventElapsedTime(&ms_pre, e0, e1);
  cudaEventElapsedTime(&ms_dec, e1, e2);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaEventDestroy(e2);
  if (prefill_seconds) *prefill_seconds = ms_pre / 1e3;
  if (decode_seconds) *decode_seconds = ms_dec / 1e3;
  if (n_tokens) *n_tokens = n_out;
  D.cached = n_prompt + (n_out ? n_out - 1 : 0);
  return EFG_OK;
}

int efg_decoder_set_slots(efg_decoder* h, size_t n_slots) {
  if (!h) return fail(EFG_EINVAL, "set_slots: null handle");
  return efg::set_slots(*reinterpret_cast<Decoder*>(h), n_slots);
}

int efg_decoder_step_slots(efg_decoder* h, const int32_t* slots, const int32_t* tokens, const int32_t* positions,
                           size_t n, float* logits, int32_t* next_tokens) {
  if (!h || !slots || !tokens || !positions) return fail(EFG_EINVAL, "step_slots: null argument");
  Decoder& D = *reinterpret_cast<Decoder*>(h);
  if (n == 0) return fail(EFG_EINVAL, "step_slots: no rows");
  std::vector<char> seen(D.n_slots, 0);
  for (size_t b = 0; b < n; ++b) {
    if (slots[b] < 0 || static_cast<size_t>(slots[b]) >= D.n_slots)
      return fail(EFG_EINVAL, "step_slots: slot %d is outside [0, %zu)", slots[b], D.n_slots);
    if (seen[slots[b]]++) return fail(EFG_EINVAL, "step_slots: slot %d appears twice in one step", slots[b]);
    if (tokens[b] < 0 || tokens[b] >= D.c.vocab)
      return fail(EFG_EINVAL, "step_slots: token id %d is outside [0, %lld)", tokens[b],
                  static_cast<long long>(D.c.vocab));
    const size_t pos = static_cast<size_t>(positions[b]);
    if (positions[b] < 0 || pos >= D.max_seq)
      return fail(EFG_ESTATE, "step_slots: position %d exceeds the KV-cache capacity %zu", positions[b], D.max_seq);
    if (pos > efg::slot_cached(D, slots[b]))
      return fail(EFG_ESTATE, "step_slots: position %zu skips ahead of the %zu cached tokens of slot %d", pos,
                  efg::slot_cached(D, slots[b]), slots[b]);
  }
  if (int st = efg::ensure_prefill_buffers(D)) return st;
  if (!D.d_rows) {
    EFG_TRY_CUDA(cudaMalloc(&D.d_rows, 3 * D.pb_rows * sizeof(int32_t)), "step buffer allocation");
    EFG_TRY_CUDA(cudaMalloc(&D.d_lb, D.pb_rows * D.c.vocab * sizeof(float)), "step buffer allocation");
    EFG_TRY_CUDA(cudaMalloc(&D.d_next, D.pb_rows * sizeof(int32_t)), "step buffer allocation");
  }
  if (D.n_slots == 1 && !D.d_slot_k)
    if (int st = efg::set_slots(D, 1)) return st;
  for (size_t c0 = 0; c0 < n; c0 += D.pb_rows) {
    const size_t cn = std::min(D.pb_rows, n - c0);
    std::vector<int32_t> rows(3 * D.pb_rows, 0);
    for (size_t b = 0; b < cn; ++b) {
      rows[b] = tokens[c0 + b];
      rows[D.pb_rows + b] = slots[c0 + b];
      rows[2 * D.pb_rows + b] = positions[c0 + b];
    }
    EFG_TRY_CUDA(cudaMemcpyAsync(D.d_rows, rows.data(), rows.size() * sizeof(int32_t), cudaMemcpyHostToDevice, D.stream),
                 "row upload");
    if (int st = efg::step_pass(D, cn)) return st;
    if (logits)
      EFG_TRY_CUDA(cudaMemcpyAsync(logits + c0 * D.c.vocab, D.d_lb, cn * D.c.vocab * sizeof(float),
                                   cudaMemcpyDeviceToHost, D.stream),
                   "logits download");
    if (next_tokens)
      EFG_TRY_CUDA(cudaMemcpyAsync(next_tokens + c0, D.d_next, cn * sizeof(int32_t), cudaMemcpyDeviceToHost, D.stream),
                   "token download");
    EFG_TRY_CUDA(cudaStreamSynchronize(D.stream), "stream synchronize");
  }
  if (int st = efg::device_status(D)) return st;
  for (size_t b = 0; b < n; ++b) efg::slot_cached(D, slots[b]) = static_cast<size_t>(positions[b]) + 1;
  return EFG_OK;
}

int efg_decoder_set_mode(efg_decoder* h, int persistent) {
  if (!h) return fail(EFG_EINVAL, "decoder_set_mode: null handle");
  Decoder& D = *reinterpret_cast<Decoder*>(h);
  if (persistent && !D.mk_ok)
    return fail(EFG_EINVAL, "decoder_set_mode: the persistent kernel cannot run this model (%s)", D.mk_why.c_str());
  D.use_mk = persistent != 0;
  return EFG_OK;
}

int efg_decoder_mode(const efg_decoder* h) {
  if (!h) return -1;
  return reinterpret_cast<const Decoder*>(h)->use_mk ? 1 : 0;
}

}  // extern "C"
