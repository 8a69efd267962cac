// efg_decode_mk.cuh - the decode step as ONE persistent kernel (included by efg_decode.cu).
//
// One CTA per SM, launched cooperatively so every CTA is resident. A token is a fixed list
// of phases (embed; per layer q/k/v, attention, o_proj, gate/up, down; lm_head, argmax)
// separated by grid barriers. Inside each CTA:
//   * the producer warp streams the CTA's share of every matrix phase after phase, token
//     after token, through a ring of shared-memory slots (1-D bulk copies completing on
//     the slot's "full" mbarrier). Weights never depend on activations, so the stream
//     runs ahead of the consumers and across the grid barriers;
//   * 15 consumer warps run the phases. A matrix phase stages its input vector (with the
//     RMSNorm folded in), then each row group (G warps covering the row's 64-column slots)
//     takes every RG-th tile of the phase, computes the rows with the standalone matvec's
//     per-lane dot products and writes Store / Add / SwiGLU outputs, freeing the slot
//     through its "empty" mbarrier. SwiGLU is applied while the down projection stages
//     its input (silu(gate) * up), so gate and up may have different storage types.
// A slot's tile sequence number is published next to its mbarrier, so a consumer that
// runs ahead of the ring never takes a phase of the wrong generation for its own.
// Activations written in one phase are read in the next through L2 (ld.global.cg) after
// the grid barrier (release/acquire at gpu scope). Every wait is bounded: a timeout
// records EFG_ETIMEOUT and the whole grid winds down through the same checks.
#pragma once

#include <cstdint>

#include "efg_device.cuh"
#include "efg_dot.cuh"

namespace efg {
namespace mk {

constexpr int kWarps = 16;  // 15 consumer warps + the producer warp
constexpr int kConsumerWarps = 15;
constexpr int kThreads = kWarps * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr uint32_t kSlotBytes = 18432;
constexpr uint32_t kSlots = 10;
constexpr uint32_t kMaxSlotsX = 96;  // 64-column slots of an input vector (cols <= 6144)
constexpr uint32_t kXsFloats = kMaxSlotsX * 65;
constexpr int kAllConsumersBarrier = 1;  // named barrier ids: 1 all consumers, 2.. row groups
constexpr uint32_t kMaxBatches = 4;      // batches (RB rows each) per tile: the empty barrier's count
constexpr uint32_t kAttnChunk = 32;      // cached positions staged in shared memory at a time
// Copies a producer keeps in flight (issued, not landed). Landed tiles may fill the whole
// ring ahead of the consumers, but the memory system is kept shallow: with ~26 MB of
// requests queued GPU-wide, every L2 access on the critical path (barrier, activations)
// would wait microseconds behind the weight stream.
#ifndef EFG_MK_OUTSTANDING
#define EFG_MK_OUTSTANDING 3
#endif
constexpr uint32_t kOutstanding = EFG_MK_OUTSTANDING;

enum Kind : uint32_t { kEmbed = 0, kMatvec = 1, kAttn = 2, kArgmax = 3 };

struct Job {
  const uint8_t* W;
  float* y;
  uint32_t rows, rb;       // rows, bytes per row (a multiple of 16)
  uint32_t y_pos_stride;   // y += pos * stride (v written into the KV cache); y null: the logits
  uint32_t fmt, RB, TR;    // format (3 Q8_0 / 4 Q4_0), rows per batch, rows per tile (per matrix)
};

enum InMode : uint32_t { kInPlain = 0, kInNorm = 1, kInSwiGLU = 2 };

struct Phase {
  uint32_t kind, epi, n_jobs, G, cols, layer, in_mode;
  const float* x;       // matvec input (SwiGLU: the gate vector)
  const float* x2;      // SwiGLU: the up vector
  const float* norm_w;  // RMSNorm weights
  Job jobs[3];
};

// The phases of one token. A step with logits runs them all; a prompt step without
// logits runs all but the last two (lm_head, argmax) and then advances the position.
constexpr uint32_t kMaxPhases = 116;

struct Params {
  const Phase* phases;
  uint32_t n_phases, n_prefill_steps, n_full_steps;
  const uint8_t* embed;
  int embed_type;
  uint32_t vocab, dim, H, KV, hd, max_seq;
  float* kc;
  float* vc;
  const float* rcos;
  const float* rsin;
  float* q;
  float* knew;
  float* ctx;
  float* x;
  float* logits;  // argmax input; + step * vocab when kept per step
  uint32_t logits_step_stride;
  float eps;
  int32_t* pos;
  const int32_t* n_fixed;
  int32_t* tokens;
  int32_t* out_tokens;
  int32_t eos;
  int32_t* ctl;  // [0] stop (eos seen), [1] full steps done
  unsigned* bar;
  int* err;
};

// ---------------------------------------------------------------- small helpers

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ int32_t ldcg_i(const int32_t* p) { return __ldcg(p); }

__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t chunk_begin(uint32_t n, uint32_t parts, uint32_t i) {
  return static_cast<uint32_t>(static_cast<uint64_t>(n) * i / parts);
}

// Calls fn(job, r0, nrows) for the tiles this CTA owns in a matrix phase, in the order
// both the producer and the consumers walk them: job by job, TR rows at a time, over the
// contiguous row range rows * cta / grid .. rows * (cta + 1) / grid of each job.
template <class F>
__device__ __forceinline__ void for_each_tile(const Phase& P, uint32_t cta, uint32_t grid, F&& fn) {
  for (uint32_t j = 0; j < P.n_jobs; ++j) {
    const Job& J = P.jobs[j];
    const uint32_t b = chunk_begin(J.rows, grid, cta), e = chunk_begin(J.rows, grid, cta + 1);
    for (uint32_t r0 = b; r0 < e; r0 += J.TR) fn(j, r0, min(J.TR, e - r0));
  }
}

// Bounded wait for the slot to carry tile `gt` (its sequence number), then for its bytes.
__device__ __forceinline__ bool wait_tile(volatile uint32_t* tile_id, uint64_t* full, uint32_t gt, int* err) {
  const uint32_t s = gt % kSlots;
  if (tile_id[s] != gt) {
    const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
    for (uint32_t i = 0; tile_id[s] != gt; ++i) {
      if ((i & 63u) == 63u) {
        if (error_raised(err)) return false;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
          record_error(err, EFG_ETIMEOUT);
          return false;
        }
      }
    }
  }
  return mbar_wait(&full[s], (gt / kSlots) & 1u, err);
}

__device__ __forceinline__ void mbar_arrive_n(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(n) : "memory");
}

// All CTAs: a CTA arrives once its consumers are done with the phase; consumers of every
// CTA continue when all have arrived. `k` counts this launch's barriers (the counter is
// zeroed before the launch). Bounded; false on timeout or once any wait of the grid has
// recorded an error. The result is the same for every consumer thread of the CTA, and it
// alone steers the consumers' loops, so their named barriers always match.
__device__ __forceinline__ bool grid_sync(const Params& p, uint32_t k) {
  named_barrier(kAllConsumersBarrier, kConsumerThreads);
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    int ok = 1;
    __threadfence();
    atomicAdd(p.bar, 1u);
    const uint32_t target = (k + 1) * gridDim.x;
    const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
    for (uint32_t i = 0; ld_acquire_gpu(p.bar) < target; ++i) {
      __nanosleep(20);
      if ((i & 15u) == 15u) {
        if (error_raised(p.err)) {
          ok = 0;
          break;
        }
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
          record_error(p.err, EFG_ETIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
    if (error_raised(p.err)) ok = 0;  // any failure anywhere ends the launch on every CTA
    ok_s = ok;
  }
  named_barrier(kAllConsumersBarrier, kConsumerThreads);
  return ok_s != 0;
}

// ---------------------------------------------------------------- phases

// x = row tokens[pos] of the embedding table (src/qkernels.cpp:299-305); this CTA writes
// its share of the columns.
__device__ __noinline__ void phase_embed(const Params& p) {
  const int32_t pos = ldcg_i(p.pos);
  const int32_t tok = ldcg_i(p.tokens + pos);
  if (tok < 0 || static_cast<uint32_t>(tok) >= p.vocab) {
    if (threadIdx.x == 0) record_error(p.err, EFG_EINVAL);
    return;
  }
  const int type = p.embed_type;
  const uint32_t dim = p.dim;
  const uint64_t rb = type == 0 ? 4ull * dim : type <= 2 ? 2ull * dim : dim / 32ull * (type == 3 ? 34 : 18);
  const uint8_t* row = p.embed + static_cast<uint64_t>(tok) * rb;
  const uint32_t b = chunk_begin(dim, gridDim.x, blockIdx.x), e = chunk_begin(dim, gridDim.x, blockIdx.x + 1);
  for (uint32_t i = b + threadIdx.x; i < e; i += kConsumerThreads) {
    float v;
    if (type == 2) {
      v = bf16_to_f32(row[2 * i] | (row[2 * i + 1] << 8));
    } else if (type == 1) {
      v = fp16_to_f32(row[2 * i] | (row[2 * i + 1] << 8));
    } else if (type == 0) {
      v = __uint_as_float(row[4 * i] | (row[4 * i + 1] << 8) | (row[4 * i + 2] << 16) |
                          (static_cast<uint32_t>(row[4 * i + 3]) << 24));
    } else {
      const uint8_t* blk = row + (i / 32) * (type == 3 ? 34 : 18);
      const int j = i % 32;
      const float d = fp16_to_f32(blk[0] | (blk[1] << 8));
      const int code = type == 4 ? (j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4)) - 8
                                 : static_cast<int8_t>(blk[2 + j]);
      v = __fmul_rn(static_cast<float>(code), d);
    }
    p.x[i] = v;
  }
}

// One query head per CTA (src/kernels.cpp:133-174), as the standalone attention kernel:
// RoPE of q and of the new key, the key written to the cache by the first head of its
// group, scores / sqrt(hd) with 8 partial sums, softmax with a double sum, then the
// probability-weighted sum of the values in position order. Cached keys and values come
// through shared memory kAttnChunk positions at a time (all loads of a chunk in flight at
// once); the arithmetic and its order are the standalone kernel's.
__device__ __noinline__ void phase_attention(const Params& p, uint32_t layer, float* scratch) {
  const uint32_t h = blockIdx.x;
  if (h >= p.H) return;
  const int pos = ldcg_i(p.pos);
  if (pos < 0 || pos >= static_cast<int>(p.max_seq)) {
    if (threadIdx.x == 0) record_error(p.err, EFG_ESTATE);
    return;
  }
  const uint32_t hd = p.hd, half = hd / 2, kvd = p.KV * hd, group = p.H / p.KV, kv = h / group;
  float* qh = scratch;
  float* kn = qh + hd;
  float* sc = kn + hd;                 // [max_seq]
  float* ch = sc + p.max_seq;          // [kAttnChunk][hd]
  __shared__ float red_f[kConsumerWarps];
  __shared__ double red_d[kConsumerWarps];
  const uint32_t tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  float* k_layer = p.kc + static_cast<size_t>(layer) * p.max_seq * kvd;
  const float* v_layer = p.vc + static_cast<size_t>(layer) * p.max_seq * kvd;
  const float* c = p.rcos + static_cast<size_t>(pos) * half;
  const float* s = p.rsin + static_cast<size_t>(pos) * half;
  for (uint32_t i = tid; i < half; i += kConsumerThreads) {
    const float a = ldcg(p.q + h * hd + i), b = ldcg(p.q + h * hd + i + half);
    qh[i] = __fsub_rn(__fmul_rn(a, c[i]), __fmul_rn(b, s[i]));
    qh[i + half] = __fadd_rn(__fmul_rn(b, c[i]), __fmul_rn(a, s[i]));
    const float ka = ldcg(p.knew + kv * hd + i), kb = ldcg(p.knew + kv * hd + i + half);
    kn[i] = __fsub_rn(__fmul_rn(ka, c[i]), __fmul_rn(kb, s[i]));
    kn[i + half] = __fadd_rn(__fmul_rn(kb, c[i]), __fmul_rn(ka, s[i]));
  }
  named_barrier(kAllConsumersBarrier, kConsumerThreads);
  if (h % group == 0)
    for (uint32_t i = tid; i < hd; i += kConsumerThreads) k_layer[static_cast<size_t>(pos) * kvd + kv * hd + i] = kn[i];
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(hd)));
  const int n_pos = pos + 1;
  float mx = -INFINITY;
#pragma unroll 1
  for (int t0 = 0; t0 < n_pos; t0 += kAttnChunk) {
    const int nt = min(static_cast<int>(kAttnChunk), n_pos - t0);
    for (uint32_t e = tid; e < static_cast<uint32_t>(nt) * hd; e += kConsumerThreads) {
      const int t = t0 + static_cast<int>(e / hd);
      ch[e] = t == pos ? kn[e % hd] : ldcg(k_layer + static_cast<size_t>(t) * kvd + kv * hd + e % hd);
    }
    named_barrier(kAllConsumersBarrier, kConsumerThreads);
    if (tid < static_cast<uint32_t>(nt)) {
      const float* kt = ch + tid * hd;
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t i = 0;
#pragma unroll 1
      for (; i + 8 <= hd; i += 8)
#pragma unroll
        for (int q = 0; q < 8; ++q) a[q] = __fadd_rn(a[q], __fmul_rn(qh[i + q], kt[i + q]));
      for (; i < hd; ++i) a[0] = __fadd_rn(a[0], __fmul_rn(qh[i], kt[i]));
      const float dot = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                                  __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
      sc[t0 + tid] = __fmul_rn(dot, scale);
      mx = fmaxf(mx, sc[t0 + tid]);
    }
    named_barrier(kAllConsumersBarrier, kConsumerThreads);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  if (lane == 0) red_f[wid] = mx;
  named_barrier(kAllConsumersBarrier, kConsumerThreads);
  mx = red_f[0];
  for (int w = 1; w < kConsumerWarps; ++w) mx = fmaxf(mx, red_f[w]);
  double sum = 0.0;
#pragma unroll 1
  for (int t = tid; t < n_pos; t += kConsumerThreads) {
    const float e = expf(__fsub_rn(sc[t], mx));
    sc[t] = e;
    sum += static_cast<double>(e);
  }
  sum = warp_sum_d(sum);
  if (lane == 0) red_d[wid] = sum;
  named_barrier(kAllConsumersBarrier, kConsumerThreads);
  double tot = 0.0;
  for (int w = 0; w < kConsumerWarps; ++w) tot += red_d[w];
  const float inv = static_cast<float>(1.0 / tot);
#pragma unroll 1
  for (int t = tid; t < n_pos; t += kConsumerThreads) sc[t] = __fmul_rn(sc[t], inv);
  float acc = 0.f;  // thread d < hd: output d, summed over positions in order
#pragma unroll 1
  for (int t0 = 0; t0 < n_pos; t0 += kAttnChunk) {
    const int nt = min(static_cast<int>(kAttnChunk), n_pos - t0);
    named_barrier(kAllConsumersBarrier, kConsumerThreads);  // sc final / previous chunk consumed
    for (uint32_t e = tid; e < static_cast<uint32_t>(nt) * hd; e += kConsumerThreads)
      ch[e] = ldcg(v_layer + static_cast<size_t>(t0 + e / hd) * kvd + kv * hd + e % hd);
    named_barrier(kAllConsumersBarrier, kConsumerThreads);
    if (tid < hd)
#pragma unroll 1
      for (int t = 0; t < nt; ++t) acc = __fadd_rn(acc, __fmul_rn(sc[t0 + t], ch[t * hd + tid]));
  }
  if (tid < hd) p.ctx[h * hd + tid] = acc;
}

// First maximum of the logits (src/kernels.cpp:105-111) on CTA 0, then the state update
// of generate_greedy: record it, make it the next token unless that token is given,
// advance the position, count the step, stop at eos.
__device__ __noinline__ void phase_argmax(const Params& p, uint32_t step_k) {
  if (blockIdx.x != 0) return;
  __shared__ float bv[kConsumerWarps];
  __shared__ uint32_t bi[kConsumerWarps];
  const float* logits = p.logits + static_cast<size_t>(step_k) * p.logits_step_stride;
  const uint32_t n = p.vocab, tid = threadIdx.x;
  float best = -INFINITY;
  uint32_t idx = 0xFFFFFFFFu;
#pragma unroll 1
  for (uint32_t i0 = tid; i0 < n; i0 += 4 * kConsumerThreads) {  // 4 loads in flight per thread
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t i = i0 + u * kConsumerThreads;
      v[u] = i < n ? ldcg(logits + i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t i = i0 + u * kConsumerThreads;
      if (i < n && (idx == 0xFFFFFFFFu ? !(v[u] != v[u]) : v[u] > best)) {
        best = v[u];
        idx = i;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
    if (oi != 0xFFFFFFFFu && (idx == 0xFFFFFFFFu || ov > best || (ov == best && oi < idx))) {
      best = ov;
      idx = oi;
    }
  }
  if ((tid & 31) == 0) {
    bv[tid >> 5] = best;
    bi[tid >> 5] = idx;
  }
  named_barrier(kAllConsumersBarrier, kConsumerThreads);
  if (tid == 0) {
    best = bv[0];
    idx = bi[0];
    for (int w = 1; w < kConsumerWarps; ++w)
      if (bi[w] != 0xFFFFFFFFu && (idx == 0xFFFFFFFFu || bv[w] > best || (bv[w] == best && bi[w] < idx))) {
        best = bv[w];
        idx = bi[w];
      }
    // a NaN at index 0 is never replaced by the reference's strict comparison
    const float first = ldcg(logits);
    if (first != first || idx == 0xFFFFFFFFu) idx = 0;
    const int32_t pos = ldcg_i(p.pos);
    p.out_tokens[pos] = static_cast<int32_t>(idx);
    if (pos + 1 < static_cast<int32_t>(p.max_seq) && pos + 1 >= ldcg_i(p.n_fixed)) p.tokens[pos + 1] = static_cast<int32_t>(idx);
    p.pos[0] = pos + 1;
    p.ctl[1] += 1;
    if (p.eos >= 0 && static_cast<int32_t>(idx) == p.eos) p.ctl[0] = 1;
  }
}

// ---------------------------------------------------------------- matrix phases

struct MvShared {
  float* xs;        // staged input [S][65]
  float* red;       // row-group partial sums [RG][2][4][3]
  double* dred;     // [16]
  uint8_t* ring;
  uint64_t* full;
  uint64_t* empty;
  volatile uint32_t* tile_id;
};

template <Fmt F>
__device__ __forceinline__ void load_xp(const float* xs, uint32_t slot, bool active, float2 (&xp)[32]) {
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    float lo = 0.f, hi = 0.f;
    if (active) {
      const float* xr = xs + slot * 65 + pair_col<F>(k);
      lo = xr[0];
      hi = xr[pair_step<F>()];
    }
    xp[k] = f2(lo, hi);
  }
}

// One batch (RB rows) of a tile by one row group; the G warps of the group combine their
// slots' partial dots through shared memory. The slot is free once every batch of its tile
// has arrived on its "empty" mbarrier (kMaxBatches arrivals: the tile's last batch makes up
// for batches a short tile does not have).
template <Fmt F, int RB>
__device__ __forceinline__ void mv_batch(const Params& p, const Job& J, const MvShared& sh, uint32_t gt, uint32_t r0,
                                         uint32_t nrows, uint32_t b, const float2 (&xp)[32], uint32_t g, uint32_t G,
                                         uint32_t rg, uint32_t slot, bool active, uint32_t lane, float* y, bool add,
                                         uint32_t& buf) {
  const bool ok = wait_tile(sh.tile_id, sh.full, gt, p.err);
  const uint32_t s = gt % kSlots;
  const uint32_t sbase = smem_addr(sh.ring) + s * kSlotBytes + slot * slot_words<F>() * 4u;
  const uint32_t nb = (nrows + RB - 1) / RB;
  const uint32_t arrivals = b + 1 == nb ? kMaxBatches - nb + 1 : 1;
  float acc[RB];
  uint32_t addr[RB];
  bool valid[RB];
#pragma unroll
  for (int i = 0; i < RB; ++i) {
    const uint32_t lr = b * RB + i;
    addr[i] = sbase + lr * J.rb;
    valid[i] = ok && active && lr < nrows;
  }
  slot_dots<F, RB>(addr, valid, xp, acc);
  if (G == 1) {
    __syncwarp();
    if (ok && lane == 0) mbar_arrive_n(&sh.empty[s], arrivals);
  }
  const float v = warp_reduce_rows<RB>(acc, lane);
  const float mine = __shfl_sync(0xFFFFFFFFu, v, (lane % RB) * (32 / RB));
  float total = mine;
  bool writer = lane < static_cast<uint32_t>(RB);
  if (G > 1) {
    float* rbuf = sh.red + rg * 2 * 4 * 3 + buf * 4 * 3;
    if (lane < static_cast<uint32_t>(RB)) rbuf[lane * G + g] = mine;
    named_barrier(2 + rg, G * 32);
    if (g == 0 && ok && lane == 0) mbar_arrive_n(&sh.empty[s], arrivals);  // the group is past its reads
    writer = writer && g == 0;
    if (writer) {
      total = 0.f;
      for (uint32_t q = 0; q < G; ++q) total += rbuf[lane * G + q];
    }
    buf ^= 1u;
  }
  const uint32_t lr = b * RB + lane;
  if (ok && writer && lr < nrows) y[r0 + lr] = add ? ldcg(y + r0 + lr) + total : total;
}

// This row group's batches of one job: the x pairs of the lane's slot are loaded into
// registers once, then each batch (gt: the tile's sequence number, k: the phase's batch
// counter) with mine % RG == rg is computed. Separate function: its registers are not
// shared with the phase's staging. Returns the group's reduction buffer toggle.
template <Fmt F, int RB>
__device__ __noinline__ uint32_t mv_job(const Params& p, const Job& J, const MvShared& sh, uint32_t gt, uint32_t k,
                                        uint32_t G, uint32_t RG, uint32_t g, uint32_t rg, uint32_t slot, bool active,
                                        uint32_t lane, float* y, bool add, uint32_t buf) {
  float2 xp[32];
  load_xp<F>(sh.xs, slot, active, xp);
  const uint32_t b0 = chunk_begin(J.rows, gridDim.x, blockIdx.x), e0 = chunk_begin(J.rows, gridDim.x, blockIdx.x + 1);
#pragma unroll 1
  for (uint32_t r0 = b0; r0 < e0; r0 += J.TR, ++gt) {
    const uint32_t nrows = min(J.TR, e0 - r0);
    const uint32_t nb = (nrows + RB - 1) / RB;
#pragma unroll 1
    for (uint32_t b = 0; b < nb; ++b, ++k)
      if (k % RG == rg) mv_batch<F, RB>(p, J, sh, gt, r0, nrows, b, xp, g, G, rg, slot, active, lane, y, add, buf);
  }
  return buf;
}

// silu(g) * u (src/kernels.cpp:94-99) of four pairs; out of line so the exp and the IEEE
// division are not repeated in the phase's code.
__device__ __noinline__ float4 swiglu4(float4 g, float4 u) {
  float4 r;
  r.x = swiglu_value(g.x, u.x);
  r.y = swiglu_value(g.y, u.y);
  r.z = swiglu_value(g.z, u.z);
  r.w = swiglu_value(g.w, u.w);
  return r;
}

// A matrix phase on the consumers: stage the input (with RMSNorm), then this row group's
// share of the CTA's tiles. Returns false after a failed wait.
__device__ __noinline__ bool phase_matvec(const Params& p, const Phase& P, const MvShared& sh, uint32_t gt_base, uint32_t step_k) {
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t cols = P.cols;
  // Input staging, cols a multiple of 64: every thread issues all its float4 loads (x, and
  // the norm weights or the up vector) before using any, so the phase pays one L2 round trip.
  constexpr uint32_t kMaxV = (kMaxSlotsX * 64 / 4 + kConsumerThreads - 1) / kConsumerThreads;  // float4 per thread
  const uint32_t nv = cols / 4;
  float4 xv[kMaxV], wv[kMaxV];
#pragma unroll
  for (uint32_t u = 0; u < kMaxV; ++u) {
    const uint32_t v = tid + u * kConsumerThreads;
    if (v < nv) {
      xv[u] = __ldcg(reinterpret_cast<const float4*>(P.x) + v);
      if (P.in_mode == kInSwiGLU) wv[u] = __ldcg(reinterpret_cast<const float4*>(P.x2) + v);
      else if (P.in_mode == kInNorm) wv[u] = __ldg(reinterpret_cast<const float4*>(P.norm_w) + v);
    }
  }
  if (P.in_mode == kInSwiGLU) {  // silu(gate) * up (src/kernels.cpp:94-99)
#pragma unroll
    for (uint32_t u = 0; u < kMaxV; ++u) xv[u] = swiglu4(xv[u], wv[u]);
  }
  if (P.in_mode == kInNorm) {  // rmsnorm (src/kernels.cpp:69-75): double sum of squares, w * (x * inv)
    double ss = 0.0;
#pragma unroll
    for (uint32_t u = 0; u < kMaxV; ++u)
      if (tid + u * kConsumerThreads < nv) {
        const double a = xv[u].x, b = xv[u].y, c = xv[u].z, d = xv[u].w;
        ss += a * a + b * b + c * c + d * d;
      }
    ss = warp_sum_d(ss);
    if (lane == 0) sh.dred[warp] = ss;
    named_barrier(kAllConsumersBarrier, kConsumerThreads);
    double tot = 0.0;
    for (int w = 0; w < kConsumerWarps; ++w) tot += sh.dred[w];
    const double mean = cols ? tot / static_cast<double>(cols) : 0.0;
    const float inv = static_cast<float>(1.0 / sqrt(mean + static_cast<double>(p.eps)));
#pragma unroll
    for (uint32_t u = 0; u < kMaxV; ++u) {
      xv[u].x = wv[u].x * (xv[u].x * inv);
      xv[u].y = wv[u].y * (xv[u].y * inv);
      xv[u].z = wv[u].z * (xv[u].z * inv);
      xv[u].w = wv[u].w * (xv[u].w * inv);
    }
  }
#pragma unroll
  for (uint32_t u = 0; u < kMaxV; ++u) {
    const uint32_t v = tid + u * kConsumerThreads;
    if (v < nv) {
      const uint32_t i = 4 * v;
      float* d = sh.xs + (i >> 6) * 65 + (i & 63);
      d[0] = xv[u].x;
      d[1] = xv[u].y;
      d[2] = xv[u].z;
      d[3] = xv[u].w;
    }
  }
  named_barrier(kAllConsumersBarrier, kConsumerThreads);
  const uint32_t G = P.G, RG = kConsumerWarps / G;
  const uint32_t g = warp % G, rg = warp / G;
  const uint32_t slot = g * 32 + lane;
  const bool active = slot < cols / 64;
  const int32_t pos = ldcg_i(p.pos);
  // work unit = one batch of one tile; batch k of the phase goes to row group k % RG
  uint32_t gt = gt_base, k = 0, buf = 0;
  for (uint32_t j = 0; j < P.n_jobs; ++j) {
    const Job& J = P.jobs[j];
    // the lm_head job writes the launch's logits buffer (one row per step when kept)
    float* y = J.y ? J.y + static_cast<size_t>(pos) * J.y_pos_stride
                   : p.logits + static_cast<size_t>(step_k) * p.logits_step_stride;
    const bool add = P.epi == static_cast<uint32_t>(Epi::Add);
    if (rg < RG) {
      if (J.fmt == static_cast<uint32_t>(Fmt::Q4))  // batches of 2 rows (mk_job)
        buf = mv_job<Fmt::Q4, 2>(p, J, sh, gt, k, G, RG, g, rg, slot, active, lane, y, add, buf);
      else
        buf = mv_job<Fmt::Q8, 2>(p, J, sh, gt, k, G, RG, g, rg, slot, active, lane, y, add, buf);
    }
    const uint32_t b0 = chunk_begin(J.rows, gridDim.x, blockIdx.x), e0 = chunk_begin(J.rows, gridDim.x, blockIdx.x + 1);
    for (uint32_t r0 = b0; r0 < e0; r0 += J.TR) {
      ++gt;
      k += (min(J.TR, e0 - r0) + J.RB - 1) / J.RB;
    }
  }
  return true;
}

__device__ __forceinline__ uint32_t phase_tiles(const Phase& P) {
  uint32_t n = 0;
  if (P.kind == kMatvec) for_each_tile(P, blockIdx.x, gridDim.x, [&](uint32_t, uint32_t, uint32_t) { ++n; });
  return n;
}

// ---------------------------------------------------------------- the kernel

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  MvShared sh;
  sh.ring = smem;
  sh.full = reinterpret_cast<uint64_t*>(smem + kSlots * kSlotBytes);
  sh.empty = sh.full + kSlots;
  sh.dred = reinterpret_cast<double*>(sh.empty + kSlots);                  // 16 doubles
  sh.tile_id = reinterpret_cast<volatile uint32_t*>(sh.dred + 16);         // kSlots
  volatile uint32_t* done = sh.tile_id + kSlots;                           // consumers finished
  sh.red = const_cast<float*>(reinterpret_cast<volatile float*>(done + 2));  // up to 7 groups x 2 x 4 x 3
  sh.xs = sh.red + 192;                                                    // kXsFloats
  Phase* phases = reinterpret_cast<Phase*>(sh.xs + kXsFloats);             // the token's phase list
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {  // the phase list, once per launch: every later read of it is a shared-memory read
    const uint4* src = reinterpret_cast<const uint4*>(p.phases);
    uint4* dst = reinterpret_cast<uint4*>(phases);
    for (uint32_t i = threadIdx.x; i < p.n_phases * sizeof(Phase) / 16; i += kThreads) dst[i] = __ldg(src + i);
  }
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kSlots; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], kMaxBatches);
      sh.tile_id[s] = 0xFFFFFFFFu;
    }
    *done = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const uint32_t steps = p.n_prefill_steps + p.n_full_steps;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    const uint64_t pol = l2_evict_first_policy();
    uint32_t gt = 0;
    bool ok = true;
    for (uint32_t st = 0; st < steps && ok; ++st) {
      const uint32_t np = st < p.n_prefill_steps ? p.n_phases - 2 : p.n_phases;
      for (uint32_t pi = 0; pi < np && ok; ++pi) {
        const Phase& P = phases[pi];
        if (P.kind != kMatvec) continue;
        for_each_tile(P, blockIdx.x, gridDim.x, [&](uint32_t j, uint32_t r0, uint32_t nrows) {
          if (!ok) return;
          const uint32_t s = gt % kSlots, gen = gt / kSlots;
          if (gen > 0) {  // the slot's previous tile must have been consumed
            const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
            for (uint32_t i = 0; !mbar_try_wait(&sh.empty[s], (gen - 1) & 1u); ++i) {
              if ((i & 63u) == 63u) {
                if (*done || error_raised(p.err)) {
                  ok = false;
                  return;
                }
                if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                  record_error(p.err, EFG_ETIMEOUT);
                  ok = false;
                  return;
                }
              }
            }
          }
          if (gt >= kOutstanding) {  // tile gt - kOutstanding has landed
            const uint32_t q = gt - kOutstanding;
            const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
            for (uint32_t i = 0; !mbar_try_wait(&sh.full[q % kSlots], (q / kSlots) & 1u); ++i) {
              if ((i & 63u) == 63u && globaltimer_ns() - t0 > kWaitTimeoutNs) {
                record_error(p.err, EFG_ETIMEOUT);
                ok = false;
                return;
              }
            }
          }
          sh.tile_id[s] = gt;
          const Job& J = P.jobs[j];
          const uint32_t bytes = nrows * J.rb;
          mbar_arrive_expect_tx(&sh.full[s], bytes);
          bulk_g2s(sh.ring + s * kSlotBytes, J.W + static_cast<size_t>(r0) * J.rb, bytes, &sh.full[s], pol);
          ++gt;
        });
      }
    }
    // copies still in flight land before the CTA may exit (bounded)
    const uint32_t first = gt > kSlots ? gt - kSlots : 0;
    for (uint32_t q = first; q < gt; ++q) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&sh.full[q % kSlots], (q / kSlots) & 1u))
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) break;
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  uint32_t gt_base = 0, bar_k = 0, step_k = 0;
  bool ok = true;
  for (uint32_t st = 0; st < steps && ok; ++st) {
    const bool pre = st < p.n_prefill_steps;
    const uint32_t np = pre ? p.n_phases - 2 : p.n_phases;
    for (uint32_t pi = 0; pi <= np && ok; ++pi) {
      if (pi == np) {  // after a prompt step without logits: advance the position
        if (!pre) break;
        if (blockIdx.x == 0 && threadIdx.x == 0) p.pos[0] = ldcg_i(p.pos) + 1;
      } else {
        const Phase& P = phases[pi];
        switch (P.kind) {
          case kEmbed: phase_embed(p); break;
          case kMatvec:
            (void)phase_matvec(p, P, sh, gt_base, step_k);  // a failed wait has recorded its error
            gt_base += phase_tiles(P);
            break;
          case kAttn: phase_attention(p, P.layer, sh.xs); break;
          default: phase_argmax(p, step_k); break;
        }
      }
      ok = grid_sync(p, bar_k++);
    }
    if (!pre) ++step_k;
    if (ok && ldcg_i(p.ctl) != 0) break;  // eos (written before the barrier: every thread reads 1)
  }
  named_barrier(kAllConsumersBarrier, kConsumerThreads);
  if (threadIdx.x == 0) *done = 1;
}

constexpr size_t smem_bytes() {
  return kSlots * kSlotBytes + 2 * kSlots * 8 + 16 * 8 + kSlots * 4 + 8 + 192 * 4 + kXsFloats * 4 +
         kMaxPhases * sizeof(Phase);
}

}  // namespace mk
}  // namespace efg
