// efg_gather.cuh - the all-gather of the row-sharded matvec done by the matvec kernels
// themselves: every CTA stores the outputs of its rows straight into every peer GPU's y
// (plain stores to peer memory mapped over NVLink), and the launch ends only once every
// peer's rows have landed in this GPU's y. No collective library call, no extra launch.
//
// Each rank owns a small flag area (uint32 words) in its own memory that the peers write:
//   ready[q] (word kReadyOff + q): the epoch at which rank q's kernel started, i.e. when
//            every earlier kernel in q's stream (readers of q's y included) had finished;
//            a rank stores into q's y for epoch e only after it has seen ready[q] >= e.
//   done[q]  (word kDoneOff + q):  the last epoch whose rows rank q has stored here.
//   epoch    (word kEpochOff):     the last epoch this rank finished (this rank only).
//   count    (word kCountOff):     CTAs of the current launch that finished (this rank only).
// An epoch is one launch; every rank makes the same sequence of sharded calls, so epoch e
// names the same call everywhere. A launch reads its epoch from device memory (after the
// grid-dependency wait), so CUDA graphs of these launches replay correctly.
//
// Order of one launch on rank r (epoch e = epoch + 1):
//   1. CTA 0 stores ready[r] = e into every peer's area (release, system scope; one lane
//      per peer).
//   2. A warp that stores outputs first waits until ready[q] >= e here for every peer q.
//   3. Each CTA: outputs to the local y and to every peer's y; the CTA barriers, then one
//      thread fences at system scope (cumulative: it orders every store the barrier ordered
//      before it, one fence per CTA instead of one per storing thread) and counts the CTA in
//      `count`.
//   4. The last CTA of the launch resets `count`, fences, stores done[r] = e into every
//      peer's area, then waits until done[q] >= e here for every peer q, and writes epoch.
// Every wait is bounded (kWaitTimeoutNs) and records EFG_ETIMEOUT in the device error word;
// after that the flags no longer agree between ranks and the communicator must be rebuilt.
#pragma once

#include <cstdint>

#include "efg_device.cuh"
#include "efg_matvec.cuh"

namespace efg {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ bool epoch_reached(uint32_t seen, uint32_t epoch) {
  return static_cast<int32_t>(seen - epoch) >= 0;
}

// The epoch of this launch. Call after the grid-dependency wait (pdl_wait): the previous
// launch's last CTA wrote the word just before that launch ended.
__device__ __forceinline__ uint32_t gather_epoch(const GatherDev& g) {
  return *reinterpret_cast<const volatile uint32_t*>(g.flags + kEpochOff) + 1u;
}

// Step 1, the first warp of CTA 0 after the grid-dependency wait: lane q stores into rank
// q's area, so the peers are told at once rather than one after another.
__device__ __forceinline__ void gather_announce(const GatherDev& g, uint32_t epoch) {
  const int q = threadIdx.x & 31;
  if (q < g.nranks && q != g.rank) st_release_sys(g.peer_flags[q] + kReadyOff + g.rank, epoch);
}

// Waits (bounded) until flags[off + q] >= epoch for every peer q. Lane q of the calling
// warp polls rank q's word; the whole warp must call it. True when every peer got there.
__device__ __forceinline__ bool gather_wait_flags(const GatherDev& g, uint32_t off, uint32_t epoch, int* err) {
  const int lane = threadIdx.x & 31;
  bool ok = true;
  if (lane < g.nranks && lane != g.rank) {
    const uint32_t* f = g.flags + off + lane;
    if (!epoch_reached(ld_acquire_sys(f), epoch)) {
      const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
      for (uint32_t i = 0; !epoch_reached(ld_acquire_sys(f), epoch); ++i) {
        __nanosleep(64);
        if ((i & 63u) == 63u && (error_raised(err) || globaltimer_ns() - t0 > kWaitTimeoutNs)) {
          record_error(err, EFG_ETIMEOUT);
          ok = false;
          break;
        }
      }
    }
  }
  return __all_sync(0xFFFFFFFFu, ok);
}

// Step 2: a whole warp, before its first store into a peer's y.
__device__ __forceinline__ bool gather_wait_ready(const GatherDev& g, uint32_t epoch, int* err) {
  return gather_wait_flags(g, kReadyOff, epoch, err);
}

// Step 3's stores: row `row` (relative to the launch's first row) of value v into every
// peer's y.
__device__ __forceinline__ void gather_store(const GatherDev& g, uint32_t row, float v) {
  for (int q = 0; q < g.nranks; ++q)
    if (q != g.rank) g.peer_y[q][row] = v;
}

// Steps 3 (count) and 4, by one full warp of each CTA after a CTA barrier that follows every
// store of the CTA into the peers' y.
__device__ __forceinline__ void gather_finish(const GatherDev& g, uint32_t epoch, int* err) {
  const int lane = threadIdx.x & 31;
  uint32_t prev = 0;
  if (lane == 0) {
    __threadfence_system();  // the CTA's peer stores (ordered before by the barrier), then the count
    prev = atomicAdd(g.flags + kCountOff, 1u);
  }
  prev = __shfl_sync(0xFFFFFFFFu, prev, 0);
  if (prev + 1u != gridDim.x) return;
  // The last CTA of this launch on this rank: every CTA fenced its stores before counting
  // itself; the fence below (after the count was read) orders them all before the done flags.
  if (lane == 0) {
    __threadfence_system();
    *reinterpret_cast<volatile uint32_t*>(g.flags + kCountOff) = 0u;  // the next launch starts from 0
  }
  __syncwarp();
  if (lane < g.nranks && lane != g.rank) st_release_sys(g.peer_flags[lane] + kDoneOff + g.rank, epoch);
  gather_wait_flags(g, kDoneOff, epoch, err);
  if (lane == 0) *reinterpret_cast<volatile uint32_t*>(g.flags + kEpochOff) = epoch;
}

}  // namespace efg
