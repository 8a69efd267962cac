// efg_matvec.cuh - host-visible description of the packed matvec kernels (efg_matvec.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace efg {

enum class Fmt : int { Q8 = 3, Q4 = 4 };  // values = ef::QType
enum class Epi : int { Store = 0, Add = 1, SwiGLU = 2 };

constexpr int kMaxJobs = 4;

// The all-gather that the matvec kernels can do in their epilogue (efg_gather.cuh): flag
// words of each rank's area, and the per-launch description (nranks == 0: no exchange).
constexpr int kMaxGatherRanks = 8;
constexpr uint32_t kReadyOff = 0;
constexpr uint32_t kDoneOff = 32;
constexpr uint32_t kEpochOff = 64;
constexpr uint32_t kCountOff = 96;
// The row-sharded argmax's exchange (efg_argmax.cu) in the same area: [2 call parities][rank]
// (value bits, index) pairs, their flags (the call number that wrote them), and this rank's
// count of exchanges.
constexpr uint32_t kPairOff = 128;
constexpr uint32_t kPairFlagOff = kPairOff + 2 * kMaxGatherRanks * 2;
constexpr uint32_t kPairEpochOff = kPairFlagOff + 2 * kMaxGatherRanks;
constexpr size_t kGatherFlagBytes = 256 * 4;
static_assert(kPairEpochOff < kGatherFlagBytes / 4, "flag area too small");

struct GatherDev {
  int nranks = 0, rank = 0;
  uint32_t* flags = nullptr;                   // this rank's flag area
  uint32_t* peer_flags[kMaxGatherRanks] = {};  // every rank's flag area (mapped)
  float* peer_y[kMaxGatherRanks] = {};         // every rank's y at the launch's first row
};

struct MatvecJobDev {
  const uint8_t* W;
  float* y;
  uint32_t rows;
  uint32_t y_pos_stride;  // y += (*pos) * y_pos_stride when MatvecArgs::pos is set
};

// One fused matvec launch: n_jobs matrices with the same type and cols applied to the
// same x (q/k/v or gate/up), or, for Epi::SwiGLU, jobs[0] = gate, jobs[1] = up with the
// result silu(gate . x) * (up . x) written to jobs[0].y.
struct MatvecArgs {
  Fmt fmt = Fmt::Q4;
  Epi epi = Epi::Store;
  const float* x = nullptr;
  const float* norm_w = nullptr;  // when set, x is replaced by rmsnorm(x) * norm_w first; with pdl,
                                  // read before the previous kernel ends (model weights only)
  float norm_eps = 1e-5f;
  const int32_t* pos = nullptr;   // device-side position for y_pos_stride (decode step)
  size_t cols = 0;
  int n_jobs = 0;
  MatvecJobDev jobs[kMaxJobs] = {};
  bool pdl = false;               // launch with programmatic stream serialization
  bool small_kernel = true;       // the small-matrix MMA kernel may take the call (the decode step
                                  // turns it off: measured slower inside that chain of launches)
  GatherDev gather;               // nranks > 0: store every output into each peer's y too, and
                                  // return only once every peer's rows are here (one job, Store,
                                  // no norm; efg_gather.cuh)
};

// Validates and launches. Returns an EFG_* status; on EFG_EINVAL/ECUDA the message is
// left in the thread-local error string.
int launch_matvec(const MatvecArgs& a, int* d_err, cudaStream_t stream);

// y = W x for W stored as 0 = F32, 1 = F16, 2 = BF16 ([rows][cols], any alignment).
int launch_dense_matvec(int qtype, float* y, const uint8_t* W, const float* x, size_t rows, size_t cols,
                        cudaStream_t stream, bool pdl);

struct DeviceInfo;
// The Q4_0 kernel on the integer tensor-core MMA (efg_matvec_mma.cu): taken for Q4_0
// matrices of 48 MB and more with 2048 <= cols <= 8192, cols % 256 == 0, 16-byte aligned
// W, x and norm weights, store / add epilogues. Uses no library-owned state.
bool matvec_mma_ok(const MatvecArgs& a, const DeviceInfo& dev);
int launch_matvec_q4_mma(const MatvecArgs& a, const DeviceInfo& dev, int* d_err, cudaStream_t stream,
                         bool direct_smem_attr);

// The Q4_0 kernel for small matrices (efg_matvec_mma.cu): each CTA fetches all of its rows
// into shared memory at once and is small enough that the next launch's CTA runs beside it,
// fetching its own weights meanwhile. Taken for Q4_0 calls whose per-CTA share fits (a few MB
// per matrix: the decode-step shapes), 2048 <= cols <= 8192, cols % 256 == 0, 16-byte aligned
// W, x and norm weights; every epilogue, no in-kernel gather.
bool matvec_small_ok(const MatvecArgs& a, const DeviceInfo& dev);
int launch_matvec_q4_small(const MatvecArgs& a, const DeviceInfo& dev, int* d_err, cudaStream_t stream,
                           bool direct_smem_attr);

// launch_matvec on a caller-described device. With direct_smem_attr the kernel's
// shared-memory limit is set by cudaFuncSetAttribute on every launch instead of through
// the library's per-kernel cache, so the call touches no library-owned state.
int launch_matvec_on(const MatvecArgs& a, const DeviceInfo& dev, int* d_err, cudaStream_t stream,
                     bool direct_smem_attr);

// True when the fast (bulk-copy) kernel accepts these arguments; otherwise
// launch_matvec uses the generic kernel (plain loads, any alignment).
bool matvec_fast_path_ok(const MatvecArgs& a);

}  // namespace efg
