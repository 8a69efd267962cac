// efg_static.cu - efg_host_matvec_static: the host-pointer packed matvec of
// efg_host_matvec, staged through a fixed device area instead of library buffers.
//
// The area is one file-scope __device__ array of kStaticScratchBytes (8 MiB), 256-byte
// aligned. Its device address is taken with cudaGetSymbolAddress once per device, in a
// set-up step run by the first call on that device (make that first call before any
// stream capture begins on the thread). After set-up a call performs no device or host
// allocation: no cudaMalloc/cudaFree, no allocating library call, no library-owned
// buffers, streams or caches; it copies on cudaStreamPerThread and synchronizes it.
//
// Layout of the area per call:
//   [0, 256)          the device error word (int at offset 0) that bounded waits write;
//                     it must start at zero: static storage starts zeroed, and a call
//                     that finds it set returns that status and writes zero back
//   then x (cols floats), y (rows floats), W (rows packed rows), each 256-byte aligned.
// Every byte of x, y and W is written before it is read in the same call, so nothing
// else must start at zero. A call whose x, y and W do not fit is rejected (EFG_EINVAL).
// Each device that loads the library holds its own copy of the area. Calls that overlap
// in time on the same device (from several host threads) race on that device's copy;
// callers serialize them. Calls on different devices do not share storage.
#include <cstdint>
#include <mutex>

#include "../../include/efg.h"
#include "efg_host.h"
#include "efg_matvec.cuh"

namespace efg {
namespace {

constexpr size_t kStaticScratchBytes = 8u << 20;
constexpr size_t kErrBytes = 256;

__device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

constexpr int kMaxStaticDevices = 64;

struct StaticDevice {
  bool ready = false;
  uint8_t* base = nullptr;
  DeviceInfo info;
};

std::mutex g_static_mu;
StaticDevice g_static[kMaxStaticDevices];

size_t al256(size_t n) { return (n + 255) / 256 * 256; }

// Set-up, once per device: the area's address, SM count and shared-memory limit.
int static_setup(StaticDevice** out) {
  int dev = -1;
  EFG_TRY_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxStaticDevices) return fail(EFG_ECUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_static_mu);
  StaticDevice& d = g_static[dev];
  if (!d.ready) {
    void* p = nullptr;
    EFG_TRY_CUDA(cudaGetSymbolAddress(&p, g_static_scratch), "static scratch address");
    int sms = 0, smem = 0;
    EFG_TRY_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device attribute");
    EFG_TRY_CUDA(cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev), "device attribute");
    d.base = static_cast<uint8_t*>(p);
    d.info.device = dev;
    d.info.sm_count = sms;
    d.info.smem_optin = static_cast<size_t>(smem);
    d.info.d_err = reinterpret_cast<int*>(d.base);
    d.ready = true;
  }
  *out = &d;
  return EFG_OK;
}

}  // namespace
}  // namespace efg

extern "C" int efg_host_matvec_static(int qtype, float* y, const uint8_t* W, const float* x, size_t rows,
                                      size_t cols) {
  using namespace efg;
  if (qtype != EFG_Q4_0 && qtype != EFG_Q8_0)
    return fail(EFG_EINVAL, "matvec_static: type %d is not a packed type (Q4_0, Q8_0)", qtype);
  if (cols % 32 != 0)
    return fail(EFG_EINVAL, "%s needs a row length divisible by 32, got %zu", qtype == EFG_Q4_0 ? "Q4_0" : "Q8_0",
                cols);
  if (rows == 0) return EFG_OK;
  if (!y || (!W && cols) || (!x && cols)) return fail(EFG_EINVAL, "matvec_static: null pointer");
  const size_t wbytes = rows * (cols / 32) * (qtype == EFG_Q4_0 ? 18 : 34);
  const size_t need = kErrBytes + al256(cols * sizeof(float)) + al256(rows * sizeof(float)) + al256(wbytes);
  if (rows >= (1ull << 31) || cols >= (1ull << 31) || need > kStaticScratchBytes)
    return fail(EFG_EINVAL, "matvec_static: needs %zu bytes of device scratch, the static area holds %zu", need,
                kStaticScratchBytes);
  StaticDevice* sd = nullptr;
  if (int st = static_setup(&sd)) return st;
  uint8_t* xs = sd->base + kErrBytes;
  uint8_t* ys = xs + al256(cols * sizeof(float));
  uint8_t* ws = ys + al256(rows * sizeof(float));
  const cudaStream_t s = cudaStreamPerThread;
  if (cols) {
    EFG_TRY_CUDA(cudaMemcpyAsync(xs, x, cols * sizeof(float), cudaMemcpyHostToDevice, s), "x upload");
    EFG_TRY_CUDA(cudaMemcpyAsync(ws, W, wbytes, cudaMemcpyHostToDevice, s), "weight upload");
  }
  MatvecArgs a;
  a.fmt = qtype == EFG_Q4_0 ? Fmt::Q4 : Fmt::Q8;
  a.x = reinterpret_cast<const float*>(xs);
  a.cols = cols;
  a.n_jobs = 1;
  a.jobs[0] = MatvecJobDev{ws, reinterpret_cast<float*>(ys), static_cast<uint32_t>(rows), 0};
  if (int st = launch_matvec_on(a, sd->info, sd->info.d_err, s, true)) return st;
  int derr = 0;
  EFG_TRY_CUDA(cudaMemcpyAsync(y, ys, rows * sizeof(float), cudaMemcpyDeviceToHost, s), "y download");
  EFG_TRY_CUDA(cudaMemcpyAsync(&derr, sd->info.d_err, sizeof derr, cudaMemcpyDeviceToHost, s), "error word read");
  EFG_TRY_CUDA(cudaStreamSynchronize(s), "stream synchronize");
  if (derr != 0) {
    EFG_TRY_CUDA(cudaMemsetAsync(sd->info.d_err, 0, sizeof(int), s), "error word reset");
    EFG_TRY_CUDA(cudaStreamSynchronize(s), "stream synchronize");
    return fail(derr, "matvec_static: the kernel reported %s", efg_status_string(derr));
  }
  return EFG_OK;
}
