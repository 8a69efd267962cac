// efg_host.cpp - thread-local error messages and per-device state.
#include "efg_host.h"

#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>

namespace efg {

namespace {
thread_local std::string g_error;
std::mutex g_dev_mu;
constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
}  // namespace

bool& weight_prefetch_flag() {
  static thread_local bool on = false;
  return on;
}

bool& q4_mma_flag() {
  static thread_local bool on = true;
  return on;
}

bool& small_gemm_flag() {
  static thread_local bool on = false;
  return on;
}

int ensure_smem_attr(const void* fn, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> done;
  int dev = 0;
  EFG_TRY_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lk(mu);
  size_t& cur = done[{dev, fn}];
  if (cur >= bytes) return EFG_OK;
  EFG_TRY_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
               "kernel shared-memory attribute");
  cur = bytes;
  return EFG_OK;
}

int fail(int status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return status;
}

void clear_error() { g_error.clear(); }

const char* last_error() { return g_error.c_str(); }

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return EFG_OK;
  const int status = e == cudaErrorMemoryAllocation ? EFG_ENOMEM : EFG_ECUDA;
  return fail(status, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

DeviceInfo* current_device() {
  int dev = -1;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cuda_check(e, "cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    fail(EFG_ECUDA, "device index %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_devices[dev];
  if (d.device == dev) return &d;
  int sms = 0, smem = 0;
  if (cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device attribute") != EFG_OK)
    return nullptr;
  if (cuda_check(cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev), "device attribute") !=
      EFG_OK)
    return nullptr;
  int* err = nullptr;
  if (cuda_check(cudaMalloc(&err, sizeof(int)), "error word allocation") != EFG_OK) return nullptr;
  if (cuda_check(cudaMemset(err, 0, sizeof(int)), "error word init") != EFG_OK) return nullptr;
  d.sm_count = sms;
  d.smem_optin = static_cast<size_t>(smem);
  d.d_err = err;
  d.device = dev;
  return &d;
}

}  // namespace efg

namespace efg {
namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static const EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}
}  // namespace

bool encode_u64_rows_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_elems,
                         uint32_t box_rows) {
  const EncodeTiledFn fn = encode_tiled();
  if (!fn || rows == 0 || row_bytes % 16 != 0 || reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
  const cuuint64_t dims[2] = {row_bytes / 8, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_elems, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace efg
