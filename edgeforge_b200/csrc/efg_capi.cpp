// efg_capi.cpp - the extern "C" boundary (include/efg.h): argument validation with the
// reference's error messages, dispatch to the kernels, and the synchronous host-pointer
// forms that keep the reference's signatures.
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/efg.h"
#include "efg_host.h"
#include "efg_matvec.cuh"
#include "efg_quant.cuh"

using namespace efg;

namespace {

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool is_block(int qtype) { return qtype == EFG_Q4_0 || qtype == EFG_Q8_0; }

const char* type_name(int qtype) {
  switch (qtype) {
    case EFG_F32: return "F32";
    case EFG_F16: return "F16";
    case EFG_BF16: return "BF16";
    case EFG_Q8_0: return "Q8_0";
    case EFG_Q4_0: return "Q4_0";
    default: return "?";
  }
}

// Same message as qtype_row_bytes' ef::Error (src/quant.cpp:143-145).
int check_cols(int qtype, uint64_t cols) {
  if (is_block(qtype) && cols % 32 != 0)
    return fail(EFG_EINVAL, "%s needs a row length divisible by 32, got %llu", type_name(qtype),
                static_cast<unsigned long long>(cols));
  return EFG_OK;
}

bool is_plain(int qtype) { return qtype == EFG_F32 || qtype == EFG_F16 || qtype == EFG_BF16; }

int matvec_one(int qtype, float* y, const uint8_t* W, const float* x, size_t rows, size_t cols, cudaStream_t s) {
  if (is_plain(qtype)) return launch_dense_matvec(qtype, y, W, x, rows, cols, s, weight_prefetch_flag());
  if (!is_block(qtype)) return fail(EFG_EINVAL, "matvec: unknown type %d", qtype);
  if (int st = check_cols(qtype, cols)) return st;
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  MatvecArgs a;
  a.fmt = qtype == EFG_Q4_0 ? Fmt::Q4 : Fmt::Q8;
  a.x = x;
  a.cols = cols;
  a.pdl = weight_prefetch_flag();
  a.n_jobs = 1;
  a.jobs[0] = MatvecJobDev{W, y, static_cast<uint32_t>(rows), 0};
  if (rows >= (1ull << 31)) return fail(EFG_EINVAL, "matvec: too many rows");
  return launch_matvec(a, dev->d_err, s);
}

// ---- host-pointer forms: one library stream and grow-only buffers per device --------
struct HostCtx {
  std::mutex mu;
  cudaStream_t stream = nullptr;
  void* in = nullptr;
  size_t in_cap = 0;
  void* out = nullptr;
  size_t out_cap = 0;
  void* wtmp = nullptr;  // per-call upload of an unregistered W
  size_t wtmp_cap = 0;
  // registered host ranges: start -> (bytes, device copy)
  std::map<const uint8_t*, std::pair<size_t, void*>> ranges;
};

// Device address of [p, p + n) if it lies inside a registered range, else nullptr.
const uint8_t* resident(const HostCtx* h, const uint8_t* p, size_t n) {
  auto it = h->ranges.upper_bound(p);
  if (it == h->ranges.begin()) return nullptr;
  --it;
  const uint8_t* base = it->first;
  const size_t len = it->second.first;
  if (p < base || static_cast<size_t>(p - base) > len || n > len - static_cast<size_t>(p - base)) return nullptr;
  return static_cast<const uint8_t*>(it->second.second) + (p - base);
}

HostCtx g_host[64];

int ensure(void*& p, size_t& cap, size_t need) {
  if (need <= cap) return EFG_OK;
  if (p) cudaFree(p);
  p = nullptr;
  cap = 0;
  EFG_TRY_CUDA(cudaMalloc(&p, need), "host-call buffer");
  cap = need;
  return EFG_OK;
}

HostCtx* host_ctx(int& status) {
  DeviceInfo* dev = current_device();
  if (!dev) {
    status = EFG_ECUDA;
    return nullptr;
  }
  HostCtx* h = &g_host[dev->device];
  status = EFG_OK;
  return h;
}

int host_stream(HostCtx* h) {
  if (!h->stream) EFG_TRY_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking), "stream create");
  return EFG_OK;
}

using PointerAttrFn = CUresult (*)(void*, CUpointer_attribute, CUdeviceptr);

// cuPointerGetAttribute from the driver, looked up once (the library links the CUDA
// runtime statically and has no link-time dependency on libcuda).
PointerAttrFn pointer_attr_fn() {
  static const PointerAttrFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuPointerGetAttribute", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PointerAttrFn>(f);
  }();
  return fn;
}

// Device address of page-locked host memory that the device may write (null for pageable
// memory, and for page-locked memory whose access flags the driver does not report as
// read-write, e.g. a range registered with cudaHostRegisterReadOnly): kernels can store
// into it directly over the bus.
void* mapped_host(void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a.type != cudaMemoryTypeHost || !a.devicePointer) return nullptr;
  const PointerAttrFn fn = pointer_attr_fn();
  unsigned int flags = 0;
  if (!fn || fn(&flags, CU_POINTER_ATTRIBUTE_ACCESS_FLAGS, reinterpret_cast<CUdeviceptr>(a.devicePointer)) !=
                 CUDA_SUCCESS)
    return nullptr;
  return flags == CU_POINTER_ATTRIBUTE_ACCESS_FLAG_READWRITE ? a.devicePointer : nullptr;
}

}  // namespace

extern "C" {

int efg_abi_version(void) { return 1; }

const char* efg_last_error(void) { return last_error(); }

const char* efg_status_string(int s) {
  switch (s) {
    case EFG_OK: return "EFG_OK";
    case EFG_EINVAL: return "EFG_EINVAL";
    case EFG_ECUDA: return "EFG_ECUDA";
    case EFG_ENCCL: return "EFG_ENCCL";
    case EFG_ETIMEOUT: return "EFG_ETIMEOUT";
    case EFG_ENOMEM: return "EFG_ENOMEM";
    case EFG_EFORMAT: return "EFG_EFORMAT";
    case EFG_ESTATE: return "EFG_ESTATE";
    default: return "EFG_UNKNOWN";
  }
}

int efg_device_error(int* code) {
  if (!code) return fail(EFG_EINVAL, "efg_device_error: null pointer");
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  EFG_TRY_CUDA(cudaDeviceSynchronize(), "device synchronize");
  EFG_TRY_CUDA(cudaMemcpy(code, dev->d_err, sizeof(int), cudaMemcpyDeviceToHost), "read error word");
  EFG_TRY_CUDA(cudaMemset(dev->d_err, 0, sizeof(int)), "clear error word");
  return EFG_OK;
}

int efg_set_weight_prefetch(int enable) {
  const bool old = weight_prefetch_flag();
  weight_prefetch_flag() = enable != 0;
  return old ? 1 : 0;
}

int efg_set_small_gemm(int enable) {
  const bool old = small_gemm_flag();
  small_gemm_flag() = enable != 0;
  return old ? 1 : 0;
}

int efg_set_q4_mma(int enable) {
  const bool old = q4_mma_flag();
  q4_mma_flag() = enable != 0;
  return old ? 1 : 0;
}

uint64_t efg_row_bytes(int qtype, uint64_t cols) {
  switch (qtype) {
    case EFG_F32: return cols * 4;
    case EFG_F16:
    case EFG_BF16: return cols * 2;
    case EFG_Q8_0:
    case EFG_Q4_0:
      if (check_cols(qtype, cols) != EFG_OK) return 0;
      return cols / 32 * (qtype == EFG_Q8_0 ? 34 : 18);
    default: fail(EFG_EINVAL, "unknown type %d", qtype); return 0;
  }
}

int efg_matvec_q4_0(float* y, const uint8_t* W, const float* x, size_t rows, size_t cols, void* stream) {
  return matvec_one(EFG_Q4_0, y, W, x, rows, cols, as_stream(stream));
}

int efg_matvec_q8_0(float* y, const uint8_t* W, const float* x, size_t rows, size_t cols, void* stream) {
  return matvec_one(EFG_Q8_0, y, W, x, rows, cols, as_stream(stream));
}

int efg_matvec(int qtype, float* y, const uint8_t* W, const float* x, size_t rows, size_t cols, void* stream) {
  return matvec_one(qtype, y, W, x, rows, cols, as_stream(stream));
}

int efg_dot_q4_0(float* out, const uint8_t* row, const float* x, size_t n, void* stream) {
  return matvec_one(EFG_Q4_0, out, row, x, 1, n, as_stream(stream));
}

int efg_dot_q8_0(float* out, const uint8_t* row, const float* x, size_t n, void* stream) {
  return matvec_one(EFG_Q8_0, out, row, x, 1, n, as_stream(stream));
}

int efg_matvec_jobs(const efg_matvec_job* jobs, size_t n_jobs, void* stream) {
  if (n_jobs && !jobs) return fail(EFG_EINVAL, "matvec_jobs: null job list");
  DeviceInfo* dev = current_device();
  if (!dev) return EFG_ECUDA;
  size_t i = 0;
  while (i < n_jobs) {
    // Greedily group consecutive jobs that share type, cols and x (one launch each).
    MatvecArgs a;
    const efg_matvec_job& f = jobs[i];
    if (is_plain(f.qtype)) {  // plain storage types: one launch per job
      if (int st = launch_dense_matvec(f.qtype, f.d_y, f.d_W, f.d_x, f.rows, f.cols, as_stream(stream),
                                       weight_prefetch_flag()))
        return st;
      ++i;
      continue;
    }
    if (!is_block(f.qtype)) return fail(EFG_EINVAL, "matvec_jobs: job %zu has type %s", i, type_name(f.qtype));
    if (int st = check_cols(f.qtype, f.cols)) return st;
    a.fmt = f.qtype == EFG_Q4_0 ? Fmt::Q4 : Fmt::Q8;
    a.pdl = weight_prefetch_flag();
    a.x = f.d_x;
    a.cols = f.cols;
    size_t k = i;
    while (k < n_jobs && a.n_jobs < kMaxJobs && jobs[k].qtype == f.qtype && jobs[k].cols == f.cols &&
           jobs[k].d_x == f.d_x) {
      if (jobs[k].rows >= (1ull << 31)) return fail(EFG_EINVAL, "matvec_jobs: too many rows");
      a.jobs[a.n_jobs++] = MatvecJobDev{jobs[k].d_W, jobs[k].d_y, static_cast<uint32_t>(jobs[k].rows), 0};
      ++k;
    }
    if (int st = launch_matvec(a, dev->d_err, as_stream(stream))) return st;
    i = k;
  }
  return EFG_OK;
}

int efg_quantize_row(int qtype, const float* x, size_t n, void* out, int search, void* stream) {
  if (!is_block(qtype) && !is_plain(qtype)) return fail(EFG_EINVAL, "quantize_row: unknown type %d", qtype);
  return launch_quantize(qtype, x, n, out, search != 0, as_stream(stream));
}

int efg_fake_quant_q4_group(const float* x, size_t n, float* out, int search, void* stream) {
  return launch_fake_quant_q4_group(x, n, out, search != 0, as_stream(stream));
}

int efg_dequantize_row(int qtype, const void* in, size_t n, float* out, void* stream) {
  return launch_dequantize(qtype, in, n, out, as_stream(stream));
}

int efg_quantize_rows(int qtype, const float* X, size_t rows, size_t cols, void* out, int search, void* stream) {
  if (!is_block(qtype) && !is_plain(qtype)) return fail(EFG_EINVAL, "quantize_rows: unknown type %d", qtype);
  if (int st = check_cols(qtype, cols)) return st;
  if (cols && rows > UINT64_MAX / cols) return fail(EFG_EINVAL, "quantize_rows: size overflows");
  return launch_quantize(qtype, X, static_cast<uint64_t>(rows) * cols, out, search != 0, as_stream(stream));
}

int efg_dequantize_rows(int qtype, const void* in, size_t rows, size_t cols, float* out, void* stream) {
  if (int st = check_cols(qtype, cols)) return st;
  if (cols && rows > UINT64_MAX / cols) return fail(EFG_EINVAL, "dequantize_rows: size overflows");
  return launch_dequantize(qtype, in, static_cast<uint64_t>(rows) * cols, out, as_stream(stream));
}

int efg_row_f32(float* out, int qtype, const uint8_t* W, size_t rows, size_t cols, const int32_t* d_r, size_t r_host,
                void* stream) {
  return launch_row_f32(qtype, W, rows, cols, d_r, r_host, out, as_stream(stream));
}

// ---- host-pointer forms -------------------------------------------------------------

int efg_host_matvec(int qtype, float* y, const uint8_t* W, const float* x, size_t rows, size_t cols) {
  if (!is_block(qtype) && !is_plain(qtype)) return fail(EFG_EINVAL, "matvec: unknown type %d", qtype);
  if (int st = check_cols(qtype, cols)) return st;
  if (rows == 0) return EFG_OK;
  if (!y || (!W && cols) || (!x && cols)) return fail(EFG_EINVAL, "matvec: null pointer");
  int st;
  HostCtx* h = host_ctx(st);
  if (!h) return st;
  std::lock_guard<std::mutex> lk(h->mu);
  if ((st = host_stream(h))) return st;
  const size_t wbytes = rows * static_cast<size_t>(efg_row_bytes(qtype, cols));
  const void* dW = resident(h, W, wbytes);
  if (!dW) {
    if ((st = ensure(h->wtmp, h->wtmp_cap, wbytes + 16))) return st;
    if (wbytes) EFG_TRY_CUDA(cudaMemcpyAsync(h->wtmp, W, wbytes, cudaMemcpyHostToDevice, h->stream), "weight upload");
    dW = h->wtmp;
  }
  if ((st = ensure(h->in, h->in_cap, cols * sizeof(float) + 16))) return st;
  if ((st = ensure(h->out, h->out_cap, rows * sizeof(float) + 16))) return st;
  if (cols) EFG_TRY_CUDA(cudaMemcpyAsync(h->in, x, cols * sizeof(float), cudaMemcpyHostToDevice, h->stream), "x upload");
  // A page-locked y is written by the matvec's own stores, as rows finish, instead of by a
  // copy after the kernel (which adds a copy-engine round trip to every call).
  float* y_dev = static_cast<float*>(mapped_host(y));
  if ((st = matvec_one(qtype, y_dev ? y_dev : static_cast<float*>(h->out), static_cast<const uint8_t*>(dW),
                       static_cast<const float*>(h->in), rows, cols, h->stream)))
    return st;
  if (!y_dev)
    EFG_TRY_CUDA(cudaMemcpyAsync(y, h->out, rows * sizeof(float), cudaMemcpyDeviceToHost, h->stream), "y download");
  EFG_TRY_CUDA(cudaStreamSynchronize(h->stream), "stream synchronize");
  return EFG_OK;
}

int efg_host_quantize_row(int qtype, const float* x, size_t n, void* out, int search) {
  if (!is_block(qtype) && !is_plain(qtype)) return fail(EFG_EINVAL, "quantize_row: unknown type %d", qtype);
  if (int st = check_cols(qtype, n)) return st;
  if (n == 0) return EFG_OK;
  if (!x || !out) return fail(EFG_EINVAL, "quantize_row: null pointer");
  int st;
  HostCtx* h = host_ctx(st);
  if (!h) return st;
  std::lock_guard<std::mutex> lk(h->mu);
  if ((st = host_stream(h))) return st;
  const size_t ob = static_cast<size_t>(efg_row_bytes(qtype, n));
  if ((st = ensure(h->in, h->in_cap, n * sizeof(float)))) return st;
  if ((st = ensure(h->out, h->out_cap, ob))) return st;
  EFG_TRY_CUDA(cudaMemcpyAsync(h->in, x, n * sizeof(float), cudaMemcpyHostToDevice, h->stream), "x upload");
  if ((st = launch_quantize(qtype, static_cast<const float*>(h->in), n, h->out, search != 0, h->stream))) return st;
  EFG_TRY_CUDA(cudaMemcpyAsync(out, h->out, ob, cudaMemcpyDeviceToHost, h->stream), "download");
  EFG_TRY_CUDA(cudaStreamSynchronize(h->stream), "stream synchronize");
  return EFG_OK;
}

int efg_host_fake_quant_q4_group(const float* x, size_t n, float* out, int search) {
  const size_t m = n < 256 ? n : 256;
  if (m == 0) return EFG_OK;
  if (!x || !out) return fail(EFG_EINVAL, "fake_quant_q4_group: null pointer");
  int st;
  HostCtx* h = host_ctx(st);
  if (!h) return st;
  std::lock_guard<std::mutex> lk(h->mu);
  if ((st = host_stream(h))) return st;
  if ((st = ensure(h->in, h->in_cap, m * sizeof(float)))) return st;
  if ((st = ensure(h->out, h->out_cap, m * sizeof(float)))) return st;
  EFG_TRY_CUDA(cudaMemcpyAsync(h->in, x, m * sizeof(float), cudaMemcpyHostToDevice, h->stream), "x upload");
  if ((st = launch_fake_quant_q4_group(static_cast<const float*>(h->in), m, static_cast<float*>(h->out), search != 0,
                                       h->stream)))
    return st;
  EFG_TRY_CUDA(cudaMemcpyAsync(out, h->out, m * sizeof(float), cudaMemcpyDeviceToHost, h->stream), "download");
  EFG_TRY_CUDA(cudaStreamSynchronize(h->stream), "stream synchronize");
  return EFG_OK;
}

int efg_host_dequantize_row(int qtype, const void* in, size_t n, float* out) {
  if (qtype < 0 || qtype > 4) return fail(EFG_EINVAL, "dequantize_row: unknown type %d", qtype);
  if (int st = check_cols(qtype, n)) return st;
  if (n == 0) return EFG_OK;
  if (!in || !out) return fail(EFG_EINVAL, "dequantize_row: null pointer");
  int st;
  HostCtx* h = host_ctx(st);
  if (!h) return st;
  std::lock_guard<std::mutex> lk(h->mu);
  if ((st = host_stream(h))) return st;
  const size_t ib = efg_row_bytes(qtype, n);
  if ((st = ensure(h->in, h->in_cap, ib))) return st;
  if ((st = ensure(h->out, h->out_cap, n * sizeof(float)))) return st;
  EFG_TRY_CUDA(cudaMemcpyAsync(h->in, in, ib, cudaMemcpyHostToDevice, h->stream), "upload");
  if ((st = launch_dequantize(qtype, h->in, n, static_cast<float*>(h->out), h->stream))) return st;
  EFG_TRY_CUDA(cudaMemcpyAsync(out, h->out, n * sizeof(float), cudaMemcpyDeviceToHost, h->stream), "download");
  EFG_TRY_CUDA(cudaStreamSynchronize(h->stream), "stream synchronize");
  return EFG_OK;
}

int efg_host_register_weights(const void* host, size_t bytes) {
  if (!host || bytes == 0) return fail(EFG_EINVAL, "register_weights: empty range");
  int st;
  HostCtx* h = host_ctx(st);
  if (!h) return st;
  std::lock_guard<std::mutex> lk(h->mu);
  if ((st = host_stream(h))) return st;
  const auto* p = static_cast<const uint8_t*>(host);
  auto it = h->ranges.find(p);
  if (it != h->ranges.end() && it->second.first != bytes) {
    EFG_TRY_CUDA(cudaStreamSynchronize(h->stream), "stream synchronize");
    cudaFree(it->second.second);
    h->ranges.erase(it);
    it = h->ranges.end();
  }
  if (it == h->ranges.end()) {
    for (const auto& kv : h->ranges) {  // overlapping ranges would make lookups ambiguous
      if (p < kv.first + kv.second.first && kv.first < p + bytes)
        return fail(EFG_EINVAL, "register_weights: range overlaps a registered range");
    }
    void* d = nullptr;
    EFG_TRY_CUDA(cudaMalloc(&d, bytes), "resident weight allocation");
    it = h->ranges.emplace(p, std::make_pair(bytes, d)).first;
  }
  EFG_TRY_CUDA(cudaMemcpyAsync(it->second.second, host, bytes, cudaMemcpyHostToDevice, h->stream), "weight upload");
  EFG_TRY_CUDA(cudaStreamSynchronize(h->stream), "stream synchronize");
  return EFG_OK;
}

int efg_host_unregister_weights(const void* host) {
  int st;
  HostCtx* h = host_ctx(st);
  if (!h) return st;
  std::lock_guard<std::mutex> lk(h->mu);
  auto it = h->ranges.find(static_cast<const uint8_t*>(host));
  if (it == h->ranges.end()) return fail(EFG_EINVAL, "unregister_weights: range not registered");
  if (h->stream) EFG_TRY_CUDA(cudaStreamSynchronize(h->stream), "stream synchronize");
  cudaFree(it->second.second);
  h->ranges.erase(it);
  return EFG_OK;
}

int efg_host_release_weights(void) {
  int st;
  HostCtx* h = host_ctx(st);
  if (!h) return st;
  std::lock_guard<std::mutex> lk(h->mu);
  if (h->stream) EFG_TRY_CUDA(cudaStreamSynchronize(h->stream), "stream synchronize");
  for (auto& kv : h->ranges) cudaFree(kv.second.second);
  h->ranges.clear();
  return EFG_OK;
}

}  // extern "C"
