// efg_shard.cpp - the row-sharded packed matvec across the GPUs of one node.
//
// Rank r of n holds the contiguous rows [rows*r/n, rows*(r+1)/n) of W (the split of the
// reference's ThreadPool::chunk_begin, include/ef/threadpool.h:52-54), computes that slice of
// y into its place in a full-size y, and the slices are exchanged in place over NVLink:
// one ncclAllGather when every rank holds the same number of rows, else one grouped
// ncclBroadcast per rank. The communicator is the library's own (ncclCommInitRank from a
// unique id the caller distributes); NCCL is loaded with dlopen on first use, so the
// library has no link-time NCCL dependency and shares the NCCL already loaded in the
// process (e.g. by torch) when there is one.
#include <dlfcn.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/efg.h"
#include "efg_argmax.cuh"
#include "efg_host.h"
#include "efg_matvec.cuh"

namespace efg {
namespace {

struct Nccl {
  bool tried = false, ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

Nccl g_nccl;
std::mutex g_nccl_mu;

template <class F>
bool sym(void* h, const char* name, F& f) {
  f = reinterpret_cast<F>(dlsym(h, name));
  return f != nullptr;
}

int load_nccl(Nccl** out) {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (!g_nccl.tried) {
    g_nccl.tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's NCCL, if loaded
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      g_nccl.ok = sym(h, "ncclGetUniqueId", g_nccl.get_unique_id) && sym(h, "ncclCommInitRank", g_nccl.comm_init_rank) &&
                  sym(h, "ncclCommDestroy", g_nccl.comm_destroy) && sym(h, "ncclAllGather", g_nccl.all_gather) &&
                  sym(h, "ncclBroadcast", g_nccl.broadcast) && sym(h, "ncclGroupStart", g_nccl.group_start) &&
                  sym(h, "ncclGroupEnd", g_nccl.group_end) && sym(h, "ncclGetErrorString", g_nccl.error_string);
    }
  }
  if (!g_nccl.ok) return fail(EFG_ENCCL, "NCCL (libnccl.so.2) could not be loaded");
  *out = &g_nccl;
  return EFG_OK;
}

int nccl_check(Nccl* n, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return EFG_OK;
  return fail(EFG_ENCCL, "%s: %s", what, n->error_string ? n->error_string(r) : "NCCL error");
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange from the driver, looked up once: the allocation that holds a pointer.
AddressRangeFn address_range_fn() {
  static const AddressRangeFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<AddressRangeFn>(f);
  }();
  return fn;
}

// What each rank tells the others when a buffer is registered for peer stores.
struct RegRecord {
  cudaIpcMemHandle_t buf;    // the allocation holding the buffer
  cudaIpcMemHandle_t flags;  // the rank's gather flag area
  uint64_t offset;           // of the buffer inside its allocation
  uint64_t bytes;
  int32_t ok;                // 0: this rank could not export its buffer
  int32_t pad;
};

}  // namespace
}  // namespace efg

// A buffer registered on every rank: this rank's copy and the mapped copies of the peers.
struct EfgRegBuf {
  uint8_t* local = nullptr;
  size_t bytes = 0;
  uint8_t* peer[efg::kMaxGatherRanks] = {};  // peer[rank] == local
  void* map_buf[efg::kMaxGatherRanks] = {};    // the peers' mapped allocations (to close)
  void* map_flags[efg::kMaxGatherRanks] = {};  // the peers' mapped flag areas (to close)
};

struct efg_comm {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0, device = -1;
  efg::ArgmaxPair* d_pairs = nullptr;  // one per rank: the row-sharded argmax's exchange
  // the in-kernel gather (efg_gather.cuh): flag areas and the registered buffers
  uint32_t* d_flags = nullptr;
  uint32_t* peer_flags[efg::kMaxGatherRanks] = {};
  std::map<std::string, std::pair<void*, int>> opened;  // peer IPC handle -> (mapping, users)
  std::vector<EfgRegBuf> bufs;
};

namespace efg {
namespace {

// All-gathers `n` bytes from every rank into all[nranks][n] (host memory), blocking.
int allgather_host(efg_comm* c, const void* mine, size_t n, void* all) {
  Nccl* nc = nullptr;
  if (int st = load_nccl(&nc)) return st;
  uint8_t* d = nullptr;
  cudaStream_t s = nullptr;
  int st = EFG_OK;
  if (cudaMalloc(&d, n * static_cast<size_t>(c->nranks + 1)) != cudaSuccess ||
      cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
    st = fail(EFG_ECUDA, "comm: exchange buffer");
  } else if (cudaMemcpyAsync(d + n * c->nranks, mine, n, cudaMemcpyHostToDevice, s) != cudaSuccess) {
    st = fail(EFG_ECUDA, "comm: exchange upload");
  } else if ((st = nccl_check(nc, nc->all_gather(d + n * c->nranks, d, n, ncclUint8, c->comm, s), "ncclAllGather"))) {
  } else if (cudaMemcpyAsync(all, d, n * c->nranks, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
             cudaStreamSynchronize(s) != cudaSuccess) {
    st = fail(EFG_ECUDA, "comm: exchange download");
  }
  if (s) cudaStreamDestroy(s);
  if (d) cudaFree(d);
  return st;
}

std::string handle_key(int rank, const cudaIpcMemHandle_t& h) {
  return std::to_string(rank) + ":" + std::string(reinterpret_cast<const char*>(&h), sizeof h);
}

// Maps rank q's allocation (reference counted per communicator).
void* open_peer(efg_comm* c, int q, const cudaIpcMemHandle_t& h) {
  const std::string key = handle_key(q, h);
  auto it = c->opened.find(key);
  if (it != c->opened.end()) {
    ++it->second.second;
    return it->second.first;
  }
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  c->opened.emplace(key, std::make_pair(p, 1));
  return p;
}

void close_peer(efg_comm* c, void* p) {
  for (auto it = c->opened.begin(); it != c->opened.end(); ++it) {
    if (it->second.first != p) continue;
    if (--it->second.second == 0) {
      cudaIpcCloseMemHandle(p);
      c->opened.erase(it);
    }
    return;
  }
}

const EfgRegBuf* registered(const efg_comm* c, const void* p, size_t n) {
  const auto* b = static_cast<const uint8_t*>(p);
  for (const EfgRegBuf& r : c->bufs)
    if (b >= r.local && static_cast<size_t>(b - r.local) <= r.bytes && n <= r.bytes - static_cast<size_t>(b - r.local))
      return &r;
  return nullptr;
}

}  // namespace
}  // namespace efg

using efg::fail;

extern "C" {

int efg_shard_rows(size_t rows, int nranks, int rank, size_t* begin, size_t* count) {
  if (nranks < 1 || rank < 0 || rank >= nranks || !begin || !count)
    return fail(EFG_EINVAL, "shard_rows: bad rank %d of %d", rank, nranks);
  const uint64_t b = static_cast<uint64_t>(rows) * static_cast<uint64_t>(rank) / static_cast<uint64_t>(nranks);
  const uint64_t e = static_cast<uint64_t>(rows) * static_cast<uint64_t>(rank + 1) / static_cast<uint64_t>(nranks);
  *begin = static_cast<size_t>(b);
  *count = static_cast<size_t>(e - b);
  return EFG_OK;
}

int efg_comm_unique_id(void* id) {
  if (!id) return fail(EFG_EINVAL, "comm_unique_id: null buffer");
  efg::Nccl* n = nullptr;
  if (int st = efg::load_nccl(&n)) return st;
  ncclUniqueId u;
  if (int st = efg::nccl_check(n, n->get_unique_id(&u), "ncclGetUniqueId")) return st;
  std::memcpy(id, &u, sizeof u);
  return EFG_OK;
}

int efg_comm_init(const void* id, int nranks, int rank, efg_comm** out) {
  if (!id || !out) return fail(EFG_EINVAL, "comm_init: null argument");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(EFG_EINVAL, "comm_init: bad rank %d of %d", rank, nranks);
  efg::Nccl* n = nullptr;
  if (int st = efg::load_nccl(&n)) return st;
  auto* c = new efg_comm;
  c->nranks = nranks;
  c->rank = rank;
  if (cudaGetDevice(&c->device) != cudaSuccess) {
    delete c;
    return fail(EFG_ECUDA, "comm_init: no current device");
  }
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof u);
  if (int st = efg::nccl_check(n, n->comm_init_rank(&c->comm, nranks, u, rank), "ncclCommInitRank")) {
    delete c;
    return st;
  }
  if (cudaMalloc(&c->d_pairs, sizeof(efg::ArgmaxPair) * static_cast<size_t>(nranks)) != cudaSuccess) {
    n->comm_destroy(c->comm);
    delete c;
    return fail(EFG_ECUDA, "comm_init: exchange buffer allocation");
  }
  *out = c;
  return EFG_OK;
}

int efg_comm_destroy(efg_comm* c) {
  if (!c) return EFG_OK;
  efg::Nccl* n = nullptr;
  int st = EFG_OK;
  if (c->device >= 0) cudaDeviceSynchronize();  // no kernel of ours may still store into a mapping
  for (auto& kv : c->opened) cudaIpcCloseMemHandle(kv.second.first);
  c->opened.clear();
  if (c->comm && efg::load_nccl(&n) == EFG_OK) st = efg::nccl_check(n, n->comm_destroy(c->comm), "ncclCommDestroy");
  if (c->d_pairs) cudaFree(c->d_pairs);
  if (c->d_flags) cudaFree(c->d_flags);
  delete c;
  return st;
}

int efg_comm_register(efg_comm* c, void* d_buf, size_t bytes) {
  using namespace efg;
  if (!c || !c->comm) return fail(EFG_EINVAL, "comm_register: null communicator");
  if (!d_buf || bytes == 0) return fail(EFG_EINVAL, "comm_register: empty buffer");
  int dev = -1;
  EFG_TRY_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != c->device)
    return fail(EFG_EINVAL, "comm_register: current device %d is not the communicator's device %d", dev, c->device);
  if (c->nranks > kMaxGatherRanks)  // the same on every rank: all of them return here
    return fail(EFG_EINVAL, "comm_register: peer stores are limited to %d ranks, this communicator has %d",
                kMaxGatherRanks, c->nranks);
  if (registered(c, d_buf, bytes)) return fail(EFG_EINVAL, "comm_register: buffer already registered");
  EfgRegBuf reg;
  reg.local = static_cast<uint8_t*>(d_buf);
  reg.bytes = bytes;
  reg.peer[c->rank] = reg.local;
  if (c->nranks == 1) {
    c->bufs.push_back(reg);
    return EFG_OK;
  }
  // this rank's record: the allocation holding the buffer and the flag area, exported
  RegRecord mine{};
  mine.bytes = bytes;
  mine.ok = 1;
  if (!c->d_flags) {
    if (cudaMalloc(&c->d_flags, kGatherFlagBytes) != cudaSuccess ||
        cudaMemset(c->d_flags, 0, kGatherFlagBytes) != cudaSuccess) {
      cudaGetLastError();
      if (c->d_flags) cudaFree(c->d_flags);
      c->d_flags = nullptr;
      mine.ok = 0;
    }
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  const AddressRangeFn range = address_range_fn();
  if (mine.ok && (!range || range(&base, &size, reinterpret_cast<CUdeviceptr>(d_buf)) != CUDA_SUCCESS ||
                  reinterpret_cast<uintptr_t>(d_buf) + bytes > base + size))
    mine.ok = 0;
  mine.offset = reinterpret_cast<uintptr_t>(d_buf) - base;
  if (mine.ok && (cudaIpcGetMemHandle(&mine.buf, reinterpret_cast<void*>(base)) != cudaSuccess ||
                  cudaIpcGetMemHandle(&mine.flags, c->d_flags) != cudaSuccess)) {
    cudaGetLastError();
    mine.ok = 0;
  }
  std::vector<RegRecord> all(static_cast<size_t>(c->nranks));
  if (int st = allgather_host(c, &mine, sizeof mine, all.data())) return st;
  // every rank maps every peer's buffer and flag area; then all agree on the outcome
  int32_t local_ok = 1;
  for (int q = 0; q < c->nranks; ++q)
    if (!all[q].ok || all[q].bytes != bytes) local_ok = 0;
  std::vector<void*> mapped;
  uint32_t* pflags[kMaxGatherRanks] = {};
  for (int q = 0; q < c->nranks && local_ok; ++q) {
    if (q == c->rank) continue;
    void* pb = open_peer(c, q, all[q].buf);
    void* pf = pb ? open_peer(c, q, all[q].flags) : nullptr;
    if (pb) mapped.push_back(pb);
    if (pf) mapped.push_back(pf);
    if (!pb || !pf) {
      local_ok = 0;
      break;
    }
    reg.peer[q] = static_cast<uint8_t*>(pb) + all[q].offset;
    reg.map_buf[q] = pb;
    reg.map_flags[q] = pf;
    pflags[q] = static_cast<uint32_t*>(pf);
  }
  std::vector<int32_t> oks(static_cast<size_t>(c->nranks));
  if (int st = allgather_host(c, &local_ok, sizeof local_ok, oks.data())) {
    for (void* p : mapped) close_peer(c, p);
    return st;
  }
  for (int32_t v : oks) {
    if (!v) {
      for (void* p : mapped) close_peer(c, p);
      return fail(EFG_ECUDA, "comm_register: a rank could not export or map the buffer for peer stores "
                             "(cudaMalloc'd memory of one process per GPU is required)");
    }
  }
  for (int q = 0; q < c->nranks; ++q) c->peer_flags[q] = q == c->rank ? c->d_flags : pflags[q];
  c->bufs.push_back(reg);
  return EFG_OK;
}

int efg_comm_deregister(efg_comm* c, void* d_buf) {
  using namespace efg;
  if (!c) return fail(EFG_EINVAL, "comm_deregister: null communicator");
  for (auto it = c->bufs.begin(); it != c->bufs.end(); ++it) {
    if (it->local != d_buf) continue;
    cudaDeviceSynchronize();
    for (int q = 0; q < c->nranks; ++q) {
      if (it->map_buf[q]) close_peer(c, it->map_buf[q]);
      if (it->map_flags[q]) close_peer(c, it->map_flags[q]);
    }
    c->bufs.erase(it);
    if (c->bufs.empty())  // the last registration held the peers' flag mappings
      for (int q = 0; q < c->nranks; ++q)
        if (q != c->rank) c->peer_flags[q] = nullptr;
    return EFG_OK;
  }
  return fail(EFG_EINVAL, "comm_deregister: buffer not registered");
}

int efg_matvec_sharded(int qtype, float* d_y, const uint8_t* d_W_shard, const float* d_x, size_t rows, size_t cols,
                       efg_comm* comm, void* stream) {
  using namespace efg;
  if (!comm || !comm->comm) return fail(EFG_EINVAL, "matvec_sharded: null communicator");
  if (qtype != EFG_Q4_0 && qtype != EFG_Q8_0)
    return fail(EFG_EINVAL, "matvec_sharded: type %d is not a packed type (Q4_0, Q8_0)", qtype);
  if (cols % 32 != 0)
    return fail(EFG_EINVAL, "%s needs a row length divisible by 32, got %zu", qtype == EFG_Q4_0 ? "Q4_0" : "Q8_0",
                cols);
  if (rows >= (1ull << 31)) return fail(EFG_EINVAL, "matvec_sharded: too many rows");
  int dev = -1;
  EFG_TRY_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != comm->device)
    return fail(EFG_EINVAL, "matvec_sharded: current device %d is not the communicator's device %d", dev,
                comm->device);
  if (rows == 0) return EFG_OK;
  if (!d_y) return fail(EFG_EINVAL, "matvec_sharded: null y");
  size_t b = 0, cnt = 0;
  if (int st = efg_shard_rows(rows, comm->nranks, comm->rank, &b, &cnt)) return st;
  auto s = static_cast<cudaStream_t>(stream);
  // The in-kernel gather: y registered on every rank (efg_comm_register) and at least one
  // row per rank, which every rank decides alike. Each CTA stores its outputs into every
  // rank's y; the launch returns once all ranks' rows are in this rank's y.
  const EfgRegBuf* reg = comm->nranks > 1 ? registered(comm, d_y, rows * sizeof(float)) : nullptr;
  if (reg && rows >= static_cast<size_t>(comm->nranks)) {
    if (cols == 0) {  // every dot is over zero blocks: every rank fills its whole y with 0
      EFG_TRY_CUDA(cudaMemsetAsync(d_y, 0, rows * sizeof(float), s), "matvec_sharded zero fill");
      return EFG_OK;
    }
    DeviceInfo* di = current_device();
    if (!di) return EFG_ECUDA;
    MatvecArgs a;
    a.fmt = qtype == EFG_Q4_0 ? Fmt::Q4 : Fmt::Q8;
    a.x = d_x;
    a.cols = cols;
    a.pdl = weight_prefetch_flag();
    a.n_jobs = 1;
    a.jobs[0] = MatvecJobDev{d_W_shard, d_y + b, static_cast<uint32_t>(cnt), 0};
    a.gather.nranks = comm->nranks;
    a.gather.rank = comm->rank;
    a.gather.flags = comm->d_flags;
    const size_t off = reinterpret_cast<const uint8_t*>(d_y) - reg->local;
    for (int q = 0; q < comm->nranks; ++q) {
      a.gather.peer_flags[q] = comm->peer_flags[q];
      a.gather.peer_y[q] = reinterpret_cast<float*>(reg->peer[q] + off) + b;
    }
    return launch_matvec(a, di->d_err, s);
  }
  if (cnt) {
    DeviceInfo* di = current_device();
    if (!di) return EFG_ECUDA;
    MatvecArgs a;
    a.fmt = qtype == EFG_Q4_0 ? Fmt::Q4 : Fmt::Q8;
    a.x = d_x;
    a.cols = cols;
    a.pdl = weight_prefetch_flag();
    a.n_jobs = 1;
    a.jobs[0] = MatvecJobDev{d_W_shard, d_y + b, static_cast<uint32_t>(cnt), 0};
    if (int st = launch_matvec(a, di->d_err, s)) return st;
  }
  if (comm->nranks == 1) return EFG_OK;
  Nccl* n = nullptr;
  if (int st = load_nccl(&n)) return st;
  if (rows % static_cast<size_t>(comm->nranks) == 0)  // in-place all-gather: send buffer = own slot
    return nccl_check(n, n->all_gather(d_y + b, d_y, cnt, ncclFloat32, comm->comm, s), "ncclAllGather");
  if (int st = nccl_check(n, n->group_start(), "ncclGroupStart")) return st;
  for (int r = 0; r < comm->nranks; ++r) {
    size_t rb = 0, rc = 0;
    efg_shard_rows(rows, comm->nranks, r, &rb, &rc);
    if (rc == 0) continue;
    const ncclResult_t res = n->broadcast(d_y + rb, d_y + rb, rc, ncclFloat32, r, comm->comm, s);
    if (res != ncclSuccess) {
      n->group_end();
      return nccl_check(n, res, "ncclBroadcast");
    }
  }
  return nccl_check(n, n->group_end(), "ncclGroupEnd");
}

int efg_lm_head_argmax_sharded(int qtype, float* d_logits_shard, int32_t* d_token, const uint8_t* d_W_shard,
                               const float* d_x, const float* d_norm_w, float eps, size_t rows, size_t cols,
                               efg_comm* comm, void* stream) {
  using namespace efg;
  if (!comm || !comm->comm) return fail(EFG_EINVAL, "lm_head_argmax_sharded: null communicator");
  if (qtype != EFG_Q4_0 && qtype != EFG_Q8_0)
    return fail(EFG_EINVAL, "lm_head_argmax_sharded: type %d is not a packed type (Q4_0, Q8_0)", qtype);
  if (cols % 32 != 0)
    return fail(EFG_EINVAL, "%s needs a row length divisible by 32, got %zu", qtype == EFG_Q4_0 ? "Q4_0" : "Q8_0",
                cols);
  if (rows == 0 || rows >= (1ull << 31)) return fail(EFG_EINVAL, "lm_head_argmax_sharded: bad row count %zu", rows);
  if (!d_token || !d_x) return fail(EFG_EINVAL, "lm_head_argmax_sharded: null pointer");
  int dev = -1;
  EFG_TRY_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != comm->device)
    return fail(EFG_EINVAL, "lm_head_argmax_sharded: current device %d is not the communicator's device %d", dev,
                comm->device);
  size_t b = 0, cnt = 0;
  if (int st = efg_shard_rows(rows, comm->nranks, comm->rank, &b, &cnt)) return st;
  auto s = static_cast<cudaStream_t>(stream);
  if (cnt) {
    if (!d_logits_shard || !d_W_shard) return fail(EFG_EINVAL, "lm_head_argmax_sharded: null shard pointer");
    DeviceInfo* di = current_device();
    if (!di) return EFG_ECUDA;
    MatvecArgs a;
    a.fmt = qtype == EFG_Q4_0 ? Fmt::Q4 : Fmt::Q8;
    a.x = d_x;
    a.norm_w = d_norm_w;
    a.norm_eps = eps;
    a.cols = cols;
    a.n_jobs = 1;
    a.jobs[0] = MatvecJobDev{d_W_shard, d_logits_shard, static_cast<uint32_t>(cnt), 0};
    if (int st = launch_matvec(a, di->d_err, s)) return st;
  }
  // Every rank's flag area mapped (some buffer registered, an outcome all ranks share): the
  // pairs travel by peer stores inside the argmax launch itself.
  bool mapped = comm->nranks > 1 && comm->nranks <= kMaxGatherRanks && comm->d_flags && !comm->bufs.empty();
  for (int q = 0; mapped && q < comm->nranks; ++q) mapped = comm->peer_flags[q] != nullptr;
  if (mapped) {
    DeviceInfo* di = current_device();
    if (!di) return EFG_ECUDA;
    GatherDev g;
    g.nranks = comm->nranks;
    g.rank = comm->rank;
    g.flags = comm->d_flags;
    for (int q = 0; q < comm->nranks; ++q) g.peer_flags[q] = comm->peer_flags[q];
    return launch_argmax_exchange(d_logits_shard, cnt, b, g, d_token, di->d_err, s);
  }
  ArgmaxPair* mine = comm->d_pairs + comm->rank;
  if (int st = launch_argmax_local(d_logits_shard, cnt, b, mine, s)) return st;
  if (comm->nranks > 1) {
    Nccl* n = nullptr;
    if (int st = load_nccl(&n)) return st;
    // in place: each rank's pair (8 bytes as two 4-byte words) lands in its slot everywhere
    if (int st = nccl_check(n, n->all_gather(mine, comm->d_pairs, 2, ncclFloat32, comm->comm, s), "ncclAllGather"))
      return st;
  }
  return launch_argmax_combine(comm->d_pairs, comm->nranks, d_token, s);
}

}  // extern "C"
