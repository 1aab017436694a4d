// NCCL halo exchange of per-atom rows and the collective step result (include/ljx_halo.h).
//
// The reference moves feature rows between the XLA program and LAMMPS's MPI comm through an
// FFI callback that stages the rows, wakes the LAMMPS thread and blocks until the exchange is
// done (cpp/pjrt/model_comm.cpp:392-472, serviced by PairJaxKokkos's comm hooks,
// cpp/pair_jax_kokkos.cpp:444-571). Here an exchange is a few stream-ordered launches: per stage
// one gather kernel (the rows each peer needs, and the periodic self images), one grouped
// ncclSend/ncclRecv that receives straight into the ghost rows, and in reverse one scatter-add
// kernel. No host thread waits; the only host wait is the bounded one of ljx_read_result_all.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "halo_internal.h"
#include "ljx_halo.h"

namespace {

thread_local std::string g_create_error;

// NCCL entry points, bound once per process.
struct Nccl {
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
  std::string error;  // empty when every symbol was found
};

template <typename F>
bool bind(void *handle, const char *name, F &fn)
{
  fn = reinterpret_cast<F>(dlsym(handle, name));
  return fn != nullptr;
}

const Nccl &nccl()
{
  static Nccl api;
  static std::once_flag once;
  std::call_once(once, [] {
    // The copy the process already has (the framework that started the ranks loaded one), so
    // both sides share one NCCL; else the library path's libnccl.so.2, or LJX_NCCL_LIBRARY.
    void *h = nullptr;
    const char *env = std::getenv("LJX_NCCL_LIBRARY");
    if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char *why = dlerror();
      api.error = std::string("cannot load NCCL (libnccl.so.2): ") + (why ? why : "unknown");
      return;
    }
    const bool ok = bind(h, "ncclGetUniqueId", api.GetUniqueId) &&
                    bind(h, "ncclCommInitRank", api.CommInitRank) &&
                    bind(h, "ncclCommDestroy", api.CommDestroy) &&
                    bind(h, "ncclCommAbort", api.CommAbort) &&
                    bind(h, "ncclCommGetAsyncError", api.CommGetAsyncError) &&
                    bind(h, "ncclGroupStart", api.GroupStart) &&
                    bind(h, "ncclGroupEnd", api.GroupEnd) && bind(h, "ncclSend", api.Send) &&
                    bind(h, "ncclRecv", api.Recv) && bind(h, "ncclAllReduce", api.AllReduce) &&
                    bind(h, "ncclGetErrorString", api.GetErrorString);
    if (!ok) api.error = "the loaded NCCL library lacks a required symbol";
  });
  return api;
}

constexpr int kStageSwaps = 16;  // swaps per stage (LAMMPS brick comm: 2 per dimension and layer)
constexpr int kThreads = 256;

// One stage's swaps for the row kernels. Gather (forward): rows list[k] -> row at + k of either
// the row array (local self images) or the staging buffer (peers). Scatter-add (reverse): rows
// at + k of either array added into rows list[k]; the zero ranges clear received ghost rows.
struct StageRows {
  const int *list[kStageSwaps];
  long long at[kStageSwaps];  // destination (gather) or source (scatter) first row
  int local[kStageSwaps];     // 1: `at` indexes the row array, 0: the staging buffer
  int prefix[kStageSwaps + 1];
  long long zfirst[kStageSwaps];
  int zprefix[kStageSwaps + 1];
  int n;
};

__device__ __forceinline__ int find_swap(const int *prefix, int n, long long flat_row)
{
  int s = 0;
  while (s + 1 < n && flat_row >= prefix[s + 1]) ++s;
  return s;
}

__global__ void __launch_bounds__(kThreads)
k_halo_gather(const StageRows d, uint32_t *rows, uint32_t *stage, int words)
{
  const long long total = static_cast<long long>(d.prefix[d.n]) * words;
  for (long long flat = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; flat < total;
       flat += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = flat / words;
    const int w = static_cast<int>(flat - r * words);
    const int s = find_swap(d.prefix, d.n, r);
    const int k = static_cast<int>(r - d.prefix[s]);
    const uint32_t v = rows[static_cast<long long>(d.list[s][k]) * words + w];
    uint32_t *dst = d.local[s] ? rows : stage;
    dst[(d.at[s] + k) * words + w] = v;
  }
}

template <typename S>
__global__ void __launch_bounds__(kThreads)
k_halo_scatter_add(const StageRows d, S *rows, S *stage, int width, int zero)
{
  const long long adds = static_cast<long long>(d.prefix[d.n]) * width;
  const long long zeros = zero ? static_cast<long long>(d.zprefix[d.n]) * width : 0;
  for (long long flat = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       flat < adds + zeros; flat += static_cast<long long>(gridDim.x) * blockDim.x) {
    if (flat < adds) {
      const long long r = flat / width;
      const int w = static_cast<int>(flat - r * width);
      const int s = find_swap(d.prefix, d.n, r);
      const int k = static_cast<int>(r - d.prefix[s]);
      S *src = (d.local[s] ? rows : stage) + (d.at[s] + k) * width + w;
      // Several images (or swaps) may share an owner row: the add is atomic.
      atomicAdd(rows + static_cast<long long>(d.list[s][k]) * width + w, *src);
      if (zero && d.local[s]) *src = S(0);
    } else {
      // Ghost rows this stage received from peers; NCCL has already sent them back.
      const long long r = (flat - adds) / width;
      const int w = static_cast<int>((flat - adds) - r * width);
      const int s = find_swap(d.zprefix, d.n, r);
      const int k = static_cast<int>(r - d.zprefix[s]);
      rows[(d.zfirst[s] + k) * width + w] = S(0);
    }
  }
}

int flat_grid(long long items)
{
  const long long need = (items + kThreads - 1) / kThreads;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(need, 148LL * 8)));
}

}  // namespace

struct ljx_halo {
  ncclComm_t comm = nullptr;
  int rank = 0;
  int nranks = 1;
  int device = 0;
  int timeout_ms = 60000;
  int flags = 0;
  bool aborted = false;
  std::vector<ljx_swap> swaps;                  // ordered by stage, then as given
  std::vector<long long> buf_row;               // per swap: first staging row (peer swaps)
  std::vector<std::pair<int, int>> stage_span;  // [first swap, end) per stage, ascending
  int max_row_bytes = 0;
  void *stage = nullptr;
  size_t stage_bytes = 0;
  double *scalars = nullptr;
  double *host = nullptr;
  cudaEvent_t done = nullptr;
  long long launches = 0;
  std::string error;

  ~ljx_halo()
  {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    // An aborted communicator was already released by ncclCommAbort.
    if (comm && !aborted && nccl().CommDestroy) nccl().CommDestroy(comm);
    if (stage) cudaFree(stage);
    if (scalars) cudaFree(scalars);
    if (host) cudaFreeHost(host);
    if (done) cudaEventDestroy(done);
    if (prev >= 0) cudaSetDevice(prev);
  }

  bool local(const ljx_swap &s) const
  {
    return s.send_rank == rank && s.recv_rank == rank && !(flags & LJX_HALO_SELF_BY_NCCL);
  }
};

namespace {

ljx_status fail(ljx_halo *h, ljx_status st, const std::string &msg)
{
  h->error = msg;
  return st;
}

ljx_status nccl_fail(ljx_halo *h, ncclResult_t r, const char *what)
{
  const Nccl &api = nccl();
  return fail(h, LJX_ERR_CUDA,
              std::string(what) + ": " + (api.GetErrorString ? api.GetErrorString(r) : "NCCL error"));
}

struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int device)
  {
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
  }
  ~DeviceScope()
  {
    int now = -1;
    if (prev >= 0 && cudaGetDevice(&now) == cudaSuccess && now != prev) cudaSetDevice(prev);
  }
};

// The row-kernel view of the swaps [first, end) of one stage. Local swaps read (gather) or write
// (scatter) their ghost rows in place; peer swaps go through the staging buffer.
StageRows stage_rows(const ljx_halo *h, int first, int end)
{
  StageRows d{};
  d.n = end - first;
  d.prefix[0] = 0;
  d.zprefix[0] = 0;
  for (int q = 0; q < d.n; ++q) {
    const ljx_swap &s = h->swaps[first + q];
    const bool loc = h->local(s);
    d.list[q] = s.sendlist;
    d.local[q] = loc ? 1 : 0;
    d.at[q] = loc ? s.firstrecv : h->buf_row[first + q];
    d.prefix[q + 1] = d.prefix[q] + s.sendnum;
    d.zfirst[q] = s.firstrecv;
    d.zprefix[q + 1] = d.zprefix[q] + (loc ? 0 : s.recvnum);
  }
  return d;
}

bool row_shape(ljx_halo *h, int width, int elem_bytes, int &row_bytes)
{
  if (width <= 0 || (elem_bytes != 4 && elem_bytes != 8)) {
    fail(h, LJX_ERR_INVALID, "halo rows need width > 0 and 4- or 8-byte elements");
    return false;
  }
  row_bytes = width * elem_bytes;
  if (row_bytes > h->max_row_bytes) {
    fail(h, LJX_ERR_INVALID,
         "halo rows of " + std::to_string(row_bytes) + " bytes exceed the " +
             std::to_string(h->max_row_bytes) + " bytes the swap table was sized for");
    return false;
  }
  return true;
}

bool stage_has_peers(const ljx_halo *h, const std::pair<int, int> &span)
{
  for (int q = span.first; q < span.second; ++q)
    if (!h->local(h->swaps[q])) return true;
  return false;
}

}  // namespace

namespace ljx {

double *halo_scalars(ljx_halo *halo) { return halo ? halo->scalars : nullptr; }

ljx_status halo_reduce_fetch(ljx_halo *h, cudaStream_t s, int nsum, int nmax, int ncopy,
                             double *host, std::string &error)
{
  const Nccl &api = nccl();
  if (h->aborted) {
    error = "the halo's communicator was aborted after an earlier failure";
    return LJX_ERR_INVALID;
  }
  DeviceScope scope(h->device);
  ncclResult_t r = api.GroupStart();
  if (r == ncclSuccess && nsum > 0)
    r = api.AllReduce(h->scalars, h->scalars, nsum, ncclFloat64, ncclSum, h->comm, s);
  if (r == ncclSuccess && nmax > 0)
    r = api.AllReduce(h->scalars + nsum, h->scalars + nsum, nmax, ncclFloat64, ncclMax, h->comm, s);
  const ncclResult_t r2 = api.GroupEnd();
  if (r == ncclSuccess) r = r2;
  if (r != ncclSuccess) {
    error = std::string("ncclAllReduce: ") + api.GetErrorString(r);
    return LJX_ERR_CUDA;
  }
  if (cudaMemcpyAsync(h->host, h->scalars, ncopy * sizeof(double), cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaEventRecord(h->done, s) != cudaSuccess) {
    error = "cudaMemcpyAsync(halo result)";
    return LJX_ERR_CUDA;
  }
  // Bounded wait: a peer that never joins leaves the all-reduce waiting; after the timeout the
  // communicator is aborted, which ends the waiting NCCL kernels.
  const auto t0 = std::chrono::steady_clock::now();
  for (long long spin = 0;; ++spin) {
    const cudaError_t q = cudaEventQuery(h->done);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      error = std::string("halo wait: ") + cudaGetErrorString(q);
      return LJX_ERR_CUDA;
    }
    if ((spin & 255) == 255) {
      ncclResult_t async = ncclSuccess;
      api.CommGetAsyncError(h->comm, &async);
      const auto waited = std::chrono::duration_cast<std::chrono::milliseconds>(
                              std::chrono::steady_clock::now() - t0)
                              .count();
      const bool failed = async != ncclSuccess && async != ncclInProgress;
      if (failed || waited > h->timeout_ms) {
        api.CommAbort(h->comm);
        h->aborted = true;
        error = failed ? std::string("NCCL failed: ") + api.GetErrorString(async)
                       : "halo step did not complete within " + std::to_string(h->timeout_ms) +
                             " ms (a peer rank never joined); the communicator was aborted";
        return LJX_ERR_CUDA;
      }
      std::this_thread::yield();
    }
  }
  std::memcpy(host, h->host, ncopy * sizeof(double));
  return LJX_OK;
}

}  // namespace ljx

extern "C" {

const char *ljx_halo_create_error(void) { return g_create_error.c_str(); }

ljx_status ljx_halo_unique_id(unsigned char id[LJX_HALO_ID_BYTES])
{
  if (id == nullptr) return LJX_ERR_INVALID;
  const Nccl &api = nccl();
  if (!api.error.empty()) {
    g_create_error = api.error;
    return LJX_ERR_UNSUPPORTED;
  }
  static_assert(sizeof(ncclUniqueId) == LJX_HALO_ID_BYTES, "NCCL unique id size");
  ncclUniqueId uid;
  const ncclResult_t r = api.GetUniqueId(&uid);
  if (r != ncclSuccess) {
    g_create_error = std::string("ncclGetUniqueId: ") + api.GetErrorString(r);
    return LJX_ERR_CUDA;
  }
  std::memcpy(id, &uid, sizeof(uid));
  return LJX_OK;
}

ljx_status ljx_halo_create(const unsigned char id[LJX_HALO_ID_BYTES], int nranks, int rank,
                           int device, int timeout_ms, int flags, ljx_halo **out)
{
  if (id == nullptr || out == nullptr || nranks <= 0 || rank < 0 || rank >= nranks) {
    g_create_error = "ljx_halo_create: bad id, rank or rank count";
    return LJX_ERR_INVALID;
  }
  *out = nullptr;
  const Nccl &api = nccl();
  if (!api.error.empty()) {
    g_create_error = api.error;
    return LJX_ERR_UNSUPPORTED;
  }
  auto *h = new ljx_halo();
  h->rank = rank;
  h->nranks = nranks;
  h->device = device;
  h->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  h->flags = flags;
  DeviceScope scope(device);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  const ncclResult_t r = api.CommInitRank(&h->comm, nranks, uid, rank);
  if (r != ncclSuccess) {
    g_create_error = std::string("ncclCommInitRank: ") + api.GetErrorString(r);
    h->comm = nullptr;
    delete h;
    return LJX_ERR_CUDA;
  }
  if (cudaMalloc(reinterpret_cast<void **>(&h->scalars), ljx::kHaloScalars * sizeof(double)) !=
          cudaSuccess ||
      cudaMemset(h->scalars, 0, ljx::kHaloScalars * sizeof(double)) != cudaSuccess ||
      cudaMallocHost(reinterpret_cast<void **>(&h->host), ljx::kHaloScalars * sizeof(double)) !=
          cudaSuccess ||
      cudaEventCreateWithFlags(&h->done, cudaEventDisableTiming) != cudaSuccess) {
    g_create_error = "ljx_halo_create: device buffers";
    delete h;
    return LJX_ERR_CUDA;
  }
  *out = h;
  return LJX_OK;
}

void ljx_halo_destroy(ljx_halo *halo) { delete halo; }

const char *ljx_halo_error(const ljx_halo *halo) { return halo ? halo->error.c_str() : "null halo"; }

long long ljx_halo_launches(const ljx_halo *halo) { return halo ? halo->launches : 0; }

ljx_status ljx_halo_set_swaps(ljx_halo *h, const ljx_swap *swaps, int nswaps, int max_row_bytes)
{
  if (h == nullptr) return LJX_ERR_INVALID;
  if (nswaps < 0 || (nswaps > 0 && swaps == nullptr))
    return fail(h, LJX_ERR_INVALID, "swap table is missing");
  if (max_row_bytes <= 0 || max_row_bytes % 4)
    return fail(h, LJX_ERR_INVALID, "max_row_bytes must be a positive multiple of 4");
  std::vector<ljx_swap> table(swaps, swaps + nswaps);
  std::stable_sort(table.begin(), table.end(),
                   [](const ljx_swap &a, const ljx_swap &b) { return a.stage < b.stage; });
  std::map<int, int> per_stage;
  for (const ljx_swap &s : table) {
    if (s.send_rank < 0 || s.send_rank >= h->nranks || s.recv_rank < 0 || s.recv_rank >= h->nranks)
      return fail(h, LJX_ERR_INVALID, "swap rank outside the communicator");
    if (s.sendnum < 0 || s.recvnum < 0 || s.firstrecv < 0 || (s.sendnum > 0 && !s.sendlist))
      return fail(h, LJX_ERR_INVALID, "swap counts, first row or send list are invalid");
    if (h->local(s) && s.sendnum != s.recvnum)
      return fail(h, LJX_ERR_INVALID, "a self swap sends and receives the same number of rows");
    if (++per_stage[s.stage] > kStageSwaps)
      return fail(h, LJX_ERR_INVALID,
                  "more than " + std::to_string(kStageSwaps) + " swaps in one stage");
  }
  std::vector<long long> buf_row(table.size(), 0);
  long long rows = 0;
  for (size_t q = 0; q < table.size(); ++q) {
    if (h->local(table[q])) continue;
    buf_row[q] = rows;
    rows += table[q].sendnum;
  }
  const size_t bytes = static_cast<size_t>(std::max<long long>(rows, 1)) * max_row_bytes;
  DeviceScope scope(h->device);
  if (bytes > h->stage_bytes) {
    if (h->stage) cudaFree(h->stage);
    h->stage = nullptr;
    h->stage_bytes = 0;
    if (cudaMalloc(&h->stage, bytes) != cudaSuccess)
      return fail(h, LJX_ERR_CUDA, "cudaMalloc(halo staging)");
    h->stage_bytes = bytes;
  }
  h->swaps = std::move(table);
  h->buf_row = std::move(buf_row);
  h->max_row_bytes = max_row_bytes;
  h->stage_span.clear();
  for (size_t q = 0; q < h->swaps.size();) {
    size_t e = q;
    while (e < h->swaps.size() && h->swaps[e].stage == h->swaps[q].stage) ++e;
    h->stage_span.emplace_back(static_cast<int>(q), static_cast<int>(e));
    q = e;
  }
  return LJX_OK;
}

ljx_status ljx_halo_forward(ljx_halo *h, void *stream, void *rows, int width, int elem_bytes)
{
  if (h == nullptr) return LJX_ERR_INVALID;
  if (h->aborted) return fail(h, LJX_ERR_INVALID, "the halo's communicator was aborted");
  int rb = 0;
  if (!row_shape(h, width, elem_bytes, rb)) return LJX_ERR_INVALID;
  if (rows == nullptr && !h->swaps.empty()) return fail(h, LJX_ERR_INVALID, "rows are missing");
  const Nccl &api = nccl();
  auto s = static_cast<cudaStream_t>(stream);
  DeviceScope scope(h->device);
  auto *base = static_cast<unsigned char *>(rows);
  auto *stage = static_cast<unsigned char *>(h->stage);
  const int words = rb / 4;
  for (const auto &span : h->stage_span) {
    const StageRows d = stage_rows(h, span.first, span.second);
    if (d.prefix[d.n] > 0) {
      k_halo_gather<<<flat_grid(static_cast<long long>(d.prefix[d.n]) * words), kThreads, 0, s>>>(
          d, static_cast<uint32_t *>(rows), static_cast<uint32_t *>(h->stage), words);
      if (cudaGetLastError() != cudaSuccess) return fail(h, LJX_ERR_CUDA, "k_halo_gather");
      h->launches++;
    }
    if (!stage_has_peers(h, span)) continue;
    ncclResult_t r = api.GroupStart();
    for (int q = span.first; q < span.second && r == ncclSuccess; ++q) {
      const ljx_swap &sw = h->swaps[q];
      if (h->local(sw)) continue;
      if (sw.recvnum > 0)
        r = api.Recv(base + static_cast<size_t>(sw.firstrecv) * rb,
                     static_cast<size_t>(sw.recvnum) * rb, ncclUint8, sw.recv_rank, h->comm, s);
      if (r == ncclSuccess && sw.sendnum > 0)
        r = api.Send(stage + static_cast<size_t>(h->buf_row[q]) * rb,
                     static_cast<size_t>(sw.sendnum) * rb, ncclUint8, sw.send_rank, h->comm, s);
    }
    const ncclResult_t r2 = api.GroupEnd();
    if (r != ncclSuccess) return nccl_fail(h, r, "forward send/recv");
    if (r2 != ncclSuccess) return nccl_fail(h, r2, "ncclGroupEnd (forward)");
  }
  return LJX_OK;
}

ljx_status ljx_halo_reverse(ljx_halo *h, void *stream, void *rows, int width, int elem_bytes,
                            int zero_ghosts)
{
  if (h == nullptr) return LJX_ERR_INVALID;
  if (h->aborted) return fail(h, LJX_ERR_INVALID, "the halo's communicator was aborted");
  int rb = 0;
  if (!row_shape(h, width, elem_bytes, rb)) return LJX_ERR_INVALID;
  if (rows == nullptr && !h->swaps.empty()) return fail(h, LJX_ERR_INVALID, "rows are missing");
  const Nccl &api = nccl();
  auto s = static_cast<cudaStream_t>(stream);
  DeviceScope scope(h->device);
  auto *base = static_cast<unsigned char *>(rows);
  auto *stage = static_cast<unsigned char *>(h->stage);
  for (auto it = h->stage_span.rbegin(); it != h->stage_span.rend(); ++it) {
    const auto &span = *it;
    if (stage_has_peers(h, span)) {
      ncclResult_t r = api.GroupStart();
      for (int q = span.first; q < span.second && r == ncclSuccess; ++q) {
        const ljx_swap &sw = h->swaps[q];
        if (h->local(sw)) continue;
        // Ghost rows go back to the rank they came from; this rank's sent rows come back as
        // partial sums into the staging buffer.
        if (sw.recvnum > 0)
          r = api.Send(base + static_cast<size_t>(sw.firstrecv) * rb,
                       static_cast<size_t>(sw.recvnum) * rb, ncclUint8, sw.recv_rank, h->comm, s);
        if (r == ncclSuccess && sw.sendnum > 0)
          r = api.Recv(stage + static_cast<size_t>(h->buf_row[q]) * rb,
                       static_cast<size_t>(sw.sendnum) * rb, ncclUint8, sw.send_rank, h->comm, s);
      }
      const ncclResult_t r2 = api.GroupEnd();
      if (r != ncclSuccess) return nccl_fail(h, r, "reverse send/recv");
      if (r2 != ncclSuccess) return nccl_fail(h, r2, "ncclGroupEnd (reverse)");
    }
    const StageRows d = stage_rows(h, span.first, span.second);
    const long long items =
        (static_cast<long long>(d.prefix[d.n]) + (zero_ghosts ? d.zprefix[d.n] : 0)) * width;
    if (items <= 0) continue;
    if (elem_bytes == 8)
      k_halo_scatter_add<double><<<flat_grid(items), kThreads, 0, s>>>(
          d, static_cast<double *>(rows), static_cast<double *>(h->stage), width, zero_ghosts);
    else
      k_halo_scatter_add<float><<<flat_grid(items), kThreads, 0, s>>>(
          d, static_cast<float *>(rows), static_cast<float *>(h->stage), width, zero_ghosts);
    if (cudaGetLastError() != cudaSuccess) return fail(h, LJX_ERR_CUDA, "k_halo_scatter_add");
    h->launches++;
  }
  return LJX_OK;
}

ljx_status ljx_halo_allreduce_sum(ljx_halo *h, void *stream, double *values, int n)
{
  if (h == nullptr) return LJX_ERR_INVALID;
  if (h->aborted) return fail(h, LJX_ERR_INVALID, "the halo's communicator was aborted");
  if (n <= 0) return LJX_OK;
  if (values == nullptr) return fail(h, LJX_ERR_INVALID, "values are missing");
  DeviceScope scope(h->device);
  const ncclResult_t r = nccl().AllReduce(values, values, n, ncclFloat64, ncclSum, h->comm,
                                          static_cast<cudaStream_t>(stream));
  if (r != ncclSuccess) return nccl_fail(h, r, "ncclAllReduce");
  return LJX_OK;
}

}  // extern "C"
