// Multi-GPU entry points of libb2g_gemm.so: M-row-slab sharding of C = A.B over NCCL.
//
// The reference is single-GPU; this is the partition BASELINE configs[4] asks for (32768^3 as
// M-row slabs over 1/2/4/8 GPUs, B broadcast once over NVLink, C written locally with no
// reduction).  NCCL is loaded at run time (dlopen of libnccl.so.2, which in a process that
// already loaded NCCL -- e.g. through torch -- resolves to that same library), so callers of
// the single-GPU entry points never need it.
//
// Pipelining: B is broadcast in row panels B[k0:k1, :] (contiguous in memory) on an internal
// stream; the slab GEMM of panel p waits only for that panel, so the transfer of panel p+1
// overlaps the GEMM of panel p.  Panel 0 overwrites C, later panels add into it (beta = 1, TMA
// reduce-add), each element receiving one addition per panel in panel order: deterministic.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "../../include/b2g_gemm.h"
#include "errors.h"

using b2g::kErrPeerFailed;

// Device error word of this file's kernels: 0, or kErrPeerFailed once a reduction found that a
// peer's part of the call had failed.
__device__ int g_shard_error;

int b2g::shard_device_error(int clear, int* value) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_shard_error, sizeof(int));
  if (e == cudaSuccess && clear) {
    const int z = 0;
    e = cudaMemcpyToSymbol(g_shard_error, &z, sizeof(int));
  }
  return (int)e;
}

namespace {

struct NcclApi {
  decltype(&ncclBroadcast) bcast = nullptr;
  decltype(&ncclReduceScatter) reduce_scatter = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclGetErrorString) errstr = nullptr;
  decltype(&ncclGetUniqueId) unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclCommCount) count = nullptr;
  decltype(&ncclCommUserRank) user_rank = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommFinalize) finalize = nullptr;
  std::string error;
};

int sfail(int code, const std::string& msg) {
  b2g::set_error(msg.c_str());
  return code;
}

NcclApi* nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.error = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    api.bcast = reinterpret_cast<decltype(api.bcast)>(dlsym(h, "ncclBroadcast"));
    api.reduce_scatter = reinterpret_cast<decltype(api.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(dlsym(h, "ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(dlsym(h, "ncclGroupEnd"));
    api.errstr = reinterpret_cast<decltype(api.errstr)>(dlsym(h, "ncclGetErrorString"));
    api.unique_id = reinterpret_cast<decltype(api.unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.init_rank = reinterpret_cast<decltype(api.init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(h, "ncclCommDestroy"));
    api.count = reinterpret_cast<decltype(api.count)>(dlsym(h, "ncclCommCount"));
    api.user_rank = reinterpret_cast<decltype(api.user_rank)>(dlsym(h, "ncclCommUserRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.init_rank_config =
        reinterpret_cast<decltype(api.init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
    api.async_error = reinterpret_cast<decltype(api.async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    api.abort = reinterpret_cast<decltype(api.abort)>(dlsym(h, "ncclCommAbort"));
    api.finalize = reinterpret_cast<decltype(api.finalize)>(dlsym(h, "ncclCommFinalize"));
    if (!api.bcast || !api.errstr || !api.unique_id || !api.init_rank || !api.destroy ||
        !api.count || !api.user_rank || !api.reduce_scatter || !api.all_gather ||
        !api.group_start || !api.group_end || !api.all_reduce || !api.init_rank_config ||
        !api.async_error || !api.abort || !api.finalize)
      api.error = "libnccl.so.2 lacks an expected symbol";
  });
  return api.error.empty() ? &api : nullptr;
}

int nccl_fail(ncclResult_t r, const char* what) {
  NcclApi* n = nccl();
  return sfail(B2G_ERR_NCCL,
               std::string(what) + ": " + (n ? n->errstr(r) : "NCCL unavailable"));
}

// Communicators this library aborted (after a bounded wait ran out).  Their handles are freed
// by NCCL; every entry point given one, or a plan built on one, refuses with B2G_ERR_NCCL
// instead of queueing work that could wait for a peer forever.
std::mutex g_abort_mu;
std::set<void*> g_aborted;

bool comm_aborted(void* comm) {
  std::lock_guard<std::mutex> lk(g_abort_mu);
  return g_aborted.count(comm) != 0;
}

int refuse_aborted() {
  return sfail(B2G_ERR_NCCL, "the communicator was aborted after a peer stopped answering");
}

// Abort `c` (its kernels in flight return) and remember that it is gone.
void abort_comm(ncclComm_t c) {
  NcclApi* n = nccl();
  if (n) n->abort(c);
  std::lock_guard<std::mutex> lk(g_abort_mu);
  g_aborted.insert(c);
}

double now_ms() {
  return std::chrono::duration<double, std::milli>(
             std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Result of an NCCL call on `c`.  A non-blocking communicator returns ncclInProgress while the
// call (or the communicator's set-up) completes in the background: poll its state, for at
// most the library's communicator timeout; if that runs out the communicator is aborted and
// the call reports B2G_ERR_TIMEOUT.
int nccl_settle(ncclComm_t c, ncclResult_t r, const char* what) {
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  if (r == ncclInProgress) {
    const double deadline = now_ms() + (double)b2g::comm_timeout_ms();
    ncclResult_t st = ncclInProgress;
    while (true) {
      if (n->async_error(c, &st) != ncclSuccess) st = ncclSystemError;
      if (st != ncclInProgress) break;
      if (now_ms() > deadline) {
        abort_comm(c);
        return sfail(B2G_ERR_TIMEOUT, std::string(what) +
                                          ": did not complete within the communicator timeout; "
                                          "the communicator was aborted");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    r = st;
  }
  if (r != ncclSuccess) return nccl_fail(r, what);
  return B2G_OK;
}

// Wait (bounded by the communicator timeout) for `s`, whose last work is an NCCL collective on
// `c`.  If the limit runs out the communicator is aborted (its kernels return) and the wait
// reports B2G_ERR_TIMEOUT.
int nccl_sync(ncclComm_t c, cudaStream_t s, const char* what) {
  const double deadline = now_ms() + (double)b2g::comm_timeout_ms();
  while (true) {
    const cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return B2G_OK;
    if (q != cudaErrorNotReady)
      return sfail(B2G_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(q));
    if (now_ms() > deadline) break;
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
  abort_comm(c);
  const double drain = now_ms() + 10000.0;
  while (cudaStreamQuery(s) == cudaErrorNotReady && now_ms() < drain)
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  return sfail(B2G_ERR_TIMEOUT, std::string(what) + ": a peer did not answer within the "
                                                    "communicator timeout; the communicator was "
                                                    "aborted");
}

// One non-blocking stream per device for the broadcasts.
cudaStream_t comm_stream(int dev) {
  static std::mutex mu;
  static cudaStream_t streams[64] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!streams[dev]) cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking);
  return streams[dev];
}

}  // namespace

extern "C" int b2g_slab_rows(int64_t M, int world, int rank, int64_t* row0, int64_t* rows) {
  if (M < 0 || world < 1 || rank < 0 || rank >= world || !row0 || !rows)
    return sfail(B2G_ERR_INVALID_ARG, "bad slab arguments");
  const int64_t base = M / world, rem = M % world;
  *rows = base + (rank < rem ? 1 : 0);
  *row0 = (int64_t)rank * base + std::min<int64_t>(rank, rem);
  return B2G_OK;
}

extern "C" int b2g_comm_unique_id(void* id_out) {
  if (!id_out) return sfail(B2G_ERR_INVALID_ARG, "null id buffer");
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  ncclUniqueId id;
  ncclResult_t r = n->unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(id_out, &id, sizeof(id));
  return B2G_OK;
}

extern "C" int b2g_comm_init(void** comm, int world, int rank, const void* id) {
  if (!comm || !id || world < 1 || rank < 0 || rank >= world)
    return sfail(B2G_ERR_INVALID_ARG, "bad communicator arguments");
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  // Non-blocking (the default): the set-up runs in the background and is polled here for at
  // most the communicator timeout, so a rank that never joins ends in an error, not a hang.
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = b2g::comm_nonblocking() ? 0 : 1;
  ncclResult_t r = n->init_rank_config(&c, world, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclCommInitRankConfig");
  {
    std::lock_guard<std::mutex> lk(g_abort_mu);
    g_aborted.erase(c);  // a new communicator may reuse a freed handle's address
  }
  const int rc = nccl_settle(c, r, "ncclCommInitRankConfig");
  if (rc != B2G_OK) return rc;
  *comm = c;
  return B2G_OK;
}

extern "C" int b2g_comm_destroy(void* comm) {
  if (!comm) return B2G_OK;
  {
    std::lock_guard<std::mutex> lk(g_abort_mu);
    if (g_aborted.erase(comm)) return B2G_OK;  // already freed by ncclCommAbort
  }
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  // flush this rank's operations (bounded), then free the communicator
  int rc = nccl_settle(c, n->finalize(c), "ncclCommFinalize");
  if (rc == B2G_ERR_TIMEOUT) {
    std::lock_guard<std::mutex> lk(g_abort_mu);
    g_aborted.erase(comm);  // aborted (freed) by the settle
    return rc;
  }
  ncclResult_t r = n->destroy(c);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclCommDestroy");
  return rc;
}

extern "C" int b2g_comm_check(void* comm, int64_t timeout_ms, void* stream) {
  b2g::set_error("");
  if (!comm || timeout_ms <= 0) return sfail(B2G_ERR_INVALID_ARG, "bad check arguments");
  if (comm_aborted(comm)) return refuse_aborted();
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return sfail(B2G_ERR_UNSUPPORTED, "device ordinal out of range");
  // one int per device for the liveness all-reduce (allocated at the first check)
  static std::mutex mu;
  static int32_t* word[64] = {};
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!word[dev] && cudaMalloc(&word[dev], 256) != cudaSuccess)
      return sfail(B2G_ERR_CUDA, "cudaMalloc(liveness word)");
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : comm_stream(dev);
  if (!s) return sfail(B2G_ERR_CUDA, "no communication stream");
  const double deadline = now_ms() + (double)timeout_ms;
  int rc = nccl_settle(c, n->all_reduce(word[dev], word[dev], 1, ncclInt32, ncclSum, c, s),
                       "ncclAllReduce(liveness)");
  if (rc != B2G_OK) return rc;
  // The all-reduce completes only when every rank has joined it.  Poll; if the limit runs
  // out, abort the communicator (its kernels in flight return) and report the peer as gone.
  while (true) {
    const cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return B2G_OK;
    if (q != cudaErrorNotReady) return sfail(B2G_ERR_CUDA, std::string("liveness check: ") +
                                                               cudaGetErrorString(q));
    ncclResult_t st = ncclSuccess;
    if (n->async_error(c, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
      abort_comm(c);
      return nccl_fail(st, "liveness check (communicator aborted)");
    }
    if (now_ms() > deadline) break;
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
  abort_comm(c);
  // the aborted all-reduce leaves the stream; wait for that (bounded) so it is usable again
  const double drain = now_ms() + 10000.0;
  while (cudaStreamQuery(s) == cudaErrorNotReady && now_ms() < drain)
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  return sfail(B2G_ERR_TIMEOUT, "liveness check: a peer did not answer within " +
                                    std::to_string(timeout_ms) +
                                    " ms; the communicator was aborted");
}

extern "C" int b2g_gemm_sharded(const void* A_slab, void* B, float* C_slab, int64_t M, int64_t N,
                                int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* comm,
                                int root, int k_panels, void* stream) {
  b2g::set_error("");
  if (M < 0 || N < 0 || K < 0 || !comm) return sfail(B2G_ERR_INVALID_ARG, "bad sharded arguments");
  if (ldb < std::max<int64_t>(N, 1)) return sfail(B2G_ERR_INVALID_ARG, "ldb < N");
  if (comm_aborted(comm)) return refuse_aborted();
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  int world = 0, rank = 0;
  ncclResult_t r = n->count(c, &world);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommCount");
  r = n->user_rank(c, &rank);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommUserRank");
  if (root < 0 || root >= world) return sfail(B2G_ERR_INVALID_ARG, "root out of range");
  int64_t row0 = 0, rows = 0;
  b2g_slab_rows(M, world, rank, &row0, &rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0;
  cudaGetDevice(&dev);
  cudaStream_t cs = comm_stream(dev);
  if (!cs) return sfail(B2G_ERR_CUDA, "no communication stream");

  // K panels: multiples of 64 (the kernel's K block) except possibly the last.
  int P = std::max(1, k_panels);
  int64_t kp = K > 0 ? (K + P - 1) / P : 0;
  kp = (kp + 63) / 64 * 64;
  if (kp == 0) P = 1;
  else P = (int)((K + kp - 1) / kp);

  cudaEvent_t start, done[64];
  if (P > 64) return sfail(B2G_ERR_INVALID_ARG, "at most 64 panels");
  cudaError_t e = cudaEventCreateWithFlags(&start, cudaEventDisableTiming);
  if (e != cudaSuccess) return sfail(B2G_ERR_CUDA, cudaGetErrorString(e));
  for (int p = 0; p < P; ++p) cudaEventCreateWithFlags(&done[p], cudaEventDisableTiming);
  // the broadcasts start after everything already queued on the caller's stream (e.g. the
  // root writing B)
  cudaEventRecord(start, s);
  cudaStreamWaitEvent(cs, start, 0);
  int rc = B2G_OK;
  for (int p = 0; p < P && rc == B2G_OK; ++p) {
    const int64_t k0 = (int64_t)p * kp, k1 = std::min<int64_t>(K, k0 + kp);
    if (k1 > k0) {
      char* bp = static_cast<char*>(B) + k0 * ldb * 2;
      rc = nccl_settle(c, n->bcast(bp, bp, (size_t)((k1 - k0) * ldb * 2), ncclUint8, root, c, cs),
                       "ncclBroadcast");
      if (rc != B2G_OK) break;
    }
    cudaEventRecord(done[p], cs);
    cudaStreamWaitEvent(s, done[p], 0);
    if (rows > 0) {
      const char* ap = static_cast<const char*>(A_slab) + k0 * 2;
      const char* bp = static_cast<const char*>(B) + k0 * ldb * 2;
      rc = b2g_gemm_ex(ap, bp, C_slab, rows, N, k1 - k0, lda, ldb, ldc, 1.0f,
                       p == 0 ? 0.0f : 1.0f, s);
    }
  }
  cudaEventDestroy(start);
  for (int p = 0; p < P; ++p) cudaEventDestroy(done[p]);
  return rc;
}

// ------------------------------------------------------------------ tensor-parallel variants
namespace {

// Stream-ordered scratch for the partial / gathered fp32 matrices of the sharded variants.
cudaMemPool_t shard_pool(int dev) {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    if (cudaMemPoolCreate(&pools[dev], &props) != cudaSuccess) return nullptr;
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
  }
  return pools[dev];
}

int comm_info(void* comm, int* world, int* rank) {
  if (comm_aborted(comm)) return refuse_aborted();
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  ncclResult_t r = n->count(static_cast<ncclComm_t>(comm), world);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommCount");
  r = n->user_rank(static_cast<ncclComm_t>(comm), rank);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommUserRank");
  return B2G_OK;
}

}  // namespace

extern "C" int b2g_gemm_sharded_k(const void* A_kslab, const void* B_kslab, float* C_slab,
                                  int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                  int64_t ldc, void* comm, void* stream) {
  b2g::set_error("");
  if (M < 0 || N < 0 || K < 0 || !comm) return sfail(B2G_ERR_INVALID_ARG, "bad sharded arguments");
  int world = 0, rank = 0;
  int rc = comm_info(comm, &world, &rank);
  if (rc) return rc;
  if (M % world != 0) return sfail(B2G_ERR_INVALID_ARG, "M must be a multiple of the rank count");
  if (ldc < std::max<int64_t>(N, 1)) return sfail(B2G_ERR_INVALID_ARG, "ldc < N");
  NcclApi* n = nccl();
  int64_t k0 = 0, kr = 0;
  b2g_slab_rows(K, world, rank, &k0, &kr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0;
  cudaGetDevice(&dev);
  cudaMemPool_t pool = shard_pool(dev);
  if (!pool) return sfail(B2G_ERR_CUDA, "no scratch pool");
  const int64_t rows = M / world;
  const bool direct = (ldc == N);  // the reduce-scatter can land in C_slab itself
  const size_t pbytes = (size_t)M * N * sizeof(float);
  const size_t tbytes = direct ? 0 : (size_t)rows * N * sizeof(float);
  void* scratch = nullptr;
  cudaError_t e = cudaMallocFromPoolAsync(&scratch, pbytes + tbytes + 256, pool, s);
  if (e != cudaSuccess) return sfail(B2G_ERR_CUDA, cudaGetErrorString(e));
  float* P = static_cast<float*>(scratch);
  float* recv = direct ? C_slab : reinterpret_cast<float*>(static_cast<char*>(scratch) + pbytes);
  // this rank's partial product over its K slab (kr == 0: zeros)
  rc = b2g_gemm_ex(A_kslab, B_kslab, P, M, N, kr, kr > 0 ? lda : 1, ldb, N, 1.0f, 0.0f, s);
  if (rc == B2G_OK) {
    rc = nccl_settle(static_cast<ncclComm_t>(comm),
                     n->reduce_scatter(P, recv, (size_t)rows * N, ncclFloat32, ncclSum,
                                       static_cast<ncclComm_t>(comm), s),
                     "ncclReduceScatter");
  }
  if (rc == B2G_OK && !direct && rows > 0) {
    e = cudaMemcpy2DAsync(C_slab, ldc * sizeof(float), recv, N * sizeof(float), N * sizeof(float),
                          rows, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) rc = sfail(B2G_ERR_CUDA, cudaGetErrorString(e));
  }
  cudaFreeAsync(scratch, s);
  return rc;
}

extern "C" int b2g_gemm_sharded_n(void* A, const void* B_nslab, float* C_nslab, int64_t M,
                                  int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                                  void* comm, int root, int m_panels, float* C_full,
                                  void* stream) {
  b2g::set_error("");
  if (M < 0 || N < 0 || K < 0 || !comm) return sfail(B2G_ERR_INVALID_ARG, "bad sharded arguments");
  int world = 0, rank = 0;
  int rc = comm_info(comm, &world, &rank);
  if (rc) return rc;
  if (root < 0 || root >= world) return sfail(B2G_ERR_INVALID_ARG, "root out of range");
  if (lda < std::max<int64_t>(K, 1)) return sfail(B2G_ERR_INVALID_ARG, "lda < K");
  if (C_full && N % world != 0)
    return sfail(B2G_ERR_INVALID_ARG, "the gathered C needs N to be a multiple of the rank count");
  NcclApi* n = nccl();
  int64_t n0 = 0, nr = 0;
  b2g_slab_rows(N, world, rank, &n0, &nr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0;
  cudaGetDevice(&dev);
  cudaStream_t cs = comm_stream(dev);
  if (!cs) return sfail(B2G_ERR_CUDA, "no communication stream");
  // A is broadcast in row panels (contiguous); the slab GEMM of a panel writes its own rows
  // of C, so panel p's GEMM overlaps panel p+1's transfer and nothing accumulates.
  const int P = std::max(1, std::min<int>(m_panels, 64));
  const int64_t mp = M > 0 ? (M + P - 1) / P : 0;
  cudaEvent_t start, done[64];
  cudaEventCreateWithFlags(&start, cudaEventDisableTiming);
  for (int p = 0; p < P; ++p) cudaEventCreateWithFlags(&done[p], cudaEventDisableTiming);
  cudaEventRecord(start, s);
  cudaStreamWaitEvent(cs, start, 0);
  for (int p = 0; p < P && rc == B2G_OK; ++p) {
    const int64_t m0 = (int64_t)p * mp, m1 = std::min<int64_t>(M, m0 + mp);
    if (m1 > m0) {
      char* ap = static_cast<char*>(A) + m0 * lda * 2;
      rc = nccl_settle(static_cast<ncclComm_t>(comm),
                       n->bcast(ap, ap, (size_t)((m1 - m0) * lda * 2), ncclUint8, root,
                                static_cast<ncclComm_t>(comm), cs),
                       "ncclBroadcast");
      if (rc != B2G_OK) break;
    }
    cudaEventRecord(done[p], cs);
    cudaStreamWaitEvent(s, done[p], 0);
    if (m1 > m0 && nr > 0)
      rc = b2g_gemm_ex(static_cast<const char*>(A) + m0 * lda * 2, B_nslab, C_nslab + m0 * ldc,
                       m1 - m0, nr, K, lda, ldb, ldc, 1.0f, 0.0f, s);
  }
  cudaEventDestroy(start);
  for (int p = 0; p < P; ++p) cudaEventDestroy(done[p]);
  if (rc != B2G_OK || !C_full) return rc;
  // all-gather the column slabs: [rank][M][N/world] in a scratch buffer, then into the
  // row-major full C (one strided copy per rank)
  const int64_t nw = N / world;
  cudaMemPool_t pool = shard_pool(dev);
  if (!pool) return sfail(B2G_ERR_CUDA, "no scratch pool");
  const size_t gbytes = (size_t)world * M * nw * sizeof(float);
  const size_t sbytes = (ldc == nw) ? 0 : (size_t)M * nw * sizeof(float);
  void* scratch = nullptr;
  cudaError_t e = cudaMallocFromPoolAsync(&scratch, gbytes + sbytes + 256, pool, s);
  if (e != cudaSuccess) return sfail(B2G_ERR_CUDA, cudaGetErrorString(e));
  float* G = static_cast<float*>(scratch);
  const float* send = C_nslab;
  if (sbytes) {  // pack the slab contiguously first
    float* packed = reinterpret_cast<float*>(static_cast<char*>(scratch) + gbytes);
    e = cudaMemcpy2DAsync(packed, nw * sizeof(float), C_nslab, ldc * sizeof(float),
                          nw * sizeof(float), M, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) rc = sfail(B2G_ERR_CUDA, cudaGetErrorString(e));
    send = packed;
  }
  if (rc == B2G_OK) {
    rc = nccl_settle(static_cast<ncclComm_t>(comm),
                     n->all_gather(send, G, (size_t)M * nw, ncclFloat32,
                                   static_cast<ncclComm_t>(comm), s),
                     "ncclAllGather");
  }
  for (int q = 0; q < world && rc == B2G_OK; ++q) {
    e = cudaMemcpy2DAsync(C_full + q * nw, N * sizeof(float), G + (size_t)q * M * nw,
                          nw * sizeof(float), nw * sizeof(float), M, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) rc = sfail(B2G_ERR_CUDA, cudaGetErrorString(e));
  }
  cudaFreeAsync(scratch, s);
  return rc;
}

// ------------------------------------------------------------------ copy-engine broadcast chain
// B reaches the ranks along a chain root -> root+1 -> ... through the copy engines: rank
// r pulls each K panel from the previous rank's buffer (CUDA IPC mapping, peer copy over
// NVLink) as soon as that rank has it, and tells the next rank so.  The signalling is done by
// stream memory operations on 32-bit epoch flags -- the upstream rank writes "panel p of call
// e is here" into the downstream rank's flag array, the downstream copy stream waits for it --
// so the broadcast occupies no SM and never waits on a kernel: the slab GEMMs keep every SM
// while the next panels travel.  (An NCCL broadcast kernel cannot be resident beside the
// persistent GEMM, which holds each SM's shared memory, so it only runs between GEMMs.)
namespace {

constexpr int kMaxPanels = 64;

using PFN_wait32 = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
using PFN_write32 = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
using PFN_range = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

struct DrvApi {
  PFN_wait32 wait32 = nullptr;
  PFN_write32 write32 = nullptr;
  PFN_range range = nullptr;
};

const DrvApi* drv() {
  static DrvApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char* name) -> void* {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess &&
          q == cudaDriverEntryPointSuccess)
        return p;
      return nullptr;
    };
    api.wait32 = reinterpret_cast<PFN_wait32>(get("cuStreamWaitValue32"));
    api.write32 = reinterpret_cast<PFN_write32>(get("cuStreamWriteValue32"));
    api.range = reinterpret_cast<PFN_range>(get("cuMemGetAddressRange"));
  });
  return (api.wait32 && api.write32 && api.range) ? &api : nullptr;
}

// What every rank publishes at plan creation (gathered over NCCL).
struct PeerInfo {
  cudaIpcMemHandle_t buf_handle;    // allocation holding the rank's B buffer
  uint64_t buf_offset;              // B buffer offset inside that allocation
  cudaIpcMemHandle_t flag_handle;   // the rank's flag array
  int64_t bytes;                    // B buffer size
  int32_t dev;
};

}  // namespace

struct b2g_chain_plan {
  ncclComm_t comm = nullptr;
  int world = 1, rank = 0, root = 0, prev = -1, next = -1, dev = 0;
  char* buf = nullptr;
  int64_t bytes = 0;
  uint32_t* flags = nullptr;          // [kMaxPanels] panel arrived (written by prev),
                                      // [kMaxPanels] done (written by next)
  char* prev_buf = nullptr;           // prev's B buffer, mapped here
  uint32_t* prev_flags = nullptr;     // prev's flag array, mapped here
  uint32_t* next_flags = nullptr;     // next's flag array, mapped here
  void* opened[3] = {nullptr, nullptr, nullptr};
  uint32_t epoch = 0;
  cudaStream_t cs = nullptr;
  cudaEvent_t start = nullptr, done_ev = nullptr, panel_ev[kMaxPanels] = {};
};

namespace {

void plan_free(b2g_chain_plan* p) {
  if (!p) return;
  for (void* o : p->opened)
    if (o) cudaIpcCloseMemHandle(o);
  if (p->flags) cudaFree(p->flags);
  if (p->cs) cudaStreamDestroy(p->cs);
  if (p->start) cudaEventDestroy(p->start);
  if (p->done_ev) cudaEventDestroy(p->done_ev);
  for (cudaEvent_t e : p->panel_ev)
    if (e) cudaEventDestroy(e);
  delete p;
}

int cuda_sfail(cudaError_t e, const char* what) {
  return sfail(B2G_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" int b2g_chain_plan_create(void* comm, void* B, int64_t bytes, int root, void** plan_out) {
  b2g::set_error("");
  if (!comm || !plan_out || bytes < 0 || (bytes > 0 && !B))
    return sfail(B2G_ERR_INVALID_ARG, "bad chain-plan arguments");
  *plan_out = nullptr;
  if (comm_aborted(comm)) return refuse_aborted();
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  const DrvApi* d = drv();
  if (!d) return sfail(B2G_ERR_UNSUPPORTED, "stream memory operations unavailable");
  auto* p = new b2g_chain_plan();
  p->comm = static_cast<ncclComm_t>(comm);
  ncclResult_t r = n->count(p->comm, &p->world);
  if (r == ncclSuccess) r = n->user_rank(p->comm, &p->rank);
  if (r != ncclSuccess) {
    plan_free(p);
    return nccl_fail(r, "ncclCommCount/UserRank");
  }
  if (root < 0 || root >= p->world) {
    plan_free(p);
    return sfail(B2G_ERR_INVALID_ARG, "root out of range");
  }
  p->root = root;
  p->buf = static_cast<char*>(B);
  p->bytes = bytes;
  cudaGetDevice(&p->dev);
  const int pos = (p->rank - root + p->world) % p->world;
  p->prev = pos > 0 ? (p->rank - 1 + p->world) % p->world : -1;
  p->next = pos < p->world - 1 ? (p->rank + 1) % p->world : -1;

  cudaError_t e = cudaMalloc(&p->flags, 2 * kMaxPanels * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(p->flags, 0, 2 * kMaxPanels * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->cs, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->start, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->done_ev, cudaEventDisableTiming);
  for (int i = 0; i < kMaxPanels && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&p->panel_ev[i], cudaEventDisableTiming);
  if (e != cudaSuccess) {
    plan_free(p);
    return cuda_sfail(e, "chain plan set-up");
  }
  int rc = B2G_OK;
  if (p->world > 1) {
    PeerInfo mine = {};
    CUdeviceptr base = 0;
    size_t sz = 0;
    if (bytes > 0 && d->range(&base, &sz, reinterpret_cast<CUdeviceptr>(B)) != CUDA_SUCCESS)
      rc = sfail(B2G_ERR_INVALID_ARG, "B is not device memory");
    if (rc == B2G_OK && bytes > 0) {
      e = cudaIpcGetMemHandle(&mine.buf_handle, reinterpret_cast<void*>(base));
      mine.buf_offset = reinterpret_cast<CUdeviceptr>(B) - base;
      if (e != cudaSuccess) rc = cuda_sfail(e, "cudaIpcGetMemHandle(B)");
    }
    if (rc == B2G_OK) {
      e = cudaIpcGetMemHandle(&mine.flag_handle, p->flags);
      if (e != cudaSuccess) rc = cuda_sfail(e, "cudaIpcGetMemHandle(flags)");
    }
    mine.bytes = bytes;
    mine.dev = p->dev;
    // gather everyone's handles (every rank takes part even after a local failure, so that no
    // rank is left waiting in the collective)
    void* dbuf = nullptr;
    const size_t one = sizeof(PeerInfo);
    e = cudaMalloc(&dbuf, one * (p->world + 1));
    if (e != cudaSuccess) {
      plan_free(p);
      return cuda_sfail(e, "cudaMalloc(handle exchange)");
    }
    cudaMemcpy(static_cast<char*>(dbuf) + one * p->world, &mine, one, cudaMemcpyHostToDevice);
    int xrc = nccl_settle(p->comm, n->all_gather(static_cast<char*>(dbuf) + one * p->world, dbuf,
                                                 one, ncclUint8, p->comm, p->cs),
                          "ncclAllGather(handles)");
    if (xrc == B2G_OK) xrc = nccl_sync(p->comm, p->cs, "handle exchange");
    std::vector<PeerInfo> all(p->world);
    if (xrc == B2G_OK) {
      e = cudaMemcpy(all.data(), dbuf, one * p->world, cudaMemcpyDeviceToHost);
      if (e != cudaSuccess && rc == B2G_OK) rc = cuda_sfail(e, "handle exchange");
    } else {
      cudaFree(dbuf);
      plan_free(p);
      return xrc;  // the communicator is unusable: no status exchange can follow
    }
    cudaFree(dbuf);
    if (rc == B2G_OK) {
      for (const PeerInfo& q : all)
        if (q.bytes != bytes) rc = sfail(B2G_ERR_INVALID_ARG, "B buffer sizes differ across ranks");
    }
    if (rc == B2G_OK && p->prev >= 0) {
      void* q = nullptr;
      if (bytes > 0) {
        e = cudaIpcOpenMemHandle(&q, all[p->prev].buf_handle, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) rc = cuda_sfail(e, "cudaIpcOpenMemHandle(previous rank's B)");
        p->opened[0] = q;
        p->prev_buf = static_cast<char*>(q) + all[p->prev].buf_offset;
      }
      if (rc == B2G_OK) {
        e = cudaIpcOpenMemHandle(&q, all[p->prev].flag_handle, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) rc = cuda_sfail(e, "cudaIpcOpenMemHandle(previous rank's flags)");
        p->opened[1] = q;
        p->prev_flags = static_cast<uint32_t*>(q);
      }
    }
    if (rc == B2G_OK && p->next >= 0) {
      void* q = nullptr;
      e = cudaIpcOpenMemHandle(&q, all[p->next].flag_handle, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) rc = cuda_sfail(e, "cudaIpcOpenMemHandle(next rank's flags)");
      p->opened[2] = q;
      p->next_flags = static_cast<uint32_t*>(q);
    }
    // Every rank learns every rank's outcome, so that all of them either keep the plan or
    // free it: a rank left holding a plan whose peer failed would wait for flags that never
    // come.
    int32_t* dst = nullptr;
    e = cudaMalloc(&dst, sizeof(int32_t) * (p->world + 1));
    if (e == cudaSuccess) {
      const int32_t mine_rc = rc;
      cudaMemcpy(dst + p->world, &mine_rc, sizeof(int32_t), cudaMemcpyHostToDevice);
      int xrc = nccl_settle(p->comm, n->all_gather(dst + p->world, dst, 1, ncclInt32, p->comm,
                                                   p->cs),
                            "ncclAllGather(status)");
      if (xrc == B2G_OK) xrc = nccl_sync(p->comm, p->cs, "chain plan status exchange");
      std::vector<int32_t> rcs(p->world, 0);
      if (xrc == B2G_OK &&
          cudaMemcpy(rcs.data(), dst, sizeof(int32_t) * p->world, cudaMemcpyDeviceToHost) ==
              cudaSuccess) {
        for (int q = 0; q < p->world; ++q)
          if (rcs[q] != B2G_OK && rc == B2G_OK)
            rc = sfail(rcs[q], "chain plan set-up failed on rank " + std::to_string(q));
      } else if (rc == B2G_OK) {
        rc = xrc != B2G_OK ? xrc : sfail(B2G_ERR_NCCL, "chain plan status exchange failed");
      }
      cudaFree(dst);
    } else if (rc == B2G_OK) {
      rc = cuda_sfail(e, "cudaMalloc(status exchange)");
    }
  }
  if (rc != B2G_OK) {
    plan_free(p);
    return rc;
  }
  *plan_out = p;
  return B2G_OK;
}

extern "C" int b2g_chain_plan_destroy(void* plan) {
  auto* p = static_cast<b2g_chain_plan*>(plan);
  if (!p) return B2G_OK;
  // Collective.  Every queued call (its copies and its final waits on the caller's stream)
  // finishes first; then each rank drops its mappings of the neighbours' memory, and only after
  // all ranks have done so (a small NCCL exchange) does anyone free the flag array the others
  // had mapped.
  cudaDeviceSynchronize();
  for (void*& o : p->opened) {
    if (o) cudaIpcCloseMemHandle(o);
    o = nullptr;
  }
  int rc = B2G_OK;
  // With an aborted communicator (a peer is gone) there is no barrier to take: the mappings
  // are dropped and this rank's memory is freed.
  if (p->world > 1 && !comm_aborted(p->comm)) {
    NcclApi* n = nccl();
    int32_t* d = nullptr;
    if (!n) {
      rc = sfail(B2G_ERR_NCCL, "NCCL unavailable");
    } else if (cudaMalloc(&d, sizeof(int32_t) * (p->world + 1)) != cudaSuccess) {
      rc = sfail(B2G_ERR_CUDA, "cudaMalloc(chain plan barrier)");
    } else {
      rc = nccl_settle(p->comm, n->all_gather(d + p->world, d, 1, ncclInt32, p->comm, p->cs),
                       "ncclAllGather(chain plan barrier)");
      if (rc == B2G_OK) rc = nccl_sync(p->comm, p->cs, "chain plan barrier");
      cudaFree(d);
    }
  }
  plan_free(p);
  return rc;
}

namespace {

// Row panels [r0, r1) of a buffer of `rows` rows: multiples of 64 rows except the last, the
// first two a quarter of the others (so that the first GEMM starts early) when there are peers.
std::vector<std::pair<int64_t, int64_t>> chain_panels(int64_t rows, int panels, int world) {
  const int P = std::max(1, std::min(panels, kMaxPanels - 2));
  int64_t kp = rows > 0 ? (rows + P - 1) / P : 0;
  kp = std::max<int64_t>(64, (kp + 63) / 64 * 64);
  std::vector<std::pair<int64_t, int64_t>> out;
  int64_t r0 = 0;
  const int64_t small = std::max<int64_t>(64, (kp / 4 + 63) / 64 * 64);
  for (int i = 0; r0 < rows; ++i) {
    const int64_t len = (i < 2 && world > 1) ? small : kp;
    out.emplace_back(r0, std::min(rows, r0 + len));
    r0 += len;
  }
  if (out.empty()) out.emplace_back(0, 0);
  return out;
}

// One call of the chain: rows [r0, r1) of panel i (row pitch `row_bytes`) are pulled from the
// previous rank (unless this is the root), announced to the next rank, and then handed to
// `on_panel(i, r0, r1)`, which queues its work on `s` after the panel has arrived.
template <typename F>
int chain_pipeline(b2g_chain_plan* p, const std::vector<std::pair<int64_t, int64_t>>& panels,
                   int64_t row_bytes, cudaStream_t s, F&& on_panel) {
  const DrvApi* d = drv();
  if (!d) return sfail(B2G_ERR_UNSUPPORTED, "stream memory operations unavailable");
  if (p->world > 1 && comm_aborted(p->comm)) return refuse_aborted();
  if ((int)panels.size() > kMaxPanels) return sfail(B2G_ERR_INVALID_ARG, "too many panels");
  if (!panels.empty() && panels.back().second * row_bytes > p->bytes)
    return sfail(B2G_ERR_INVALID_ARG, "the broadcast operand exceeds the plan's buffer");
  CUstream ccs = reinterpret_cast<CUstream>(p->cs);
  const uint32_t ep = ++p->epoch;
  const bool has_prev = p->prev >= 0, has_next = p->next >= 0;
  auto flag_ptr = [](uint32_t* base, int i) { return reinterpret_cast<CUdeviceptr>(base + i); };
  int rc = B2G_OK;
  auto cu = [&](CUresult r, const char* what) {
    if (r != CUDA_SUCCESS && rc == B2G_OK)
      rc = sfail(B2G_ERR_CUDA, std::string(what) + " failed (CUresult " + std::to_string((int)r) + ")");
  };
  auto rt = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && rc == B2G_OK) rc = cuda_sfail(e, what);
  };
  // the chain starts after everything queued on the caller's stream (the root writing the
  // operand, the previous call's GEMMs reading it)
  rt(cudaEventRecord(p->start, s), "cudaEventRecord");
  rt(cudaStreamWaitEvent(p->cs, p->start, 0), "cudaStreamWaitEvent");
  // this rank's buffer is overwritten only after the next rank finished pulling the previous
  // call's panels from it
  if (has_prev && has_next)
    cu(d->wait32(ccs, flag_ptr(p->flags, kMaxPanels), ep - 1, CU_STREAM_WAIT_VALUE_GEQ),
       "cuStreamWaitValue32(done)");
  for (size_t i = 0; i < panels.size() && rc == B2G_OK; ++i) {
    const int64_t r0 = panels[i].first, r1 = panels[i].second;
    const size_t off = (size_t)(r0 * row_bytes), len = (size_t)((r1 - r0) * row_bytes);
    if (has_prev) {
      cu(d->wait32(ccs, flag_ptr(p->flags, (int)i), ep, CU_STREAM_WAIT_VALUE_GEQ),
         "cuStreamWaitValue32(panel)");
      if (len)
        rt(cudaMemcpyAsync(p->buf + off, p->prev_buf + off, len, cudaMemcpyDeviceToDevice, p->cs),
           "cudaMemcpyAsync(peer panel)");
    }
    if (has_next)
      cu(d->write32(ccs, flag_ptr(p->next_flags, (int)i), ep, 0), "cuStreamWriteValue32(panel)");
    if (has_prev) {
      rt(cudaEventRecord(p->panel_ev[i], p->cs), "cudaEventRecord(panel)");
      rt(cudaStreamWaitEvent(s, p->panel_ev[i], 0), "cudaStreamWaitEvent(panel)");
    }
    if (rc == B2G_OK) rc = on_panel(i, r0, r1);
  }
  if (has_prev)  // tell the previous rank that its buffer is free again
    cu(d->write32(ccs, flag_ptr(p->prev_flags, kMaxPanels), ep, 0), "cuStreamWriteValue32(done)");
  // the call completes (on the caller's stream) once the copy stream is done and the next rank
  // has pulled everything from this rank's buffer
  rt(cudaEventRecord(p->done_ev, p->cs), "cudaEventRecord(done)");
  rt(cudaStreamWaitEvent(s, p->done_ev, 0), "cudaStreamWaitEvent(done)");
  if (has_next)
    cu(d->wait32(reinterpret_cast<CUstream>(s), flag_ptr(p->flags, kMaxPanels), ep,
                 CU_STREAM_WAIT_VALUE_GEQ),
       "cuStreamWaitValue32(next done)");
  return rc;
}

}  // namespace

extern "C" int b2g_gemm_sharded_chain(void* plan, const void* A_slab, float* C_slab, int64_t M,
                                      int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                                      int k_panels, void* stream) {
  b2g::set_error("");
  auto* p = static_cast<b2g_chain_plan*>(plan);
  if (!p || M < 0 || N < 0 || K < 0) return sfail(B2G_ERR_INVALID_ARG, "bad sharded arguments");
  if (ldb < std::max<int64_t>(N, 1)) return sfail(B2G_ERR_INVALID_ARG, "ldb < N");
  int64_t row0 = 0, rows = 0;
  b2g_slab_rows(M, p->world, p->rank, &row0, &rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // B arrives in K-row panels; the slab GEMM of panel i covers that K range (panel 0
  // overwrites C, the others add into it)
  return chain_pipeline(p, chain_panels(K, k_panels, p->world), ldb * 2, s,
                        [&](size_t i, int64_t k0, int64_t k1) -> int {
                          if (rows <= 0) return B2G_OK;
                          return b2g_gemm_ex(static_cast<const char*>(A_slab) + k0 * 2,
                                             p->buf + k0 * ldb * 2, C_slab, rows, N, k1 - k0, lda,
                                             ldb, ldc, 1.0f, i == 0 ? 0.0f : 1.0f, s);
                        });
}

extern "C" int b2g_chain_broadcast(void* plan, int64_t bytes, int panels, void* stream) {
  b2g::set_error("");
  auto* p = static_cast<b2g_chain_plan*>(plan);
  if (!p || bytes < 0) return sfail(B2G_ERR_INVALID_ARG, "bad broadcast arguments");
  if (bytes > p->bytes) return sfail(B2G_ERR_INVALID_ARG, "bytes exceed the plan's buffer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Panels in 64 KiB units (the chain's panel rule works on 64-row multiples; a row here is
  // 1 KiB), the last one holding the remainder bytes.
  const int64_t unit = 1024;
  const int64_t rows = (bytes + unit - 1) / unit;
  auto pan = chain_panels(rows, panels, p->world);
  for (auto& q : pan) {
    q.first = std::min(bytes, q.first * unit);
    q.second = std::min(bytes, q.second * unit);
  }
  return chain_pipeline(p, pan, 1, s, [](size_t, int64_t, int64_t) { return B2G_OK; });
}

extern "C" int b2g_gemm_sharded_n_chain(void* plan, const void* B_nslab, float* C_nslab, int64_t M,
                                        int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                        int64_t ldc, int m_panels, void* stream) {
  b2g::set_error("");
  auto* p = static_cast<b2g_chain_plan*>(plan);
  if (!p || M < 0 || N < 0 || K < 0) return sfail(B2G_ERR_INVALID_ARG, "bad sharded arguments");
  if (lda < std::max<int64_t>(K, 1)) return sfail(B2G_ERR_INVALID_ARG, "lda < K");
  int64_t n0 = 0, nr = 0;
  b2g_slab_rows(N, p->world, p->rank, &n0, &nr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // A arrives in row panels; panel i's GEMM writes rows [m0, m1) of this rank's column slab
  return chain_pipeline(p, chain_panels(M, m_panels, p->world), lda * 2, s,
                        [&](size_t, int64_t m0, int64_t m1) -> int {
                          if (nr <= 0 || m1 <= m0) return B2G_OK;
                          return b2g_gemm_ex(p->buf + m0 * lda * 2, B_nslab, C_nslab + m0 * ldc,
                                             m1 - m0, nr, K, lda, ldb, ldc, 1.0f, 0.0f, s);
                        });
}

// ------------------------------------------------------------------ peer-memory reduce-scatter
// K-split tensor parallelism with the reduce-scatter fused into the GEMMs.  Rank r computes its
// partial product A_r.B_r one row slab at a time, and the GEMM of slab q stores its tiles (the
// epilogue's TMA stores) straight into rank q's receive slot r, mapped here through CUDA IPC:
// the partials cross NVLink tile by tile while the next tiles are computed.  The other ranks'
// slabs go first, this rank's own slab last.  Epoch flags written and waited for by stream
// memory operations order the calls, so no kernel waits on another GPU:
//   - rank r writes into rank q's slots only after q has reduced the previous call's;
//   - after its GEMMs, rank r tells every peer that its partial has landed (the flag write
//     follows the GEMMs in stream order, behind a memory fence);
//   - rank r reduces its slots once every peer has said so, summing them in rank order
//     (deterministic), then tells every peer that its slots are free again.
struct b2g_rs_plan {
  ncclComm_t comm = nullptr;
  int world = 1, rank = 0, dev = 0;
  int64_t M = 0, N = 0, rows = 0;
  float* recv = nullptr;         // [world][rows][N]: slot s holds rank s's partial of my rows
  uint32_t* flags = nullptr;     // [world] partial of rank s landed, [world] rank q's slots free,
                                 // [world] call status of rank s (the epoch, or the epoch with
                                 // bit 31 set when that rank's part failed)
  std::vector<float*> peer_recv;       // rank q's receive slots, mapped here (q == rank: recv)
  std::vector<uint32_t*> peer_flags;   // rank q's flag array, mapped here
  std::vector<void*> opened;
  uint32_t epoch = 0;
  // Staged form (option "rs_stage" at plan creation): the partials of the peers' slabs are
  // computed into local buffers and pushed to the peers' slots by the copy engine on `copy`,
  // while the next GEMM runs.  min(2, world - 1) buffers of rows x N fp32.
  float* stage[2] = {nullptr, nullptr};
  int nstage = 0;
  cudaStream_t copy = nullptr;
  cudaEvent_t gemm_done[2] = {nullptr, nullptr}, copy_done[2] = {nullptr, nullptr};
  cudaEvent_t copies_done = nullptr;  // the last call's copies (the buffers may be rewritten)
};

namespace {

struct RsPeerInfo {
  cudaIpcMemHandle_t recv_handle;
  cudaIpcMemHandle_t flag_handle;
  int64_t M, N;
};

void rs_plan_free(b2g_rs_plan* p) {
  if (!p) return;
  for (void* o : p->opened)
    if (o) cudaIpcCloseMemHandle(o);
  if (p->recv) cudaFree(p->recv);
  if (p->flags) cudaFree(p->flags);
  for (int b = 0; b < 2; ++b) {
    if (p->stage[b]) cudaFree(p->stage[b]);
    if (p->gemm_done[b]) cudaEventDestroy(p->gemm_done[b]);
    if (p->copy_done[b]) cudaEventDestroy(p->copy_done[b]);
  }
  if (p->copies_done) cudaEventDestroy(p->copies_done);
  if (p->copy) cudaStreamDestroy(p->copy);
  delete p;
}

// C[i][j] = sum over s in rank order of R[s][i][j]: rows x N, slots `rows * N` floats apart.
// status[s] is the call status rank s wrote before announcing its partial: the call's epoch
// when its part succeeded.  If any peer's part failed, its slot holds a stale partial: C is
// filled with NaN instead and the library's device error word records ERR_PEER_FAILED.
__global__ void rs_reduce_kernel(const float* __restrict__ R, float* __restrict__ C, int64_t rows,
                                 int64_t N, int64_t ldc, int world, int vec,
                                 const uint32_t* status, uint32_t epoch, int self) {
  const int64_t slot = rows * N;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  bool peer_failed = false;
  for (int s = 0; s < world; ++s)
    if (s != self && __ldcv(status + s) != epoch) peer_failed = true;
  if (peer_failed) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(&g_shard_error, 0, kErrPeerFailed);
    const float nan = __int_as_float(0x7fc00000);
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < slot; v += stride) {
      const int64_t i = v / N, j = v - i * N;
      C[i * ldc + j] = nan;
    }
    return;
  }
  if (vec) {
    const int64_t n4 = N / 4;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < rows * n4; v += stride) {
      const int64_t i = v / n4, j = (v - i * n4) * 4;
      const float* src = R + i * N + j;
      float4 a = __ldcs(reinterpret_cast<const float4*>(src));
      for (int s = 1; s < world; ++s) {
        const float4 x = __ldcs(reinterpret_cast<const float4*>(src + s * slot));
        a.x += x.x;
        a.y += x.y;
        a.z += x.z;
        a.w += x.w;
      }
      *reinterpret_cast<float4*>(C + i * ldc + j) = a;
    }
  } else {
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < slot; v += stride) {
      const int64_t i = v / N, j = v - i * N;
      float a = R[v];
      for (int s = 1; s < world; ++s) a += R[v + s * slot];
      C[i * ldc + j] = a;
    }
  }
}

}  // namespace

extern "C" int b2g_rs_plan_create(void* comm, int64_t M, int64_t N, void** plan_out) {
  b2g::set_error("");
  if (!comm || !plan_out || M < 0 || N < 0) return sfail(B2G_ERR_INVALID_ARG, "bad plan arguments");
  *plan_out = nullptr;
  if (comm_aborted(comm)) return refuse_aborted();
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  if (!drv()) return sfail(B2G_ERR_UNSUPPORTED, "stream memory operations unavailable");
  auto* p = new b2g_rs_plan();
  p->comm = static_cast<ncclComm_t>(comm);
  ncclResult_t r = n->count(p->comm, &p->world);
  if (r == ncclSuccess) r = n->user_rank(p->comm, &p->rank);
  if (r != ncclSuccess) {
    rs_plan_free(p);
    return nccl_fail(r, "ncclCommCount/UserRank");
  }
  // every rank evaluates the same arguments, so an invalid M fails on all of them alike
  if (M % p->world != 0) {
    rs_plan_free(p);
    return sfail(B2G_ERR_INVALID_ARG, "M must be a multiple of the rank count");
  }
  p->M = M;
  p->N = N;
  p->rows = M / p->world;
  cudaGetDevice(&p->dev);
  const size_t rbytes = std::max<size_t>(16, (size_t)p->world * p->rows * N * sizeof(float));
  cudaError_t e = cudaMalloc(&p->recv, rbytes);
  if (e == cudaSuccess) e = cudaMalloc(&p->flags, 3 * p->world * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(p->flags, 0, 3 * p->world * sizeof(uint32_t));
  if (e == cudaSuccess && p->world > 1 && b2g::rs_stage()) {
    p->nstage = std::min(2, p->world - 1);
    const size_t sbytes = std::max<size_t>(16, (size_t)p->rows * N * sizeof(float));
    for (int b = 0; b < p->nstage && e == cudaSuccess; ++b) {
      e = cudaMalloc(&p->stage[b], sbytes);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->gemm_done[b], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->copy_done[b], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->copy, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->copies_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(p->copies_done, p->copy);
  }
  int rc = e == cudaSuccess ? B2G_OK : cuda_sfail(e, "reduce-scatter plan set-up");
  p->peer_recv.assign(p->world, nullptr);
  p->peer_flags.assign(p->world, nullptr);
  if (rc == B2G_OK) {
    p->peer_recv[p->rank] = p->recv;
    p->peer_flags[p->rank] = p->flags;
  }
  if (p->world > 1) {
    // Exchange the IPC handles of every rank's slots and flags.  Every rank takes part in both
    // collectives below even after a local failure, so that none is left waiting.
    RsPeerInfo mine = {};
    if (rc == B2G_OK) {
      e = cudaIpcGetMemHandle(&mine.recv_handle, p->recv);
      if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine.flag_handle, p->flags);
      if (e != cudaSuccess) rc = cuda_sfail(e, "cudaIpcGetMemHandle");
    }
    mine.M = M;
    mine.N = N;
    const size_t one = sizeof(RsPeerInfo);
    void* dbuf = nullptr;
    e = cudaMalloc(&dbuf, one * (p->world + 1));
    if (e != cudaSuccess) {
      rs_plan_free(p);
      return cuda_sfail(e, "cudaMalloc(handle exchange)");
    }
    cudaStream_t xs = nullptr;
    cudaStreamCreateWithFlags(&xs, cudaStreamNonBlocking);
    cudaMemcpy(static_cast<char*>(dbuf) + one * p->world, &mine, one, cudaMemcpyHostToDevice);
    int xrc = nccl_settle(p->comm, n->all_gather(static_cast<char*>(dbuf) + one * p->world, dbuf,
                                                 one, ncclUint8, p->comm, xs),
                          "ncclAllGather(handles)");
    if (xrc == B2G_OK) xrc = nccl_sync(p->comm, xs, "handle exchange");
    std::vector<RsPeerInfo> all(p->world);
    if (xrc == B2G_OK) {
      e = cudaMemcpy(all.data(), dbuf, one * p->world, cudaMemcpyDeviceToHost);
      if (e != cudaSuccess && rc == B2G_OK) rc = cuda_sfail(e, "handle exchange");
    } else {
      cudaFree(dbuf);
      cudaStreamDestroy(xs);
      rs_plan_free(p);
      return xrc;  // the communicator is unusable: no status exchange can follow
    }
    cudaFree(dbuf);
    if (rc == B2G_OK)
      for (const RsPeerInfo& q : all)
        if (q.M != M || q.N != N) rc = sfail(B2G_ERR_INVALID_ARG, "M or N differ across ranks");
    for (int q = 0; q < p->world && rc == B2G_OK; ++q) {
      if (q == p->rank) continue;
      void* a = nullptr;
      e = cudaIpcOpenMemHandle(&a, all[q].recv_handle, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        rc = cuda_sfail(e, "cudaIpcOpenMemHandle(peer slots)");
        break;
      }
      p->opened.push_back(a);
      p->peer_recv[q] = static_cast<float*>(a);
      e = cudaIpcOpenMemHandle(&a, all[q].flag_handle, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        rc = cuda_sfail(e, "cudaIpcOpenMemHandle(peer flags)");
        break;
      }
      p->opened.push_back(a);
      p->peer_flags[q] = static_cast<uint32_t*>(a);
    }
    // every rank learns every rank's outcome: all keep the plan or all free it
    int32_t* dst = nullptr;
    e = cudaMalloc(&dst, sizeof(int32_t) * (p->world + 1));
    if (e == cudaSuccess) {
      const int32_t mine_rc = rc;
      cudaMemcpy(dst + p->world, &mine_rc, sizeof(int32_t), cudaMemcpyHostToDevice);
      int xrc2 = nccl_settle(p->comm, n->all_gather(dst + p->world, dst, 1, ncclInt32, p->comm, xs),
                             "ncclAllGather(status)");
      if (xrc2 == B2G_OK) xrc2 = nccl_sync(p->comm, xs, "reduce-scatter plan status exchange");
      std::vector<int32_t> rcs(p->world, 0);
      if (xrc2 == B2G_OK &&
          cudaMemcpy(rcs.data(), dst, sizeof(int32_t) * p->world, cudaMemcpyDeviceToHost) ==
              cudaSuccess) {
        for (int q = 0; q < p->world; ++q)
          if (rcs[q] != B2G_OK && rc == B2G_OK)
            rc = sfail(rcs[q], "reduce-scatter plan set-up failed on rank " + std::to_string(q));
      } else if (rc == B2G_OK) {
        rc = xrc2 != B2G_OK ? xrc2
                            : sfail(B2G_ERR_NCCL, "reduce-scatter plan status exchange failed");
      }
      cudaFree(dst);
    } else if (rc == B2G_OK) {
      rc = cuda_sfail(e, "cudaMalloc(status exchange)");
    }
    cudaStreamDestroy(xs);
  }
  if (rc != B2G_OK) {
    rs_plan_free(p);
    return rc;
  }
  *plan_out = p;
  return B2G_OK;
}

extern "C" int b2g_rs_plan_destroy(void* plan) {
  auto* p = static_cast<b2g_rs_plan*>(plan);
  if (!p) return B2G_OK;
  // Collective: this rank's queued calls finish, it drops its mappings of the peers' memory,
  // and only after every rank has done so does anyone free the memory the others had mapped.
  cudaDeviceSynchronize();
  for (void*& o : p->opened) {
    if (o) cudaIpcCloseMemHandle(o);
    o = nullptr;
  }
  int rc = B2G_OK;
  if (p->world > 1 && !comm_aborted(p->comm)) {
    NcclApi* n = nccl();
    int32_t* d = nullptr;
    cudaStream_t xs = nullptr;
    if (!n) {
      rc = sfail(B2G_ERR_NCCL, "NCCL unavailable");
    } else if (cudaMalloc(&d, sizeof(int32_t) * (p->world + 1)) != cudaSuccess ||
               cudaStreamCreateWithFlags(&xs, cudaStreamNonBlocking) != cudaSuccess) {
      rc = sfail(B2G_ERR_CUDA, "reduce-scatter plan barrier set-up");
    } else {
      rc = nccl_settle(p->comm, n->all_gather(d + p->world, d, 1, ncclInt32, p->comm, xs),
                       "ncclAllGather(plan barrier)");
      if (rc == B2G_OK) rc = nccl_sync(p->comm, xs, "reduce-scatter plan barrier");
    }
    if (d) cudaFree(d);
    if (xs) cudaStreamDestroy(xs);
  }
  rs_plan_free(p);
  return rc;
}

extern "C" int b2g_gemm_sharded_k_p2p(void* plan, const void* A_kslab, const void* B_kslab,
                                      float* C_slab, int64_t M, int64_t N, int64_t K, int64_t lda,
                                      int64_t ldb, int64_t ldc, void* stream) {
  b2g::set_error("");
  auto* p = static_cast<b2g_rs_plan*>(plan);
  if (!p) return sfail(B2G_ERR_INVALID_ARG, "null plan");
  if (p->world > 1 && comm_aborted(p->comm)) return refuse_aborted();
  const DrvApi* d = drv();
  if (!d) return sfail(B2G_ERR_UNSUPPORTED, "stream memory operations unavailable");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUstream cs = reinterpret_cast<CUstream>(s);
  const uint32_t ep = ++p->epoch;
  const int W = p->world, R = p->rank;
  const int64_t rows = p->rows;
  int64_t k0 = 0, kr = 0;
  b2g_slab_rows(K, W, R, &k0, &kr);
  // From here on every flag of the protocol is written and waited for even after a local
  // error (which only skips this rank's GEMMs and reduction), so that no peer's stream is left
  // waiting for this rank.
  int rc = B2G_OK;
  if (M != p->M || N != p->N || K < 0)
    rc = sfail(B2G_ERR_INVALID_ARG, "M or N differ from the plan's, or K < 0");
  else if (ldc < std::max<int64_t>(N, 1))
    rc = sfail(B2G_ERR_INVALID_ARG, "ldc < N");
  else if (kr > 0 && (lda < kr || ldb < std::max<int64_t>(N, 1)))
    rc = sfail(B2G_ERR_INVALID_ARG, "lda < the K slab or ldb < N");
  auto flag = [](uint32_t* base, int i) { return reinterpret_cast<CUdeviceptr>(base + i); };
  auto cu = [&](CUresult r, const char* what) {
    if (r != CUDA_SUCCESS && rc == B2G_OK)
      rc = sfail(B2G_ERR_CUDA, std::string(what) + " failed (CUresult " + std::to_string((int)r) + ")");
  };
  // Three forms, all giving the same bits (slot s of rank q holds rank s's partial of q's rows
  // and C_slab is the sum of the slots in rank order):
  //  - staged (option "rs_stage", default): the peers' partials are computed into local
  //    buffers, and the copy engine pushes each to its peer's slot on the plan's copy stream
  //    while the next GEMM runs, so no GEMM stores over NVLink (measured: a GEMM whose C is a
  //    peer's memory runs 8-40% slower, its epilogue stalled on the link); the own partial
  //    goes to slot R and rs_reduce_kernel sums the slots;
  //  - direct: the GEMMs of the peers' slabs store their tiles straight into the peers' slots;
  //  - direct and fused (option "rs_fused"): as direct, but the own slab is computed last,
  //    after every peer's partial of it has landed, by a GEMM whose epilogue adds the peers'
  //    slots in rank order (its own product standing in for slot R) and stores C_slab; it
  //    needs the tensor-core path (16-byte aligned operands and pitches), and where the
  //    planner finds no tensor-core launch the own partial goes to slot R as in the others.
  const char* A_base = static_cast<const char*>(A_kslab);
  const int64_t lda_e = kr > 0 ? lda : 1;
  const bool stage = W > 1 && b2g::rs_stage() && p->nstage > 0;
  const bool fused = !stage && W > 1 && b2g::rs_fused() && rc == B2G_OK && rows > 0 && N > 0 &&
                     kr > 0 && N % 4 == 0 && ldc % 4 == 0 && lda % 8 == 0 && ldb % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(C_slab) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(A_base) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(B_kslab) & 15) == 0 &&
                     b2g_get_option("force_generic") == 0;
  const bool work = rows > 0 && N > 0;
  auto ce = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && rc == B2G_OK) rc = cuda_sfail(e, what);
  };
  CUstream ccs = reinterpret_cast<CUstream>(p->copy);
  // staged: the previous call's pushes out of the staging buffers finish before they are
  // rewritten (whatever stream that call ran on)
  if (stage) ce(cudaStreamWaitEvent(s, p->copies_done, 0), "cudaStreamWaitEvent(previous pushes)");
  // the partial of rows [q*rows, (q+1)*rows) goes to rank q's slot R; the other ranks first
  for (int t = 1; t <= W; ++t) {
    const int q = (R + t) % W;
    const char* A_q = A_base + (size_t)(q * rows) * lda_e * 2;
    if (q == R) {
      if (!fused && rc == B2G_OK && work)
        rc = b2g_gemm_ex(A_q, B_kslab, p->recv + (size_t)R * rows * N, rows, N, kr, lda_e, ldb, N,
                         1.0f, 0.0f, s);
      continue;
    }
    if (!stage) {
      // rank q has reduced the previous call's slots
      cu(d->wait32(cs, flag(p->flags, W + q), ep - 1, CU_STREAM_WAIT_VALUE_GEQ),
         "cuStreamWaitValue32(slots free)");
      if (rc == B2G_OK && work)
        rc = b2g_gemm_ex(A_q, B_kslab, p->peer_recv[q] + (size_t)R * rows * N, rows, N, kr, lda_e,
                         ldb, N, 1.0f, 0.0f, s);
      continue;
    }
    const int b = (t - 1) % p->nstage;
    if (t - 1 >= p->nstage)  // buffer b's earlier push in this call is done
      ce(cudaStreamWaitEvent(s, p->copy_done[b], 0), "cudaStreamWaitEvent(push done)");
    if (rc == B2G_OK && work)
      rc = b2g_gemm_ex(A_q, B_kslab, p->stage[b], rows, N, kr, lda_e, ldb, N, 1.0f, 0.0f, s);
    ce(cudaEventRecord(p->gemm_done[b], s), "cudaEventRecord(partial)");
    ce(cudaStreamWaitEvent(p->copy, p->gemm_done[b], 0), "cudaStreamWaitEvent(partial)");
    cu(d->wait32(ccs, flag(p->flags, W + q), ep - 1, CU_STREAM_WAIT_VALUE_GEQ),
       "cuStreamWaitValue32(slots free)");
    if (rc == B2G_OK && work)
      ce(cudaMemcpyAsync(p->peer_recv[q] + (size_t)R * rows * N, p->stage[b],
                         (size_t)rows * N * sizeof(float), cudaMemcpyDeviceToDevice, p->copy),
         "cudaMemcpyAsync(push partial)");
    ce(cudaEventRecord(p->copy_done[b], p->copy), "cudaEventRecord(push)");
  }
  if (stage) {  // the flags below announce partials that have arrived
    ce(cudaEventRecord(p->copies_done, p->copy), "cudaEventRecord(pushes)");
    ce(cudaStreamWaitEvent(s, p->copies_done, 0), "cudaStreamWaitEvent(pushes)");
  }
  // announce this rank's partials (the default write orders the GEMMs' stores before it), then
  // wait for every peer's.  The status word goes first: the epoch if this rank's part
  // succeeded, the epoch with bit 31 set if it did not, so that the peers' reductions do not
  // sum a stale partial as if it were this call's.
  const uint32_t st = rc == B2G_OK ? ep : (ep | 0x80000000u);
  for (int q = 0; q < W; ++q)
    if (q != R) cu(d->write32(cs, flag(p->peer_flags[q], 2 * W + R), st, 0), "cuStreamWriteValue32(status)");
  for (int q = 0; q < W; ++q)
    if (q != R) cu(d->write32(cs, flag(p->peer_flags[q], R), ep, 0), "cuStreamWriteValue32(landed)");
  for (int q = 0; q < W; ++q)
    if (q != R)
      cu(d->wait32(cs, flag(p->flags, q), ep, CU_STREAM_WAIT_VALUE_GEQ), "cuStreamWaitValue32(landed)");
  bool reduce = !fused;
  if (fused && rc == B2G_OK && work) {
    const char* A_own = A_base + (size_t)(R * rows) * lda_e * 2;
    rc = b2g::gemm_rank_sum(A_own, B_kslab, C_slab, rows, N, kr, lda_e, ldb, ldc, p->recv,
                            rows * N, W, R, p->flags + 2 * W, ep, s);
    if (rc == B2G_ERR_UNSUPPORTED) {  // no tensor-core launch: the unfused form
      rc = b2g_gemm_ex(A_own, B_kslab, p->recv + (size_t)R * rows * N, rows, N, kr, lda_e, ldb,
                       N, 1.0f, 0.0f, s);
      reduce = true;
    }
  }
  if (reduce && rc == B2G_OK && work) {
    const int vec = (N % 4 == 0 && ldc % 4 == 0 && (reinterpret_cast<uintptr_t>(C_slab) & 15) == 0);
    const int64_t items = vec ? rows * (N / 4) : rows * N;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p->dev);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, (int64_t)sms * 8));
    rs_reduce_kernel<<<grid, 256, 0, s>>>(p->recv, C_slab, rows, N, ldc, W, vec, p->flags + 2 * W,
                                          ep, R);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_sfail(e, "rs_reduce_kernel");
    else b2g::count_launch();
  }
  // this rank's slots may be overwritten by the next call
  for (int q = 0; q < W; ++q)
    if (q != R) cu(d->write32(cs, flag(p->peer_flags[q], W + R), ep, 0), "cuStreamWriteValue32(free)");
  return rc;
}
