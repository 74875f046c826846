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
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/b2g_gemm.h"
#include "errors.h"

namespace {

struct NcclApi {
  decltype(&ncclBroadcast) bcast = nullptr;
  decltype(&ncclGetErrorString) errstr = nullptr;
  decltype(&ncclGetUniqueId) unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclCommCount) count = nullptr;
  decltype(&ncclCommUserRank) user_rank = nullptr;
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
    api.errstr = reinterpret_cast<decltype(api.errstr)>(dlsym(h, "ncclGetErrorString"));
    api.unique_id = reinterpret_cast<decltype(api.unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.init_rank = reinterpret_cast<decltype(api.init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(h, "ncclCommDestroy"));
    api.count = reinterpret_cast<decltype(api.count)>(dlsym(h, "ncclCommCount"));
    api.user_rank = reinterpret_cast<decltype(api.user_rank)>(dlsym(h, "ncclCommUserRank"));
    if (!api.bcast || !api.errstr || !api.unique_id || !api.init_rank || !api.destroy ||
        !api.count || !api.user_rank)
      api.error = "libnccl.so.2 lacks an expected symbol";
  });
  return api.error.empty() ? &api : nullptr;
}

int nccl_fail(ncclResult_t r, const char* what) {
  NcclApi* n = nccl();
  return sfail(B2G_ERR_NCCL,
               std::string(what) + ": " + (n ? n->errstr(r) : "NCCL unavailable"));
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
  ncclResult_t r = n->init_rank(&c, world, uid, rank);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
  *comm = c;
  return B2G_OK;
}

extern "C" int b2g_comm_destroy(void* comm) {
  if (!comm) return B2G_OK;
  NcclApi* n = nccl();
  if (!n) return sfail(B2G_ERR_NCCL, "NCCL unavailable");
  ncclResult_t r = n->destroy(static_cast<ncclComm_t>(comm));
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommDestroy");
  return B2G_OK;
}

extern "C" int b2g_gemm_sharded(const void* A_slab, void* B, float* C_slab, int64_t M, int64_t N,
                                int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* comm,
                                int root, int k_panels, void* stream) {
  b2g::set_error("");
  if (M < 0 || N < 0 || K < 0 || !comm) return sfail(B2G_ERR_INVALID_ARG, "bad sharded arguments");
  if (ldb < std::max<int64_t>(N, 1)) return sfail(B2G_ERR_INVALID_ARG, "ldb < N");
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
      r = n->bcast(bp, bp, (size_t)((k1 - k0) * ldb * 2), ncclUint8, root, c, cs);
      if (r != ncclSuccess) {
        rc = nccl_fail(r, "ncclBroadcast");
        break;
      }
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
