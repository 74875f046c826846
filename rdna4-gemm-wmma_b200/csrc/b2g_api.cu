// Host side of libb2g_gemm.so: the C ABI declared in include/b2g_gemm.h.
//
// Per call: validate shapes/strides, coalesce contraction modes whose strides allow it,
// classify the layout (K-major A; N- or K-contiguous B; N- or M-contiguous C), encode the
// TMA tensor maps directly on the caller's strides, pick one CTA or a CTA pair per tile,
// and launch the persistent tcgen05 kernel (gemm_sm100.cuh) on the caller's stream.
// Layouts outside TMA's addressing rules run on gemm_generic_kernel below, which computes
// exactly GEMM_Naive's arithmetic (mmm.cpp:52-62).  There is no host/CPU compute path.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/b2g_gemm.h"
#include "errors.h"
#include "plan.h"
#include "gemm_sm100.cuh"

namespace b2g {

// ------------------------------------------------------------------ errors / options
static thread_local std::string t_err;
static thread_local int t_path = B2G_PATH_NONE;
// Split-K workspace bytes (partial tiles) of the calling thread's last tensor-core launch: 0
// when it split nothing or reduced through distributed shared memory.
static thread_local int64_t t_split_ws = 0;
// Set while run() plans a call again without half-height pair tiles (see there).
static thread_local bool t_no_half = false;

static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

void set_error(const char* msg) { t_err = msg; }

static int cuda_fail(cudaError_t e, const char* what) {
  return fail(B2G_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static std::atomic<int64_t> opt_cta_group{0};
static std::atomic<int64_t> opt_raster_group{0};
static std::atomic<int64_t> opt_timeout_ns{2000000000LL};
static std::atomic<int64_t> opt_force_generic{0};
static std::atomic<int64_t> opt_fault_flags{0};
static std::atomic<int64_t> opt_tile_n{0};  // 0 = choose by shape, else 256 or 512
static std::atomic<int64_t> opt_store_hint{0};
static std::atomic<int64_t> opt_split_k{0};  // 0 = choose by shape, else the split count
static std::atomic<int64_t> opt_tail_split{1};  // split the tail wave's tiles (auto mode)
static std::atomic<int64_t> opt_pdl{1};  // launch with programmatic stream serialization
static std::atomic<int64_t> opt_pair_rows{0};  // 0 = choose, 64 = half-height pair tiles, 128 = never
static std::atomic<int64_t> opt_epi_warps{8};  // epilogue warps of the 256 x 512 pair tile (4 or 8)
static std::atomic<int64_t> opt_rs_fused{0};  // peer-memory K-split: rank-order sum in the own GEMM
static std::atomic<int64_t> opt_rs_stage{1};  // peer-memory K-split: partials pushed by the copy engine
// Kernels this library has launched (every GEMM, scale and fill kernel), for callers that
// count launches (b2g_get_option("launches")).
static std::atomic<int64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
static std::atomic<int64_t> opt_comm_timeout_ms{60000};  // bound of the library's NCCL waits
static std::atomic<int64_t> opt_comm_nonblocking{1};    // b2g_comm_init: non-blocking NCCL
int64_t comm_timeout_ms() { return opt_comm_timeout_ms.load(); }
bool comm_nonblocking() { return opt_comm_nonblocking.load() != 0; }
static std::atomic<int64_t> opt_cluster_fixup{1};  // split-K fix-up through distributed smem
static std::atomic<int64_t> opt_serial_fixup{0};  // 1 = always the last-arriver fix-up

// ------------------------------------------------------------------ driver entry point
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// ------------------------------------------------------------------ tensor-map cache
// A tensor map is a pure function of (base address, type, dims, strides, box, swizzle, L2
// promotion), so repeated calls on the same buffers reuse the encoded map instead of calling
// the driver again.  Small and bounded: cleared when full.
struct MapKey {
  uint64_t w[24];
  bool operator==(const MapKey& o) const { return std::memcmp(w, o.w, sizeof(w)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = 1469598103934665603ull;
    for (uint64_t x : k.w) h = (h ^ x) * 1099511628211ull;
    return (size_t)h;
  }
};
static std::mutex g_map_mu;
static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_map_cache;

static CUresult encode_cached(CUtensorMap* out, CUtensorMapDataType dt, cuuint32_t rank, void* addr,
                              const cuuint64_t* dims, const cuuint64_t* strides,
                              const cuuint32_t* box, CUtensorMapSwizzle swz,
                              CUtensorMapL2promotion l2) {
  MapKey key;
  std::memset(key.w, 0, sizeof(key.w));
  key.w[0] = (uint64_t)(uintptr_t)addr;
  key.w[1] = ((uint64_t)dt << 32) | ((uint64_t)rank << 24) | ((uint64_t)swz << 8) | (uint64_t)l2;
  for (cuuint32_t i = 0; i < rank; ++i) {
    key.w[2 + i] = dims[i];
    key.w[7 + i] = box[i];
    if (i + 1 < rank) key.w[12 + i] = strides[i];
  }
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_map_cache.find(key);
    if (it != g_map_cache.end()) {
      *out = it->second;
      return CUDA_SUCCESS;
    }
  }
  auto encode = get_encode();
  if (!encode) return CUDA_ERROR_NOT_SUPPORTED;
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  CUresult r = encode(out, dt, rank, addr, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      swz, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) {
    std::lock_guard<std::mutex> lk(g_map_mu);
    if (g_map_cache.size() >= 1024) g_map_cache.clear();
    g_map_cache.emplace(key, *out);
  }
  return r;
}

// ------------------------------------------------------------------ per-device state
struct DevState {
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  // [kind: 0 fp16, 1 fp8, 2 fp16 with the epilogue rank-order sum][variant][b_kmajor][c_mcontig]
  bool attr_set[3][6][2][2] = {};
  int max_clusters[3][6][2][2] = {};
  // clusters of s split units resident at once (cluster fix-up): one-CTA tiles, or s CTA pairs
  // of half-height pair tiles
  int max_clusters_cg1[3][6][2][2][9] = {};
};
static std::mutex g_dev_mu;
static DevState g_dev[64];

static int device_state(int dev, DevState** out) {
  if (dev < 0 || dev >= 64) return fail(B2G_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DevState& d = g_dev[dev];
  if (d.sm_count == 0) {
    cudaError_t e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
  }
  *out = &d;
  return B2G_OK;
}

// ------------------------------------------------------------------ generic kernel
// Any shape, any strides: one thread per C element, fp32 accumulator, K visited in
// ascending flattened (j, k) order -- GEMM_Naive's arithmetic (mmm.cpp:52-62).  With K == 0
// it writes zeros.  Used when TMA cannot address the operands.
struct Geo {
  int64_t as[5], ast[5];  // a,b,i,j,k
  int64_t bst[3];         // j,k,n strides
  int64_t b_batch;        // B stride along mode a (0: B is shared by every a)
  int64_t n;              // N
  int64_t cst[4];         // a,b,i,n strides
};

// Operand element -> float (exact for every supported type).
template <int DT>
__device__ __forceinline__ float elem_f32(const void* base, int64_t i) {
  if constexpr (DT == B2G_DTYPE_F16)
    return __half2float(static_cast<const __half*>(base)[i]);
  else if constexpr (DT == B2G_DTYPE_BF16)
    return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
  else if constexpr (DT == B2G_DTYPE_E4M3)
    return float(static_cast<const __nv_fp8_e4m3*>(base)[i]);
  else
    return float(static_cast<const __nv_fp8_e5m2*>(base)[i]);
}

// c_type: 0 = fp32 C (C = alpha*A.B + bias + beta*C), 1 = fp16 C, 2 = bf16 C (beta is 0 for
// the 16-bit types: C = round(alpha*A.B + bias)).  bias: per-column fp32 vector or null.
template <int DT>
__global__ void gemm_generic_kernel(const void* __restrict__ A, const void* __restrict__ B,
                                    void* __restrict__ C, const Geo g, float alpha, float beta,
                                    const float* __restrict__ bias, int c_type) {
  const int64_t rows = g.as[0] * g.as[1] * g.as[2];
  const int64_t total = rows * g.n;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / g.n, col = idx - row * g.n;
    const int64_t ii = row % g.as[2];
    const int64_t ib = (row / g.as[2]) % g.as[1];
    const int64_t ia = row / (g.as[2] * g.as[1]);
    const int64_t ar = ia * g.ast[0] + ib * g.ast[1] + ii * g.ast[2];
    const int64_t bc = col * g.bst[2] + ia * g.b_batch;
    float acc = 0.0f;
    for (int64_t j = 0; j < g.as[3]; ++j)
      for (int64_t k = 0; k < g.as[4]; ++k)
        acc += elem_f32<DT>(A, ar + j * g.ast[3] + k * g.ast[4]) *
               elem_f32<DT>(B, bc + j * g.bst[0] + k * g.bst[1]);
    const int64_t ci = ia * g.cst[0] + ib * g.cst[1] + ii * g.cst[2] + col * g.cst[3];
    float out = alpha == 1.0f ? acc : alpha * acc;
    if (bias) out += bias[col];
    if (c_type == 0) {
      float* c = static_cast<float*>(C) + ci;
      *c = beta == 0.0f ? out : out + beta * *c;  // beta == 0: C is not read
    } else if (c_type == 1) {
      static_cast<__half*>(C)[ci] = __float2half_rn(out);
    } else {
      static_cast<__nv_bfloat16*>(C)[ci] = __float2bfloat16_rn(out);
    }
  }
}

// C *= beta over the strided (a, b, i, n) view (the beta part of C = alpha*A.B + beta*C when
// the tensor-core kernel then adds alpha*A.B with a TMA reduce).
__global__ void scale_c_kernel(float* __restrict__ C, const Geo g, float beta) {
  const int64_t total = g.as[0] * g.as[1] * g.as[2] * g.n;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / g.n, col = idx - row * g.n;
    const int64_t ii = row % g.as[2];
    const int64_t ib = (row / g.as[2]) % g.as[1];
    const int64_t ia = row / (g.as[2] * g.as[1]);
    float* c = C + ia * g.cst[0] + ib * g.cst[1] + ii * g.cst[2] + col * g.cst[3];
    *c = beta * *c;
  }
}

// ------------------------------------------------------------------ RNG kernel
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

template <int DT>
__global__ void fill_uniform_kernel(void* __restrict__ dst, int64_t n, uint64_t seed,
                                    uint64_t offset) {
  const uint64_t key = mix64(seed);
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t h = mix64(key + offset + (uint64_t)e);
    const int32_t r = (int32_t)(h >> 40) - 8388608;
    const float v = (float)r * (1.0f / 8388608.0f);  // exact; rounded to nearest even below
    if constexpr (DT == B2G_DTYPE_F16)
      static_cast<__half*>(dst)[e] = __float2half_rn(v);
    else if constexpr (DT == B2G_DTYPE_BF16)
      static_cast<__nv_bfloat16*>(dst)[e] = __float2bfloat16_rn(v);
    else if constexpr (DT == B2G_DTYPE_E4M3)
      static_cast<__nv_fp8_e4m3*>(dst)[e] = __nv_fp8_e4m3(v);
    else
      static_cast<__nv_fp8_e5m2*>(dst)[e] = __nv_fp8_e5m2(v);
  }
}

// ------------------------------------------------------------------ split-K workspace pool
// Stream-ordered pool of the split-K workspaces, one per device, that keeps freed memory for
// reuse (release threshold: unlimited) instead of returning it to the driver at every
// synchronisation as the default pool does.
static int split_pool(cudaMemPool_t* out) {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B2G_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    e = cudaMemPoolCreate(&pool, &props);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemPoolCreate(split-K)");
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    pools[dev] = pool;
  }
  *out = pools[dev];
  return B2G_OK;
}

// ------------------------------------------------------------------ fixed scratch
// Split-K scratch for b2g_gemm_f16_f32_noalloc: a file-scope device array, so that entry point
// never allocates.  Each device that loads the library holds it until the process exits.
// Host code must not use `g_noalloc_scratch` as an address (on the host it is only a stand-in
// symbol); its device address comes from cudaGetSymbolAddress, once per device.
constexpr size_t kNoAllocScratchBytes = (size_t)32 << 20;  // 32 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct FixedScratch {
  void* ptr;
  size_t bytes;
};

// Device address of g_noalloc_scratch on the current device (set-up on the first call).
static int noalloc_scratch(FixedScratch* out) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B2G_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    addr[dev] = p;
  }
  out->ptr = addr[dev];
  out->bytes = kNoAllocScratchBytes;
  return B2G_OK;
}

// ------------------------------------------------------------------ split-K counters
// Arrival counters of split tiles come from a per-device ring in a file-scope device array
// (zero at module load).  Every kernel returns the counters it used to zero (the last unit of
// each split tile resets its counter), so a call needs no memset: it takes the next range of
// the ring.  A kernel that gave up on a bounded wait may leave counters non-zero; clearing the
// device error (b2g_device_status(1)) marks the ring for one full reset before its next use.
// Calls captured into a CUDA graph do not use the ring (a graph replays fixed addresses long
// after the ring has moved on); they zero their counters with a memset node instead.
//
// Streams: calls on several streams share the ring.  Each call that takes counters records an
// event on its stream after its launch (under the ring's lock, so no other call can wrap the
// ring in between).  Before the ring wraps to its start, or is reset, the calling stream waits
// for the last such event of every other stream that used the ring since the previous wrap, so
// a range is never handed out again while a kernel on another stream may still use it.
constexpr size_t kCounterSlots = (size_t)1 << 20;  // 4 MiB of ints per device
static __device__ int g_split_counters[kCounterSlots];

struct CounterRing {
  int* base = nullptr;
  size_t next = 0;
  bool dirty = false;
  std::vector<std::pair<cudaStream_t, cudaEvent_t>> users;  // since the last wrap
  std::vector<cudaEvent_t> spare;
};
static std::mutex g_ring_mu;
static CounterRing g_ring[64];

// Holds the ring of one device locked from the hand-out of a range until the launch that uses
// it has been recorded (commit), or until it goes out of scope.
struct RingLease {
  std::unique_lock<std::mutex> lk;
  CounterRing* ring = nullptr;
  RingLease() : lk(g_ring_mu, std::defer_lock) {}
  // after the launch: record this stream's use of the ring
  void commit(cudaStream_t stream) {
    if (!ring) return;
    cudaEvent_t ev = nullptr;
    for (auto& u : ring->users)
      if (u.first == stream) ev = u.second;
    if (!ev) {
      if (!ring->spare.empty()) {
        ev = ring->spare.back();
        ring->spare.pop_back();
      } else if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
        ev = nullptr;
      }
      if (ev) ring->users.emplace_back(stream, ev);
    }
    if (ev) cudaEventRecord(ev, stream);
    ring = nullptr;
    lk.unlock();
  }
};

// The calling stream waits for every other stream's last use of the ring; the list restarts.
static int ring_fence(CounterRing& r, cudaStream_t stream) {
  for (auto& u : r.users) {
    if (u.first != stream) {
      cudaError_t e = cudaStreamWaitEvent(stream, u.second, 0);
      if (e != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent(split-K counter ring)");
    }
    r.spare.push_back(u.second);
  }
  r.users.clear();
  return B2G_OK;
}

// `n` zeroed counters on the current device, or nullptr when `n` is too large for the ring.
// On success with a non-null range the lease holds the ring until lease.commit(stream).
static std::atomic<int64_t> opt_ring_slots{(int64_t)kCounterSlots};  // test knob: usable slots

static int ring_counters(size_t n, cudaStream_t stream, int** out, RingLease* lease) {
  *out = nullptr;
  const size_t cap = std::min(kCounterSlots, (size_t)opt_ring_slots.load());
  if (n == 0 || n > cap / 8) return B2G_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B2G_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  lease->lk.lock();
  CounterRing& r = g_ring[dev];
  if (!r.base) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_split_counters);
    if (e != cudaSuccess) {
      lease->lk.unlock();
      return cuda_fail(e, "cudaGetSymbolAddress(split-K counters)");
    }
    r.base = static_cast<int*>(p);
  }
  const size_t m = (n + 63) / 64 * 64;  // 256-byte granules
  const bool wrap = r.next + m > cap;
  if (r.dirty || wrap) {
    int rc = ring_fence(r, stream);
    if (rc != B2G_OK) {
      lease->lk.unlock();
      return rc;
    }
  }
  if (r.dirty) {
    e = cudaMemsetAsync(r.base, 0, kCounterSlots * sizeof(int), stream);
    if (e != cudaSuccess) {
      lease->lk.unlock();
      return cuda_fail(e, "cudaMemsetAsync(split-K counter ring)");
    }
    r.dirty = false;
    r.next = 0;
  }
  if (r.next + m > cap) r.next = 0;
  *out = r.base + r.next;
  r.next += m;
  lease->ring = &r;
  return B2G_OK;
}

static void ring_mark_dirty() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
  std::lock_guard<std::mutex> lk(g_ring_mu);
  g_ring[dev].dirty = true;
}

// ------------------------------------------------------------------ planning
struct Mode {
  int64_t size, sa, sc;  // extent, stride in the first operand, stride in the second
};

// Merge adjacent modes (outer first) whose strides in both operands are "outer = inner *
// size_inner"; drop size-1 modes.  Returns the number of modes kept, innermost last.
static int coalesce(Mode* m, int n) {
  Mode out[5];
  int k = 0;
  for (int t = 0; t < n; ++t)
    if (m[t].size != 1) out[k++] = m[t];
  bool merged = true;
  while (merged) {
    merged = false;
    for (int t = k - 1; t > 0; --t) {
      const Mode& ot = out[t - 1];
      Mode& in = out[t];
      if (ot.sa == in.sa * in.size && ot.sc == in.sc * in.size) {
        in.size *= ot.size;  // the merged mode keeps the inner strides
        for (int u = t - 1; u < k - 1; ++u) out[u] = out[u + 1];
        --k;
        merged = true;
        break;
      }
    }
  }
  for (int t = 0; t < k; ++t) m[t] = out[t];
  return k;
}

static inline bool al16(int64_t bytes) { return (bytes & 15) == 0; }

// ------------------------------------------------------------------ operand types
static inline int dt_size(int dt) { return dt >= B2G_DTYPE_E4M3 ? 1 : 2; }
// UMMA operand format code: kind::f16 0 = F16, 1 = BF16; kind::f8f6f4 0 = E4M3, 1 = E5M2
static inline int dt_fmt(int dt) { return (dt == B2G_DTYPE_BF16 || dt == B2G_DTYPE_E5M2) ? 1 : 0; }
static inline CUtensorMapDataType dt_map(int dt) {
  return dt == B2G_DTYPE_F16    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
         : dt == B2G_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                : CU_TENSOR_MAP_DATA_TYPE_UINT8;  // fp8: bytes
}

// ------------------------------------------------------------------ core dispatch
// Rank-order sum in the epilogue (see GemmParams::add_*): the stored C is the sum, in slot
// order, of `count` terms, term `self` being A.B and term s the fp32 slot base + s * slot.
struct AddendSpec {
  const float* base;
  int64_t slot;
  int count, self;
  const uint32_t* status;
  uint32_t epoch;
};

// c_type: 0 = fp32 C, 1 = fp16 C, 2 = bf16 C (16-bit C requires beta == 0); bias: optional
// per-column fp32 vector of N elements added once to every row of alpha*A.B.
static int run(const void* A, const int64_t as[5], const int64_t ast[5], const void* B,
               const int64_t bs[3], const int64_t bst[3], void* Cv, const int64_t cs[4],
               const int64_t cst[4], int dtype, float alpha, float beta, cudaStream_t stream,
               const FixedScratch* fixed = nullptr, const float* bias = nullptr, int c_type = 0,
               int64_t b_batch = -1, const AddendSpec* add = nullptr) {
  // b_batch >= 0: mode a is a batch mode, B[a][j][k][n] with stride b_batch along a
  if (dtype < B2G_DTYPE_F16 || dtype > B2G_DTYPE_E5M2)
    return fail(B2G_ERR_INVALID_ARG, "unknown operand type code %d", dtype);
  if (c_type < 0 || c_type > 2) return fail(B2G_ERR_INVALID_ARG, "unknown output type");
  if (c_type != 0 && beta != 0.0f)
    return fail(B2G_ERR_INVALID_ARG, "a 16-bit C takes beta = 0 only (got %g)", (double)beta);
  float* Cp = static_cast<float*>(Cv);
  const int c_esz = c_type == 0 ? 4 : 2;
  const int esz = dt_size(dtype);
  const int kb_elems = kRowBytes / esz;  // K elements per 128-byte stage row
  const CUtensorMapDataType map_type = dt_map(dtype);
  // ---- validation
  for (int t = 0; t < 5; ++t)
    if (as[t] < 0) return fail(B2G_ERR_INVALID_ARG, "negative A extent");
  for (int t = 0; t < 3; ++t)
    if (bs[t] < 0) return fail(B2G_ERR_INVALID_ARG, "negative B extent");
  if (bs[0] != as[3] || bs[1] != as[4])
    return fail(B2G_ERR_INVALID_ARG, "contracted modes differ: A (j,k)=(%lld,%lld) B=(%lld,%lld)",
                (long long)as[3], (long long)as[4], (long long)bs[0], (long long)bs[1]);
  if (cs[0] != as[0] || cs[1] != as[1] || cs[2] != as[2] || cs[3] != bs[2])
    return fail(B2G_ERR_INVALID_ARG, "C shape does not match A/B free modes");
  const int64_t M = as[0] * as[1] * as[2], N = bs[2], K = as[3] * as[4];
  if (M == 0 || N == 0) {
    t_path = B2G_PATH_EMPTY;
    return B2G_OK;
  }
  if (!Cp) return fail(B2G_ERR_INVALID_ARG, "C is null");
  if (K > 0 && (!A || !B)) return fail(B2G_ERR_INVALID_ARG, "A or B is null");

  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  DevState* ds = nullptr;
  int rc = device_state(dev, &ds);
  if (rc) return rc;

  auto make_geo = [&]() {
    Geo g;
    for (int t = 0; t < 5; ++t) {
      g.as[t] = as[t];
      g.ast[t] = ast[t];
    }
    for (int t = 0; t < 3; ++t) g.bst[t] = bst[t];
    for (int t = 0; t < 4; ++t) g.cst[t] = cst[t];
    g.b_batch = b_batch >= 0 ? b_batch : 0;
    g.n = N;
    return g;
  };
  const int64_t total = M * N;
  const int eth = 256;
  const unsigned eblocks =
      (unsigned)std::min<int64_t>((total + eth - 1) / eth, (int64_t)ds->sm_count * 32);
  auto launch_generic = [&](int path) -> int {
    if (add)  // the rank-order sum exists on the tensor-core path only
      return fail(B2G_ERR_UNSUPPORTED, "the epilogue rank-order sum needs the tensor-core path");
    const Geo g = make_geo();
    switch (dtype) {
      case B2G_DTYPE_F16:
        gemm_generic_kernel<B2G_DTYPE_F16><<<eblocks, eth, 0, stream>>>(A, B, Cv, g, alpha, beta, bias, c_type);
        break;
      case B2G_DTYPE_BF16:
        gemm_generic_kernel<B2G_DTYPE_BF16><<<eblocks, eth, 0, stream>>>(A, B, Cv, g, alpha, beta, bias, c_type);
        break;
      case B2G_DTYPE_E4M3:
        gemm_generic_kernel<B2G_DTYPE_E4M3><<<eblocks, eth, 0, stream>>>(A, B, Cv, g, alpha, beta, bias, c_type);
        break;
      default:
        gemm_generic_kernel<B2G_DTYPE_E5M2><<<eblocks, eth, 0, stream>>>(A, B, Cv, g, alpha, beta, bias, c_type);
        break;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "generic kernel launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    t_path = path;
    return B2G_OK;
  };

  if (K == 0 || alpha == 0.0f) {  // C = beta*C (+ bias)
    if (beta == 1.0f && !bias) {
      t_path = B2G_PATH_ZERO;
      return B2G_OK;
    }
    return launch_generic(B2G_PATH_ZERO);
  }
  if (opt_force_generic.load()) return launch_generic(B2G_PATH_GENERIC);
  if (ds->cc_major != 10) return launch_generic(B2G_PATH_GENERIC);

  // ---- coalesce modes
  const bool batched = b_batch >= 0 && as[0] > 1;
  Mode mm[3] = {{as[0], ast[0], cst[0]}, {as[1], ast[1], cst[1]}, {as[2], ast[2], cst[2]}};
  // a batch mode stays a mode of its own (B follows it), only (b, i) may merge
  int nm = batched ? 1 + coalesce(mm + 1, 2) : coalesce(mm, 3);
  Mode km[2] = {{as[3], ast[3], bst[0]}, {as[4], ast[4], bst[1]}};
  int nk = coalesce(km, 2);
  // pad to fixed arity: M -> (a, b, i), K -> (j, k); padded modes have size 1
  Mode M3[3], K2[2];
  for (int t = 0; t < 3; ++t) M3[t] = {1, 0, 0};
  for (int t = 0; t < 2; ++t) K2[t] = {1, 0, 0};
  if (nm > 3 || nk > 2) return launch_generic(B2G_PATH_GENERIC);
  if (batched) {
    // the batch mode keeps the a slot (the kernel indexes B with the tile's a coordinate);
    // the compacted (b, i) modes are right-aligned after it
    M3[0] = mm[0];
    for (int t = 1; t < nm; ++t) M3[3 - (nm - 1) + (t - 1)] = mm[t];
    if (nm == 1) M3[2] = {1, 1, 1};
  } else {
    for (int t = 0; t < nm; ++t) M3[3 - nm + t] = mm[t];
    if (nm == 0) M3[2] = {1, 1, 1};
  }
  for (int t = 0; t < nk; ++t) K2[2 - nk + t] = km[t];
  if (nk == 0) K2[1] = {1, 1, 1};
  const int64_t b_sn = bst[2], c_sn = cst[3];

  // ---- layout classes
  const bool a_ok = K2[1].sa == 1;                  // K-major A
  const bool b_mn = (b_sn == 1) || N == 1;          // N contiguous
  const bool b_k = !b_mn && K2[1].sc == 1;          // K contiguous
  const bool c_n = (c_sn == 1) || N == 1;           // N contiguous
  const bool c_m = !c_n && M3[2].sc == 1;           // innermost M mode contiguous
  if (!a_ok || !(b_mn || b_k) || !(c_n || c_m)) return launch_generic(B2G_PATH_GENERIC);
  // 16-bit C: row-major (N-contiguous) layouts only; the bias is read 16 bytes at a time
  if ((c_type != 0 && !c_n) || (bias && !al16((int64_t)(uintptr_t)bias)))
    return launch_generic(B2G_PATH_GENERIC);

  // ---- M decomposition: 128-row load box over (i, b, a)
  const int64_t isz = M3[2].size, bsz = M3[1].size, asz = M3[0].size;
  const int64_t jsz = K2[0].size, ksz = K2[1].size;
  if (isz > INT32_MAX / 2 || bsz > INT32_MAX / 2 || asz > INT32_MAX / 2 || N > INT32_MAX / 2 ||
      jsz > INT32_MAX / 2 || ksz > INT32_MAX / 2)
    return launch_generic(B2G_PATH_GENERIC);
  int bi, bb, ba;
  // the load box of one CTA's `rows` rows (128, or 64 for half-height pair tiles) over (i, b, a)
  auto decompose = [&](int rows) {
    if (batched) {
      // a tile never spans two batch entries: the box covers (i, b) only, rows past b's
      // extent are zero-filled on load and clipped on store
      bi = (isz >= rows || (rows % isz) != 0) ? rows : (int)isz;
      bb = rows / bi;
      ba = 1;
    } else if (isz >= rows || (rows % isz) != 0 || bsz * asz == 1) {
      bi = rows; bb = 1; ba = 1;
    } else {
      bi = (int)isz;
      const int rem = rows / bi;
      if (bsz >= rem || (rem % bsz) != 0) {
        bb = rem; ba = 1;
      } else {
        bb = (int)bsz; ba = rem / bb;
      }
    }
  };
  decompose(128);
  int si = std::min(bi, 32);
  if (c_m && si < 4) return launch_generic(B2G_PATH_GENERIC);  // TMA inner box >= 16 bytes

  // ---- TMA legality: 16-byte aligned bases and strides (size-1 modes do not matter)
  auto stride_ok = [](const Mode& m, bool first, int esz) {
    return m.size == 1 || al16((first ? m.sa : m.sc) * esz);
  };
  bool tma_ok = al16((int64_t)(uintptr_t)A) && al16((int64_t)(uintptr_t)B) &&
                al16((int64_t)(uintptr_t)Cp);
  // every M mode is an outer dimension of A; of C too, except the innermost one when C is
  // M-contiguous (it is then the map's unit-stride dimension 0)
  for (int t = 0; t < 3; ++t)
    tma_ok = tma_ok && stride_ok(M3[t], true, esz) && ((c_m && t == 2) || stride_ok(M3[t], false, c_esz));
  tma_ok = tma_ok && stride_ok(K2[0], true, esz) && stride_ok(K2[0], false, esz);
  if (b_mn) tma_ok = tma_ok && stride_ok(K2[1], false, esz);
  if (b_k) tma_ok = tma_ok && (N == 1 || al16(b_sn * esz));
  if (c_m) tma_ok = tma_ok && (N == 1 || al16(c_sn * c_esz));
  if (batched) tma_ok = tma_ok && al16(b_batch * esz);
  if (!tma_ok) return launch_generic(B2G_PATH_GENERIC);

  if (!get_encode()) return fail(B2G_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");

  // filler stride for size-1 modes: anything 16-byte aligned works (coordinate is always 0)
  auto fill = [](int64_t s, int64_t size, int64_t prev_extent_bytes) -> cuuint64_t {
    if (size == 1) return (cuuint64_t)((std::max<int64_t>(prev_extent_bytes, 16) + 15) & ~15LL);
    return (cuuint64_t)s;
  };

  CUtensorMap tmA, tmB, tmC;
  // choose CTA grouping (on 128-row tiles)
  int num_m_tiles_i = (int)((isz + bi - 1) / bi);
  int num_m_tiles_b = (int)((bsz + bb - 1) / bb);
  int num_m_tiles_a = (int)((asz + ba - 1) / ba);
  int64_t nmt64 = (int64_t)num_m_tiles_i * num_m_tiles_b * num_m_tiles_a;
  // batched: a CTA pair holds M tiles 2p and 2p+1, whose rows must be of one batch entry (the
  // pair's MMA shares both halves of B); with an odd number of M tiles per batch entry, tiles
  // are one-CTA
  const bool pair_ok = !batched || ((int64_t)num_m_tiles_i * num_m_tiles_b) % 2 == 0;
  const int64_t kit = ((ksz + kb_elems - 1) / kb_elems) * jsz;
  // half-height pair tiles need the cluster fix-up whenever they split K
  int half_opt = (batched || t_no_half) ? 128 : (int)opt_pair_rows.load();
  if (half_opt == 0 && (!opt_cluster_fixup.load() || opt_serial_fixup.load() || opt_split_k.load() > 4))
    half_opt = 128;
  TileChoice tc = choose_tiles(nmt64, N, kit, ds->sm_count, pair_ok ? (int)opt_cta_group.load() : 1,
                               (int)opt_tile_n.load(), half_opt);
  if (tc.half) {
    // half-height pair tiles: each CTA loads 64 rows; the M tiles are 64-row tiles, a pair
    // holds tiles 2p and 2p+1
    decompose(64);
    si = std::min(bi, 32);
    if (c_m && si < 4) {  // the 32-row store box of a warp would be too narrow: plain tiles
      decompose(128);
      si = std::min(bi, 32);
      tc = choose_tiles(nmt64, N, kit, ds->sm_count, pair_ok ? (int)opt_cta_group.load() : 1,
                        (int)opt_tile_n.load(), 128);
    } else {
      num_m_tiles_i = (int)((isz + bi - 1) / bi);
      num_m_tiles_b = (int)((bsz + bb - 1) / bb);
      num_m_tiles_a = (int)((asz + ba - 1) / ba);
      nmt64 = (int64_t)num_m_tiles_i * num_m_tiles_b * num_m_tiles_a;
    }
  }
  const int sb = std::min(bb, 32 / si);
  const int sa = 32 / (si * sb);
  // A: dims (k, j, i, b, a)
  {
    cuuint64_t dims[5] = {(cuuint64_t)ksz, (cuuint64_t)jsz, (cuuint64_t)isz, (cuuint64_t)bsz,
                          (cuuint64_t)asz};
    cuuint64_t st[4];
    st[0] = fill(K2[0].sa * esz, jsz, ksz * esz);
    st[1] = fill(M3[2].sa * esz, isz, (int64_t)st[0] * jsz);
    st[2] = fill(M3[1].sa * esz, bsz, (int64_t)st[1] * isz);
    st[3] = fill(M3[0].sa * esz, asz, (int64_t)st[2] * bsz);
    cuuint32_t box[5] = {(cuuint32_t)kb_elems, 1, (cuuint32_t)bi, (cuuint32_t)bb, (cuuint32_t)ba};
    CUresult r = encode_cached(&tmA, map_type, 5, const_cast<void*>(A), dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (r != CUDA_SUCCESS) return launch_generic(B2G_PATH_GENERIC);  // tensor map A not encodable
  }
  const int cg = tc.cg, bn = tc.bn;
  const int64_t nnt64 = (N + bn - 1) / bn;
  if (nmt64 * nnt64 > INT32_MAX / 4) return launch_generic(B2G_PATH_GENERIC);
  const int bph = std::min(bn, 256) / cg;  // B columns of one N-half held by one CTA
  // B
  // B: a batch mode adds a 4th dimension (the batch, stride b_batch) after the others
  const cuuint32_t b_rank = batched ? 4 : 3;
  if (b_mn) {  // dims (n, k, j[, l])
    cuuint64_t dims[4] = {(cuuint64_t)N, (cuuint64_t)ksz, (cuuint64_t)jsz, (cuuint64_t)asz};
    cuuint64_t st[3];
    st[0] = fill(K2[1].sc * esz, ksz, N * esz);
    st[1] = fill(K2[0].sc * esz, jsz, (int64_t)st[0] * ksz);
    st[2] = (cuuint64_t)(batched ? b_batch * esz : 16);
    cuuint32_t box[4] = {(cuuint32_t)kb_elems, (cuuint32_t)kb_elems, 1, 1};  // one MN-major atom
    CUresult r = encode_cached(&tmB, map_type, b_rank, const_cast<void*>(B), dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (r != CUDA_SUCCESS) return launch_generic(B2G_PATH_GENERIC);  // tensor map B (N-major) not encodable
  } else {  // dims (k, j, n[, l])
    cuuint64_t dims[4] = {(cuuint64_t)ksz, (cuuint64_t)jsz, (cuuint64_t)N, (cuuint64_t)asz};
    cuuint64_t st[3];
    st[0] = fill(K2[0].sc * esz, jsz, ksz * esz);
    st[1] = fill(b_sn * esz, N, (int64_t)st[0] * jsz);
    st[2] = (cuuint64_t)(batched ? b_batch * esz : 16);
    cuuint32_t box[4] = {(cuuint32_t)kb_elems, 1, (cuuint32_t)bph, 1};
    CUresult r = encode_cached(&tmB, map_type, b_rank, const_cast<void*>(B), dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (r != CUDA_SUCCESS) return launch_generic(B2G_PATH_GENERIC);  // tensor map B (K-major) not encodable
  }
  // C
  if (c_n) {  // dims (n, i, b, a), 32x32 boxes: fp32 rows of 128 bytes (128-byte swizzle) or
              // 16-bit rows of 64 bytes (64-byte swizzle)
    cuuint64_t dims[4] = {(cuuint64_t)N, (cuuint64_t)isz, (cuuint64_t)bsz, (cuuint64_t)asz};
    cuuint64_t st[3];
    st[0] = fill(M3[2].sc * c_esz, isz, N * c_esz);
    st[1] = fill(M3[1].sc * c_esz, bsz, (int64_t)st[0] * isz);
    st[2] = fill(M3[0].sc * c_esz, asz, (int64_t)st[1] * bsz);
    cuuint32_t box[4] = {32, (cuuint32_t)si, (cuuint32_t)sb, (cuuint32_t)sa};
    const CUtensorMapDataType ct = c_type == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : c_type == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUresult r = encode_cached(&tmC, ct, 4, Cv, dims, st, box,
                               c_type == 0 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                               CU_TENSOR_MAP_L2_PROMOTION_NONE);
    if (r != CUDA_SUCCESS) return launch_generic(B2G_PATH_GENERIC);  // tensor map C (N-major) not encodable
  } else {  // dims (i, n, b, a), unswizzled si x 32 boxes
    cuuint64_t dims[4] = {(cuuint64_t)isz, (cuuint64_t)N, (cuuint64_t)bsz, (cuuint64_t)asz};
    cuuint64_t st[3];
    st[0] = fill(c_sn * 4, N, isz * 4);
    st[1] = fill(M3[1].sc * 4, bsz, (int64_t)st[0] * N);
    st[2] = fill(M3[0].sc * 4, asz, (int64_t)st[1] * bsz);
    cuuint32_t box[4] = {(cuuint32_t)si, 32, (cuuint32_t)sb, (cuuint32_t)sa};
    CUresult r = encode_cached(&tmC, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Cp, dims, st, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_NONE);
    if (r != CUDA_SUCCESS) return launch_generic(B2G_PATH_GENERIC);  // tensor map C (M-major) not encodable
  }

  GemmParams p{};
  p.i_size = (int)isz;
  p.b_size = (int)bsz;
  p.a_size = (int)asz;
  p.bi = bi; p.bb = bb; p.ba = ba;
  p.ti = num_m_tiles_i;
  p.tb = num_m_tiles_b;
  p.si = si; p.sb = sb; p.sa = sa;
  p.num_m_tiles = (int)nmt64;
  p.num_pm_tiles = (int)((nmt64 + cg - 1) / cg);
  p.n_size = (int)N;
  p.num_n_tiles = (int)nnt64;
  p.k_blocks_per_j = (int)((ksz + kb_elems - 1) / kb_elems);
  p.ab_format = dt_fmt(dtype);
  p.k_iters = (int)(jsz * p.k_blocks_per_j);
  p.num_tiles = p.num_pm_tiles * p.num_n_tiles;
  int rg = (int)opt_raster_group.load();
  p.raster_group = rg > 0 ? rg : (cg == 2 ? 8 : 16);  // measured best on 8192^3
  p.store_hint = (int)opt_store_hint.load();
  p.c_type = c_type;
  p.bias = bias;
  p.b_batched = batched ? 1 : 0;
  p.alpha = alpha;
  p.accumulate = beta != 0.0f ? 1 : 0;
  p.timeout_ns = (unsigned long long)opt_timeout_ns.load();
  p.fault_flags = (int)opt_fault_flags.load();
  if (add) {
    if (batched || !c_n || c_type != 0 || beta != 0.0f || as[0] * as[1] != 1 || bias)
      return fail(B2G_ERR_UNSUPPORTED, "the epilogue rank-order sum takes a plain row-major fp32 C");
    p.add_base = add->base;
    p.add_slot = (long long)add->slot;
    p.add_count = add->count;
    p.add_self = add->self;
    p.add_status = add->status;
    p.add_epoch = add->epoch;
  }

  // ---- launch
  using KernFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const GemmParams);
  const int bk = b_k ? 1 : 0, cm = c_m ? 1 : 0;
  const int variant = tc.half ? 4
                      : cg == 1 ? (bn == 128 ? 3 : 0)
                      : bn == 256 ? 1
                      : (opt_epi_warps.load() == 8 ? 5 : 2);
  static const KernFn table[2][6][2][2] = {
      {{{gemm_tc_kernel<1, 256, false, false, 2>, gemm_tc_kernel<1, 256, false, true, 2>},
        {gemm_tc_kernel<1, 256, true, false, 2>, gemm_tc_kernel<1, 256, true, true, 2>}},
       {{gemm_tc_kernel<2, 256, false, false, 2>, gemm_tc_kernel<2, 256, false, true, 2>},
        {gemm_tc_kernel<2, 256, true, false, 2>, gemm_tc_kernel<2, 256, true, true, 2>}},
       {{gemm_tc_kernel<2, 512, false, false, 2>, gemm_tc_kernel<2, 512, false, true, 2>},
        {gemm_tc_kernel<2, 512, true, false, 2>, gemm_tc_kernel<2, 512, true, true, 2>}},
       {{gemm_tc_kernel<1, 128, false, false, 2>, gemm_tc_kernel<1, 128, false, true, 2>},
        {gemm_tc_kernel<1, 128, true, false, 2>, gemm_tc_kernel<1, 128, true, true, 2>}},
       {{gemm_tc_kernel<2, 256, false, false, 2, 64>, gemm_tc_kernel<2, 256, false, true, 2, 64>},
        {gemm_tc_kernel<2, 256, true, false, 2, 64>, gemm_tc_kernel<2, 256, true, true, 2, 64>}},
       {{gemm_tc_kernel<2, 512, false, false, 2, 128, 8>, gemm_tc_kernel<2, 512, false, true, 2, 128, 8>},
        {gemm_tc_kernel<2, 512, true, false, 2, 128, 8>, gemm_tc_kernel<2, 512, true, true, 2, 128, 8>}}},
      {{{gemm_tc_kernel<1, 256, false, false, 1>, gemm_tc_kernel<1, 256, false, true, 1>},
        {gemm_tc_kernel<1, 256, true, false, 1>, gemm_tc_kernel<1, 256, true, true, 1>}},
       {{gemm_tc_kernel<2, 256, false, false, 1>, gemm_tc_kernel<2, 256, false, true, 1>},
        {gemm_tc_kernel<2, 256, true, false, 1>, gemm_tc_kernel<2, 256, true, true, 1>}},
       {{gemm_tc_kernel<2, 512, false, false, 1>, gemm_tc_kernel<2, 512, false, true, 1>},
        {gemm_tc_kernel<2, 512, true, false, 1>, gemm_tc_kernel<2, 512, true, true, 1>}},
       {{gemm_tc_kernel<1, 128, false, false, 1>, gemm_tc_kernel<1, 128, false, true, 1>},
        {gemm_tc_kernel<1, 128, true, false, 1>, gemm_tc_kernel<1, 128, true, true, 1>}},
       {{gemm_tc_kernel<2, 256, false, false, 1, 64>, gemm_tc_kernel<2, 256, false, true, 1, 64>},
        {gemm_tc_kernel<2, 256, true, false, 1, 64>, gemm_tc_kernel<2, 256, true, true, 1, 64>}},
       {{gemm_tc_kernel<2, 512, false, false, 1, 128, 8>, gemm_tc_kernel<2, 512, false, true, 1, 128, 8>},
        {gemm_tc_kernel<2, 512, true, false, 1, 128, 8>, gemm_tc_kernel<2, 512, true, true, 1, 128, 8>}}}};
  static const uint32_t smem_of[6] = {Cfg<1, 256>::SMEM_BYTES, Cfg<2, 256>::SMEM_BYTES,
                                      Cfg<2, 512>::SMEM_BYTES, Cfg<1, 128>::SMEM_BYTES,
                                      Cfg<2, 256, 64>::SMEM_BYTES, Cfg<2, 512, kBM, 8>::SMEM_BYTES};
  static const int threads_of[6] = {Cfg<1, 256>::THREADS, Cfg<2, 256>::THREADS,
                                    Cfg<2, 512>::THREADS, Cfg<1, 128>::THREADS,
                                    Cfg<2, 256, 64>::THREADS, Cfg<2, 512, kBM, 8>::THREADS};
  // the epilogue rank-order sum: fp16 operands, row-major C (the ADD instances)
  static const KernFn table_add[6][2] = {
      {gemm_tc_kernel<1, 256, false, false, 2, kBM, 4, true>,
       gemm_tc_kernel<1, 256, true, false, 2, kBM, 4, true>},
      {gemm_tc_kernel<2, 256, false, false, 2, kBM, 4, true>,
       gemm_tc_kernel<2, 256, true, false, 2, kBM, 4, true>},
      {gemm_tc_kernel<2, 512, false, false, 2, kBM, 4, true>,
       gemm_tc_kernel<2, 512, true, false, 2, kBM, 4, true>},
      {gemm_tc_kernel<1, 128, false, false, 2, kBM, 4, true>,
       gemm_tc_kernel<1, 128, true, false, 2, kBM, 4, true>},
      {gemm_tc_kernel<2, 256, false, false, 2, 64, 4, true>,
       gemm_tc_kernel<2, 256, true, false, 2, 64, 4, true>},
      {gemm_tc_kernel<2, 512, false, false, 2, kBM, 8, true>,
       gemm_tc_kernel<2, 512, true, false, 2, kBM, 8, true>}};
  const int nthreads = threads_of[variant];
  if (add && (esz != 2 || cm != 0))
    return fail(B2G_ERR_UNSUPPORTED, "the epilogue rank-order sum takes 16-bit operands and a row-major C");
  const int e8 = add ? 2 : esz == 1 ? 1 : 0;
  KernFn kern = add ? table_add[variant][bk] : table[e8][variant][bk][cm];
  const uint32_t smem = smem_of[variant];
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!ds->attr_set[e8][variant][bk][cm]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(smem)");
      if (cg == 2) {
        cudaLaunchConfig_t qc = {};
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = 2;
        qa[0].val.clusterDim.y = 1;
        qa[0].val.clusterDim.z = 1;
        qc.gridDim = dim3(2 * (ds->sm_count / 2), 1, 1);
        qc.blockDim = dim3((unsigned)nthreads, 1, 1);
        qc.dynamicSmemBytes = smem;
        qc.attrs = qa;
        qc.numAttrs = 1;
        int nclu = 0;
        e = cudaOccupancyMaxActiveClusters(&nclu, (void*)kern, &qc);
        if (e != cudaSuccess || nclu <= 0) nclu = ds->sm_count / 2;
        ds->max_clusters[e8][variant][bk][cm] = nclu;
      }
      ds->attr_set[e8][variant][bk][cm] = true;
    }
  }
  const int group_cap = cg == 1 ? ds->sm_count : ds->max_clusters[e8][variant][bk][cm];
  // ---- split-K: when the tiles cannot fill the GPU, split K so that every CTA group has a
  // unit; each split keeps at least 8 K blocks.
  // Tail split: when the tiles fill whole waves plus a partial one, split only the tiles of
  // the partial wave so that its units fill the CTA groups.
  const SplitChoice sc = choose_splits(p.num_tiles, p.k_iters, group_cap, cg, (int)opt_split_k.load(),
                                       opt_tail_split.load() != 0, tc.half);
  p.k_per_split = sc.k_per_split;
  p.k_splits = sc.k_splits;
  int full = sc.num_full;
  if (fixed && full > 0 && full < p.num_tiles) {
    // the tail split is an optimisation: under a fixed scratch it is dropped if it does not fit
    const size_t need = (size_t)(p.num_tiles - full) * p.k_splits * cg * 128 * bn * sizeof(float) +
                        ((size_t)(p.num_tiles - full) * cg * sizeof(int) + 255) / 256 * 256;
    if (need > fixed->bytes) {
      full = p.num_tiles;
      p.k_splits = 1;
      p.k_per_split = p.k_iters;
    }
  }
  p.num_full = full;
  p.num_units = full + (p.num_tiles - full) * p.k_splits;
  t_split_ws = 0;
  p.ws = nullptr;
  p.counters = nullptr;
  // Cluster fix-up: one-CTA tiles (at most 8 splits) or half-height pair tiles (at most 4
  // splits: 2 CTAs each), every tile split, one unit per CTA group, and every cluster resident
  // at once (checked against the cluster occupancy).
  p.cluster_fixup = 0;
  if ((cg == 1 || tc.half) && p.k_splits > 1 && p.k_splits * cg <= 8 && p.num_full == 0 &&
      opt_cluster_fixup.load() && !opt_serial_fixup.load()) {
    const int S = p.k_splits;
    int nclu = 0;
    {
      std::lock_guard<std::mutex> lk(g_dev_mu);
      nclu = ds->max_clusters_cg1[e8][variant][bk][cm][S];
      if (nclu == 0) {
        cudaLaunchConfig_t qc = {};
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = (unsigned)(cg * S);
        qa[0].val.clusterDim.y = 1;
        qa[0].val.clusterDim.z = 1;
        qc.gridDim = dim3((unsigned)(cg * S * (ds->sm_count / (cg * S))), 1, 1);
        qc.blockDim = dim3((unsigned)nthreads, 1, 1);
        qc.dynamicSmemBytes = smem;
        qc.attrs = qa;
        qc.numAttrs = 1;
        cudaError_t e = cudaOccupancyMaxActiveClusters(&nclu, (void*)kern, &qc);
        if (e != cudaSuccess || nclu <= 0) {
          cudaGetLastError();
          nclu = -1;  // not launchable in clusters of S: never use this mode for S
        }
        ds->max_clusters_cg1[e8][variant][bk][cm][S] = nclu;
      }
    }
    if (nclu > 0 && p.num_units <= nclu * S) p.cluster_fixup = 1;
  }
  if (tc.half && p.k_splits > 1 && !p.cluster_fixup) {
    // Half-height pair tiles reduce split partials only through distributed shared memory.
    // Forced by the caller: refuse; chosen by the planner: plan again without them.
    if (opt_pair_rows.load() == 64)
      return fail(B2G_ERR_UNSUPPORTED,
                  "half-height pair tiles split K only with the cluster fix-up (at most 4 "
                  "splits, every cluster resident)");
    t_no_half = true;
    const int rc2 = run(A, as, ast, B, bs, bst, Cv, cs, cst, dtype, alpha, beta, stream, fixed, bias,
                        c_type, b_batch);
    t_no_half = false;
    return rc2;
  }
  void* scratch = nullptr;
  const size_t split_tiles = (size_t)(p.num_tiles - p.num_full);
  int* ring = nullptr;  // counters from the ring: no memset
  RingLease lease;      // holds the ring until the launch is recorded
  if (p.k_splits > 1 && !p.cluster_fixup) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
    if (cap == cudaStreamCaptureStatusNone) {
      int rrc = ring_counters(split_tiles * cg, stream, &ring, &lease);
      if (rrc != B2G_OK) return rrc;
    }
  }
  if (p.k_splits > 1 && !p.cluster_fixup)
    t_split_ws = (int64_t)(split_tiles * p.k_splits * cg * 128 * bn * sizeof(float));
  if (p.cluster_fixup) {
    // partials stay in shared memory: no workspace, no counters
  } else if (p.k_splits > 1 && fixed) {
    // caller-supplied scratch (b2g_gemm_f16_f32_noalloc): no allocation
    const size_t ws_bytes = split_tiles * p.k_splits * cg * 128 * bn * sizeof(float);
    const size_t ctr_bytes = ring ? 0 : (split_tiles * cg * sizeof(int) + 255) / 256 * 256;
    if (ctr_bytes + ws_bytes > fixed->bytes)
      return fail(B2G_ERR_INVALID_ARG,
                  "split-K scratch of %zu bytes exceeds the %zu-byte static scratch of "
                  "b2g_gemm_f16_f32_noalloc",
                  ctr_bytes + ws_bytes, fixed->bytes);
    p.ws = reinterpret_cast<float*>(static_cast<char*>(fixed->ptr) + ctr_bytes);
    if (ring) {
      p.counters = ring;
    } else {
      p.counters = static_cast<int*>(fixed->ptr);
      cudaError_t e = cudaMemsetAsync(p.counters, 0, ctr_bytes, stream);  // counters start at 0
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(split-K counters)");
    }
  } else if (p.k_splits > 1) {
    const size_t ws_bytes = split_tiles * p.k_splits * cg * 128 * bn * sizeof(float);
    const size_t ctr_bytes = ring ? 0 : (split_tiles * cg * sizeof(int) + 255) / 256 * 256;
    cudaMemPool_t pool = nullptr;
    int prc = split_pool(&pool);
    if (prc != B2G_OK) return prc;
    cudaError_t e = cudaMallocFromPoolAsync(&scratch, ctr_bytes + ws_bytes, pool, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocFromPoolAsync(split-K workspace)");
    p.ws = reinterpret_cast<float*>(static_cast<char*>(scratch) + ctr_bytes);
    if (ring) {
      p.counters = ring;
    } else {
      p.counters = static_cast<int*>(scratch);
      e = cudaMemsetAsync(p.counters, 0, ctr_bytes, stream);
      if (e != cudaSuccess) {
        cudaFreeAsync(scratch, stream);
        return cuda_fail(e, "cudaMemsetAsync(split-K counters)");
      }
    }
  }
  int groups = std::min(group_cap, p.num_units);
  if (groups < 1) groups = 1;
  // parallel fix-up only when each CTA group holds at most one split unit (all split units of
  // the launch then run at the same time, so their mutual waits always end)
  if (p.cluster_fixup) groups = p.num_units;  // one unit per CTA, whole clusters
  p.fixup_parallel = (p.k_splits > 1 && p.num_full % groups == 0 &&
                      p.num_units - p.num_full <= groups && !opt_serial_fixup.load())
                         ? 1
                         : 0;

  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.gridDim = dim3((unsigned)(groups * cg), 1, 1);
  cfg.blockDim = dim3((unsigned)nthreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (cg == 2 || p.cluster_fixup) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[cfg.numAttrs].val.clusterDim.x = p.cluster_fixup ? (unsigned)(cg * p.k_splits) : 2u;
    attr[cfg.numAttrs].val.clusterDim.y = 1;
    attr[cfg.numAttrs].val.clusterDim.z = 1;
    ++cfg.numAttrs;
  }
  if (opt_pdl.load() && !add) {
    // programmatic dependent launch: the kernel's set-up overlaps the previous kernel's tail
    // (the kernel waits with griddepcontrol.wait before it touches global memory).  Not for
    // the rank-order sum, whose launch follows a stream wait on the peers' flags.
    attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
    ++cfg.numAttrs;
  }
  if (beta != 0.0f && beta != 1.0f) {  // C = beta*C first; the kernel then adds alpha*A.B
    scale_c_kernel<<<eblocks, eth, 0, stream>>>(Cp, make_geo(), beta);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      if (scratch) cudaFreeAsync(scratch, stream);
      return cuda_fail(e, "scale kernel launch");
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmC, p);
  lease.commit(stream);
  if (scratch) cudaFreeAsync(scratch, stream);  // stream-ordered: freed after the kernel
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  t_path = cg == 1 ? B2G_PATH_TC_1CTA : B2G_PATH_TC_2CTA;
  return B2G_OK;
}

int gemm_rank_sum(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K,
                  int64_t lda, int64_t ldb, int64_t ldc, const float* add_base, int64_t add_slot,
                  int add_count, int add_self, const uint32_t* status, uint32_t epoch,
                  void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(B2G_ERR_INVALID_ARG, "negative dimension");
  if (lda < std::max<int64_t>(K, 1) || ldb < std::max<int64_t>(N, 1) || ldc < std::max<int64_t>(N, 1))
    return fail(B2G_ERR_INVALID_ARG, "leading dimension smaller than the row length");
  if (M == 0 || N == 0) return B2G_OK;  // nothing to store (run() would return before adding)
  if (K == 0) return fail(B2G_ERR_UNSUPPORTED, "the epilogue rank-order sum needs K > 0");
  const int64_t as[5] = {1, 1, M, 1, K}, ast[5] = {0, 0, lda, 0, 1};
  const int64_t bs[3] = {1, K, N}, bst[3] = {0, ldb, 1};
  const int64_t cs[4] = {1, 1, M, N}, cst[4] = {0, 0, ldc, 1};
  const AddendSpec add = {add_base, add_slot, add_count, add_self, status, epoch};
  return run(A, as, ast, B, bs, bst, C, cs, cst, B2G_DTYPE_F16, 1.0f, 0.0f,
             static_cast<cudaStream_t>(stream), nullptr, nullptr, 0, -1, &add);
}

bool rs_fused() { return opt_rs_fused.load() != 0; }
bool rs_stage() { return opt_rs_stage.load() != 0; }

// The rank-order sum as a separate pass, for calls the tensor-core epilogue does not take:
// C (holding A.B) becomes the sum over s of term s in order, term `self` being C itself and
// the others slots[s * slot_stride + i * N + j].  Failed status words give NaN, as in the
// kernel's epilogue.
__global__ void slot_sum_kernel(float* __restrict__ C, int64_t M, int64_t N, int64_t ldc,
                                const float* __restrict__ slots, int64_t slot_stride, int count,
                                int self, const uint32_t* status, uint32_t epoch) {
  bool failed = false;
  if (status)
    for (int s = 0; s < count; ++s)
      if (s != self && __ldcg(status + s) != epoch) failed = true;
  if (failed && blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(&g_device_error, 0, ERR_PEER_FAILED);
  const int64_t total = M * N, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += stride) {
    const int64_t i = v / N, j = v - i * N;
    float a = 0.0f;
    for (int s = 0; s < count; ++s) {
      const float t = s == self ? C[i * ldc + j] : __ldcg(slots + s * slot_stride + v);
      a = s == 0 ? t : a + t;
    }
    C[i * ldc + j] = failed ? __int_as_float(0x7fc00000) : a;
  }
}

}  // namespace b2g

// ==================================================================== C ABI
using namespace b2g;

extern "C" int b2g_gemm_ex(const void* A, const void* B, float* C, int64_t M, int64_t N,
                           int64_t K, int64_t lda, int64_t ldb, int64_t ldc, float alpha,
                           float beta, void* stream) {
  t_err.clear();
  if (M < 0 || N < 0 || K < 0) return fail(B2G_ERR_INVALID_ARG, "negative dimension");
  if (lda < std::max<int64_t>(K, 1) || ldb < std::max<int64_t>(N, 1) || ldc < std::max<int64_t>(N, 1))
    return fail(B2G_ERR_INVALID_ARG, "leading dimension smaller than the row length");
  const int64_t as[5] = {1, 1, M, 1, K}, ast[5] = {0, 0, lda, 0, 1};
  const int64_t bs[3] = {1, K, N}, bst[3] = {0, ldb, 1};
  const int64_t cs[4] = {1, 1, M, N}, cst[4] = {0, 0, ldc, 1};
  return run(A, as, ast, B, bs, bst, C, cs, cst, B2G_DTYPE_F16, alpha, beta,
             static_cast<cudaStream_t>(stream));
}

extern "C" int b2g_gemm_f16_f32(const void* A, const void* B, float* C, int64_t M, int64_t N,
                                int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  return b2g_gemm_ex(A, B, C, M, N, K, lda, ldb, ldc, 1.0f, 0.0f, stream);
}

extern "C" int b2g_gemm_sum_slots(const void* A, const void* B, float* C, int64_t M, int64_t N,
                                  int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                                  const float* slots, int64_t slot_stride, int count, int self,
                                  const uint32_t* status, uint32_t epoch, void* stream) {
  t_err.clear();
  if (M < 0 || N < 0 || K < 0) return fail(B2G_ERR_INVALID_ARG, "negative dimension");
  if (lda < std::max<int64_t>(K, 1) || ldb < std::max<int64_t>(N, 1) || ldc < std::max<int64_t>(N, 1))
    return fail(B2G_ERR_INVALID_ARG, "leading dimension smaller than the row length");
  if (count < 1 || count > 1024 || self < 0 || self >= count)
    return fail(B2G_ERR_INVALID_ARG, "count outside [1, 1024] or self outside [0, count)");
  if (count > 1 && (!slots || slot_stride < M * N || slot_stride % 4 != 0 ||
                    (reinterpret_cast<uintptr_t>(slots) & 15) != 0))
    return fail(B2G_ERR_INVALID_ARG,
                "slots must be 16-byte aligned, slot_stride >= M * N and a multiple of 4");
  if (M == 0 || N == 0) return B2G_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = K > 0 ? gemm_rank_sum(A, B, C, M, N, K, lda, ldb, ldc, slots, slot_stride, count, self,
                                 status, epoch, stream)
                 : (int)B2G_ERR_UNSUPPORTED;
  if (rc != B2G_ERR_UNSUPPORTED) return rc;
  // no tensor-core launch for this call: the GEMM, then the sum as its own pass
  rc = b2g_gemm_ex(A, B, C, M, N, K, lda, ldb, ldc, 1.0f, 0.0f, stream);
  if (rc != B2G_OK || count == 1) return rc;
  const int64_t blocks = std::min<int64_t>((M * N + 255) / 256, 148 * 8);
  slot_sum_kernel<<<(unsigned)blocks, 256, 0, s>>>(C, M, N, ldc, slots, slot_stride, count, self,
                                                   status, epoch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "slot_sum_kernel");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return B2G_OK;
}

extern "C" int b2g_gemm_f16_f32_noalloc(const void* A, const void* B, float* C, int64_t M,
                                        int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                        int64_t ldc, void* stream) {
  t_err.clear();
  if (M < 0 || N < 0 || K < 0) return fail(B2G_ERR_INVALID_ARG, "negative dimension");
  if (lda < std::max<int64_t>(K, 1) || ldb < std::max<int64_t>(N, 1) || ldc < std::max<int64_t>(N, 1))
    return fail(B2G_ERR_INVALID_ARG, "leading dimension smaller than the row length");
  // an empty problem needs no device (as in b2g_gemm_f16_f32): the scratch is looked up only
  // for a non-empty one
  FixedScratch fs = {nullptr, 0};
  if (M > 0 && N > 0) {
    const int rc = noalloc_scratch(&fs);
    if (rc != B2G_OK) return rc;
  }
  const int64_t as[5] = {1, 1, M, 1, K}, ast[5] = {0, 0, lda, 0, 1};
  const int64_t bs[3] = {1, K, N}, bst[3] = {0, ldb, 1};
  const int64_t cs[4] = {1, 1, M, N}, cst[4] = {0, 0, ldc, 1};
  return run(A, as, ast, B, bs, bst, C, cs, cst, B2G_DTYPE_F16, 1.0f, 0.0f,
             static_cast<cudaStream_t>(stream),
             &fs);
}

extern "C" int b2g_gemm(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K) {
  return b2g_gemm_f16_f32(A, B, C, M, N, K, std::max<int64_t>(K, 1), std::max<int64_t>(N, 1),
                          std::max<int64_t>(N, 1), nullptr);
}

extern "C" int b2g_contract5d_ex(const void* A, const int64_t a_shape[5],
                                 const int64_t a_stride[5], const void* B,
                                 const int64_t b_shape[3], const int64_t b_stride[3], float* C,
                                 const int64_t c_shape[4], const int64_t c_stride[4], float alpha,
                                 float beta, void* stream) {
  t_err.clear();
  if (!a_shape || !a_stride || !b_shape || !b_stride || !c_shape || !c_stride)
    return fail(B2G_ERR_INVALID_ARG, "null shape/stride array");
  return run(A, a_shape, a_stride, B, b_shape, b_stride, C, c_shape, c_stride, B2G_DTYPE_F16,
             alpha, beta,
             static_cast<cudaStream_t>(stream));
}

extern "C" int b2g_contract5d_f16_f32(const void* A, const int64_t a_shape[5],
                                      const int64_t a_stride[5], const void* B,
                                      const int64_t b_shape[3], const int64_t b_stride[3], float* C,
                                      const int64_t c_shape[4], const int64_t c_stride[4],
                                      void* stream) {
  return b2g_contract5d_ex(A, a_shape, a_stride, B, b_shape, b_stride, C, c_shape, c_stride, 1.0f,
                           0.0f, stream);
}

extern "C" int b2g_fill_uniform(void* dst, int64_t n, int dtype, uint64_t seed, uint64_t offset,
                                void* stream) {
  t_err.clear();
  if (n < 0) return fail(B2G_ERR_INVALID_ARG, "negative length");
  if (dtype < B2G_DTYPE_F16 || dtype > B2G_DTYPE_E5M2)
    return fail(B2G_ERR_INVALID_ARG, "unknown operand type code %d", dtype);
  if (n == 0) return B2G_OK;
  if (!dst) return fail(B2G_ERR_INVALID_ARG, "dst is null");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DevState* ds = nullptr;
  int rc = device_state(dev, &ds);
  if (rc) return rc;
  const int threads = 256;
  const unsigned blocks =
      (unsigned)std::min<int64_t>((n + threads - 1) / threads, (int64_t)ds->sm_count * 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case B2G_DTYPE_F16:
      fill_uniform_kernel<B2G_DTYPE_F16><<<blocks, threads, 0, s>>>(dst, n, seed, offset);
      break;
    case B2G_DTYPE_BF16:
      fill_uniform_kernel<B2G_DTYPE_BF16><<<blocks, threads, 0, s>>>(dst, n, seed, offset);
      break;
    case B2G_DTYPE_E4M3:
      fill_uniform_kernel<B2G_DTYPE_E4M3><<<blocks, threads, 0, s>>>(dst, n, seed, offset);
      break;
    default:
      fill_uniform_kernel<B2G_DTYPE_E5M2><<<blocks, threads, 0, s>>>(dst, n, seed, offset);
      break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fill kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return B2G_OK;
}

extern "C" int b2g_fill_uniform_f16(void* dst, int64_t n, uint64_t seed, uint64_t offset,
                                    void* stream) {
  return b2g_fill_uniform(dst, n, B2G_DTYPE_F16, seed, offset, stream);
}

extern "C" int b2g_gemm_typed(const void* A, const void* B, float* C, int64_t M, int64_t N,
                              int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int dtype,
                              float alpha, float beta, void* stream) {
  t_err.clear();
  if (M < 0 || N < 0 || K < 0) return fail(B2G_ERR_INVALID_ARG, "negative dimension");
  if (lda < std::max<int64_t>(K, 1) || ldb < std::max<int64_t>(N, 1) || ldc < std::max<int64_t>(N, 1))
    return fail(B2G_ERR_INVALID_ARG, "leading dimension smaller than the row length");
  const int64_t as[5] = {1, 1, M, 1, K}, ast[5] = {0, 0, lda, 0, 1};
  const int64_t bs[3] = {1, K, N}, bst[3] = {0, ldb, 1};
  const int64_t cs[4] = {1, 1, M, N}, cst[4] = {0, 0, ldc, 1};
  return run(A, as, ast, B, bs, bst, C, cs, cst, dtype, alpha, beta,
             static_cast<cudaStream_t>(stream));
}

extern "C" int b2g_contract5d_typed(const void* A, const int64_t a_shape[5],
                                    const int64_t a_stride[5], const void* B,
                                    const int64_t b_shape[3], const int64_t b_stride[3], float* C,
                                    const int64_t c_shape[4], const int64_t c_stride[4], int dtype,
                                    float alpha, float beta, void* stream) {
  t_err.clear();
  if (!a_shape || !a_stride || !b_shape || !b_stride || !c_shape || !c_stride)
    return fail(B2G_ERR_INVALID_ARG, "null shape/stride array");
  return run(A, a_shape, a_stride, B, b_shape, b_stride, C, c_shape, c_stride, dtype, alpha, beta,
             static_cast<cudaStream_t>(stream));
}

static int out_type(int c_dtype, int* c_type) {
  switch (c_dtype) {
    case B2G_DTYPE_F32: *c_type = 0; return B2G_OK;
    case B2G_DTYPE_F16: *c_type = 1; return B2G_OK;
    case B2G_DTYPE_BF16: *c_type = 2; return B2G_OK;
    default: return fail(B2G_ERR_INVALID_ARG, "unsupported output type code %d", c_dtype);
  }
}

extern "C" int b2g_gemm_epilogue(const void* A, const void* B, void* C, int64_t M, int64_t N,
                                 int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int dtype,
                                 float alpha, float beta, const float* bias, int c_dtype,
                                 void* stream) {
  t_err.clear();
  int c_type = 0;
  int rc = out_type(c_dtype, &c_type);
  if (rc) return rc;
  if (M < 0 || N < 0 || K < 0) return fail(B2G_ERR_INVALID_ARG, "negative dimension");
  if (lda < std::max<int64_t>(K, 1) || ldb < std::max<int64_t>(N, 1) || ldc < std::max<int64_t>(N, 1))
    return fail(B2G_ERR_INVALID_ARG, "leading dimension smaller than the row length");
  const int64_t as[5] = {1, 1, M, 1, K}, ast[5] = {0, 0, lda, 0, 1};
  const int64_t bs[3] = {1, K, N}, bst[3] = {0, ldb, 1};
  const int64_t cs[4] = {1, 1, M, N}, cst[4] = {0, 0, ldc, 1};
  return run(A, as, ast, B, bs, bst, C, cs, cst, dtype, alpha, beta,
             static_cast<cudaStream_t>(stream), nullptr, bias, c_type);
}

extern "C" int b2g_contract5d_epilogue(const void* A, const int64_t a_shape[5],
                                       const int64_t a_stride[5], const void* B,
                                       const int64_t b_shape[3], const int64_t b_stride[3], void* C,
                                       const int64_t c_shape[4], const int64_t c_stride[4],
                                       int dtype, float alpha, float beta, const float* bias,
                                       int c_dtype, void* stream) {
  t_err.clear();
  int c_type = 0;
  int rc = out_type(c_dtype, &c_type);
  if (rc) return rc;
  if (!a_shape || !a_stride || !b_shape || !b_stride || !c_shape || !c_stride)
    return fail(B2G_ERR_INVALID_ARG, "null shape/stride array");
  return run(A, a_shape, a_stride, B, b_shape, b_stride, C, c_shape, c_stride, dtype, alpha, beta,
             static_cast<cudaStream_t>(stream), nullptr, bias, c_type);
}

extern "C" int b2g_contract5d_batched(const void* A, const int64_t a_shape[5],
                                      const int64_t a_stride[5], const void* B,
                                      const int64_t b_shape[3], const int64_t b_stride[3],
                                      int64_t b_batch_stride, float* C, const int64_t c_shape[4],
                                      const int64_t c_stride[4], int dtype, float alpha,
                                      float beta, void* stream) {
  t_err.clear();
  if (!a_shape || !a_stride || !b_shape || !b_stride || !c_shape || !c_stride)
    return fail(B2G_ERR_INVALID_ARG, "null shape/stride array");
  if (b_batch_stride < 0) return fail(B2G_ERR_INVALID_ARG, "negative batch stride");
  return run(A, a_shape, a_stride, B, b_shape, b_stride, C, c_shape, c_stride, dtype, alpha, beta,
             static_cast<cudaStream_t>(stream), nullptr, nullptr, 0, b_batch_stride);
}

extern "C" int b2g_gemm_batched(const void* A, const void* B, float* C, int64_t L, int64_t M,
                                int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                                int64_t stride_a, int64_t stride_b, int64_t stride_c,
                                void* stream) {
  t_err.clear();
  if (L < 0 || M < 0 || N < 0 || K < 0) return fail(B2G_ERR_INVALID_ARG, "negative dimension");
  if (lda < std::max<int64_t>(K, 1) || ldb < std::max<int64_t>(N, 1) || ldc < std::max<int64_t>(N, 1))
    return fail(B2G_ERR_INVALID_ARG, "leading dimension smaller than the row length");
  if (stride_a < 0 || stride_b < 0 || stride_c < 0)
    return fail(B2G_ERR_INVALID_ARG, "negative batch stride");
  const int64_t as[5] = {L, 1, M, 1, K}, ast[5] = {stride_a, 0, lda, 0, 1};
  const int64_t bs[3] = {1, K, N}, bst[3] = {0, ldb, 1};
  const int64_t cs[4] = {L, 1, M, N}, cst[4] = {stride_c, 0, ldc, 1};
  return run(A, as, ast, B, bs, bst, C, cs, cst, B2G_DTYPE_F16, 1.0f, 0.0f,
             static_cast<cudaStream_t>(stream), nullptr, nullptr, 0, stride_b);
}

extern "C" const char* b2g_last_error_string(void) { return t_err.c_str(); }

extern "C" int b2g_last_path(void) { return t_path; }

extern "C" int b2g_device_status(int clear) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    fail(B2G_ERR_CUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(e));
    return -1;
  }
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) {
    fail(B2G_ERR_CUDA, "read device error word: %s", cudaGetErrorString(e));
    return -1;
  }
  int vs = 0;  // the multi-GPU kernels' word (a peer's failed part of a reduce-scatter)
  const int se = shard_device_error(clear, &vs);
  if (se != 0) {
    fail(B2G_ERR_CUDA, "read shard error word: %s", cudaGetErrorString((cudaError_t)se));
    return -1;
  }
  if (v == 0) v = vs;
  if (clear) {
    if (v != 0) ring_mark_dirty();  // a kernel that gave up may have left counters set
    const int z = 0;
    e = cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
    if (e != cudaSuccess) {
      fail(B2G_ERR_CUDA, "clear device error word: %s", cudaGetErrorString(e));
      return -1;
    }
  }
  return v;
}

extern "C" int b2g_set_option(const char* key, int64_t value) {
  if (!key) return B2G_ERR_INVALID_ARG;
  if (!strcmp(key, "cta_group")) {
    if (value < 0 || value > 2) return B2G_ERR_INVALID_ARG;
    opt_cta_group = value;
  } else if (!strcmp(key, "raster_group")) {
    if (value < 0) return B2G_ERR_INVALID_ARG;
    opt_raster_group = value;
  } else if (!strcmp(key, "timeout_ns")) {
    if (value <= 0) return B2G_ERR_INVALID_ARG;
    opt_timeout_ns = value;
  } else if (!strcmp(key, "force_generic")) {
    opt_force_generic = value ? 1 : 0;
  } else if (!strcmp(key, "fault_flags")) {
    opt_fault_flags = value;
  } else if (!strcmp(key, "serial_fixup")) {
    opt_serial_fixup = value ? 1 : 0;
  } else if (!strcmp(key, "pdl")) {
    opt_pdl = value ? 1 : 0;
  } else if (!strcmp(key, "cluster_fixup")) {
    opt_cluster_fixup = value ? 1 : 0;
  } else if (!strcmp(key, "tail_split")) {
    opt_tail_split = value ? 1 : 0;
  } else if (!strcmp(key, "split_k")) {
    if (value < 0 || value > 64) return B2G_ERR_INVALID_ARG;
    opt_split_k = value;
  } else if (!strcmp(key, "store_hint")) {
    opt_store_hint = value ? 1 : 0;
  } else if (!strcmp(key, "comm_timeout_ms")) {
    if (value <= 0) return B2G_ERR_INVALID_ARG;
    opt_comm_timeout_ms = value;
  } else if (!strcmp(key, "comm_nonblocking")) {
    opt_comm_nonblocking = value ? 1 : 0;
  } else if (!strcmp(key, "rs_fused")) {
    opt_rs_fused = value ? 1 : 0;
  } else if (!strcmp(key, "rs_stage")) {
    opt_rs_stage = value ? 1 : 0;
  } else if (!strcmp(key, "epi_warps")) {
    if (value != 4 && value != 8) return B2G_ERR_INVALID_ARG;
    opt_epi_warps = value;
  } else if (!strcmp(key, "pair_rows")) {
    if (value != 0 && value != 64 && value != 128) return B2G_ERR_INVALID_ARG;
    opt_pair_rows = value;
  } else if (!strcmp(key, "ring_slots")) {
    if (value < 512 || value > (int64_t)kCounterSlots || value % 64) return B2G_ERR_INVALID_ARG;
    opt_ring_slots = value;
  } else if (!strcmp(key, "tile_n")) {
    if (value != 0 && value != 128 && value != 256 && value != 512) return B2G_ERR_INVALID_ARG;
    opt_tile_n = value;
  } else {
    return B2G_ERR_INVALID_ARG;
  }
  return B2G_OK;
}

extern "C" int64_t b2g_get_option(const char* key) {
  if (!key) return -1;
  if (!strcmp(key, "launches")) return g_launches.load();
  if (!strcmp(key, "last_split_ws_bytes")) return t_split_ws;
  if (!strcmp(key, "cta_group")) return opt_cta_group;
  if (!strcmp(key, "raster_group")) return opt_raster_group;
  if (!strcmp(key, "timeout_ns")) return opt_timeout_ns;
  if (!strcmp(key, "force_generic")) return opt_force_generic;
  if (!strcmp(key, "fault_flags")) return opt_fault_flags;
  if (!strcmp(key, "tile_n")) return opt_tile_n;
  if (!strcmp(key, "store_hint")) return opt_store_hint;
  if (!strcmp(key, "split_k")) return opt_split_k;
  if (!strcmp(key, "tail_split")) return opt_tail_split;
  if (!strcmp(key, "pdl")) return opt_pdl;
  if (!strcmp(key, "cluster_fixup")) return opt_cluster_fixup;
  if (!strcmp(key, "serial_fixup")) return opt_serial_fixup;
  if (!strcmp(key, "ring_slots")) return opt_ring_slots;
  if (!strcmp(key, "pair_rows")) return opt_pair_rows;
  if (!strcmp(key, "epi_warps")) return opt_epi_warps;
  if (!strcmp(key, "rs_fused")) return opt_rs_fused;
  if (!strcmp(key, "rs_stage")) return opt_rs_stage;
  if (!strcmp(key, "comm_timeout_ms")) return opt_comm_timeout_ms;
  if (!strcmp(key, "comm_nonblocking")) return opt_comm_nonblocking;
  return -1;
}

extern "C" void b2g_tile_coord(int t, int num_m, int num_n, int group, int* tm, int* tn) {
  b2g_sched_tile(t, num_m, num_n, group, tm, tn);
}

extern "C" const char* b2g_version(void) { return "b2g_gemm 0.1 (sm_100a tcgen05)"; }

extern "C" int b2g_plan_preview(int64_t M, int64_t N, int64_t K, int dtype, int sm_count, int* cg,
                                int* bn, int* k_splits, int* num_full, int* cta_rows) {
  if (M < 1 || N < 1 || K < 1 || sm_count < 2 || !cg || !bn || !k_splits || !num_full)
    return fail(B2G_ERR_INVALID_ARG, "bad plan-preview arguments");
  if (dtype < B2G_DTYPE_F16 || dtype > B2G_DTYPE_E5M2)
    return fail(B2G_ERR_INVALID_ARG, "unknown operand type code %d", dtype);
  const int64_t kb = dtype >= B2G_DTYPE_E4M3 ? 128 : 64;  // K elements per 128-byte stage row
  const int64_t nmt = (M + 127) / 128;
  int half_opt = (int)opt_pair_rows.load();
  if (half_opt == 0 && (!opt_cluster_fixup.load() || opt_serial_fixup.load() || opt_split_k.load() > 4))
    half_opt = 128;
  const TileChoice t = choose_tiles(nmt, N, (K + kb - 1) / kb, sm_count, (int)opt_cta_group.load(),
                                    (int)opt_tile_n.load(), half_opt);
  const int64_t rows = t.half ? 64 : 128;
  const int64_t tiles = ((((M + rows - 1) / rows) + t.cg - 1) / t.cg) * ((N + t.bn - 1) / t.bn);
  if (tiles > INT32_MAX / 4) return fail(B2G_ERR_UNSUPPORTED, "too many tiles");
  const int group_cap = t.cg == 1 ? sm_count : sm_count / 2;  // CTA pairs: full occupancy assumed
  const SplitChoice s = choose_splits((int)tiles, (int)((K + kb - 1) / kb), group_cap, t.cg,
                                      (int)opt_split_k.load(), opt_tail_split.load() != 0, t.half);
  *cg = t.cg;
  *bn = t.bn;
  *k_splits = s.k_splits;
  *num_full = s.num_full;
  if (cta_rows) *cta_rows = (int)rows;
  return B2G_OK;
}
