// sm_100a GEMM / contraction kernel: C (fp32) = A (fp16) x B (fp16), fp32 accumulation in
// tensor memory.
//
// Replaces the reference's WMMA_Swizzled_Full (mmm.cpp:1214-1374) and its tensor variant
// (mmmTensor.cpp:44-257).  Same result definition (GEMM_Naive, mmm.cpp:52-62: every C element
// is the fp32-accumulated dot product of an A row and a B column, C overwritten), different
// machine: the gfx12 WMMA ladder, LDS XOR swizzles and register-blocking templates give way to
//   * TMA tensor-map loads into 128-byte-swizzled shared memory (the tensor maps carry the
//     operand strides, so the 5-D contraction is read in place, with no packing pass),
//   * a STAGES-deep mbarrier ring between one TMA producer thread and one MMA thread,
//   * tcgen05.mma (kind::f16) with the fp32 accumulator in TMEM, double-buffered so the
//     epilogue of tile t overlaps the main loop of tile t+1,
//   * CG = 2: a CTA pair (cluster of 2) shares one 256x256 tile: each CTA loads its own 128
//     A rows and half of the B columns, the even CTA issues cta_group::2 MMAs over both
//     halves.  No TMA load uses cluster multicast.
//   * an epilogue of 4 warps: TMEM -> registers -> swizzled shared memory -> TMA store,
//     which also clips ragged M/N edges (TMA zero-fill covers ragged K on the load side),
//   * a persistent grid walking the tiles in grouped order (sched.h).
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer,
// warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ptx.cuh"
#include "sched.h"

namespace b2g {

// Device-side error word: 0 = fine, otherwise the code of the first bounded wait that gave up.
// Read and cleared by b2g_device_status().
__device__ int g_device_error;

enum : int {
  ERR_WAIT_EMPTY = 1,   // producer waiting for a free pipeline stage
  ERR_WAIT_FULL = 2,    // MMA waiting for operands
  ERR_WAIT_TEMPTY = 3,  // MMA waiting for the epilogue to release an accumulator
  ERR_WAIT_TFULL = 4,   // epilogue waiting for an accumulator
  ERR_WAIT_DRAIN = 5,   // teardown waiting for copies / MMAs in flight
  ERR_WAIT_FIXUP = 6,   // split-K unit waiting for the partial tiles of its siblings
  ERR_PEER_FAILED = 7,  // a peer's part of a peer-memory reduce-scatter failed (its status word)
};

// Problem description computed on the host (b2g_api.cu) and passed by value.
//
// Rows of C are the flattened M-modes (a, b, i), i innermost; the K axis is the flattened
// (j, k), k innermost.  A 128-row CTA tile is one TMA box of bi x bb x ba rows over (i, b, a),
// bi*bb*ba == 128; each epilogue warp stores a 32-row sub-box si x sb x sa.
struct GemmParams {
  int i_size, b_size, a_size;  // M-mode extents
  int bi, bb, ba;              // load box per M-mode
  int ti, tb;                  // tiles along i and b (tiles along a = num_m_tiles/(ti*tb))
  int si, sb, sa;              // per-warp store sub-box
  int num_m_tiles;             // 128-row tiles
  int num_pm_tiles;            // tiles of 128*CG rows (one per CTA group)
  int n_size;                  // N extent
  int num_n_tiles;             // BN-column tiles
  int k_blocks_per_j;          // K blocks (128 bytes of k: 64 16-bit or 128 8-bit elements) per j
  int k_iters;                 // j * k_blocks_per_j
  int num_tiles;               // num_pm_tiles * num_n_tiles
  int raster_group;            // strip height of the tile order, in CTA-group tiles
  int store_hint;              // 1 = C stores carry an L2 evict-first hint
  int accumulate;              // 1 = C += alpha*A.B (TMA reduce-add), 0 = C = alpha*A.B
  float alpha;                 // scale of A.B
  int c_type;                  // C element type: 0 = fp32, 1 = fp16, 2 = bf16 (16-bit: row-major
                               // C, no accumulate)
  const float* bias;           // per-column fp32 bias added to alpha*A.B, or null
  int b_batched;               // 1 = mode a is a batch mode: B has a 4th tensor-map dimension
                               // indexed by the tile's a (a tile then spans a single a)
  // Work units: the first num_full tiles (in tile order) are one unit each over all of K; each
  // remaining tile is split into k_splits units, split s covering the K blocks
  // [s*k_per_split, min(k_iters, (s+1)*k_per_split)).  num_full = 0 is plain split-K (too few
  // tiles to fill the GPU); num_full = (waves)*(CTA groups) splits only the tail wave.  Unless
  // cluster_fixup is set, a split unit writes its fp32 partial tile to `ws` and bumps
  // counters[split tile*CG + cta]; the partials are summed in split order (deterministic) by the
  // parallel or the serial fix-up below, which also return the counter to zero.
  int num_full;
  int k_splits;
  int k_per_split;
  int num_units;               // num_full + (num_tiles - num_full) * k_splits
  float* ws;                   // (num_tiles - num_full) * k_splits * CG * 128 * BN floats
  int* counters;               // (num_tiles - num_full) * CG ints, zero between calls
  // 1 = parallel fix-up: every CTA group holds at most one split unit, so all splits of a tile
  // run at the same time; each waits (bounded) for the tile's partials and reduces 1/k_splits
  // of it.  0 = the unit that arrives last reduces the whole tile (no waiting).
  int fixup_parallel;
  // 1 = cluster fix-up (CG = 1, num_full = 0, one unit per CTA): the k_splits splits of a tile
  // are the CTAs of one cluster; each leaves its partial in its own shared memory and reduces
  // 1/k_splits of the tile from all of them through distributed shared memory.  No workspace.
  int cluster_fixup;
  int ab_format;               // UMMA operand format code (see make_idesc)
  unsigned long long timeout_ns;
  int fault_flags;             // test-only: bit 0 = producer issues no loads (forces a timeout)
  // Rank-order sum in the epilogue (the own row slab of the peer-memory K-split; the kernel
  // instances with ADD = true only): with add_count > 0 every stored element is the sum over
  // s = 0 .. add_count-1, in that order, of term s, where term add_self is this launch's A.B
  // and every other term is add_base[s * add_slot + row * n_size + col] (fp32 slots, e.g.
  // written by the peers).  Plain row-major C only (one M mode).  With add_status set,
  // add_status[s] must equal add_epoch for every s other than add_self, else the result is
  // NaN and the device error word records ERR_PEER_FAILED.
  const float* add_base;
  long long add_slot;
  int add_count;
  int add_self;
  const unsigned* add_status;
  unsigned add_epoch;
};

constexpr int kBM = 128;  // rows per CTA (UMMA M per CTA)
constexpr int kRowBytes = 128;  // bytes of K per stage and operand row: one 128-byte swizzle row
constexpr int kUN = 256;  // N of one UMMA instruction
constexpr int kEpiWarps = 4;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;      // all of TMEM
constexpr uint32_t kCBuf = 32 * 32 * 4;  // one 32x32 fp32 staging buffer
constexpr uint32_t kSmemLimit = 232448;  // max dynamic shared memory per CTA on sm_100

// CG: CTAs per tile (1, or 2 = cta_group::2 pair).  BN: tile width in columns (128, 256 or
// 512); a tile is (BMC*CG) x BN.  BN <= 256 keeps two accumulators in TMEM (the epilogue of
// tile t overlaps the main loop of tile t+1); BN = 512 fills TMEM with one accumulator and cuts
// the operand bytes each CTA pulls from L2 per FLOP by a quarter; BN = 128 (one CTA only)
// gives small problems four times as many tiles as the 256x512 pair tile.
// BMC: A rows per CTA.  128, or 64 for the half-height pair tile (CG = 2, BN = 256: a 128 x 256
// tile, UMMA M = 128 over the pair).  That accumulator is folded into the TMEM of each CTA:
// its 64 rows x 256 columns sit in 128 lanes x 128 columns, columns [0, 128) of the tile in
// lanes 0-63 and columns [128, 256) in lanes 64-127 (the "2x2" data-path layout of M = 128
// with cta_group::2).  It halves the partial tile a CTA holds when K is split, which is what
// bounds the split-K reduction of skinny problems.
// EW: epilogue warps, 4, or 8 for the 256 x 512 pair tile.  With one accumulator filling TMEM
// the MMA of the next tile waits for the epilogue to hand back each N-half.  Eight warps pull a
// whole N-half into registers (each warp 32 rows x 128 columns) and hand it back before they
// store it, instead of after storing 7/8 of it.
template <int CG, int BN, int BMC = kBM, int EW = 4>
struct Cfg {
  static_assert(CG == 1 || CG == 2, "CTA group");
  static_assert(EW == 4 || (EW == 8 && CG == 2 && BN == 512 && BMC == kBM), "epilogue warps");
  static_assert(BN == 256 || BN == 512 || (BN == 128 && CG == 1), "tile width");
  static_assert(BMC == kBM || (BMC == 64 && CG == 2 && BN == 256), "half-height pair tile");
  static constexpr int UN = BN < kUN ? BN : kUN;      // N of one UMMA instruction
  static constexpr int NH = BN / UN;                  // UMMA N-halves per k step
  static constexpr int ACC_COLS = BMC == kBM ? BN : BN / 2;  // TMEM columns of one accumulator
  static constexpr int UN_COLS = BMC == kBM ? UN : UN / 2;   // TMEM columns written by one UMMA
  static constexpr int ACC_BUFS = ACC_COLS <= 256 ? 2 : 1;   // accumulators held in TMEM
  static constexpr int BPH = UN / CG;                 // B columns per N-half held by one CTA
  static constexpr int BN_CTA = BN / CG;              // B columns loaded per CTA
  static constexpr uint32_t A_BYTES = BMC * kRowBytes;  // 16 KiB (8 KiB for BMC = 64)
  static constexpr uint32_t B_BYTES = BN_CTA * kRowBytes;
  static constexpr uint32_t HALF_BYTES = BPH * kRowBytes;  // one N-half of B in shared memory
  static constexpr int EPI_WARPS = EW;
  static constexpr int EPI_BUFS = EW == 8 ? 1 : 2;  // 32x32 staging buffers per epilogue warp
  static constexpr int THREADS = 64 + 32 * EW;
  static constexpr uint32_t EPI_BYTES = EW * EPI_BUFS * kCBuf;
  static constexpr int NUM_BARS_FIXED = 2 + 2 + 1 + 1;
  static constexpr int STAGES =
      (int)((kSmemLimit - 1024 - EPI_BYTES - 256) / (A_BYTES + B_BYTES)) > 8
          ? 8
          : (int)((kSmemLimit - 1024 - EPI_BYTES - 256) / (A_BYTES + B_BYTES));
  static constexpr uint32_t OFF_B = STAGES * A_BYTES;
  static constexpr uint32_t OFF_C = OFF_B + STAGES * B_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_C + EPI_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + NUM_BARS_FIXED;
  static constexpr uint32_t OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
  static constexpr uint32_t TX_BYTES = CG * (A_BYTES + B_BYTES);  // bytes per stage per group
  static constexpr int CHUNKS = ACC_COLS / 32;  // 32-column epilogue chunks per warp and tile
  static constexpr int WARP_COLS = ACC_COLS;     // tile columns one epilogue warp stores
};

static_assert(Cfg<1, 256>::SMEM_BYTES <= kSmemLimit && Cfg<1, 256>::STAGES >= 4, "CG=1 shared-memory fit");
static_assert(Cfg<2, 256>::SMEM_BYTES <= kSmemLimit && Cfg<2, 256>::STAGES >= 6, "CG=2 shared-memory fit");
static_assert(Cfg<2, 512>::SMEM_BYTES <= kSmemLimit && Cfg<2, 512>::STAGES >= 4, "BN=512 shared-memory fit");
static_assert(Cfg<2, 512, kBM, 8>::SMEM_BYTES <= kSmemLimit && Cfg<2, 512, kBM, 8>::STAGES >= 4,
              "BN=512 eight-warp shared-memory fit");
static_assert(Cfg<1, 128>::SMEM_BYTES <= kSmemLimit && Cfg<1, 128>::STAGES >= 6, "BN=128 shared-memory fit");
static_assert(Cfg<2, 256, 64>::SMEM_BYTES <= kSmemLimit && Cfg<2, 256, 64>::STAGES >= 8, "half-pair shared-memory fit");
// the cluster fix-up keeps a CTA's 128 x BN fp32 partial in its (then idle) operand stages
static_assert(Cfg<1, 128>::OFF_C >= 128u * 128u * 4u && Cfg<1, 256>::OFF_C >= 128u * 256u * 4u &&
                  Cfg<2, 256, 64>::OFF_C >= 64u * 256u * 4u,
              "partial tile fits in the operand stages");

// Instruction descriptor (kind::f16 and kind::f8f6f4 share the layout): D fp32 (bit 4), A and
// B format at bits 7 and 10 (kind::f16: 0 = F16, 1 = BF16; kind::f8f6f4: 0 = E4M3,
// 1 = E5M2), A K-major, B major per template (bit 16), N>>3 at bit 17, M>>4 at bit 24.
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, bool b_mn_major, uint32_t fmt) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Unit u -> (tile, split index, number of splits of that tile, K-block range).
__device__ __forceinline__ void unit_info(const GemmParams& p, int u, int& t, int& sp, int& ns,
                                          int& kb_lo, int& kb_hi) {
  if (u < p.num_full) {
    t = u;
    sp = 0;
    ns = 1;
    kb_lo = 0;
    kb_hi = p.k_iters;
  } else {
    const int v = u - p.num_full;
    const int st = v / p.k_splits;
    t = p.num_full + st;
    sp = v - st * p.k_splits;
    ns = p.k_splits;
    kb_lo = sp * p.k_per_split;
    kb_hi = min(p.k_iters, kb_lo + p.k_per_split);
  }
}

__device__ __forceinline__ void m_tile_origin(const GemmParams& p, int mt, int& i0, int& b0,
                                              int& a0) {
  const int ii = mt % p.ti;
  const int r = mt / p.ti;
  const int ib = r % p.tb;
  const int ia = r / p.tb;
  i0 = ii * p.bi;
  b0 = ib * p.bb;
  a0 = ia * p.ba;
}

// ESZ: operand element size in bytes (2 = fp16/bf16 via kind::f16, 1 = fp8 via kind::f8f6f4).
// A K block is 128 bytes of K (64 or 128 elements), consumed by 4 UMMAs of 32 bytes of K each.
template <int CG, int BN, bool B_KMAJOR, bool C_MCONTIG, int ESZ, int BMC = kBM, int EW = 4,
          bool ADD = false>
__global__ void __launch_bounds__(Cfg<CG, BN, BMC, EW>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using C = Cfg<CG, BN, BMC, EW>;
  constexpr int KB = kRowBytes / ESZ;                 // K elements per stage
  constexpr int ATOM = kRowBytes / ESZ;               // MN-major swizzle atom width (elements)
  constexpr uint32_t ATOM_BYTES = (uint32_t)kRowBytes * KB;  // one atom: ATOM x KB elements
  constexpr uint32_t MN_STEP = 32u / ESZ * kRowBytes;  // MN-major descriptor advance per UMMA
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint32_t base = ptx::smem_u32(smem_raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  base += pad;
  uint8_t* smem = smem_raw + pad;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA pairs are cluster ranks (2i, 2i+1); a cluster may hold several pairs (the cluster
  // fix-up of half-height pair tiles).  pair0 is the cluster rank of this CTA's pair leader.
  const uint32_t crank = (CG == 2 || p.cluster_fixup) ? ptx::cluster_ctarank() : 0u;
  const uint32_t cta_rank = (CG == 2) ? (crank & 1u) : 0u;
  const uint32_t pair0 = (CG == 2) ? (crank & ~1u) : 0u;
  const uint16_t pair_mask = (uint16_t)(0x3u << pair0);
  const bool leader = (cta_rank == 0);

  auto full_bar = [&](int s) { return base + C::OFF_BAR + 8u * s; };
  auto empty_bar = [&](int s) { return base + C::OFF_BAR + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int a) { return base + C::OFF_BAR + 8u * (2 * C::STAGES + a); };
  auto tempty_bar = [&](int a) { return base + C::OFF_BAR + 8u * (2 * C::STAGES + 2 + a); };
  const uint32_t mma_done_bar = base + C::OFF_BAR + 8u * (2 * C::STAGES + 4);
  const uint32_t ready_bar = base + C::OFF_BAR + 8u * (2 * C::STAGES + 5);  // cluster fix-up
  const uint32_t tmem_slot = base + C::OFF_MISC;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  int* err = &g_device_error;
  const unsigned long long lim = p.timeout_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(tfull_bar(a), 1);
      ptx::mbar_init(tempty_bar(a), C::EPI_WARPS * CG);
    }
    ptx::mbar_init(mma_done_bar, 1);
    ptx::mbar_init(ready_bar, p.cluster_fixup ? (uint32_t)p.k_splits : 1u);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    ptx::tma_prefetch_desc(&tmA);
    ptx::tma_prefetch_desc(&tmB);
    ptx::tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    ptx::tmem_alloc<CG>(tmem_slot, kTmemCols);
    ptx::tmem_relinquish<CG>();
  }
  ptx::tc_fence_before();
  __syncthreads();
  // CTA pairs, and the clusters of the cluster fix-up, start only once every CTA of the cluster
  // has initialised its barriers (peers arrive on them remotely).
  if (CG == 2 || p.cluster_fixup) ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(smem + C::OFF_MISC);
  // Launched with programmatic stream serialization: everything above (barrier set-up, TMEM
  // allocation, descriptor prefetch) may overlap the tail of the previous kernel in the stream;
  // no global memory is touched before the wait below, which returns once that kernel has
  // completed.  The next kernel may start its own set-up as soon as this one is running.
  ptx::grid_launch_dependents();
  ptx::grid_dependency_wait();

  const int group_id = blockIdx.x / CG;
  const int num_groups = gridDim.x / CG;

  // B columns of N-half h held by this CTA start at n0 + h*UN + cta_rank*BPH.
  auto issue_b = [&](uint32_t sb, uint32_t fb, int n0, int kc, int jj, int lb) {
#pragma unroll
    for (int h = 0; h < C::NH; ++h) {
      const int nh = n0 + h * C::UN + (int)cta_rank * C::BPH;
      const uint32_t dst = sb + (uint32_t)h * C::HALF_BYTES;
      if constexpr (B_KMAJOR) {
        if (p.b_batched)
          ptx::tma_load_4d<CG>(dst, &tmB, fb, kc, jj, nh, lb);
        else
          ptx::tma_load_3d<CG>(dst, &tmB, fb, kc, jj, nh);
      } else {
#pragma unroll
        for (int c = 0; c < C::BPH / ATOM; ++c)
          if (p.b_batched)
            ptx::tma_load_4d<CG>(dst + (uint32_t)c * ATOM_BYTES, &tmB, fb, nh + ATOM * c, kc, jj, lb);
          else
            ptx::tma_load_3d<CG>(dst + (uint32_t)c * ATOM_BYTES, &tmB, fb, nh + ATOM * c, kc, jj);
      }
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = group_id; u < p.num_units && ok; u += num_groups) {
        int t, sp, ns, kb_lo, kb_hi;
        unit_info(p, u, t, sp, ns, kb_lo, kb_hi);
        int pm, tn;
        b2g_sched_tile(t, p.num_pm_tiles, p.num_n_tiles, p.raster_group, &pm, &tn);
        const int mt = pm * CG + (int)cta_rank;
        int i0, b0, a0;
        m_tile_origin(p, mt, i0, b0, a0);
        const int n0 = tn * BN;
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          if (!ptx::mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, err, ERR_WAIT_EMPTY, lim)) {
            ok = false;
            break;
          }
          const uint32_t fb = (CG == 1) ? full_bar(s) : ptx::mapa(full_bar(s), pair0);
          if (leader) ptx::mbar_arrive_expect_tx(full_bar(s), C::TX_BYTES);
          if (p.fault_flags & 1) continue;
          const int jj = kb / p.k_blocks_per_j;
          const int kc = (kb - jj * p.k_blocks_per_j) * KB;
          ptx::tma_load_5d<CG>(base + s * C::A_BYTES, &tmA, fb, kc, jj, i0, b0, a0);
          issue_b(base + C::OFF_B + s * C::B_BYTES, fb, n0, kc, jj, a0);
        }
      }
      // Teardown: every load this thread issued must land before the CTA can exit.  With
      // CG == 1 the last min(it, STAGES) loads each completed (or will complete) a phase of
      // their stage's full barrier; wait for those phases.  (With CG == 2 in a normal exit the
      // leader's MMA thread consumed every stage before the final cluster barrier.)
      if (CG == 1 && !(p.fault_flags & 1)) {
        const int pending = it < C::STAGES ? it : C::STAGES;
        for (int q = 0; q < pending; ++q) {
          const int i2 = it - 1 - q;
          ptx::mbar_wait_drain(full_bar(i2 % C::STAGES), (uint32_t)(i2 / C::STAGES) & 1u, err,
                               ERR_WAIT_DRAIN, lim);
        }
      }
      if (!ok || *abort_flag) ptx::spin_ns(200000ull);  // abnormal exit: grace period for copies
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (leader && lane == 0) {
      const uint32_t idesc = make_idesc(BMC * CG, C::UN, !B_KMAJOR, (uint32_t)p.ab_format);
      int it = 0, tc = 0;
      bool ok = true;
      // Issue the MMAs of K block kb from stage s into N-halves [h_lo, h_hi).
      auto issue_mma = [&](uint32_t d, int s, int kb, int h_lo, int h_hi) {
        const uint32_t sa = base + s * C::A_BYTES;
        const uint32_t sb = base + C::OFF_B + s * C::B_BYTES;
#pragma unroll
        for (int k16 = 0; k16 < 4; ++k16) {  // 4 UMMAs of 32 bytes of K
          const uint64_t ad = ptx::smem_desc_sw128(sa + 32u * k16, 16u, 1024u);
#pragma unroll
          for (int h = 0; h < C::NH; ++h) {
            if (h < h_lo || h >= h_hi) continue;
            const uint32_t bh = sb + (uint32_t)h * C::HALF_BYTES;
            const uint64_t bd = B_KMAJOR ? ptx::smem_desc_sw128(bh + 32u * k16, 16u, 1024u)
                                         : ptx::smem_desc_sw128(bh + MN_STEP * k16, ATOM_BYTES, 1024u);
            ptx::umma<CG, ESZ>(d + (uint32_t)h * C::UN_COLS, ad, bd, idesc, (kb | k16) != 0 ? 1u : 0u);
          }
        }
      };
      for (int u = group_id; u < p.num_units && ok; u += num_groups, ++tc) {
        int t, sp, ns, kb_lo, kb_hi;
        unit_info(p, u, t, sp, ns, kb_lo, kb_hi);
        const int nkb = kb_hi - kb_lo;
        // BN <= 256: two accumulators, tempty[acc] guards accumulator acc.
        // BN = 512: one accumulator, tempty[h] guards its N-half h (the epilogue frees the
        // halves one after the other).
        const int acc = (C::ACC_BUFS == 2) ? (tc & 1) : 0;
        const uint32_t aph = (uint32_t)(C::ACC_BUFS == 2 ? (tc >> 1) : tc) & 1u;
        if (!ptx::mbar_wait(tempty_bar(acc), aph ^ 1u, abort_flag, err, ERR_WAIT_TEMPTY, lim)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)acc * C::ACC_COLS;
        int kb = 0;  // K block of this unit, relative to kb_lo
        if constexpr (C::NH == 2) {
          // Half 0 of every K block already in shared memory first, then wait for half 1 of
          // the accumulator (still being read by the epilogue) and complete those blocks.
          const int pro = nkb < C::STAGES ? nkb : C::STAGES;
          for (; kb < pro; ++kb) {
            const int s = (it + kb) % C::STAGES;
            const uint32_t ph = (uint32_t)((it + kb) / C::STAGES) & 1u;
            if (!ptx::mbar_wait(full_bar(s), ph, abort_flag, err, ERR_WAIT_FULL, lim)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            issue_mma(d, s, kb, 0, 1);
          }
          if (!ok) break;
          if (!ptx::mbar_wait(tempty_bar(1), aph ^ 1u, abort_flag, err, ERR_WAIT_TEMPTY, lim)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          for (int k2 = 0; k2 < pro; ++k2) {
            const int s = (it + k2) % C::STAGES;
            issue_mma(d, s, k2, 1, 2);
            ptx::umma_commit<CG>(empty_bar(s), pair_mask);
          }
          it += pro;
        }
        for (; kb < nkb; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          if (!ptx::mbar_wait(full_bar(s), ph, abort_flag, err, ERR_WAIT_FULL, lim)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          issue_mma(d, s, kb, 0, C::NH);
          ptx::umma_commit<CG>(empty_bar(s), pair_mask);
        }
        if (!ok) break;
        ptx::umma_commit<CG>(tfull_bar(acc), pair_mask);
      }
      // Teardown: all MMAs issued by this thread must finish before TMEM/shared memory go away.
      ptx::umma_commit<CG>(mma_done_bar, (uint16_t)(0x1u << pair0));
      ptx::mbar_wait_drain(mma_done_bar, 0u, err, ERR_WAIT_DRAIN, lim);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter
    // EW = 8: warps 2-5 and 6-9 cover the four lane quarters twice; `part` picks the 128
    // columns of each N-half this warp handles.  EW = 4: one warp per quarter, every column.
    const int part = (warp - 2) >> 2;
    auto mine = [&](int ch) { return C::EPI_WARPS == 4 || ((ch >> 2) & 1) == part; };
    const uint32_t cbuf = base + C::OFF_C + (uint32_t)(warp - 2) * (uint32_t)C::EPI_BUFS * kCBuf;
    // This warp's 32-row sub-box inside the CTA's BMC-row tile (flattened (a, b, i) order) and
    // its columns: BMC = 128, all BN columns of rows 32q..32q+31; BMC = 64 (folded
    // accumulator), columns [(q/2)*BN/2, (q/2+1)*BN/2) of rows 32(q%2)..32(q%2)+31.
    const int r0 = BMC == kBM ? 32 * q : 32 * (q & 1);
    // rank-order sum: the peers' status words are final before the launch (the stream waited
    // for their flags), so each warp reads them once
    bool add_failed = false;
    if constexpr (ADD) {
      if (p.add_count > 0 && p.add_status != nullptr) {
        for (int s2 = 0; s2 < p.add_count; ++s2)
          if (s2 != p.add_self && __ldcg(p.add_status + s2) != p.add_epoch) add_failed = true;
        if (add_failed && lane == 0) atomicCAS(err, 0, ERR_PEER_FAILED);
      }
    }
    const int col_off = BMC == kBM ? 0 : (q >> 1) * C::WARP_COLS;
    const int a_l = r0 / (p.bi * p.bb);
    const int b_l = (r0 / p.bi) % p.bb;
    const int i_l = r0 % p.bi;
    int tc = 0, nstore = 0;
    for (int u = group_id; u < p.num_units; u += num_groups, ++tc) {
      int t, sp, ns, kb_lo, kb_hi;
      unit_info(p, u, t, sp, ns, kb_lo, kb_hi);
      int pm, tn;
      b2g_sched_tile(t, p.num_pm_tiles, p.num_n_tiles, p.raster_group, &pm, &tn);
      const int mt = pm * CG + (int)cta_rank;
      int i0, b0, a0;
      m_tile_origin(p, mt, i0, b0, a0);
      const int ci = i0 + i_l, cb = b0 + b_l, ca = a0 + a_l;
      const bool rows_valid = mt < p.num_m_tiles && ci < p.i_size && cb < p.b_size && ca < p.a_size;
      const int acc = (C::ACC_BUFS == 2) ? (tc & 1) : 0;
      const uint32_t aph = (uint32_t)(C::ACC_BUFS == 2 ? (tc >> 1) : tc) & 1u;
      if constexpr (ADD) {
        // rank-order sum: while the tile's MMAs run, bring this lane's row of every other
        // term (the columns this warp stores) into L2, so that the epilogue's reads hit there
        const int row = ci + lane;
        if (p.add_count > 1 && !add_failed && rows_valid && row < p.i_size && ns == 1) {
          const int nb = tn * BN + col_off;
          for (int s2 = 0; s2 < p.add_count; ++s2) {
            if (s2 == p.add_self) continue;
            const float* rp = p.add_base + (size_t)s2 * (size_t)p.add_slot +
                              (size_t)row * (size_t)p.n_size;
#pragma unroll
            for (int ch = 0; ch < C::CHUNKS; ++ch) {
              const int gc = nb + 32 * ch;
              if (!mine(ch) || gc >= p.n_size) continue;
              const uint32_t bytes = (uint32_t)min(32, p.n_size - gc) * 4u & ~15u;
              if (bytes && (reinterpret_cast<uintptr_t>(rp + gc) & 15) == 0)
                ptx::bulk_prefetch_l2(rp + gc, bytes);
            }
          }
        }
      }
      const bool got = ptx::mbar_wait(tfull_bar(acc), aph, abort_flag, err, ERR_WAIT_TFULL, lim);
      if (!__all_sync(0xffffffffu, got)) break;
      ptx::tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)acc * C::ACC_COLS;
      const int n0 = tn * BN + col_off;

      // Stage chunk `ch` (32 columns of this warp's 32 rows) and TMA-store it.
      auto store_chunk = [&](const uint32_t (&v)[32], int ch) {
        const int gcol = n0 + 32 * ch;
        if (!rows_valid || gcol >= p.n_size) return;
        const uint32_t buf = cbuf + (uint32_t)(C::EPI_BUFS == 2 ? (nstore & 1) : 0) * kCBuf;
        if (lane == 0) {
          if constexpr (C::EPI_BUFS == 2)
            ptx::bulk_wait_read<1>();
          else
            ptx::bulk_wait_read<0>();
        }
        __syncwarp();
        uint32_t w[32];
        if (ADD && p.add_count > 0) {
          // rank-order sum (compiled only into the ADD instances, so that the plain kernels
          // keep their registers): term add_self is v, the others come from the peers' slots
          // (row = this lane's row of the plain row-major C)
          const int row = ci + lane;
          if (add_failed) {
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = 0x7fc00000u;  // NaN
          } else {
            float a[32];
            const bool vec = gcol + 32 <= p.n_size && (p.n_size & 3) == 0;
            // each term is added straight into a (the first one assigned), so no second
            // 32-value array is live
#pragma unroll 1
            for (int s2 = 0; s2 < p.add_count; ++s2) {
              const bool first = s2 == 0;
              if (s2 == p.add_self) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  a[j] = first ? __uint_as_float(v[j]) : a[j] + __uint_as_float(v[j]);
              } else if (row < p.i_size) {
                const float* src = p.add_base + (size_t)s2 * (size_t)p.add_slot +
                                   (size_t)row * (size_t)p.n_size + gcol;
                if (vec) {
#pragma unroll
                  for (int j = 0; j < 8; ++j) {
                    const float4 x = __ldcg(reinterpret_cast<const float4*>(src) + j);
                    a[4 * j] = first ? x.x : a[4 * j] + x.x;
                    a[4 * j + 1] = first ? x.y : a[4 * j + 1] + x.y;
                    a[4 * j + 2] = first ? x.z : a[4 * j + 2] + x.z;
                    a[4 * j + 3] = first ? x.w : a[4 * j + 3] + x.w;
                  }
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j) {
                    const float x = gcol + j < p.n_size ? __ldcg(src + j) : 0.0f;
                    a[j] = first ? x : a[j] + x;
                  }
                }
              } else if (first) {
#pragma unroll
                for (int j = 0; j < 32; ++j) a[j] = 0.0f;  // a row past M: clipped by the store
              }
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(a[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) w[j] = v[j];
        }
#pragma unroll
        for (int j = 0; j < 32; ++j)
          w[j] = p.alpha == 1.0f ? w[j] : __float_as_uint(__uint_as_float(w[j]) * p.alpha);
        if (p.bias) {
          // the same 32 bias values for every lane (broadcast loads); columns past N are not
          // read (the store clips them)
          if (gcol + 32 <= p.n_size) {
            const float4* bq = reinterpret_cast<const float4*>(p.bias + gcol);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 b = __ldg(bq + j);
              w[4 * j] = __float_as_uint(__uint_as_float(w[4 * j]) + b.x);
              w[4 * j + 1] = __float_as_uint(__uint_as_float(w[4 * j + 1]) + b.y);
              w[4 * j + 2] = __float_as_uint(__uint_as_float(w[4 * j + 2]) + b.z);
              w[4 * j + 3] = __float_as_uint(__uint_as_float(w[4 * j + 3]) + b.w);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (gcol + j < p.n_size)
                w[j] = __float_as_uint(__uint_as_float(w[j]) + __ldg(p.bias + gcol + j));
          }
        }
        if (p.c_type != 0) {
          // 16-bit C: row `lane` as 4 16-byte chunks (32 values rounded to nearest), 64-byte
          // swizzle: chunk j -> j ^ ((row / 2) % 4)
          uint32_t h[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float x0 = __uint_as_float(w[2 * j]), x1 = __uint_as_float(w[2 * j + 1]);
            if (p.c_type == 1) {
              const __half2 t = __floats2half2_rn(x0, x1);
              h[j] = *reinterpret_cast<const uint32_t*>(&t);
            } else {
              const __nv_bfloat162 t = __floats2bfloat162_rn(x0, x1);
              h[j] = *reinterpret_cast<const uint32_t*>(&t);
            }
          }
          const uint32_t row = buf + (uint32_t)lane * 64u;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            ptx::st_shared_v4(row + (uint32_t)((j ^ ((lane >> 1) & 3)) << 4), h[4 * j],
                              h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
        } else         if constexpr (!C_MCONTIG) {
          // Row `lane` as 8 16-byte chunks, 128-byte swizzle: chunk j -> j ^ (row % 8).
          const uint32_t row = buf + (uint32_t)lane * 128u;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            ptx::st_shared_v4(row + (uint32_t)((j ^ (lane & 7)) << 4), w[4 * j], w[4 * j + 1],
                              w[4 * j + 2], w[4 * j + 3]);
        } else {
          // Box order (i, n, b, a): element (row, col) at ((row / si) * 32 + col) * si + row % si.
          const int blk = lane / p.si, il = lane - blk * p.si;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            ptx::st_shared_b32(buf + 4u * (uint32_t)((blk * 32 + j) * p.si + il), w[j]);
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int x0 = C_MCONTIG ? ci : gcol, x1 = C_MCONTIG ? gcol : ci;
          if (p.accumulate)
            ptx::tma_reduce_add_4d(&tmC, buf, x0, x1, cb, ca);
          else if (p.store_hint)
            ptx::tma_store_4d_hint(&tmC, buf, x0, x1, cb, ca, ptx::policy_evict_first());
          else
            ptx::tma_store_4d(&tmC, buf, x0, x1, cb, ca);
          ptx::bulk_commit();
        }
        ++nstore;
      };

      // Hand accumulator (or N-half) `rel` back to the MMA warp.
      auto release = [&](int rel) {
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 1)
            ptx::mbar_arrive(tempty_bar(rel));
          else
            ptx::mbar_arrive_cluster(tempty_bar(rel), pair0);
        }
      };

      if ((CG == 1 || BMC != kBM) && ns > 1 && p.cluster_fixup) {
        // ---- cluster fix-up: partial tile -> this CTA's shared memory (the operand stages,
        // idle after its only unit's main loop) as float4 [chunk][warp][j][lane]; then split sp
        // sums chunks sp, sp + ns, ... over the ns CTAs of the cluster that hold the same rows
        // (distributed shared memory, in split order) and stores them.  One-CTA tiles: split r
        // is cluster rank r.  Half-height pairs: split r is the pair at cluster ranks 2r, 2r+1,
        // and this CTA's counterpart in it is rank 2r + cta_rank.
        auto split_cta = [&](int r) -> uint32_t {
          return CG == 1 ? (uint32_t)r : (uint32_t)(2 * r) + cta_rank;
        };
        const uint32_t part = base + (uint32_t)(q * 8 * 32 + lane) * 16u;
        ptx::fence_proxy_async_smem();
        // four chunks of TMEM loads in flight per wait (the wait is the cost here)
        static_assert(C::CHUNKS % 4 == 0, "fix-up copies four chunks per TMEM wait");
#pragma unroll 1
        for (int ch0 = 0; ch0 < C::CHUNKS; ch0 += 4) {
          uint32_t w4[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) ptx::tmem_ld_32x32b_x32(tbase + 32u * (ch0 + c), w4[c]);
          ptx::tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 0; j < 8; ++j)
              ptx::st_shared_v4(part + (uint32_t)(((ch0 + c) * 4 * 8 + j) * 32) * 16u,
                                w4[c][4 * j], w4[c][4 * j + 1], w4[c][4 * j + 2], w4[c][4 * j + 3]);
        }
        release(acc);
        // Publish: after the epilogue warps' barrier one thread arrives (release, cluster
        // scope) on the ready barrier of every CTA of the cluster, then waits (acquire) until
        // all ns partials of the tile are in place.
        ptx::named_barrier_sync(1, C::EPI_WARPS * 32);
        volatile int* ready_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);
        if (threadIdx.x == 64) {
          for (int r = 0; r < ns; ++r) ptx::mbar_arrive_cluster(ready_bar, split_cta(r));
          *ready_flag = ptx::mbar_wait_cluster(ready_bar, 0u, abort_flag, err, ERR_WAIT_FIXUP, lim)
                            ? 1 : 0;
        }
        ptx::named_barrier_sync(1, C::EPI_WARPS * 32);
        if (*ready_flag) {
#pragma unroll 1
          for (int ch = sp; ch < C::CHUNKS; ch += ns) {
            float a[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] = 0.0f;
            // Splits in order (deterministic sums), four splits' loads in flight at a time.
            const uint32_t off = part + (uint32_t)(ch * 4 * 8 * 32) * 16u;
#pragma unroll 1
            for (int r0 = 0; r0 < ns; r0 += 4) {
              float4 x[4][8];
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                if (r0 + c >= ns) break;
                const uint32_t src = ptx::mapa(off, split_cta(r0 + c));
#pragma unroll
                for (int j = 0; j < 8; ++j) x[c][j] = ptx::ld_shared_cluster_v4(src + (uint32_t)(j * 32) * 16u);
              }
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                if (r0 + c >= ns) break;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  a[4 * j] += x[c][j].x;
                  a[4 * j + 1] += x[c][j].y;
                  a[4 * j + 2] += x[c][j].z;
                  a[4 * j + 3] += x[c][j].w;
                }
              }
            }
            uint32_t vv[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) vv[j] = __float_as_uint(a[j]);
            store_chunk(vv, ch);
          }
        }
        continue;
      }
      if (BMC != kBM && ns > 1) {
        // half-height pair tiles split K only with the cluster fix-up (the launcher never
        // plans otherwise); record the inconsistency and leave C untouched
        if (lane == 0) atomicCAS(err, 0, ERR_WAIT_FIXUP);
        release(acc);
        continue;
      }
      if (ns > 1) {
        // ---- split-K unit: partial tile -> workspace, then the fix-up reduces the tile.
        // Workspace block of (split unit, CTA): 128 x BN floats as float4 [chunk][warp][j][lane]
        // (lane = row within the warp's 32 rows, j = columns 4j..4j+3 of the 32-column chunk),
        // so every warp-wide store and load covers 512 contiguous bytes.
        const size_t blk = (size_t)128 * BN;
        const int v = u - p.num_full;   // split unit index
        const int st = t - p.num_full;  // split tile index
        float4* mine_ws = reinterpret_cast<float4*>(p.ws + ((size_t)v * CG + cta_rank) * blk) +
                          (size_t)q * 8 * 32 + lane;
        uint32_t w0[32], w1[32];
        if constexpr (C::EPI_WARPS == 8) {
          // this warp's chunks only, two at a time (no loads in flight across iterations)
#pragma unroll 1
          for (int ch = 0; ch < C::CHUNKS; ch += 2) {
            if (!mine(ch)) continue;
            ptx::tmem_ld_32x32b_x32(tbase + 32u * ch, w0);
            ptx::tmem_ld_32x32b_x32(tbase + 32u * (ch + 1), w1);
            ptx::tmem_ld_wait();
            float4* d0 = mine_ws + (size_t)ch * 4 * 8 * 32;
            float4* d1 = mine_ws + (size_t)(ch + 1) * 4 * 8 * 32;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              __stcg(d0 + 32 * j, make_float4(__uint_as_float(w0[4 * j]), __uint_as_float(w0[4 * j + 1]),
                                              __uint_as_float(w0[4 * j + 2]), __uint_as_float(w0[4 * j + 3])));
              __stcg(d1 + 32 * j, make_float4(__uint_as_float(w1[4 * j]), __uint_as_float(w1[4 * j + 1]),
                                              __uint_as_float(w1[4 * j + 2]), __uint_as_float(w1[4 * j + 3])));
            }
          }
        } else {
        ptx::tmem_ld_32x32b_x32(tbase, w0);
#pragma unroll 1
        for (int ch = 0; ch < C::CHUNKS; ch += 2) {
          ptx::tmem_ld_wait();
          ptx::tmem_ld_32x32b_x32(tbase + 32u * (ch + 1), w1);
          float4* d0 = mine_ws + (size_t)ch * 4 * 8 * 32;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(d0 + 32 * j, make_float4(__uint_as_float(w0[4 * j]), __uint_as_float(w0[4 * j + 1]),
                                            __uint_as_float(w0[4 * j + 2]), __uint_as_float(w0[4 * j + 3])));
          ptx::tmem_ld_wait();
          if (ch + 2 < C::CHUNKS) ptx::tmem_ld_32x32b_x32(tbase + 32u * (ch + 2), w0);
          float4* d1 = mine_ws + (size_t)(ch + 1) * 4 * 8 * 32;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(d1 + 32 * j, make_float4(__uint_as_float(w1[4 * j]), __uint_as_float(w1[4 * j + 1]),
                                            __uint_as_float(w1[4 * j + 2]), __uint_as_float(w1[4 * j + 3])));
        }
        }
        if constexpr (C::ACC_BUFS == 2) {
          release(acc);
        } else {
          release(0);
          release(1);
        }
        // One thread publishes the partial: the barrier orders the epilogue threads' stores
        // before its acq_rel (gpu scope) atomic, and its acquire, followed by the second
        // barrier, orders the siblings' partials before every thread's loads below.
        ptx::named_barrier_sync(1, C::EPI_WARPS * 32);
        volatile int* last_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);
        int* ctr = p.counters + (size_t)st * CG + cta_rank;
        int ch_first = 0, ch_step = 1;
        if (p.fixup_parallel) {
          // publish this partial, then wait until every split of the tile has published
          if (threadIdx.x == 64) {
            ptx::atom_add_acq_rel_gpu(ctr, 1);
            *last_flag = ptx::wait_counter_ge(ctr, ns, abort_flag, err, ERR_WAIT_FIXUP, lim) ? 1 : 0;
          }
          ch_first = sp;  // this unit reduces chunks sp, sp + ns, ...
          ch_step = ns;
        } else if (threadIdx.x == 64) {
          const int old = ptx::atom_add_acq_rel_gpu(ctr, 1);
          const int last = old == p.k_splits - 1;
          if (last) *ctr = 0;  // every split has arrived: ready for the next call
          *last_flag = last;
        }
        ptx::named_barrier_sync(1, C::EPI_WARPS * 32);
        if (*last_flag) {
          const float4* tile4 = reinterpret_cast<const float4*>(
                                    p.ws + ((size_t)st * p.k_splits * CG + cta_rank) * blk) +
                                (size_t)q * 8 * 32 + lane;
          const size_t split_stride = (size_t)CG * blk / 4;  // float4s between splits
#pragma unroll 1
          for (int ch = ch_first; ch < C::CHUNKS; ch += ch_step) {
            if (!mine(ch)) continue;
            const float4* src = tile4 + (size_t)ch * 4 * 8 * 32;
            float a[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] = 0.0f;
            // Partials are summed in split order (deterministic); two splits' loads are in
            // flight at a time.
            int sp = 0;
#pragma unroll 1
            for (; sp + 1 < p.k_splits; sp += 2) {
              float4 x[8], y[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) x[j] = __ldcg(src + sp * split_stride + 32 * j);
#pragma unroll
              for (int j = 0; j < 8; ++j) y[j] = __ldcg(src + (sp + 1) * split_stride + 32 * j);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                a[4 * j] += x[j].x;
                a[4 * j + 1] += x[j].y;
                a[4 * j + 2] += x[j].z;
                a[4 * j + 3] += x[j].w;
              }
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                a[4 * j] += y[j].x;
                a[4 * j + 1] += y[j].y;
                a[4 * j + 2] += y[j].z;
                a[4 * j + 3] += y[j].w;
              }
            }
            if (sp < p.k_splits) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 x = __ldcg(src + sp * split_stride + 32 * j);
                a[4 * j] += x.x;
                a[4 * j + 1] += x.y;
                a[4 * j + 2] += x.z;
                a[4 * j + 3] += x.w;
              }
            }
            uint32_t vv[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) vv[j] = __float_as_uint(a[j]);
            store_chunk(vv, ch);
          }
        }
        ptx::named_barrier_sync(1, C::EPI_WARPS * 32);
        if (p.fixup_parallel && threadIdx.x == 64) {
          // done reading the partials; the last split to get here resets the counter
          if (ptx::atom_add_acq_rel_gpu(ctr, 1) == 2 * ns - 1) *ctr = 0;
        }
        continue;
      }

      if constexpr (C::EPI_WARPS == 8) {
        // N-half h: this warp's four chunks (h*8 + part*4 + c) into registers, hand the half
        // back to the MMA warp as soon as all eight warps have loaded theirs, then store them.
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          const int ch0 = h * 8 + part * 4;
          uint32_t v[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) ptx::tmem_ld_32x32b_x32(tbase + 32u * (ch0 + c), v[c]);
          ptx::tmem_ld_wait();
          release(h);
#pragma unroll
          for (int c = 0; c < 4; ++c) store_chunk(v[c], ch0 + c);
        }
        continue;
      }
      // TMEM loads are software-pipelined: chunk ch+1 is in flight while chunk ch is stored.
      uint32_t v0[32], v1[32];
      ptx::tmem_ld_32x32b_x32(tbase, v0);
#pragma unroll 1
      for (int ch = 0; ch < C::CHUNKS; ch += 2) {
        ptx::tmem_ld_wait();
        ptx::tmem_ld_32x32b_x32(tbase + 32u * (ch + 1), v1);
        store_chunk(v0, ch);
        ptx::tmem_ld_wait();
        if ((ch + 2) % 8 == 0 || ch + 2 >= C::CHUNKS) {
          // An N-half (BN = 512) or the whole accumulator (BN <= 256) has been read: hand it
          // back to the MMA warp.
          release(C::ACC_BUFS == 2 ? acc : (ch + 1) / 8);
        }
        if (ch + 2 < C::CHUNKS) ptx::tmem_ld_32x32b_x32(tbase + 32u * (ch + 2), v0);
        store_chunk(v1, ch + 1);
      }
    }
    if (lane == 0) ptx::bulk_wait_all();
    __syncwarp();
  }

  // ------------------------------------------------------------ teardown
  __syncwarp();
  ptx::tc_fence_before();
  __syncthreads();
  if (CG == 2 || p.cluster_fixup) {
    // no CTA of the cluster leaves (freeing its shared memory and TMEM) while a peer may
    // still read its shared memory or signal its barriers
    __syncwarp();
    ptx::cluster_sync();
  }
  ptx::tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    ptx::tmem_dealloc<CG>(tmem_base, kTmemCols);
  }
}

}  // namespace b2g
