/*
 * b2g_gemm.h - C ABI of the B200 (sm_100a) GEMM and 5-D contraction library
 * (libb2g_gemm.so).  Plain pointers and sizes only; no CUDA or framework types.
 *
 * Reference: thrasos-g/RDNA4-GEMM-WMMA.  The reference is two benchmark programs whose
 * de-facto drop-in boundary is a kernel launch on the default stream with compile-time
 * sizes; every entry point below cites the reference interface it replaces.
 *
 * Conventions (all entry points):
 *   - Device pointers are owned by the caller.  A, B are IEEE fp16 (2-byte elements);
 *     C is fp32.  C is overwritten (beta = 0), as the reference kernel does
 *     (mmm.cpp:1372, mmmTensor.cpp:251).
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream, which is what the
 *     reference launches on, mmm.cpp:1496).  Calls are asynchronous on that stream.
 *   - Return 0 (B2G_OK) on success, else a B2G_ERR_* code; b2g_last_error_string()
 *     returns a message for the calling thread's last failure.  (The reference aborts
 *     the process from HIP_CHECK / ROCBLAS_CHECK, mmm.cpp:33-49.)
 *   - Strides are in elements.  Any shape and stride set is accepted; layouts the
 *     tensor-memory kernel cannot address through TMA (unaligned bases or strides,
 *     no unit-stride K/N/M mode, ...) run on a generic CUDA kernel instead
 *     (b2g_last_path() tells which).
 *   - Numerics: fp32 accumulation of exact fp16 products.  Results agree with an FP64
 *     reference within |err| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|ref|.
 *   - Thread-safe; calls from several host threads may run concurrently (except the
 *     no-alloc entry point, whose calls share one scratch array).
 */
#ifndef B2G_GEMM_H
#define B2G_GEMM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  B2G_OK = 0,
  B2G_ERR_INVALID_ARG = 1, /* bad shape, stride or null pointer */
  B2G_ERR_UNSUPPORTED = 2, /* valid request this build cannot run (e.g. no sm_100 device) */
  B2G_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
  B2G_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up (see b2g_device_status) */
  B2G_ERR_NCCL = 5,        /* collective failure in the sharded path */
};

/* Operand element types of the typed entry points (C is always fp32). */
enum {
  B2G_DTYPE_F16 = 0,  /* IEEE binary16 (the reference's _Float16) */
  B2G_DTYPE_BF16 = 1, /* bfloat16 */
  B2G_DTYPE_E4M3 = 2, /* fp8 e4m3 (OCP / NVIDIA __nv_fp8_e4m3) */
  B2G_DTYPE_E5M2 = 3, /* fp8 e5m2 */
  B2G_DTYPE_F32 = 4,  /* IEEE binary32: output (C) type only */
};

/* Which kernel the calling thread's last successful compute call ran. */
enum {
  B2G_PATH_NONE = 0,
  B2G_PATH_TC_1CTA = 1,   /* tcgen05 kernel, one CTA per 128x256 or 128x128 tile */
  B2G_PATH_TC_2CTA = 2,   /* tcgen05 kernel, CTA pair per 256x256 or 256x512 tile (cta_group::2) */
  B2G_PATH_GENERIC = 3,   /* generic CUDA kernel (layouts outside TMA's rules) */
  B2G_PATH_ZERO = 4,      /* K == 0: C filled with zeros */
  B2G_PATH_EMPTY = 5,     /* M == 0 or N == 0: nothing to do */
};

/*
 * C[M,N] = A[M,K] . B[K,N], all row-major: A[m*lda + k], B[k*ldb + n], C[m*ldc + n].
 * Replaces the launch of WMMA_Swizzled_Full<2,2,4,4> (mmm.cpp:1214-1215 signature,
 * 1462-1472 launch configuration, 1496 launch), whose sizes are the compile-time globals
 * DIM_I/DIM_J/DIM_K (mmm.cpp:13-15) with lda = K, ldb = N, ldc = N; here they are
 * arguments.
 */
int b2g_gemm_f16_f32(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K,
                     int64_t lda, int64_t ldb, int64_t ldc, void* stream);

/*
 * C = alpha * A.B + beta * C with the layout of b2g_gemm_f16_f32.  beta == 0 never reads C;
 * beta == 1 adds alpha*A.B into C (TMA reduce-add in the epilogue: each element receives one
 * addition per call, so the result is deterministic); any other beta scales C first.
 * Extends the reference's beta = 0 semantics (mmm.cpp:1372) with the alpha/beta epilogue of
 * its rocBLAS comparison call (rocblas_gemm_ex alpha/beta, mmm.cpp:1512-1513).
 */
int b2g_gemm_ex(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K,
                int64_t lda, int64_t ldb, int64_t ldc, float alpha, float beta, void* stream);

/*
 * b2g_gemm_ex with the operand type as an argument: A and B are both `dtype`
 * (B2G_DTYPE_*), products are exact in fp32 and accumulated in fp32 (tcgen05 kind::f16 for
 * fp16/bf16, kind::f8f6f4 for the fp8 types).  fp16 is the reference's type (mmm.cpp:27);
 * bf16 and fp8 have no counterpart in the reference.
 */
int b2g_gemm_typed(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K,
                   int64_t lda, int64_t ldb, int64_t ldc, int dtype, float alpha, float beta,
                   void* stream);

/*
 * b2g_gemm_f16_f32 for callers that can't call cudaMalloc: this entry point allocates
 * nothing.  (No counterpart in the reference, which allocates everything up front in main.)
 * Some callers can't allocate device memory per call -- a host runtime that has handed all
 * device memory to its own pool allocator, or a serving loop that must not allocate on every
 * call.  When the problem has too few output tiles to fill the GPU the library splits K and
 * needs a workspace for the partial tiles; here it comes from a 32 MiB array compiled into
 * the library (every GPU that loads the library holds it until the process exits), not from
 * cudaMallocAsync.  A request whose split-K workspace would exceed 32 MiB returns
 * B2G_ERR_INVALID_ARG with a message saying so.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) for that device.  All calls share the one
 * array, and it keeps the last call's contents
 * (each call clears the split counters it relies on): calls that overlap on the GPU -- on
 * different streams, or from different host threads -- race on it and must be serialized.
 */
int b2g_gemm_f16_f32_noalloc(const void* A, const void* B, float* C, int64_t M, int64_t N,
                             int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* stream);

/*
 * The reference's drop-in form: contiguous row-major operands, lda = K, ldb = N, ldc = N,
 * default stream.  Same as GEMM_Naive's contract (mmm.cpp:52-62).
 */
int b2g_gemm(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K);

/*
 * 5-D contraction C[a,b,i,n] = sum_{j,k} A[a,b,i,j,k] * B[j,k,n].
 *   a_shape = (a,b,i,j,k), b_shape = (j,k,n), c_shape = (a,b,i,n); *_stride in elements.
 * Read in place through TMA tensor maps on these strides: no packed copy is made.
 * Replaces mmmTensor.cpp: the host pack of G into A (329-340) plus the contraction
 * kernel launch (44-45 signature, 345-355 launch configuration, 364-369 launch) with its
 * K-major Input read (168) and remapped Output store (246-252).  The reference's own
 * form Out[m,b,r] = sum_{n,k} G[r,n,m,k] * In[b,n,k] is this call with
 *   a_shape = (mt, 1, rt, nt, rt_l), a_stride = (rt_l, 0, nt*mt*rt_l, mt*rt_l, 1),
 *   b_shape = (nt, rt_l, bt),        b_stride = (rt_l, 1, nt*rt_l),
 *   c_shape = (mt, 1, rt, bt),       c_stride = (bt*rt, 0, 1, rt).
 */
int b2g_contract5d_f16_f32(const void* A, const int64_t a_shape[5], const int64_t a_stride[5],
                           const void* B, const int64_t b_shape[3], const int64_t b_stride[3],
                           float* C, const int64_t c_shape[4], const int64_t c_stride[4],
                           void* stream);

/* The contraction with the alpha/beta epilogue of b2g_gemm_ex (the reference's contraction
 * always overwrites its Output, mmmTensor.cpp:246-252; alpha/beta follow the rocBLAS call at
 * mmmTensor.cpp:393-420). */
int b2g_contract5d_ex(const void* A, const int64_t a_shape[5], const int64_t a_stride[5],
                      const void* B, const int64_t b_shape[3], const int64_t b_stride[3],
                      float* C, const int64_t c_shape[4], const int64_t c_stride[4], float alpha,
                      float beta, void* stream);

/* The contraction with an operand type argument (see b2g_gemm_typed).  No reference
 * counterpart: the reference's contraction is fp16 only. */
int b2g_contract5d_typed(const void* A, const int64_t a_shape[5], const int64_t a_stride[5],
                         const void* B, const int64_t b_shape[3], const int64_t b_stride[3],
                         float* C, const int64_t c_shape[4], const int64_t c_stride[4], int dtype,
                         float alpha, float beta, void* stream);

/* b2g_fill_uniform_f16 for any operand type: the same exact fp32 values, rounded to nearest
 * even into `dtype` (saturating to the largest finite value for the fp8 types).  Replaces
 * randomMatrix (mmm.cpp:1409-1414) for the non-fp16 types, which the reference does not have. */
int b2g_fill_uniform(void* dst, int64_t n, int dtype, uint64_t seed, uint64_t offset, void* stream);

/*
 * Fill n fp16 elements with the seeded uniform [-1,1] sequence: element e of the logical
 * stream is f(seed, offset + e).  Bit-identical to the host oracle, so a row slab of a
 * large matrix can be generated on the GPU that owns it.  Replaces randomMatrix
 * (mmm.cpp:1409-1414, mmmTensor.cpp:271-276: rand()/RAND_MAX, U[0,1], unseeded).
 */
int b2g_fill_uniform_f16(void* dst, int64_t n, uint64_t seed, uint64_t offset, void* stream);

/*
 * Multi-GPU: one rank's part of the M-row-slab sharded GEMM C[M,N] = A[M,K].B[K,N] over NCCL
 * (the reference is single-GPU and has no counterpart).  The rank's slab
 * is rows [row0, row0 + rows) of b2g_slab_rows(M, world, rank); A_slab (rows x K, lda) and
 * C_slab (rows x N, ldc) hold those rows; B is a K x N buffer (ldb) on every rank that holds
 * B on `root`.  The call broadcasts B from root in `k_panels` row panels on an internal
 * stream and runs the slab GEMM panel by panel as the panels arrive (panel 0 overwrites
 * C_slab, later panels add into it), all ordered after prior work on `stream`; C is written
 * locally with no reduction.  `comm` is an ncclComm_t (b2g_comm_init or the caller's own);
 * every rank of the communicator must make the call with the same M, N, K, root, k_panels.
 * NCCL is loaded at run time (libnccl.so.2) only by these entry points.
 */
int b2g_gemm_sharded(const void* A_slab, void* B, float* C_slab, int64_t M, int64_t N, int64_t K,
                     int64_t lda, int64_t ldb, int64_t ldc, void* comm, int root, int k_panels,
                     void* stream);

/*
 * Copy-engine broadcast chain for the M-row-slab GEMM (collective: every rank of `comm` calls
 * it with its own B buffer of `bytes` bytes; the root's holds B).  Ranks form a chain
 * root -> root+1 -> ...; each pulls K panels from the previous rank's buffer with peer copies
 * (CUDA IPC) and signals the next rank through epoch flags written by stream memory
 * operations, so the broadcast uses no SM and overlaps the slab GEMMs.  b2g_chain_plan_destroy
 * is collective too (every rank calls it); it waits for this rank's queued calls, and frees
 * memory only after every rank has dropped its mappings of it.  No reference counterpart (the
 * reference is single-GPU); BASELINE configs[4] asks for B to be broadcast over NVLink.
 */
int b2g_chain_plan_create(void* comm, void* B, int64_t bytes, int root, void** plan);
int b2g_chain_plan_destroy(void* plan);

/*
 * b2g_gemm_sharded over a chain plan: B is the plan's buffer (ldb, K rows); A_slab / C_slab
 * as in b2g_gemm_sharded.  Panel p's GEMM waits only for panel p to arrive.  The call
 * completes on `stream` once this rank's copies are done and the next rank has pulled every
 * panel from this rank's buffer, so the caller may then overwrite B.  No reference
 * counterpart (the reference is single-GPU).
 */
int b2g_gemm_sharded_chain(void* plan, const void* A_slab, float* C_slab, int64_t M, int64_t N,
                           int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int k_panels,
                           void* stream);

/*
 * The chain on its own: the first `bytes` bytes of the plan's buffer travel from the root
 * along the chain in about `panels` panels (peer copies, no SM), ordered after prior work on
 * `stream`.  The call completes on `stream` once this rank holds every byte and the next rank
 * has pulled every panel from this rank's buffer.  A caller that keeps two plans over two
 * buffers can broadcast the operand of its next step while its current step computes with
 * the other buffer.  Every rank of the plan makes the same calls in the same order.  No
 * reference counterpart (the reference is single-GPU); BASELINE configs[4] asks for B to be
 * broadcast over NVLink.
 */
int b2g_chain_broadcast(void* plan, int64_t bytes, int panels, void* stream);

/*
 * b2g_gemm_sharded_n over a chain plan whose buffer is A (M x K, lda; the root's holds A): A
 * arrives in row panels along the chain, and panel p's GEMM writes rows of this rank's column
 * slab of C (B_nslab: K x n_r, C_nslab: M x n_r with (n0, n_r) = b2g_slab_rows(N, world,
 * rank)) as soon as that panel is here.  No NCCL kernel and no SM are used for A.  No
 * reference counterpart.
 */
int b2g_gemm_sharded_n_chain(void* plan, const void* B_nslab, float* C_nslab, int64_t M,
                             int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                             int m_panels, void* stream);

/*
 * Tensor-parallel variants for shapes whose B is too large to replicate (no reference
 * counterpart).
 *
 * K-split with reduce-scatter: rank r holds the K slab b2g_slab_rows(K, world, r) of A
 * (M x k_r, lda) and of B (k_r x N, ldb); its C_slab (M/world x N, ldc) receives rows
 * [r*M/world, (r+1)*M/world) of C = sum over ranks of A_r.B_r (fp32 partials in a
 * stream-ordered scratch buffer, ncclReduceScatter).  M must be a multiple of the rank count.
 */
int b2g_gemm_sharded_k(const void* A_kslab, const void* B_kslab, float* C_slab, int64_t M,
                       int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* comm,
                       void* stream);

/*
 * The same K-split GEMM with the reduce-scatter done over peer memory (no NCCL kernel).
 * b2g_rs_plan_create (collective, once per M x N) allocates every rank's receive slots
 * (world x M/world x N fp32) and maps every peer's through CUDA IPC; in the staged form also
 * min(2, world-1) local staging buffers of M/world x N fp32 and a copy stream.  In
 * b2g_gemm_sharded_k_p2p, rank r's partial of row slab q reaches rank q's slot r, and C_slab
 * is the sum of rank r's slots in rank order.  Three forms, all giving the same bits:
 * staged (option "rs_stage", default 1, read when the plan is created and at each call): the
 * peers' partials are computed into local staging buffers and the copy engine pushes each to
 * its peer over NVLink while the next GEMM runs; direct ("rs_stage" 0): the GEMMs store their
 * tiles straight into the peers' slots; fused ("rs_stage" 0, "rs_fused" 1): direct, and rank
 * r computes its own slab last, after the peers' partials have landed, with a GEMM whose
 * epilogue adds the slots in rank order and stores C_slab (no separate reduction kernel).
 * Staged is the fastest measured.  Epoch flags written and waited for by stream memory
 * operations order the ranks.  Every rank of the plan calls it with the same M, N, K, in the
 * same order.  b2g_rs_plan_destroy is collective.
 * The ranks are processes on one node with CUDA IPC between their GPUs.  No reference
 * counterpart.
 */
int b2g_rs_plan_create(void* comm, int64_t M, int64_t N, void** plan);
int b2g_rs_plan_destroy(void* plan);
int b2g_gemm_sharded_k_p2p(void* plan, const void* A_kslab, const void* B_kslab, float* C_slab,
                           int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                           void* stream);

/*
 * The fused form's epilogue on its own, for callers that run their own exchange:
 * C (M x N, ldc) = sum over s = 0 .. count-1, in that order, of term s, where term `self` is
 * A.B (fp16 A M x K and B K x N, row-major, fp32 accumulation) and every other term is the fp32
 * M x N block slots + s * slot_stride (row pitch N).  With status != NULL, status[s] must equal
 * `epoch` for every s != self, else C is NaN and b2g_device_status reports 7 (a peer's part
 * failed).  On the tensor-core path the sum happens in the GEMM's epilogue; elsewhere a
 * separate pass gives the same bits.  slots is 16-byte aligned and slot_stride (elements) a
 * multiple of 4, at least M * N; count is at most 1024.  No reference counterpart.
 */
int b2g_gemm_sum_slots(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K,
                       int64_t lda, int64_t ldb, int64_t ldc, const float* slots,
                       int64_t slot_stride, int count, int self, const uint32_t* status,
                       uint32_t epoch, void* stream);

/*
 * N-slabs with all-gather: rank r holds the column slab b2g_slab_rows(N, world, r) of B
 * (K x n_r, ldb) and of C (M x n_r, ldc); A (M x K, lda, every rank) is broadcast from `root`
 * in `m_panels` row panels, each followed by the GEMM of its rows.  With C_full != NULL
 * (N a multiple of the rank count) every rank also receives the whole row-major C (M x N)
 * there (ncclAllGather).  No reference counterpart.
 */
int b2g_gemm_sharded_n(void* A, const void* B_nslab, float* C_nslab, int64_t M, int64_t N,
                       int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* comm, int root,
                       int m_panels, float* C_full, void* stream);

/*
 * Launch plan the library would choose for a row-major M x N x K GEMM of operand type `dtype`
 * on a GPU with `sm_count` SMs (full cluster occupancy assumed), under the current options:
 * CTAs per tile, tile width, K splits per split tile, how many tiles run unsplit, and (if
 * cta_rows is not NULL) the A rows each CTA holds: 128, or 64 for the half-height pair tile
 * (128 x 256 over a CTA pair).  No GPU needed (no reference counterpart; for tests and
 * tuning).
 */
int b2g_plan_preview(int64_t M, int64_t N, int64_t K, int dtype, int sm_count, int* cta_group,
                     int* tile_n, int* k_splits, int* num_full, int* cta_rows);

/*
 * Fused epilogue variants: C = alpha*A.B + beta*C + bias, with C stored as fp32
 * (B2G_DTYPE_F32), fp16 (B2G_DTYPE_F16) or bf16 (B2G_DTYPE_BF16).  `bias` is an optional
 * (NULL = none) fp32 vector of N elements added to every row; `dtype` is the A/B operand type
 * as in b2g_gemm_typed.  A 16-bit C is rounded to nearest even from the fp32 result and takes
 * beta = 0 only; C's leading dimension (ldc) and strides are in C elements.  No reference
 * counterpart (the reference's kernels always write fp32 C with no bias).
 */
int b2g_gemm_epilogue(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                      int64_t lda, int64_t ldb, int64_t ldc, int dtype, float alpha, float beta,
                      const float* bias, int c_dtype, void* stream);
int b2g_contract5d_epilogue(const void* A, const int64_t a_shape[5], const int64_t a_stride[5],
                            const void* B, const int64_t b_shape[3], const int64_t b_stride[3],
                            void* C, const int64_t c_shape[4], const int64_t c_stride[4], int dtype,
                            float alpha, float beta, const float* bias, int c_dtype, void* stream);

/*
 * Batch modes: the contraction with mode a shared by B,
 *   C[a,b,i,n] = alpha * sum_{j,k} A[a,b,i,j,k] B[a,j,k,n] + beta * C[a,b,i,n],
 * B's element (a, j, k, n) at a*b_batch_stride + j*b_stride[0] + k*b_stride[1] +
 * n*b_stride[2].  b2g_gemm_batched is the strided-batched GEMM C[l] = A[l].B[l] (fp16 in,
 * fp32 out) over l < L with batch strides in elements.  Batched calls use CTA-pair tiles only
 * when every batch entry has an even number of 128-row M tiles.  No
 * reference counterpart (generalises mmmTensor.cpp's fixed (a,b,i | j,k | n) roles).
 */
int b2g_contract5d_batched(const void* A, const int64_t a_shape[5], const int64_t a_stride[5],
                           const void* B, const int64_t b_shape[3], const int64_t b_stride[3],
                           int64_t b_batch_stride, float* C, const int64_t c_shape[4],
                           const int64_t c_stride[4], int dtype, float alpha, float beta,
                           void* stream);
int b2g_gemm_batched(const void* A, const void* B, float* C, int64_t L, int64_t M, int64_t N,
                     int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int64_t stride_a,
                     int64_t stride_b, int64_t stride_c, void* stream);

/* Balanced contiguous row partition: rank r gets M/world rows, the first M%world ranks one more.
 * No reference counterpart (the reference is single-GPU). */
int b2g_slab_rows(int64_t M, int world, int rank, int64_t* row0, int64_t* rows);

/* NCCL communicator helpers for callers without their own NCCL: a 128-byte unique id made on
 * one rank and shared with the others out of band, then one b2g_comm_init per rank (with that
 * rank's device current).  The communicator is non-blocking (option "comm_nonblocking"): its
 * set-up and every NCCL call the library makes on it are polled for at most the option
 * "comm_timeout_ms" (default 60000), after which the communicator is aborted
 * (ncclCommAbort) and the call returns B2G_ERR_TIMEOUT.  b2g_comm_destroy flushes this rank's
 * operations (bounded the same way) and frees the communicator.  No reference counterpart
 * (the reference is single-GPU; its HIP_CHECK exits the process, mmm.cpp:33-39). */
int b2g_comm_unique_id(void* id_out);
int b2g_comm_init(void** comm, int world, int rank, const void* id);
int b2g_comm_destroy(void* comm);

/*
 * Liveness check between steps: a one-word all-reduce over `comm` on `stream` (NULL: an
 * internal stream), waited for on the host for at most timeout_ms.  Returns B2G_OK when every
 * rank answered.  If a rank has gone (its process exited or stopped calling), the wait runs
 * out, the communicator is aborted (its kernels return) and the call returns B2G_ERR_TIMEOUT.
 * From then on every entry point given that communicator, or a chain or reduce-scatter plan
 * built on it, returns B2G_ERR_NCCL without queueing any work, and b2g_chain_plan_destroy /
 * b2g_rs_plan_destroy only free this rank's memory.  Every rank calls it at the same point of
 * its step sequence.  The library's stream-memory-operation waits (chain and peer-memory
 * plans) have no bound of their own: a caller that may lose a rank checks between steps, so
 * that no work is queued that waits for the lost rank.  No reference counterpart.
 */
int b2g_comm_check(void* comm, int64_t timeout_ms, void* stream);

/* Message for the calling thread's last failed call ("" if none).  Replaces the messages the
 * reference prints before exiting from HIP_CHECK / ROCBLAS_CHECK (mmm.cpp:33-49). */
const char* b2g_last_error_string(void);

/* Path taken by the calling thread's last successful compute call (B2G_PATH_*).  No reference
 * counterpart (the reference launches one kernel). */
int b2g_last_path(void);

/*
 * Device-side error word of the current device: 0 if every bounded wait completed, else
 * the code of the first wait that gave up.  Synchronises the device.  clear != 0 resets
 * the word.  Returns -1 if the word could not be read.  (No reference counterpart: the
 * reference has no device-side failure detection.)
 */
int b2g_device_status(int clear);

/*
 * Tuning / test options (no reference counterpart; the reference selects kernels by
 * editing source, mmm.cpp:1489,1494).  Keys:
 *   "cta_group"    0 = choose by shape (default), 1 = one CTA per tile, 2 = CTA pairs
 *   "raster_group" strip height of the persistent tile order (0 = default)
 *   "timeout_ns"   limit of every bounded device-side wait (default 2e9)
 *   "force_generic" 1 = run the generic kernel for every call (testing)
 *   "tile_n"       0 = choose by shape (default); 128 (one CTA, 128x128 tiles), 256 or 512
 *                  columns per tile (512 needs CTA pairs)
 *   "epi_warps"    8 (default) or 4: epilogue warps of the 256 x 512 CTA-pair tile.  With 8,
 *                  each warp pulls 128 columns of an accumulator N-half into registers and
 *                  hands the half back to the MMA before storing it
 *   "pair_rows"    64 = half-height pair tiles (128 x 256 over a CTA pair, UMMA M = 128 with
 *                  cta_group::2, 64 A rows per CTA) whenever the call allows them; 0 (default)
 *                  or 128 = the planner's tiles, which never include them (measured slower on
 *                  the skinny shapes they were built for)
 *   "split_k"      0 = choose by shape (default), else split every tile's K this many ways
 *   "tail_split"   1 (default) = split only the tiles of a partial last wave; 0 = never
 *   "serial_fixup" 1 = split-K partials are always summed by the last unit to arrive
 *   "store_hint"   1 = C stores carry an L2 evict-first hint
 *   "cluster_fixup" 1 (default) = when every tile of a one-CTA-tile launch is split in K (at
 *                  most 8 ways, one unit per CTA), the splits of a tile run as one thread-block
 *                  cluster and reduce their partials through distributed shared memory; 0 = the
 *                  partials go through a global workspace
 *   "pdl"          1 (default) = tensor-core launches use programmatic dependent launch (the
 *                  kernel's set-up overlaps the previous kernel in the stream); 0 = plain launch
 *   "comm_timeout_ms" bound of every NCCL wait of the multi-GPU entry points (default 60000)
 *   "comm_nonblocking" 1 (default) = b2g_comm_init makes a non-blocking NCCL communicator
 *   "rs_stage"     1 (default) = b2g_gemm_sharded_k_p2p computes the peers' partials locally
 *                  and pushes them with the copy engine; 0 = its GEMMs store into peer memory
 *   "rs_fused"     with "rs_stage" 0: 1 = sum the slots in the own slab's GEMM epilogue; 0
 *                  (default) = a separate reduction kernel (same bits)
 *   "ring_slots"   split-K arrival counters usable in the per-device ring (default and
 *                  maximum 1048576, a multiple of 64, at least 512): a small ring makes tests
 *                  wrap it often
 *   "fault_flags"  test-only fault injection: bit 0 = the TMA producer issues no loads,
 *                  so the MMA wait runs out and the call reports B2G_ERR_TIMEOUT
 * Returns B2G_OK or B2G_ERR_INVALID_ARG for an unknown key or value.  Options are
 * process-wide.  b2g_get_option("launches") (read-only) returns how many kernels the library
 * has launched in this process; b2g_get_option("last_split_ws_bytes") (read-only) the bytes of
 * split-K partial tiles the calling thread's last tensor-core launch kept in global memory (0
 * when it split nothing or reduced its splits through distributed shared memory).
 */
int b2g_set_option(const char* key, int64_t value);
int64_t b2g_get_option(const char* key);

/*
 * Host mirror of the persistent kernel's tile order: tile index t of a num_m x num_n
 * tile grid visited in strips of `group` M-tiles -> (tm, tn).  A bijection for every
 * shape (the reference's strip remap, mmm.cpp:1219-1236, is not when the grid width is
 * not a multiple of 32).  Exposed for host-side tests.
 */
void b2g_tile_coord(int t, int num_m, int num_n, int group, int* tm, int* tn);

/* Library version string.  No reference counterpart. */
const char* b2g_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* B2G_GEMM_H */
