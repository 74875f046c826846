/*
 * CPU oracle for the fp16 x fp16 -> fp32 GEMM and the 5-D contraction.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load this library.  The
 * product path (the CUDA library in rdna4-gemm-wmma_b200/) never links, loads
 * or calls it.
 *
 * What this restates (reference = thrasos-g/RDNA4-GEMM-WMMA):
 *   - GEMM_Naive, mmm.cpp:52-62: C[r,c] = sum_k float(A[r,k]) * float(B[k,c]),
 *     fp32 accumulator, k ascending, row-major A (lda=K), B (ldb=N), C (ldc=N).
 *     orc_gemm_f32_seq() is that loop.  Because every fp16*fp16 product is
 *     exact in fp32 (11+11 significand bits <= 24), fused and unfused
 *     multiply-add give the same bits, so this matches the GPU kernel of the
 *     reference bit for bit whatever its FMA contraction.
 *   - orc_gemm_f32_blocked(): the same arithmetic (fp32 accumulate, k
 *     ascending for every element) cache-blocked and multithreaded; the CPU
 *     baseline that bench.py times.  Bit-identical to orc_gemm_f32_seq().
 *   - orc_gemm_f64(): FP64-accumulated reference used for tolerance checks.
 *   - orc_contract5d_f64(): C[a,b,i,n] = sum_{j,k} A[a,b,i,j,k] * B[j,k,n] over
 *     arbitrary element strides; the reference's own form
 *     Out[m,b,r] = sum_{n,k} G[r,n,m,k] * In[b,n,k] (mmmTensor.cpp:329-340
 *     pack, 246-252 output remap, 285-286 check remap) is this with permuted
 *     strides.
 *   - orc_fill_uniform_f16(): seeded counter-based U[-1,1] fp16 generator.  It
 *     replaces randomMatrix (mmm.cpp:1409-1414, rand()/RAND_MAX, U[0,1],
 *     unseeded) with a generator the CUDA library reproduces bit for bit.
 *   - orc_check_tolerance(): |C - R| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|R|,
 *     the abs+rel bound that replaces validateResults (mmm.cpp:1387-1407,
 *     pure relative 1e-4), which is unusable once U[-1,1] inputs cancel.
 *
 * Parity pinning: the reference ships no golden vectors or known-answer
 * tests.  tests/golden/ holds fixtures produced by the reference's own
 * GEMM_Naive body and validateResults / G-pack code, extracted from the
 * reference sources at fixture-generation time and compiled on the CPU
 * (oracle/build_ref.py); tests/test_oracle.py pins this file against them.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ------------------------------------------------------------------ */
/* fp16 <-> fp32, exact bit manipulation (IEEE 754 binary16)           */
/* ------------------------------------------------------------------ */
float orc_h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do { e++; man <<= 1; } while ((man & 0x400) == 0);
      man &= 0x3ff;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* Round-to-nearest-even fp32 -> fp16. */
uint16_t orc_f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) { /* inf / nan */
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
  }
  if (ax >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
    return (uint16_t)(sign | 0x7c00u);
  }
  if (ax < 0x38800000u) { /* below min normal half (2^-14): subnormal or 0 */
    if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25 rounds to 0 */
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    /* value = m * 2^(e-150); half subnormal unit = 2^-24 -> q = m * 2^(e-126) */
    uint32_t s = 126 - e; /* number of bits to drop, in [14, 24] */
    uint32_t q = m >> s;
    uint32_t rem = m & ((1u << s) - 1);
    uint32_t half = 1u << (s - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 127 + 15;
  uint32_t m = ax & 0x7fffffu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
  return (uint16_t)(sign | q);
}

void orc_h2f_array(const uint16_t* h, float* f, int64_t n) {
  for (int64_t i = 0; i < n; ++i) f[i] = orc_h2f(h[i]);
}

void orc_f2h_array(const float* f, uint16_t* h, int64_t n) {
  for (int64_t i = 0; i < n; ++i) h[i] = orc_f2h(f[i]);
}

/* ------------------------------------------------------------------ */
/* Counter-based generator: splitmix64 finaliser over (seed, index).    */
/* value = (r24 - 2^23) / 2^23, exact in fp32, then RNE to fp16.        */
/* The CUDA library's b2g_fill_uniform_f16 computes the same function. */
/* ------------------------------------------------------------------ */
static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint16_t orc_uniform_f16_at(uint64_t seed, uint64_t index) {
  uint64_t h = mix64(mix64(seed) + index);
  int32_t r = (int32_t)(h >> 40) - 8388608; /* [-2^23, 2^23) */
  float v = (float)r * (1.0f / 8388608.0f);
  return orc_f2h(v);
}

void orc_fill_uniform_f16(uint16_t* out, int64_t n, uint64_t seed, uint64_t offset) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_uniform_f16_at(seed, offset + (uint64_t)i);
}

/* ------------------------------------------------------------------ */
/* Thread pool helper: run fn(ctx, lo, hi) over [0, n) split in chunks. */
/* ------------------------------------------------------------------ */
typedef void (*range_fn)(void* ctx, int64_t lo, int64_t hi);
typedef struct {
  range_fn fn;
  void* ctx;
  int64_t lo, hi;
} range_job;

static void* range_thread(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->ctx, j->lo, j->hi);
  return NULL;
}

static void parallel_for(int64_t n, int nthreads, range_fn fn, void* ctx) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (n <= 0) return;
  if ((int64_t)nthreads > n) nthreads = (int)n;
  if (nthreads == 1) {
    fn(ctx, 0, n);
    return;
  }
  pthread_t th[256];
  range_job jobs[256];
  int64_t chunk = (n + nthreads - 1) / nthreads;
  int started = 0;
  for (int t = 0; t < nthreads; ++t) {
    int64_t lo = t * chunk, hi = lo + chunk < n ? lo + chunk : n;
    if (lo >= hi) break;
    jobs[t].fn = fn; jobs[t].ctx = ctx; jobs[t].lo = lo; jobs[t].hi = hi;
    if (pthread_create(&th[t], NULL, range_thread, &jobs[t]) != 0) {
      fn(ctx, lo, hi); /* run inline if the thread cannot start */
      jobs[t].fn = NULL;
    }
    started = t + 1;
  }
  for (int t = 0; t < started; ++t)
    if (jobs[t].fn) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------ */
/* GEMM_Naive semantics (mmm.cpp:52-62): fp32 accumulator, k ascending */
/* Rows [r0, r1) of C.                                                  */
/* ------------------------------------------------------------------ */
void orc_gemm_f32_seq(const uint16_t* A, const uint16_t* B, float* C, int64_t M, int64_t N,
                      int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int64_t r0, int64_t r1) {
  (void)M;
  for (int64_t r = r0; r < r1; ++r)
    for (int64_t c = 0; c < N; ++c) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) acc += orc_h2f(A[r * lda + k]) * orc_h2f(B[k * ldb + c]);
      C[r * ldc + c] = acc;
    }
}

/* ------------------------------------------------------------------ */
/* FP64-accumulated GEMM, rows [r0, r1), multithreaded over rows.       */
/* ------------------------------------------------------------------ */
typedef struct {
  const uint16_t *A, *B;
  double* C;
  int64_t N, K, lda, ldb, ldc, r0;
  const double* Bd; /* B widened to double, K x N, row stride N */
} f64_ctx;

static void f64_rows(void* p, int64_t lo, int64_t hi) {
  f64_ctx* c = (f64_ctx*)p;
  double* acc = (double*)malloc(sizeof(double) * (size_t)(c->N > 0 ? c->N : 1));
  for (int64_t rr = lo; rr < hi; ++rr) {
    int64_t r = c->r0 + rr;
    for (int64_t n = 0; n < c->N; ++n) acc[n] = 0.0;
    for (int64_t k = 0; k < c->K; ++k) {
      double a = (double)orc_h2f(c->A[r * c->lda + k]);
      if (a == 0.0) continue;
      const double* brow = c->Bd + k * c->N;
      for (int64_t n = 0; n < c->N; ++n) acc[n] += a * brow[n];
    }
    for (int64_t n = 0; n < c->N; ++n) c->C[rr * c->ldc + n] = acc[n];
  }
  free(acc);
}

/* C is (r1-r0) x N with row stride ldc (row 0 of C holds output row r0). */
int orc_gemm_f64(const uint16_t* A, const uint16_t* B, double* C, int64_t M, int64_t N, int64_t K,
                 int64_t lda, int64_t ldb, int64_t ldc, int64_t r0, int64_t r1, int nthreads) {
  (void)M;
  double* Bd = (double*)malloc(sizeof(double) * (size_t)(K * N > 0 ? K * N : 1));
  if (!Bd) return -1;
  for (int64_t k = 0; k < K; ++k)
    for (int64_t n = 0; n < N; ++n) Bd[k * N + n] = (double)orc_h2f(B[k * ldb + n]);
  f64_ctx ctx = {A, B, C, N, K, lda, ldb, ldc, r0, Bd};
  parallel_for(r1 - r0, nthreads, f64_rows, &ctx);
  free(Bd);
  return 0;
}

/* ------------------------------------------------------------------ */
/* 5-D contraction, FP64 accumulate, arbitrary element strides.         */
/* C[a,b,i,n] = sum_{j,k} A[a,b,i,j,k] * B[j,k,n]                       */
/* ------------------------------------------------------------------ */
typedef struct {
  const uint16_t *A, *B;
  double* C;
  const int64_t *as, *ass, *bs, *bss, *cs;
  const double* Bd; /* B widened, packed [j][k][n] */
} con_ctx;

static void con_rows(void* p, int64_t lo, int64_t hi) {
  con_ctx* c = (con_ctx*)p;
  const int64_t Bsz = c->as[1], Isz = c->as[2], Jsz = c->as[3], Ksz = c->as[4], Nsz = c->bs[2];
  double* acc = (double*)malloc(sizeof(double) * (size_t)(Nsz > 0 ? Nsz : 1));
  for (int64_t row = lo; row < hi; ++row) {
    int64_t ia = row / (Bsz * Isz), ib = (row / Isz) % Bsz, ii = row % Isz;
    for (int64_t n = 0; n < Nsz; ++n) acc[n] = 0.0;
    const uint16_t* arow = c->A + ia * c->ass[0] + ib * c->ass[1] + ii * c->ass[2];
    for (int64_t j = 0; j < Jsz; ++j)
      for (int64_t k = 0; k < Ksz; ++k) {
        double a = (double)orc_h2f(arow[j * c->ass[3] + k * c->ass[4]]);
        if (a == 0.0) continue;
        const double* brow = c->Bd + (j * Ksz + k) * Nsz;
        for (int64_t n = 0; n < Nsz; ++n) acc[n] += a * brow[n];
      }
    double* crow = c->C + ia * c->cs[0] + ib * c->cs[1] + ii * c->cs[2];
    for (int64_t n = 0; n < Nsz; ++n) crow[n * c->cs[3]] = acc[n];
  }
  free(acc);
}

/* a_shape/a_stride: (a,b,i,j,k); b_shape/b_stride: (j,k,n); c_stride: (a,b,i,n), all in
 * elements.  C is double with the given strides. */
int orc_contract5d_f64(const uint16_t* A, const int64_t* a_shape, const int64_t* a_stride,
                       const uint16_t* B, const int64_t* b_shape, const int64_t* b_stride,
                       double* C, const int64_t* c_stride, int nthreads) {
  const int64_t J = b_shape[0], Kk = b_shape[1], N = b_shape[2];
  if (J != a_shape[3] || Kk != a_shape[4]) return -1;
  double* Bd = (double*)malloc(sizeof(double) * (size_t)(J * Kk * N > 0 ? J * Kk * N : 1));
  if (!Bd) return -1;
  for (int64_t j = 0; j < J; ++j)
    for (int64_t k = 0; k < Kk; ++k)
      for (int64_t n = 0; n < N; ++n)
        Bd[(j * Kk + k) * N + n] =
            (double)orc_h2f(B[j * b_stride[0] + k * b_stride[1] + n * b_stride[2]]);
  con_ctx ctx = {A, B, C, a_shape, a_stride, b_shape, b_stride, c_stride, Bd};
  parallel_for(a_shape[0] * a_shape[1] * a_shape[2], nthreads, con_rows, &ctx);
  free(Bd);
  return 0;
}

/* ------------------------------------------------------------------ */
/* Blocked multithreaded fp32 GEMM with GEMM_Naive arithmetic.          */
/* Every C element is accumulated from 0 in ascending k with exact      */
/* products, so the result equals orc_gemm_f32_seq bit for bit.         */
/* Each thread owns a range of 6-row panels; it walks NC-column x       */
/* KC-deep blocks of B (kept in its cache) in ascending k and applies   */
/* each block to all of its panels, carrying partial sums in C.         */
/* ------------------------------------------------------------------ */
#define MR 6
#define NR 16
#define KC 256
#define NC 512

typedef struct {
  const uint16_t* A;
  const float* Bf; /* B widened to fp32, K x N, row stride N */
  float* C;
  int64_t N, K, lda, ldc, r0, r1;
} blk_ctx;

/* acc[rows][nw] (+)= apack[rows][k0:k0+kc] . Bf[k0:k0+kc][n0:n0+nw] */
static void micro(const float* apack, int64_t K, int64_t k0, int64_t kc, const float* Bf,
                  int64_t N, int64_t n0, int rows, int nw, float* c, int64_t ldc, int first) {
#if defined(__AVX2__) && defined(__FMA__)
  if (rows == MR && nw == NR) {
    __m256 c00, c01, c10, c11, c20, c21, c30, c31, c40, c41, c50, c51;
    if (first) {
      c00 = c01 = c10 = c11 = c20 = c21 = c30 = c31 = c40 = c41 = c50 = c51 = _mm256_setzero_ps();
    } else {
      c00 = _mm256_loadu_ps(c + 0 * ldc); c01 = _mm256_loadu_ps(c + 0 * ldc + 8);
      c10 = _mm256_loadu_ps(c + 1 * ldc); c11 = _mm256_loadu_ps(c + 1 * ldc + 8);
      c20 = _mm256_loadu_ps(c + 2 * ldc); c21 = _mm256_loadu_ps(c + 2 * ldc + 8);
      c30 = _mm256_loadu_ps(c + 3 * ldc); c31 = _mm256_loadu_ps(c + 3 * ldc + 8);
      c40 = _mm256_loadu_ps(c + 4 * ldc); c41 = _mm256_loadu_ps(c + 4 * ldc + 8);
      c50 = _mm256_loadu_ps(c + 5 * ldc); c51 = _mm256_loadu_ps(c + 5 * ldc + 8);
    }
    const float* bp = Bf + k0 * N + n0;
    const float* ap = apack + k0;
    for (int64_t k = 0; k < kc; ++k) {
      __m256 b0 = _mm256_loadu_ps(bp + k * N);
      __m256 b1 = _mm256_loadu_ps(bp + k * N + 8);
      __m256 a;
      a = _mm256_broadcast_ss(ap + 0 * K + k); c00 = _mm256_fmadd_ps(a, b0, c00); c01 = _mm256_fmadd_ps(a, b1, c01);
      a = _mm256_broadcast_ss(ap + 1 * K + k); c10 = _mm256_fmadd_ps(a, b0, c10); c11 = _mm256_fmadd_ps(a, b1, c11);
      a = _mm256_broadcast_ss(ap + 2 * K + k); c20 = _mm256_fmadd_ps(a, b0, c20); c21 = _mm256_fmadd_ps(a, b1, c21);
      a = _mm256_broadcast_ss(ap + 3 * K + k); c30 = _mm256_fmadd_ps(a, b0, c30); c31 = _mm256_fmadd_ps(a, b1, c31);
      a = _mm256_broadcast_ss(ap + 4 * K + k); c40 = _mm256_fmadd_ps(a, b0, c40); c41 = _mm256_fmadd_ps(a, b1, c41);
      a = _mm256_broadcast_ss(ap + 5 * K + k); c50 = _mm256_fmadd_ps(a, b0, c50); c51 = _mm256_fmadd_ps(a, b1, c51);
    }
    _mm256_storeu_ps(c + 0 * ldc, c00); _mm256_storeu_ps(c + 0 * ldc + 8, c01);
    _mm256_storeu_ps(c + 1 * ldc, c10); _mm256_storeu_ps(c + 1 * ldc + 8, c11);
    _mm256_storeu_ps(c + 2 * ldc, c20); _mm256_storeu_ps(c + 2 * ldc + 8, c21);
    _mm256_storeu_ps(c + 3 * ldc, c30); _mm256_storeu_ps(c + 3 * ldc + 8, c31);
    _mm256_storeu_ps(c + 4 * ldc, c40); _mm256_storeu_ps(c + 4 * ldc + 8, c41);
    _mm256_storeu_ps(c + 5 * ldc, c50); _mm256_storeu_ps(c + 5 * ldc + 8, c51);
    return;
  }
#endif
  for (int r = 0; r < rows; ++r)
    for (int j = 0; j < nw; ++j) {
      float acc = first ? 0.0f : c[r * ldc + j];
      for (int64_t k = 0; k < kc; ++k)
        acc = fmaf(apack[r * K + k0 + k], Bf[(k0 + k) * N + n0 + j], acc);
      c[r * ldc + j] = acc;
    }
}

static void blk_rows(void* p, int64_t lo, int64_t hi) {
  blk_ctx* c = (blk_ctx*)p;
  const int64_t N = c->N, K = c->K;
  const int64_t rbeg = c->r0 + lo * MR;
  const int64_t rend = c->r0 + hi * MR < c->r1 ? c->r0 + hi * MR : c->r1;
  const int64_t nrows = rend - rbeg;
  if (nrows <= 0) return;
  float* apack = (float*)malloc(sizeof(float) * (size_t)(nrows * (K > 0 ? K : 1)));
  for (int64_t r = 0; r < nrows; ++r)
    for (int64_t k = 0; k < K; ++k) apack[r * K + k] = orc_h2f(c->A[(rbeg + r) * c->lda + k]);
  if (K == 0) {
    for (int64_t r = 0; r < nrows; ++r)
      for (int64_t n = 0; n < N; ++n) c->C[(rbeg + r - c->r0) * c->ldc + n] = 0.0f;
  }
  for (int64_t n0 = 0; n0 < N; n0 += NC) {
    const int64_t nc = N - n0 < NC ? N - n0 : NC;
    for (int64_t k0 = 0; k0 < K; k0 += KC) {
      const int64_t kc = K - k0 < KC ? K - k0 : KC;
      for (int64_t r = 0; r < nrows; r += MR) {
        const int rows = (int)(nrows - r < MR ? nrows - r : MR);
        for (int64_t j = 0; j < nc; j += NR) {
          const int nw = (int)(nc - j < NR ? nc - j : NR);
          float* cp = c->C + (rbeg + r - c->r0) * c->ldc + n0 + j;
          micro(apack + r * K, K, k0, kc, c->Bf, N, n0 + j, rows, nw, cp, c->ldc, k0 == 0);
        }
      }
    }
  }
  free(apack);
}

/* Widen B once (K x N fp16 with ldb -> fp32 dense).  Exposed so a timing loop can either
 * include it (the default through orc_gemm_f32_blocked) or not. */
typedef struct {
  const uint16_t* B;
  float* Bf;
  int64_t N, ldb;
} widen_ctx;

static void widen_rows(void* p, int64_t lo, int64_t hi) {
  widen_ctx* c = (widen_ctx*)p;
  for (int64_t k = lo; k < hi; ++k)
    for (int64_t n = 0; n < c->N; ++n) c->Bf[k * c->N + n] = orc_h2f(c->B[k * c->ldb + n]);
}

int orc_widen_b_mt(const uint16_t* B, float* Bf, int64_t K, int64_t N, int64_t ldb, int nthreads) {
  widen_ctx ctx = {B, Bf, N, ldb};
  parallel_for(K, nthreads, widen_rows, &ctx);
  return 0;
}

int orc_widen_b(const uint16_t* B, float* Bf, int64_t K, int64_t N, int64_t ldb) {
  return orc_widen_b_mt(B, Bf, K, N, ldb, 1);
}

/* Rows [r0, r1) of C = A*B; C row 0 corresponds to output row r0.  Bf may be NULL (the
 * function widens B itself) or a K x N fp32 copy from orc_widen_b. */
int orc_gemm_f32_blocked(const uint16_t* A, const uint16_t* B, const float* Bf_in, float* C,
                         int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                         int64_t r0, int64_t r1, int nthreads) {
  (void)M;
  float* Bf = (float*)Bf_in;
  int own = 0;
  if (!Bf) {
    Bf = (float*)malloc(sizeof(float) * (size_t)(K * N > 0 ? K * N : 1));
    if (!Bf) return -1;
    orc_widen_b_mt(B, Bf, K, N, ldb, nthreads);
    own = 1;
  }
  blk_ctx ctx = {A, Bf, C, N, K, lda, ldc, r0, r1};
  int64_t panels = (r1 - r0 + MR - 1) / MR;
  parallel_for(panels, nthreads, blk_rows, &ctx);
  if (own) free(Bf);
  return 0;
}

int orc_simd_level(void) {
#if defined(__AVX2__) && defined(__FMA__)
  return 2;
#else
  return 0;
#endif
}

/* ------------------------------------------------------------------ */
/* Tolerance check: returns the number of violating elements and writes */
/* max abs / max rel error.  got: fp32 (rows x N, stride ldg),          */
/* ref: fp64 (rows x N, stride ldr).                                    */
/* ------------------------------------------------------------------ */
int64_t orc_check_tolerance(const float* got, int64_t ldg, const double* ref, int64_t ldr,
                            int64_t rows, int64_t N, int64_t K, double max_a, double max_b,
                            double* max_abs, double* max_rel, int64_t* first_bad) {
  double atol = 1e-3 * sqrt((double)(K > 0 ? K : 1)) * max_a * max_b;
  int64_t bad = 0;
  double ma = 0.0, mr = 0.0;
  *first_bad = -1;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t n = 0; n < N; ++n) {
      double g = (double)got[r * ldg + n], e = ref[r * ldr + n];
      double d = fabs(g - e);
      if (!(d <= atol + 1e-3 * fabs(e))) {
        if (bad == 0) *first_bad = r * N + n;
        bad++;
      }
      if (d > ma || d != d) ma = d;
      double rel = d / (fabs(e) > 1e-30 ? fabs(e) : 1e-30);
      if (fabs(e) > atol && rel > mr) mr = rel;
    }
  *max_abs = ma;
  *max_rel = mr;
  return bad;
}

/* ------------------------------------------------------------------ */
/* bf16 and fp8 (e4m3, e5m2) operands: exact decode and round-to-      */
/* nearest-even encode from the format definitions:                    */
/*   bf16: the top 16 bits of an IEEE binary32.                        */
/*   e4m3: 1 sign, 4 exponent (bias 7), 3 mantissa; no infinities,     */
/*         S.1111.111 is NaN; largest finite 448.                      */
/*   e5m2: 1 sign, 5 exponent (bias 15), 2 mantissa; IEEE-style        */
/*         infinities and NaNs; largest finite 57344.                  */
/* Encoding saturates to the largest finite value (the convention of   */
/* the CUDA library's fill kernel).  Type codes match b2g_gemm.h:      */
/* 0 f16, 1 bf16, 2 e4m3, 3 e5m2.                                      */
/* ------------------------------------------------------------------ */
float orc_bf16_to_f32(uint16_t b) {
  uint32_t x = (uint32_t)b << 16;
  float f;
  memcpy(&f, &x, 4);
  return f;
}

uint16_t orc_f32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40); /* quiet NaN */
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

float orc_fp8_to_f32(uint8_t c, int e4m3) {
  const int mb = e4m3 ? 3 : 2, eb = e4m3 ? 4 : 5, bias = e4m3 ? 7 : 15;
  const int s = c >> 7, e = (c >> mb) & ((1 << eb) - 1), m = c & ((1 << mb) - 1);
  float v;
  if (e4m3 && e == 15 && m == 7)
    v = NAN;
  else if (!e4m3 && e == 31)
    v = m ? NAN : INFINITY;
  else if (e == 0)
    v = ldexpf((float)m, 1 - bias - mb);
  else
    v = ldexpf((float)((1 << mb) | m), e - bias - mb);
  return s ? -v : v;
}

uint8_t orc_f32_to_fp8(float f, int e4m3) {
  const int maxcode = e4m3 ? 0x7e : 0x7b; /* largest finite positive code */
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint8_t sign = (uint8_t)((x >> 24) & 0x80);
  if (f != f) return (uint8_t)(sign | 0x7f);
  const double a = fabs((double)f);
  if (a >= (double)orc_fp8_to_f32((uint8_t)maxcode, e4m3)) return (uint8_t)(sign | maxcode);
  /* positive finite codes are increasing in value: find the last code <= a */
  int lo = 0, hi = maxcode;
  while (lo < hi) {
    int mid = (lo + hi + 1) / 2;
    if ((double)orc_fp8_to_f32((uint8_t)mid, e4m3) <= a)
      lo = mid;
    else
      hi = mid - 1;
  }
  const double v0 = orc_fp8_to_f32((uint8_t)lo, e4m3);
  if (v0 == a) return (uint8_t)(sign | lo);
  const double v1 = orc_fp8_to_f32((uint8_t)(lo + 1), e4m3);
  const double mid = 0.5 * (v0 + v1);
  int c = a < mid ? lo : a > mid ? lo + 1 : ((lo & 1) ? lo + 1 : lo);
  return (uint8_t)(sign | c);
}

/* dst (fp32) <- n elements of type `dt` */
void orc_typed_to_f32(const void* src, int dt, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    if (dt == 0) dst[i] = orc_h2f(((const uint16_t*)src)[i]);
    else if (dt == 1) dst[i] = orc_bf16_to_f32(((const uint16_t*)src)[i]);
    else dst[i] = orc_fp8_to_f32(((const uint8_t*)src)[i], dt == 2);
  }
}

/* dst (type `dt`) <- n fp32 values, round to nearest even */
void orc_f32_to_typed(const float* src, int dt, void* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    if (dt == 0) ((uint16_t*)dst)[i] = orc_f2h(src[i]);
    else if (dt == 1) ((uint16_t*)dst)[i] = orc_f32_to_bf16(src[i]);
    else ((uint8_t*)dst)[i] = orc_f32_to_fp8(src[i], dt == 2);
  }
}

/* The seeded U[-1,1] sequence (orc_uniform_f16_at's fp32 value) in type `dt`. */
void orc_fill_uniform(void* dst, int64_t n, int dt, uint64_t seed, uint64_t offset) {
  const uint64_t key = mix64(seed);
  for (int64_t i = 0; i < n; ++i) {
    uint64_t h = mix64(key + offset + (uint64_t)i);
    int32_t r = (int32_t)(h >> 40) - 8388608;
    float v = (float)r * (1.0f / 8388608.0f);
    orc_f32_to_typed(&v, dt, (char*)dst + i * (dt >= 2 ? 1 : 2), 1);
  }
}

/* FP64-accumulated GEMM on fp32 operands (exact widenings of any operand type), rows [r0, r1);
 * C row 0 holds output row r0. */
typedef struct {
  const float *A, *B;
  double* C;
  int64_t N, K, lda, ldb, ldc, r0;
} f64f_ctx;

static void f64f_rows(void* p, int64_t lo, int64_t hi) {
  f64f_ctx* c = (f64f_ctx*)p;
  double* acc = (double*)malloc(sizeof(double) * (size_t)(c->N > 0 ? c->N : 1));
  for (int64_t rr = lo; rr < hi; ++rr) {
    int64_t r = c->r0 + rr;
    for (int64_t n = 0; n < c->N; ++n) acc[n] = 0.0;
    for (int64_t k = 0; k < c->K; ++k) {
      double a = (double)c->A[r * c->lda + k];
      if (a == 0.0) continue;
      const float* brow = c->B + k * c->ldb;
      for (int64_t n = 0; n < c->N; ++n) acc[n] += a * (double)brow[n];
    }
    for (int64_t n = 0; n < c->N; ++n) c->C[rr * c->ldc + n] = acc[n];
  }
  free(acc);
}

int orc_gemm_f64_f32in(const float* A, const float* B, double* C, int64_t M, int64_t N, int64_t K,
                       int64_t lda, int64_t ldb, int64_t ldc, int64_t r0, int64_t r1,
                       int nthreads) {
  (void)M;
  f64f_ctx ctx = {A, B, C, N, K, lda, ldb, ldc, r0};
  parallel_for(r1 - r0, nthreads, f64f_rows, &ctx);
  return 0;
}
