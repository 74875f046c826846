// b2g_gemm.hpp - C++ drop-in surface over the C ABI of b2g_gemm.h.
//
// GEMM(A, B, C, M, N, K) replaces the reference's kernel launch
//   WMMA_Swizzled_Full<2,2,4,4><<<grid, block>>>(dA, dB, dC)         (mmm.cpp:1488,1496)
// and contract_reference_form(...) replaces its contraction pipeline
//   host pack of G (mmmTensor.cpp:329-340) + contraction launch (mmmTensor.cpp:364-369).
// Sizes are arguments instead of the compile-time DIM_I/DIM_J/DIM_K (mmm.cpp:13-15).
// Errors come back as status codes; check() turns one into an exception (the reference's
// HIP_CHECK, mmm.cpp:33-39, exits the process instead).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>

#include "b2g_gemm.h"

namespace b2g {

class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

inline void check(int rc) {
  if (rc != B2G_OK)
    throw Error(rc, std::string("b2g error ") + std::to_string(rc) + ": " + b2g_last_error_string());
}

// C[M,N] = A[M,K] * B[K,N]; fp16 A/B, fp32 C, contiguous row-major, default stream.
inline int GEMM(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K) {
  return b2g_gemm(A, B, C, M, N, K);
}

// Same with leading dimensions and a stream (cudaStream_t passed as void*).
inline int GEMM(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K,
                int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  return b2g_gemm_f16_f32(A, B, C, M, N, K, lda, ldb, ldc, stream);
}

// C[a,b,i,n] = sum_{j,k} A[a,b,i,j,k] * B[j,k,n], element strides.
inline int Contract(const void* A, const int64_t a_shape[5], const int64_t a_stride[5],
                    const void* B, const int64_t b_shape[3], const int64_t b_stride[3], float* C,
                    const int64_t c_shape[4], const int64_t c_stride[4], void* stream = nullptr) {
  return b2g_contract5d_f16_f32(A, a_shape, a_stride, B, b_shape, b_stride, C, c_shape, c_stride,
                                stream);
}

// All operands contiguous: A[a][b][i][j][k], B[j][k][n], C[a][b][i][n].
inline int contract5d_contiguous(const void* A, const void* B, float* C, int64_t a, int64_t b,
                                 int64_t i, int64_t j, int64_t k, int64_t n,
                                 void* stream = nullptr) {
  const int64_t as[5] = {a, b, i, j, k};
  const int64_t ast[5] = {b * i * j * k, i * j * k, j * k, k, 1};
  const int64_t bs[3] = {j, k, n};
  const int64_t bst[3] = {k * n, n, 1};
  const int64_t cs[4] = {a, b, i, n};
  const int64_t cst[4] = {b * i * n, i * n, n, 1};
  return Contract(A, as, ast, B, bs, bst, C, cs, cst, stream);
}

// The reference's own contraction (mmmTensor.cpp): Out[m][b][r] =
// sum_{n,k} G[r][n][m][k] * Input[b][n*rt_l + k], read in place (no packed copy of G).
inline int contract_reference_form(const void* G, const void* Input, float* Output, int64_t mt,
                                   int64_t rt, int64_t nt, int64_t rt_l, int64_t bt,
                                   void* stream = nullptr) {
  const int64_t as[5] = {mt, 1, rt, nt, rt_l};
  const int64_t ast[5] = {rt_l, 0, nt * mt * rt_l, mt * rt_l, 1};
  const int64_t bs[3] = {nt, rt_l, bt};
  const int64_t bst[3] = {rt_l, 1, nt * rt_l};
  const int64_t cs[4] = {mt, 1, rt, bt};
  const int64_t cst[4] = {bt * rt, 0, 1, rt};
  return Contract(G, as, ast, Input, bs, bst, Output, cs, cst, stream);
}

}  // namespace b2g
