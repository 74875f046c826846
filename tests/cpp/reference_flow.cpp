// The reference's host flow with the library's drop-in calls, as INTEGRATION.md describes it:
// host operands -> cudaMalloc + cudaMemcpy -> b2g::GEMM (for the kernel launch of
// mmm.cpp:1496) or b2g::contract_reference_form (for the G pack plus contraction launch of
// mmmTensor.cpp:329-369) -> cudaMemcpy back.  Operands come from files and the result goes to
// a file, so the test that runs this program checks it against the oracle and the golden
// fixtures made by the reference's own code.
//
//   reference_flow gemm M N K A.f16 B.f16 C.f32
//   reference_flow contract mt rt nt rt_l bt G.f16 Input.f16 Output.f32
//
// Exit status 0 on success; a failing CUDA or library call prints its message and exits
// non-zero (the reference's HIP_CHECK, mmm.cpp:33-39, does the same).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "b2g_gemm.hpp"

#define CUDA_OK(x)                                                                   \
  do {                                                                               \
    cudaError_t e_ = (x);                                                            \
    if (e_ != cudaSuccess) {                                                         \
      std::fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));                  \
      std::exit(3);                                                                  \
    }                                                                                \
  } while (0)

template <typename T>
static std::vector<T> read_file(const char* path, size_t n) {
  std::vector<T> v(n);
  FILE* f = std::fopen(path, "rb");
  if (!f || std::fread(v.data(), sizeof(T), n, f) != n) {
    std::fprintf(stderr, "cannot read %zu elements from %s\n", n, path);
    std::exit(2);
  }
  std::fclose(f);
  return v;
}

static void write_file(const char* path, const std::vector<float>& v) {
  FILE* f = std::fopen(path, "wb");
  if (!f || std::fwrite(v.data(), sizeof(float), v.size(), f) != v.size()) {
    std::fprintf(stderr, "cannot write %s\n", path);
    std::exit(2);
  }
  std::fclose(f);
}

int main(int argc, char** argv) {
  if (argc < 2) return 1;
  const std::string mode = argv[1];
  try {
    if (mode == "gemm" && argc == 8) {
      const int64_t M = std::atoll(argv[2]), N = std::atoll(argv[3]), K = std::atoll(argv[4]);
      auto hA = read_file<uint16_t>(argv[5], (size_t)(M * K));
      auto hB = read_file<uint16_t>(argv[6], (size_t)(K * N));
      std::vector<float> hC((size_t)(M * N));
      void *dA = nullptr, *dB = nullptr;
      float* dC = nullptr;
      CUDA_OK(cudaMalloc(&dA, hA.size() * 2));
      CUDA_OK(cudaMalloc(&dB, hB.size() * 2));
      CUDA_OK(cudaMalloc(&dC, hC.size() * 4));
      CUDA_OK(cudaMemcpy(dA, hA.data(), hA.size() * 2, cudaMemcpyHostToDevice));
      CUDA_OK(cudaMemcpy(dB, hB.data(), hB.size() * 2, cudaMemcpyHostToDevice));
      b2g::check(b2g::GEMM(dA, dB, dC, M, N, K));  // was: WMMA_Swizzled_Full<<<...>>>(dA, dB, dC)
      CUDA_OK(cudaDeviceSynchronize());
      CUDA_OK(cudaMemcpy(hC.data(), dC, hC.size() * 4, cudaMemcpyDeviceToHost));
      write_file(argv[7], hC);
      cudaFree(dA);
      cudaFree(dB);
      cudaFree(dC);
    } else if (mode == "contract" && argc == 10) {
      const int64_t mt = std::atoll(argv[2]), rt = std::atoll(argv[3]), nt = std::atoll(argv[4]),
                    rt_l = std::atoll(argv[5]), bt = std::atoll(argv[6]);
      auto hG = read_file<uint16_t>(argv[7], (size_t)(rt * nt * mt * rt_l));
      auto hIn = read_file<uint16_t>(argv[8], (size_t)(bt * nt * rt_l));
      std::vector<float> hOut((size_t)(mt * bt * rt));
      void *dG = nullptr, *dIn = nullptr;
      float* dOut = nullptr;
      CUDA_OK(cudaMalloc(&dG, hG.size() * 2));
      CUDA_OK(cudaMalloc(&dIn, hIn.size() * 2));
      CUDA_OK(cudaMalloc(&dOut, hOut.size() * 4));
      CUDA_OK(cudaMemcpy(dG, hG.data(), hG.size() * 2, cudaMemcpyHostToDevice));
      CUDA_OK(cudaMemcpy(dIn, hIn.data(), hIn.size() * 2, cudaMemcpyHostToDevice));
      // was: pack G into hA on the host, upload hA, launch the contraction kernel
      b2g::check(b2g::contract_reference_form(dG, dIn, dOut, mt, rt, nt, rt_l, bt));
      CUDA_OK(cudaDeviceSynchronize());
      CUDA_OK(cudaMemcpy(hOut.data(), dOut, hOut.size() * 4, cudaMemcpyDeviceToHost));
      write_file(argv[9], hOut);
      cudaFree(dG);
      cudaFree(dIn);
      cudaFree(dOut);
    } else {
      return 1;
    }
  } catch (const b2g::Error& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 4;
  }
  const int path = b2g_last_path();
  std::printf("ok path=%d\n", path);
  return 0;
}
