// State shared by the translation units of libb2g_gemm.so: the thread-local error message
// (read back through b2g_last_error_string()) and the count of kernels launched
// (b2g_get_option("launches")).
#pragma once
#include <cstdint>

namespace b2g {
void set_error(const char* msg);
void count_launch();
// Device error word of the multi-GPU kernels (b2g_shard.cu), merged into b2g_device_status():
// reads it and, with clear != 0, resets it; returns 0 or a cudaError_t.
int shard_device_error(int clear, int* value);
// Options of the multi-GPU entry points (b2g_set_option "comm_timeout_ms", "comm_nonblocking").
int64_t comm_timeout_ms();
bool comm_nonblocking();
// The fp16 GEMM C = A.B whose epilogue stores, for every element, the sum in slot order of
// add_count terms: term add_self is A.B, term s the fp32 matrix add_base + s * add_slot (row
// pitch N).  add_status[s] must equal epoch for every s != add_self, else C is NaN and the
// device error word records kErrPeerFailed.  Tensor-core path only (B2G_ERR_UNSUPPORTED
// otherwise).  Used by the peer-memory K-split (b2g_shard.cu).
int gemm_rank_sum(const void* A, const void* B, float* C, int64_t M, int64_t N, int64_t K,
                  int64_t lda, int64_t ldb, int64_t ldc, const float* add_base, int64_t add_slot,
                  int add_count, int add_self, const uint32_t* add_status, uint32_t epoch,
                  void* stream);
// Option "rs_fused": whether the peer-memory K-split sums its slots in the own GEMM's epilogue.
bool rs_fused();
// Option "rs_stage": whether the peer-memory K-split computes the peers' partials into local
// staging buffers and pushes them with the copy engine (instead of storing them remotely).
bool rs_stage();
// Device-side error codes beyond the bounded-wait codes of the GEMM kernel (1..6).
constexpr int kErrPeerFailed = 7;  // a peer's part of a peer-memory reduce-scatter failed
}  // namespace b2g
