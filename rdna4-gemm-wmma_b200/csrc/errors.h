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
// Device-side error codes beyond the bounded-wait codes of the GEMM kernel (1..6).
constexpr int kErrPeerFailed = 7;  // a peer's part of a peer-memory reduce-scatter failed
}  // namespace b2g
