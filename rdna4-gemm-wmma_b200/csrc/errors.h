// State shared by the translation units of libb2g_gemm.so: the thread-local error message
// (read back through b2g_last_error_string()) and the count of kernels launched
// (b2g_get_option("launches")).
#pragma once

namespace b2g {
void set_error(const char* msg);
void count_launch();
}  // namespace b2g
