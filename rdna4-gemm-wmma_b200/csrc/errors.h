// Thread-local error message shared by the translation units of libb2g_gemm.so; read back
// through b2g_last_error_string().
#pragma once

namespace b2g {
void set_error(const char* msg);
}  // namespace b2g
