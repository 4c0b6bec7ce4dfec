// Status reporting of the C ABI: a per-thread message buffer and the version number.
#include <cstdarg>
#include <cstdio>

#include "ql_common.cuh"

namespace ql {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return QL_OK;
  set_error("%s: %s (%s)", where, cudaGetErrorString(e), cudaGetErrorName(e));
  return QL_ERR_CUDA;
}

}  // namespace ql

extern "C" int ql_version(void) { return 100; }  // 0.1.0

extern "C" const char* ql_last_error(void) { return ql::g_err; }
