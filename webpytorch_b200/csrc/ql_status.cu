// Status reporting of the C ABI: a per-thread message buffer and the version number.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>

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

static std::atomic<int> g_launch_flags{0};

int launch_flags() { return g_launch_flags.load(std::memory_order_relaxed); }

// Set by the allocation-free entry point for the duration of its call: every stream-ordered
// allocation the kernels' host code would make fails instead (see stream_alloc).
static thread_local bool g_alloc_forbidden = false;

AllocGuard::AllocGuard() : prev(g_alloc_forbidden) { g_alloc_forbidden = true; }
AllocGuard::~AllocGuard() { g_alloc_forbidden = prev; }

int stream_alloc(void** p, size_t bytes, cudaStream_t st, const char* what) {
  if (g_alloc_forbidden) {
    set_error("%s: %zu bytes of scratch needed, but this call may not allocate", what, bytes);
    return QL_ERR_UNSUPPORTED;
  }
  return cuda_status(cudaMallocAsync(p, bytes, st), what);
}

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

}  // namespace ql

extern "C" int ql_set_launch_flags(int flags) { return ql::g_launch_flags.exchange(flags); }

extern "C" int ql_version(void) { return 100; }  // 0.1.0

extern "C" const char* ql_last_error(void) { return ql::g_err; }
