// Error plumbing of the C-ABI: a per-thread message and the launch check.
#include <cstdarg>
#include <cstdio>

#include "qb_common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

namespace qb {

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(QB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return QB_OK;
}

}  // namespace qb

extern "C" const char* qb_last_error(void) { return g_last_error; }

extern "C" int qb_abi_version(void) { return 2; }
