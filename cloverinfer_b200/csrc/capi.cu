// Library-wide C ABI pieces: version, last-error string, CUDA error mapping.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace clover {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return CLOVER_B200_OK;
  return set_error(CLOVER_B200_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace clover

extern "C" int clover_b200_version(void) { return 100; }  // 0.1.0

extern "C" const char* clover_b200_last_error(void) { return clover::g_last_error; }
