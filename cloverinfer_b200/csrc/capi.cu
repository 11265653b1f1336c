// Library-wide C ABI pieces: version, last-error string, CUDA error mapping.
#include <atomic>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

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

static std::atomic<int64_t> g_wait_ns{(int64_t)kWaitLimitNs};

uint64_t wait_limit_ns() { return (uint64_t)g_wait_ns.load(std::memory_order_relaxed); }

}  // namespace clover

extern "C" int clover_b200_version(void) { return 100; }  // 0.1.0

// Host-side gather of n source buffers into one destination (a pinned
// staging buffer): one native call instead of one framework op per item.
extern "C" int clover_b200_host_gather(const void* const* srcs, const int64_t* nbytes, int32_t n,
                                       void* dst) {
  if (n < 0 || (n > 0 && (!srcs || !nbytes || !dst)))
    return clover::set_error(CLOVER_B200_ERR_INVALID_ARG, "host_gather: bad arguments");
  char* d = static_cast<char*>(dst);
  for (int32_t i = 0; i < n; ++i) {
    if (nbytes[i] < 0 || (nbytes[i] > 0 && !srcs[i]))
      return clover::set_error(CLOVER_B200_ERR_INVALID_ARG, "host_gather: bad source %d", i);
    memcpy(d, srcs[i], (size_t)nbytes[i]);
    d += nbytes[i];
  }
  return CLOVER_B200_OK;
}

extern "C" const char* clover_b200_last_error(void) { return clover::g_last_error; }

extern "C" int64_t clover_b200_set_wait_limit_ns(int64_t ns) {
  constexpr int64_t kMin = 1000ll * 1000ll;             // 1 ms
  constexpr int64_t kMax = 60ll * 1000ll * 1000ll * 1000ll;  // 60 s
  if (ns <= 0) ns = (int64_t)clover::kWaitLimitNs;
  ns = ns < kMin ? kMin : (ns > kMax ? kMax : ns);
  return clover::g_wait_ns.exchange(ns);
}
