// capi_common.cu -- error reporting, launch accounting and device queries of the C ABI.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>

#include "../../include/specdec_b200.h"
#include "sd_internal.h"

namespace {
thread_local char g_last_error[512] = "";
std::atomic<int64_t> g_launches{0};
std::mutex g_sm_mutex;
int g_sm_count[64] = {0};
}  // namespace

namespace sd {

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int after_launch(const char* what, int n) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SPECDEC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  g_launches.fetch_add(n, std::memory_order_relaxed);
  return SPECDEC_OK;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(g_sm_mutex);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

}  // namespace sd

extern "C" const char* specdec_last_error(void) { return g_last_error; }
extern "C" int specdec_abi_version(void) { return SPECDEC_ABI_VERSION; }
extern "C" int64_t specdec_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }
