// ABI-level helpers: version, thread-local last error, device SM count.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/d2sd.h"

namespace d2sd {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }

int current_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace d2sd

extern "C" int d2sd_version(void) { return 100; }

extern "C" const char* d2sd_last_error(void) { return d2sd::g_last_error.c_str(); }
