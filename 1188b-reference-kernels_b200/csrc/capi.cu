// Library-wide pieces of the C ABI: per-thread error messages, the ABI
// version, and a cached SM count per device (persistent-kernel grid size).
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "moe_common.cuh"

namespace moe {

namespace {
thread_local char g_last_error[512] = {0};
}

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int num_sms(int device) {
  static std::mutex mu;
  static int cache[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (device >= 0 && device < 64 && cache[device] > 0) return cache[device];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
    n = 148;
  if (device >= 0 && device < 64) cache[device] = n;
  return n;
}

}  // namespace moe

extern "C" const char* moe_b200_last_error(void) { return moe::g_last_error; }

extern "C" int moe_b200_abi_version(void) { return 2; }
