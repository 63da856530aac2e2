// Error state, version and fault-injection hooks of the C-ABI.
#include "tocr_common.cuh"

#include <atomic>
#include <cstdarg>
#include <string>

namespace tocr {

namespace {
thread_local std::string g_last_error;
std::atomic<int> g_inject_status{TOCR_OK};
std::atomic<int> g_inject_count{0};
}  // namespace

int set_error(int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

void clear_error() { g_last_error.clear(); }

int take_injected() {
  int n = g_inject_count.load(std::memory_order_acquire);
  while (n > 0) {
    if (g_inject_count.compare_exchange_weak(n, n - 1, std::memory_order_acq_rel))
      return g_inject_status.load(std::memory_order_acquire);
  }
  return TOCR_OK;
}

int sm_count() {
  static thread_local int cached_dev = -1, cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev != cached_dev) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    cached_dev = dev;
    cached_sms = v;
  }
  return cached_sms;
}

}  // namespace tocr

extern "C" {

TOCR_API const char *tocr_last_error_string(void) { return tocr::g_last_error.c_str(); }

TOCR_API int tocr_version(void) { return 0x000100; }

TOCR_API void tocr_debug_inject_error(int status, int count) {
  if (count <= 0) {
    tocr::g_inject_count.store(0, std::memory_order_release);
    tocr::g_inject_status.store(TOCR_OK, std::memory_order_release);
    return;
  }
  tocr::g_inject_status.store(status, std::memory_order_release);
  tocr::g_inject_count.store(count, std::memory_order_release);
}

}  // extern "C"
