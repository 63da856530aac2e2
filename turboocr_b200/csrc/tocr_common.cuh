// Shared plumbing of the C-ABI entry points: status codes, the per-thread
// last-error message, host-side fault injection and launch checks.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>
#include <climits>

#include "tocr_capi.h"

namespace tocr {

// Records `msg` as this thread's last error and returns `status`.
int set_error(int status, const char *fmt, ...);
// Clears the thread's last error (called on entry of every compute call).
void clear_error();
// Returns a pending injected status (and consumes one injection), or TOCR_OK.
int take_injected();

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// Checks the launch that was just enqueued.
inline int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(TOCR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TOCR_OK;
}

inline bool aligned(const void *p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// SM count of the current device, cached per device.
int sm_count();

}  // namespace tocr

// Common prologue for a compute entry: clear error, honour injection.
#define TOCR_ENTRY()                               \
  do {                                             \
    ::tocr::clear_error();                         \
    int _inj = ::tocr::take_injected();            \
    if (_inj != TOCR_OK)                           \
      return ::tocr::set_error(_inj, "injected");  \
  } while (0)

#define TOCR_REQUIRE(cond, ...)                                 \
  do {                                                          \
    if (!(cond)) return ::tocr::set_error(TOCR_ERR_INVALID, __VA_ARGS__); \
  } while (0)
