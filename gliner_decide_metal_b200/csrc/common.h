// Shared host-side helpers: status/error plumbing and small utilities.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include <cuda_runtime.h>

#include "gdc.h"

namespace gdc {

// Sets the thread-local last-error message and returns `st`.
gdc_status set_error(gdc_status st, const char* fmt, ...);
void clear_error();

#define GDC_CUDA_TRY(expr)                                                                  \
  do {                                                                                      \
    cudaError_t e_ = (expr);                                                                \
    if (e_ != cudaSuccess) {                                                                \
      gdc_status st_ = (e_ == cudaErrorMemoryAllocation) ? GDC_ERR_OUT_OF_MEMORY : GDC_ERR_CUDA; \
      return ::gdc::set_error(st_, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_),   \
                              __FILE__, __LINE__);                                          \
    }                                                                                       \
  } while (0)

#define GDC_TRY(expr)                  \
  do {                                 \
    gdc_status s_ = (expr);            \
    if (s_ != GDC_OK) return s_;       \
  } while (0)

// Checks the launch status of the last kernel.
inline gdc_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(GDC_ERR_CUDA, "kernel launch %s failed: %s", what, cudaGetErrorString(e));
  return GDC_OK;
}

// Runs `init` once per device ordinal (0..63) over all host threads and returns its result
// on every later call. Kernel attributes and device queries are set up this way because
// distinct model handles on one device may reach a kernel's first launch concurrently.
struct PerDeviceOnce {
  std::once_flag flag[64];
  int result[64] = {};
};

template <typename F>
int per_device_once(PerDeviceOnce& once, int dev, F&& init) {
  std::call_once(once.flag[dev], [&] { once.result[dev] = int(init()); });
  return once.result[dev];
}

// Device error flag bits written by kernels (bounded waits, input checks).
enum DeviceErrorBits : int {
  kErrTimeout = 1,          // an mbarrier / flag wait exceeded its limit
  kErrBadTokenId = 2,       // input id outside [0, vocab)
  kErrBadMarkerIndex = 4,   // marker index outside [0, seq_len)
};

// fp16 <-> fp32 on the host (IEEE binary16, round-to-nearest-even).
uint16_t f32_to_f16_bits(float f);
float f16_bits_to_f32(uint16_t h);

}  // namespace gdc
