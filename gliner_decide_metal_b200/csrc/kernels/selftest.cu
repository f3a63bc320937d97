// Device-side failure detection self-test: one CTA waits on a shared-memory mbarrier
// that nothing ever arrives on, with a short time limit, exactly as every wait in the
// forward's kernels is bounded (ptx.cuh). When the limit passes it sets kErrTimeout in
// the error word and returns, leaving the context usable; the host reads the word.
#include "kernels.h"
#include "ptx.cuh"

namespace gdc {
namespace {

__global__ void wait_timeout_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  ptx::mbar_init(&bar, 1);
  ptx::fence_barrier_init();
  const unsigned long long t0 = ptx::globaltimer();
  while (!ptx::mbar_try_wait(&bar, 0)) {  // phase 0 never completes: no thread arrives
    if (ptx::globaltimer() - t0 > limit_ns) {
      atomicOr(err, kErrTimeout);
      return;
    }
  }
}

}  // namespace

gdc_status launch_wait_timeout_probe(int* err, int limit_us, cudaStream_t stream) {
  if (limit_us <= 0 || limit_us > 1000000)
    return set_error(GDC_ERR_INVALID_INPUT, "wait timeout probe: limit %d us outside (0, 1e6]", limit_us);
  wait_timeout_probe_kernel<<<1, 32, 0, stream>>>(err, (unsigned long long)limit_us * 1000ull);
  return check_launch("wait_timeout_probe_kernel");
}

}  // namespace gdc
