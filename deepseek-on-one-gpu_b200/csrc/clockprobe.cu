// Clock probe for measurement: every SM records its cycle counter and the
// global nanosecond timer. Two probes on a stream bracket a timed region;
// per SM, (cycles after - cycles before) / (ns after - ns before) is the mean
// SM clock over the region, whatever the power cap did meanwhile.
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {
namespace cp {
__global__ void probe_kernel(unsigned long long* out, int n_slots) {
  if (threadIdx.x != 0) return;
  uint32_t sm;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
  if (static_cast<int>(sm) >= n_slots) return;
  const unsigned long long c = clock64();
  const unsigned long long t = globaltimer();
  // several blocks may land on one SM: each writes a consistent pair of its own
  out[2 * sm] = c;
  out[2 * sm + 1] = t;
}
}  // namespace cp

cudaError_t launch_clock_probe(unsigned long long* out, int n_slots, int n_sm, cudaStream_t stream) {
  if (!out || n_slots <= 0 || n_sm <= 0) return cudaErrorInvalidValue;
  cp::probe_kernel<<<4 * n_sm, 32, 0, stream>>>(out, n_slots);
  return cudaGetLastError();
}
}  // namespace dsmoe
