// Device timestamps for tracing: one thread writes %globaltimer (ns) into
// slot `idx` of a device buffer after the previous kernel in the stream has
// completed (griddepcontrol.wait), then releases its dependents at once.  The
// slot index is a launch argument, so a captured CUDA graph re-stamps the
// same slots on every replay: a per-replay timeline of the decode step
// without host involvement.
#include "../common/ptx.cuh"
#include "elementwise.h"

namespace {
__global__ void stamp_kernel(unsigned long long* buf, int idx) {
  b200::pdl_wait();
  b200::pdl_launch_dependents();
  buf[idx] = b200::globaltimer_ns();
}
}  // namespace

int b200_trace_stamp(void* buf, int idx, cudaStream_t st) {
  if (idx < 0) return -1;
  b200::launch_pdl(stamp_kernel, dim3(1), dim3(1), 0, st, reinterpret_cast<unsigned long long*>(buf), idx);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
