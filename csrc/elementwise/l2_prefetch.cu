// L2 prefetch of weights a later kernel of the step will stream: the next
// projection's weights are pulled into L2 while attention (which is bound by
// its own KV reads and the softmax chain, not by weight traffic) runs, on a
// low-priority side stream.  Each CTA's first thread issues bulk L2
// prefetches (cp.async.bulk.prefetch.L2, no shared memory, no completion to
// wait for) over its share of up to four regions.
//
// Reference parity: l2pf_unit.cu:22,33 (`line_kernel` / `bulk_kernel`, the
// L2PF lever's WO-A / wo_b / router warm-up during attention, l2pf.py:4-5).
#include "../common/ptx.cuh"
#include "elementwise.h"

namespace b200 {
namespace ew {

constexpr int64_t kChunk = 64 * 1024;       // bytes per prefetch instruction

__global__ void l2_prefetch_kernel(L2Regions r) {
  if (threadIdx.x != 0) return;
  for (int k = 0; k < r.n; ++k) {
    const uint8_t* base = reinterpret_cast<const uint8_t*>(r.ptr[k]);
    const int64_t bytes = r.bytes[k] & ~int64_t(15);
    const int64_t chunks = (bytes + kChunk - 1) / kChunk;
    for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x) {
      const int64_t off = c * kChunk;
      const uint32_t sz = (uint32_t)min(kChunk, bytes - off);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off), "r"(sz) : "memory");
    }
  }
}

}  // namespace ew
}  // namespace b200

int b200_l2_prefetch(const L2Regions* r, int nctas, cudaStream_t st) {
  if (r->n <= 0) return 0;
  if (r->n > 4 || nctas <= 0) return -1;
  for (int k = 0; k < r->n; ++k)
    if ((reinterpret_cast<uintptr_t>(r->ptr[k]) & 15) != 0) return -1;   // bulk copies start on 16 bytes
  b200::ew::l2_prefetch_kernel<<<nctas, 32, 0, st>>>(*r);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
