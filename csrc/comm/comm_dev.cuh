// Device-side pieces of the NVLink push protocols (one process per GPU, peer
// buffers mapped through torch symmetric memory):
//   * every symmetric buffer starts with uint32 arrival counters
//     cnt[2 parities][kArMaxRanks];
//   * a push grid P2P-stores its rows, then each CTA fences and takes a local
//     ticket; the last CTA publishes one release.sys increment of
//     cnt[parity][my rank] on every destination rank;
//   * consumers poll cnt with ld.acquire.sys under a %globaltimer deadline.
#pragma once
#include "../common/ptx.cuh"
#include "comm.h"

namespace b200 {
namespace comm {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t* counters(uint8_t* base, int parity) {
  return reinterpret_cast<uint32_t*>(base) + parity * kArMaxRanks;
}

__device__ __forceinline__ __nv_bfloat16* recv_slot(uint8_t* base, int parity, int src, int world, int max_t,
                                                    int hidden) {
  return reinterpret_cast<__nv_bfloat16*>(base + kArRecvOff) +
         ((int64_t)(parity * world + src) * max_t) * hidden;
}

// Destinations of a push: every rank's slot recv[parity][my rank] (push
// mode), or only this rank's own NVLS input slot (mc set).
__device__ __forceinline__ int push_dests(const ArPeers& p) { return p.mc ? 1 : p.world; }
__device__ __forceinline__ __nv_bfloat16* push_slot(const ArPeers& p, int d, int parity, int hidden) {
  return p.mc ? recv_slot(p.base[p.rank], parity, 0, 1, p.max_t, hidden)
              : recv_slot(p.base[d], parity, p.rank, p.world, p.max_t, hidden);
}

__device__ __forceinline__ uint32_t* cta_counters(uint8_t* base, int parity) {
  return reinterpret_cast<uint32_t*>(base + kArCtaCntOff) + parity * kArMaxCtas;
}

__device__ __forceinline__ uint32_t* cta_counters2(uint8_t* base, int parity) {
  return reinterpret_cast<uint32_t*>(base + kArCtaCnt2Off) + parity * kArMaxCtas;
}

__device__ __forceinline__ uint32_t* counters2(uint8_t* base, int parity) {
  return reinterpret_cast<uint32_t*>(base + kNvlsCnt2Off) + parity * kArMaxRanks;
}

// Last CTA of the grid (by ticket) publishes one arrival on every rank.
__device__ __forceinline__ void publish_push(uint8_t* const* bases, int world, int rank, int parity, uint32_t* ticket) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t prev = atomicAdd(ticket, 1u);
    if (prev == gridDim.x * gridDim.y * gridDim.z - 1) {
      __threadfence_system();
      *ticket = 0u;
      for (int q = 0; q < world; ++q)
        asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(counters(bases[q], parity) + rank), "r"(1u)
                     : "memory");
    }
  }
}

// Thread 0 waits until cnt[parity][src] >= expected for every src (bounded);
// returns the block-uniform verdict.  On timeout the error word is set.
__device__ __forceinline__ bool wait_arrivals(uint8_t* mine, int parity, int world, uint32_t expected, uint32_t* err,
                                              int* ok_s) {
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint32_t* cnt = counters(mine, parity);
    const uint64_t t0 = globaltimer_ns();
    for (int src = 0; src < world && ok; ++src) {
      while (ld_acquire_sys(cnt + src) < expected) {
        if (globaltimer_ns() - t0 > kWaitBudgetNs) {
          if (err) atomicExch(err, kErrPeerTimeout);
          ok = 0;
          break;
        }
      }
    }
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s != 0;
}

}  // namespace comm
}  // namespace b200
