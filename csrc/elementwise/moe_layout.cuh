// Device-side MoE routing layout shared by the single-GPU MoE path and the
// expert-parallel dispatch path:
//
//   moe_align_body  (one CTA, 3*E ints of shared memory): from the routing
//       (ids, weights) of T tokens x K choices, build per-expert segments
//       (row starts padded to 128, counts), the per-row token / weight
//       lists, the (token, choice) -> row map and the token-tile prefix
//       sums the persistent grouped GEMMs walk.
//   moe_gather_pair (one CTA per (token, choice)): copy token t's MXFP8 row
//       (e4m3 data + UE8M0 scales in the tcgen05 scale layout) to row r of
//       the expert-sorted operand.
#pragma once
#include "../common/ptx.cuh"

namespace b200 {
namespace moe {

// Byte offset of (row, k-block) in the sf128x4 scale layout.
__device__ __forceinline__ int64_t sf_offset(int row, int kblock, int kb_total) {
  return ((int64_t)((row >> 7) * (kb_total >> 2) + (kblock >> 2)) << 9) + ((row & 31) << 4) + (((row & 127) >> 5) << 2) +
         (kblock & 3);
}

__device__ __forceinline__ void moe_align_body(const int* ids, const float* w, int T, int K, int first, int E,
                                               int* seg_start, int* seg_count, int* row_token, float* row_weight,
                                               int* pair_row, int* total_rows, int bn1, int* ttile1, int bn2,
                                               int* ttile2, int* sh, int* row_pair = nullptr) {
  int* cnt = sh;          // [E]
  int* start = sh + E;    // [E]
  int* fill = sh + 2 * E; // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) { cnt[e] = 0; fill[e] = 0; }
  __syncthreads();
  const int n = T * K;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = __ldcg(ids + i) - first;
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0, a1 = 0, a2 = 0;
    for (int e = 0; e < E; ++e) {
      start[e] = acc;
      acc += (cnt[e] + 127) & ~127;
      if (ttile1) ttile1[e] = a1;
      if (ttile2) ttile2[e] = a2;
      a1 += (cnt[e] + bn1 - 1) / bn1;
      a2 += (cnt[e] + bn2 - 1) / bn2;
    }
    if (ttile1) ttile1[E] = a1;
    if (ttile2) ttile2[E] = a2;
    *total_rows = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    seg_start[e] = start[e];
    seg_count[e] = cnt[e];
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = __ldcg(ids + i) - first;
    if (e >= 0 && e < E) {
      const int r = start[e] + atomicAdd(&fill[e], 1);
      row_token[r] = i / K;
      row_weight[r] = __ldcg(w + i);
      pair_row[i] = r;
      if (row_pair) row_pair[r] = i;
    } else {
      pair_row[i] = -1;
    }
  }
}

__device__ __forceinline__ void moe_gather_pair(const uint8_t* xq, const uint8_t* xsf, int t, int r, int Kd,
                                                uint8_t* dq, uint8_t* dsf) {
  const uint4* s = reinterpret_cast<const uint4*>(xq + (int64_t)t * Kd);
  uint4* d = reinterpret_cast<uint4*>(dq + (int64_t)r * Kd);
  for (int i = threadIdx.x; i < Kd / 16; i += blockDim.x) d[i] = __ldcg(s + i);
  const int kb = Kd / 32;
  for (int b = threadIdx.x; b < kb; b += blockDim.x) dsf[sf_offset(r, b, kb)] = __ldcg(xsf + sf_offset(t, b, kb));
}

}  // namespace moe
}  // namespace b200
