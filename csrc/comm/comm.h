// Host interface of the fused NVLink communication kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

constexpr int kArMaxRanks = 8;
constexpr int64_t kArRecvOff = 256;        // bytes: counters first, then the receive slots

// Symmetric-buffer base pointers of every rank (UVA peer mappings).
struct ArPeers {
  uint8_t* base[kArMaxRanks];
  int rank;
  int world;
  int max_t;                                // token rows per receive slot
};

inline int64_t ar_buffer_bytes(int world, int max_t, int hidden) {
  return kArRecvOff + (int64_t)2 * world * max_t * hidden * 2;
}

// Push kernels publish once per destination rank (the last CTA, by ticket);
// the reduce kernel therefore expects one arrival per source rank.
int b200_ar_push(const void* x, int T, int hidden, const ArPeers* peers, const uint32_t* epoch, uint32_t* ticket,
                 int nctas, cudaStream_t st);
int b200_ar_reduce_norm(int T, int hidden, const ArPeers* peers, uint32_t* epoch, uint32_t* ticket, int push_ctas,
                        float* residual, const float* w, float eps, void* y, uint8_t* q, uint8_t* sf, uint32_t* err,
                        cudaStream_t st);
int b200_moe_combine_push(const void* y, const int* pair_row, int T, int K, int hidden, const void* add,
                          const ArPeers* peers, const uint32_t* epoch, uint32_t* ticket, int nctas, cudaStream_t st);
