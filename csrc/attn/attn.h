// Host interface of the MLA attention kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

int b200_mla_simt(const void* q_abs, const void* q_pe, int T, int H, int L, int R, const uint8_t* cache,
                  float kv_scale, const int* block_table, int bt_stride, const int* q_seq, const int* q_pos,
                  const int* topk, int topk_n, int page_size, float sm_scale, void* out, cudaStream_t st);
