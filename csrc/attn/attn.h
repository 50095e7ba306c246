// Host interface of the MLA attention kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

int b200_mla_simt(const void* q_abs, const void* q_pe, int T, int H, int L, int R, const uint8_t* cache,
                  float kv_scale, const int* block_table, int bt_stride, const int* q_seq, const int* q_pos,
                  const int* topk, int topk_n, int page_size, float sm_scale, void* out, cudaStream_t st);

struct MlaTcArgs {
  const uint8_t* q8;        // e4m3 [T, H, 576]
  const float* q_scale;     // [T, H]
  const uint8_t* cache;     // e4m3 [cache_rows, 576]
  int64_t cache_rows;
  const int* block_table;
  int bt_stride;
  const int* q_seq;
  const int* q_pos;
  int T, H;
  int page_size;
  int nsplit;
  int split_tokens;
  float sm_scale, kv_scale;
  void* out;                // bf16 [T, H, 512]
  float* part_o;            // [nsplit, T, H, 512]
  float* part_lse;          // [nsplit, T, H]
  uint32_t* err;
};
int b200_mla_q_quant(const void* q_abs, const void* q_pe, int TH, uint8_t* q8, float* qs, cudaStream_t st);
int b200_mla_tc(const MlaTcArgs* args, cudaStream_t st);
