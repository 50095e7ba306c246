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
  const int* topk = nullptr;  // [T, topk_n] cache positions (-1 = none): sparse MLA
  int topk_n = 0;
  int hb = 0;                 // heads per CTA (16 / 32 / 64); 0 = largest that divides H
  float* lse_out = nullptr;   // [T, H] log-sum-exp (log2 of the sum of 2^(scaled score)), optional
  // compressed sparse attention: top-k entries >= kMlaCompFlag name compressed
  // block j = entry - kMlaCompFlag, whose row (same e4m3 layout and scale) is
  // page * (64 / ratio) + (j * ratio mod 64) / ratio of cache2
  const uint8_t* cache2 = nullptr;
  int64_t cache2_rows = 0;
  int ratio2 = 0;
};
constexpr int kMlaCompFlag = 1 << 30;
// Lightning indexer (sparse MLA): key store, query quantisation, tcgen05
// scores and the top-k radix select.
int b200_ix_k_store(const void* k, int f32, int64_t ld, int T, const float* ln_w, const float* ln_b, float eps,
                    const int* pos, const float* table, int R, const int64_t* slots, uint8_t* cache, float* scale,
                    cudaStream_t st);
int b200_ix_q_quant(const void* q, int q_f32, int64_t ldq, const void* wraw, int w_f32, int64_t ldw, int T, int NH,
                    float w_factor, const int* pos, const float* table, int R, uint8_t* q8, float* wq, cudaStream_t st);
int b200_ix_score(const uint8_t* q8, const float* wq, int T, int NH, const uint8_t* k_cache, int64_t cache_rows,
                  const float* k_scale, const int* block_table, int bt_stride, const int* q_seq, const int* q_pos,
                  int page_size, int nsplit, float* scores, int64_t ld, uint32_t* err, cudaStream_t st);
// max_n: the longest row (q_pos + 1) the caller knows of; above 8K the rows
// are split over a cluster of CTAs (0: one CTA per row).
int b200_topk_select(const float* scores, int64_t ld, const int* q_pos, int T, int K, int* out, cudaStream_t st,
                     int max_n = 0);

int b200_mla_q_quant(const void* q_abs, const void* q_pe, int TH, uint8_t* q8, float* qs, cudaStream_t st);
// RoPE of the un-rotated q_pe + e4m3 quantization of [q_abs | q_pe] from
// strided bf16 inputs (token stride, head stride in elements).
int b200_mla_q_prep(const void* q_abs, int64_t qa_t, int64_t qa_h, const void* q_pe, int64_t qp_t, int64_t qp_h, int T,
                    int H, const int* pos, const float* table, uint8_t* q8, float* qs, cudaStream_t st);
int b200_mla_tc(const MlaTcArgs* args, cudaStream_t st);

// ---------------------------------------------------------------------------
// Allocation-free MLA decode (absorbed MLA over the paged e4m3 latent cache,
// split-KV with merge), for callers that cannot allocate device memory: its
// scratch lives in fixed device arrays inside the library (about 10.8 MB per
// GPU, held until exit; limits T*H <= 4096 and nsplit*T*H <= 4096).  Inputs:
// q_abs bf16 [T,H,512], q_pe bf16 [T,H,64], kv_cache e4m3 [cache_rows,576],
// int32 block_table [*, bt_stride] / q_seq [T] / q_pos [T]; output bf16
// [T,H,512].  Returns 0 or a B200_NOALLOC_ERR_* code (see
// b200_mla_decode_noalloc_error).  Calls share the scratch, so calls that
// overlap on the GPU race; the first call on a device sets up the scratch
// addresses and should come before any stream capture.  The stream must
// belong to the current device (a stream of another device is rejected as
// a bad argument).  Kernel-side failures (a bounded wait that ran out of
// time) set a sticky status word in the library: b200_mla_decode_noalloc_status
// waits for the stream, returns the word (0 = fine) and clears it.
// This entry point has no counterpart in the reference.
// ---------------------------------------------------------------------------
#define B200_NOALLOC_ERR_BAD_ARG (-1)
#define B200_NOALLOC_ERR_TOO_LARGE (-2)
#define B200_NOALLOC_ERR_SETUP (-3)
#define B200_NOALLOC_ERR_LAUNCH (-4)
extern "C" int b200_mla_decode_noalloc(const void* q_abs, const void* q_pe, int T, int H, const void* kv_cache,
                                       long long cache_rows, const int* block_table, int bt_stride, const int* q_seq,
                                       const int* q_pos, int page_size, float sm_scale, float kv_scale, int nsplit,
                                       void* out, cudaStream_t stream);
extern "C" const char* b200_mla_decode_noalloc_error(int code);
extern "C" int b200_mla_decode_noalloc_status(cudaStream_t stream, unsigned int* status);
