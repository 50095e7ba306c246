// Host interface of the elementwise / routing kernels.  All take raw device
// pointers and a stream; return 0 on success.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

int b200_rmsnorm(const void* x, int x_is_f32, int ldx, float* residual, const float* w, float eps, int rows, int K,
                 void* y, int ldy, uint8_t* q, uint8_t* sf, cudaStream_t st);
int b200_quant_mxfp8(const void* x, int x_is_f32, int ldx, int rows, int K, uint8_t* q, uint8_t* sf, cudaStream_t st);
int b200_rope(void* x, int f32, int64_t st_t, int64_t st_h, int T, int H, int d, const int* pos, const float* table,
              cudaStream_t st);
int b200_kv_store(const void* kv, int f32, int64_t ld, int T, int L, int R, const float* w, float eps, const int* pos,
                  const float* table, const int64_t* slots, uint8_t* cache, float kv_scale, cudaStream_t st);
// scoring 0: sigmoid (DeepSeek-V3); 1: sqrt(softplus) (DeepSeek-V4 family).
int b200_router(const float* logits, const float* bias, int T, int E, int G, int topk_group, int K, float scaling,
                int renorm, int scoring, float* w_out, int* id_out, cudaStream_t st);
int b200_moe_align(const int* ids, const float* w, int T, int K, int first, int E, int* seg_start, int* seg_count,
                   int* row_token, float* row_weight, int* pair_row, int* total_rows, int bn1, int* ttile1, int bn2,
                   int* ttile2, cudaStream_t st);
int b200_moe_gather(const uint8_t* xq, const uint8_t* xsf, const int* pair_row, int npairs, int K, int Kd, uint8_t* dq,
                    uint8_t* dsf, cudaStream_t st);
int b200_moe_combine(const void* y, const int* pair_row, int T, int K, int D, const void* add, int add_f32, void* out,
                     int out_f32, cudaStream_t st);
int b200_fill_bytes(void* p, int64_t nbytes, uint64_t seed, uint8_t and_mask, uint8_t or_mask, cudaStream_t st);

// NVFP4 activations (see nvfp4.cu).
int b200_nvfp4_quant(const void* x, int f32, int64_t ld, int T, int K, uint8_t* q, uint8_t* sf, float* g,
                     cudaStream_t st);
int b200_moe_gather4(const uint8_t* xq, const uint8_t* xsf, const float* xg, const int* pair_row, int npairs, int K,
                     int Kx, uint8_t* dq, uint8_t* dsf, float* dg, cudaStream_t st);

// Vocab-parallel sampling (see sample.cu).  peers == nullptr: local buffers
// (out / cand = [world][B][Kc + 1] uint2); else candidates travel through
// the fused all-reduce's receive slots (ArPeers from comm/comm.h).
struct ArPeers;
int b200_lm_candidates(const void* logits, int f32, int64_t ld, int B, int n, int Kc, int vocab_off,
                       const float* temperature, void* out, const ArPeers* peers, const uint32_t* epoch,
                       uint32_t* ticket, cudaStream_t st);
int b200_sample_final(const void* cand, int B, int Kc, int world, const ArPeers* peers, uint32_t* epoch,
                      uint32_t* ticket, const float* temperature, const float* top_p, const int* top_k,
                      const float* uniform, int64_t* tokens, uint32_t* err, cudaStream_t st);

// MXFP8 quantization of rows gathered from head-major blocks: element k of
// row r at x[r * ldx + (k / seg) * seg_stride + k % seg].
int b200_quant_mxfp8_seg(const void* x, int x_is_f32, int ldx, int rows, int K, int seg, int64_t seg_stride,
                         uint8_t* q, uint8_t* sf, cudaStream_t st);

// DeepSeek-V4 family (see v4.cu): mHC stream mixing, Engram, MQA prep, E5.
int b200_hc_post(void* X, const void* y, int64_t ldy, const float* post, const float* comb, int T, int hc, int D,
                 float* sumsq, cudaStream_t st);
int b200_hc_pre(const float* raw, int ldr, int parts, int pstride, const float* sumsq, const float* scale,
                const float* base, int mode, int iters, float eps, float inv_width, const void* X, int T, int hc,
                int D, const float* norm_w, float norm_eps, float* post, float* comb, uint8_t* q, uint8_t* sf,
                void* hb, float* hf, cudaStream_t st);
// Fused hyper-connection boundary (hc_post when y is set, fp32 mixes, the
// coefficients, the normed sublayer input) of T rows; a row per cluster of
// CTAs.  mode 0 needs M = 24 (pre, post, comb), mode 1 (head) M = 4.
int b200_hc_boundary(void* X, int T, int hc, int D, const void* y, int64_t ldy, const float* post_in,
                     const float* comb_in, const float* fn, int M, const float* scale, const float* base, int mode,
                     int iters, float eps, float inv_width, const float* norm_w, float norm_eps, float* post,
                     float* comb, uint8_t* q, uint8_t* sf, void* hb, float* hf, cudaStream_t st);
int b200_hc_mean(const void* X, int T, int hc, int D, void* out, cudaStream_t st);
int b200_engram_hash(const int* ids, const int* pos, const int* q_seq, const int* block_table, int bt_stride,
                     const int64_t* out_slots, int page_size, int* tok_cache, int T, int heads, int per_head,
                     int max_n, const unsigned long long* mults, int* out, cudaStream_t st);
int b200_engram_gather(const uint8_t* table, const uint8_t* scale, const int* ids, int n, int row_lo, int row_hi,
                       void* out, cudaStream_t st);
int b200_engram_gate(void* X, int T, int hc, int D, const void* kv, int kv_f32, int64_t ldkv, const float* q_w,
                     const float* k_w, float eps, float clampv, float* sumsq, cudaStream_t st);
int b200_hc_embed(const void* embed, const int* ids, int T, int hc, int D, void* X, float* sumsq, cudaStream_t st);
int b200_kv_store_v4(const void* kv, int f32, int64_t ld, int T, int L, int rd, const float* w, float eps,
                     const int* pos, const float* table, const int64_t* slots, uint8_t* cache, float kv_scale,
                     cudaStream_t st);
int b200_mqa_q_prep(const void* q, int64_t qt, int64_t qh, int T, int H, int Hq, int rd, const int* pos,
                    const float* table, uint8_t* q8, float* qs, cudaStream_t st);
int b200_attn_fixup(void* o, int T, int H, const float* lse, const float* sink, int rd, const int* pos,
                    const float* table, cudaStream_t st);
int b200_e5_prune(int* ids, float* w, int T, int K, int E, float budget, int max_count, cudaStream_t st);

// Tracing (see trace.cu): %globaltimer into buf[idx] once the stream's
// previous kernel has completed.
int b200_trace_stamp(void* buf, int idx, cudaStream_t st);

// L2 prefetch of up to four regions (16-byte aligned) by `nctas` CTAs.
struct L2Regions {
  const void* ptr[4];
  int64_t bytes[4];
  int n;
};
int b200_l2_prefetch(const L2Regions* r, int nctas, cudaStream_t st);

// Compressed sparse attention (V4 family): store this step's gate logits g
// (column of the qkv GEMM output, stride ld, bf16 or fp32) at their slots, then
// write the compressed latent rows / indexer keys of the blocks of r
// positions the step completes (kernels in v4.cu).
int b200_compress_store(const void* g, int64_t ld, int gf32, const int64_t* slots, const int* pos, const int* q_seq,
                        const int* bt, int bt_stride, int page, int r, int T, float* gate, const float* bias,
                        const uint8_t* kv, int kvd, float kv_scale, const uint8_t* ik, const float* iks, int ikd,
                        uint8_t* ckv, uint8_t* cik, float* cis, cudaStream_t st);
