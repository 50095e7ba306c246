// Host interface of the MXFP8 tcgen05 GEMM (see gemm_mxf8.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

enum GemmEpi : int {
  kEpiStoreBf16 = 0,     // out[row, n] = bf16(acc)
  kEpiAtomicF32 = 1,     // out[row, n] += acc (fp32, split-K)
  kEpiSwiglu = 2,        // q_out/sf_out = mxfp8(silu(gate) * up)
  kEpiWeightedBf16 = 3,  // out[row, n] = bf16(acc * row_weight[row])  (grouped only)
  kEpiClusterSplit = 4,  // split-K over a thread-block cluster, DSMEM reduction, bf16 out
  kEpiClusterPush = 5,   // as kEpiClusterSplit, but the reduced tile is pushed into every
                         // rank's all-reduce receive slot (fused GEMM + all-reduce)
  kEpiClusterSwiglu = 6, // split-K over a cluster for thin gate_up GEMMs; the reduce applies
                         // SwiGLU and MXFP8 requant (q_out / sf_out)
};

struct GemmArgs {
  const uint8_t* w;        // e4m3 weights [E *] nw x k
  const uint8_t* w_sf;     // packed sf128x4 scales of w
  int64_t w_sf_estride;    // bytes between experts' scales (grouped)
  const uint8_t* x;        // e4m3 activations [x_rows, k]
  const uint8_t* x_sf;     // packed scales of x
  int64_t x_rows;          // rows addressable in x (for the TMA bounds)
  int nw;                  // weight rows per expert (dense: total rows)
  int nw_total;            // dense: rows of w
  int t;                   // dense: tokens
  int k;
  int splits;              // dense split-K factor (kEpiAtomicF32)
  int num_experts;         // > 0: grouped mode
  const int* seg_start;    // grouped: first sorted row per expert (128-aligned)
  const int* seg_count;    // grouped: rows per expert
  int max_rows_per_expert; // grouped: upper bound of seg_count (grid size)
  int epi;
  void* out;
  int ldo;
  uint8_t* q_out;
  uint8_t* sf_out;
  int ldq;
  int inter;
  const float* row_weight;
  uint32_t* err;
  int pdl;
  // kEpiClusterPush: symmetric all-reduce buffers (see comm/comm.h)
  const void* ar_peers;     // const ArPeers*
  const uint32_t* ar_epoch;
  uint32_t* ar_ticket;      // publish ticket (last CTA publishes)
};

int b200_gemm_mxf8(const GemmArgs* args, cudaStream_t stream);

// Persistent grouped GEMM over the routed experts (see gemm_grouped.cu).
struct GroupedArgs {
  const uint8_t* w;        // e4m3 [E, nw, k]
  const uint8_t* w_sf;
  int64_t w_sf_estride;
  const uint8_t* x;        // e4m3 sorted rows [x_rows, k]
  const uint8_t* x_sf;
  int64_t x_rows;
  int nw, k, E, inter;
  int bn;                  // token tile: 16/32/64 (swiglu), up to 128 (weighted)
  const int* seg_start;
  const int* seg_count;
  const int* ttile_off;    // [E+1] prefix of ceil(count/bn)
  int epi;                 // kEpiSwiglu or kEpiWeightedBf16
  void* out;
  int ldo;
  uint8_t* q_out;
  uint8_t* sf_out;
  int ldq;
  const float* row_weight;
  uint32_t* err;
  int num_ctas;
  int pdl;
  // NVFP4 operands (fp4 = 1): w / x hold packed e2m1 pairs (k / 2 bytes per
  // row, low nibble = even element), w_sf / x_sf e4m3 scales per 16 elements
  // in the same 128-row x 4-column chunk layout; fp32 global scales: w_g per
  // expert, x_g per sorted activation row (or x_g_const when null); FC1
  // writes its SwiGLU output as NVFP4 with global scale out_g.
  // a_tiled = 1: w is stored as contiguous 128-row x 128-byte tiles,
  // [E * nw / 128][k_bytes / 128][128][128], so every TMA box reads one
  // contiguous 16 KB block (short weight rows otherwise scatter each box
  // over 128 DRAM rows).
  int a_tiled;
  int fp4;
  const float* w_g;
  const float* x_g;
  float x_g_const;
  float out_g;
};
int b200_gemm_grouped(const GroupedArgs* args, cudaStream_t stream);

// Fused persistent FC1 + FC2 of the routed experts (see moe_fused.cu).
struct MoeFusedArgs {
  const uint8_t* w13;      // [E, 2 * inter, hidden] (MXFP8 e4m3 or NVFP4 pairs; optionally tiled)
  const uint8_t* w13_sf;
  int64_t w13_sf_estride;
  const uint8_t* w2;       // [E, hidden, inter]
  const uint8_t* w2_sf;
  int64_t w2_sf_estride;
  const uint8_t* x;        // sorted activation rows [rows, hidden]
  const uint8_t* x_sf;
  uint8_t* hq;             // FC1 output / FC2 operand [rows, inter]
  uint8_t* hq_sf;
  void* y;                 // bf16 [rows, ldy]
  int ldy;
  int64_t rows;
  int hidden, inter, E, bn;
  const int* seg_start;
  const int* seg_count;
  const int* ttile_off;    // [E+1] prefix of ceil(count / bn)
  const float* row_weight;
  int* work;               // [2] zero before the first launch; the kernel resets it
  int* fc1_done;           // [E] idem
  uint32_t* err;
  int num_ctas;
  int pdl;
  int a_tiled;
  int fp4;
  const float* x_g;        // NVFP4: per sorted row
  const float* w1_g;       // NVFP4: per expert
  const float* w2_g;
  float out_g;             // NVFP4: global scale of the FC1 output
  // pull = 1: the FC1 activation rows are read straight from their source
  // buffers (this GPU's or a peer's, P2P) by the producer warp instead of a
  // pre-gathered x: sorted row r is token row_token[r] = s * src_rows + t,
  // i.e. row t of source s (q rows, scales in the tcgen05 layout, NVFP4 g).
  int pull;
  const uint8_t* src_q[8];
  const uint8_t* src_sf[8];
  const float* src_g[8];
  int src_rows;
  const int* row_token;
  // sources in a two-parity buffer: every source pointer moves by
  // ((*src_epoch + src_epoch_add) & 1) * src_par_bytes (null: fixed sources)
  const uint32_t* src_epoch;
  int src_epoch_add;
  int64_t src_par_bytes;
  // expert-parallel combine in the FC2 epilogue (c_row_pair set): the
  // weighted output row of pair (token, k) is stored straight into the
  // token's owner rank (P2P), slot [parity][token's row there][k] of that
  // rank's combine region, instead of into y; the last CTA then publishes one
  // arrival on every rank.  Token = src rank * c_T_step + its row there.
  const int* c_row_pair;     // sorted row -> pair index token * c_K + k
  int c_K, c_T_step;
  uint8_t* c_base[8];
  int c_rank, c_world, c_max_t;
  int64_t c_off;             // bytes from a rank's symmetric base to its combine region
  const uint32_t* c_epoch;   // parity = *c_epoch & 1
};
int b200_moe_fused(const MoeFusedArgs* args, cudaStream_t stream);

// Batched bf16 swap-AB GEMM for the MLA weight absorptions (see gemm_bf16.cu).
struct Bf16GemmArgs {
  const void* w;           // bf16 [B][M][K] (K contiguous)
  const void* x;           // bf16 tokens: element (t, b, k) at x[t * x_ts + b * x_bs + k]
  int64_t x_ts, x_bs;
  int T, K, M, B;
  int epi;                 // 0 bf16 store, 1 absorb_q + query prep, 2 absorb_o + MXFP8 rows,
                           // 3 split-K fp32 atomic accumulate into out (zeroed by the caller)
  int splits;              // epi 3: K splits (grid z = M tiles * splits)
  void* out;               // epi 0: bf16, element (t, b, m) at out[t * out_ts + b * out_bs + m]
  int64_t out_ts, out_bs;
  const void* q_pe;        // epi 1: un-rotated rope part, (t, b, d) at q_pe[t * pe_ts + b * pe_bs + d]
  int64_t pe_ts, pe_bs;
  const int* pos;
  const float* table;
  uint8_t* q8;             // epi 1: e4m3 [T, B, 576]
  float* qs;               // epi 1: [T, B]
  uint8_t* q;              // epi 2: e4m3 [T, B * 128]
  uint8_t* sf;             // epi 2: scales (tcgen05 layout, K = B * 128)
  uint32_t* err;
};
int b200_bf16_gemm(const Bf16GemmArgs* args, cudaStream_t stream);
