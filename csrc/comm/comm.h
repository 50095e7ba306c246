// Host interface of the fused NVLink communication kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

constexpr int kArMaxRanks = 8;
// Push all-reduce buffer: [0, 64) uint32 cnt[2][kArMaxRanks] (per-source
// arrivals), [128, 192) NVLS cnt2, [kArCtaCntOff, +2 KB) uint32
// cta_cnt[2][kArMaxCtas] (per-CTA arrivals of the one-kernel all-reduces),
// [kArCtaCnt2Off, +2 KB) cta_cnt2[2][kArMaxCtas] (per-CTA "sum broadcast" of
// the one-kernel NVLS variant), then the receive slots from kArRecvOff.
constexpr int kArMaxCtas = 256;
constexpr int64_t kArCtaCntOff = 256;
constexpr int64_t kArCtaCnt2Off = kArCtaCntOff + 2 * kArMaxCtas * 4;
constexpr int64_t kArRecvOff = 8192;

// Symmetric-buffer base pointers of every rank (UVA peer mappings).
struct ArPeers {
  uint8_t* base[kArMaxRanks];
  int rank;
  int world;
  int max_t;                                // token rows per receive slot
  int hidden = 0;                           // bf16 columns per slot row (kernels that reuse the
                                            // slots as raw bytes need it to locate a slot)
  // NVLS mode (nonzero `mc`, the multicast address of the same symmetric
  // buffer): pushers store their partial only into their OWN input slot
  // (layout of nvls_in_off) and still publish one arrival on every rank; the
  // reduction then reads the sum of all ranks' slots through the switch.
  uint8_t* mc = nullptr;
};

// NVLS all-reduce buffer (symmetric + multicast-bound, identical layout on
// every rank):
//   [0, 64)     uint32 cnt_in[2][kArMaxRanks]    pushers' arrivals
//   [128, 192)  uint32 cnt_out[2][kArMaxRanks]   reduce CTAs done broadcasting
//   kArRecvOff  bf16 in[2][max_t][hidden]        each rank's own partial
//   then        bf16 out[2][max_t][hidden]       the sum, written by multimem.st
constexpr int64_t kNvlsCnt2Off = 128;
inline int64_t nvls_buffer_bytes(int max_t, int hidden) { return kArRecvOff + (int64_t)4 * max_t * hidden * 2; }

__host__ __device__ inline int64_t ar_buffer_bytes(int world, int max_t, int hidden) {
  return kArRecvOff + (int64_t)2 * world * max_t * hidden * 2;
}
// Expert-parallel buffers (DP attention) append a combine region after the
// per-source slots: bf16 comb[2][max_t][K][hidden], filled by the experts'
// FC2 epilogues of every rank (pair (t, k) of this rank's token t).
__host__ __device__ inline int64_t ep_combine_off(int world, int max_t, int hidden) {
  return ar_buffer_bytes(world, max_t, hidden);
}
inline int64_t ar_buffer_bytes_ep(int world, int max_t, int hidden, int K) {
  return ep_combine_off(world, max_t, hidden) + (int64_t)2 * max_t * K * hidden * 2;
}

// Push kernels publish once per destination rank (the last CTA, by ticket);
// the reduce kernel therefore expects one arrival per source rank.
int b200_ar_push(const void* x, int T, int hidden, const ArPeers* peers, const uint32_t* epoch, uint32_t* ticket,
                 int nctas, cudaStream_t st);
int b200_ar_reduce_norm(int T, int hidden, const ArPeers* peers, uint32_t* epoch, uint32_t* ticket, int push_ctas,
                        float* residual, const float* w, float eps, void* y, uint8_t* q, uint8_t* sf, uint32_t* err,
                        cudaStream_t st);
// One kernel: push (plain partial x, or with pair_row the MoE combine of the
// local expert rows y + add) + per-CTA arrivals + reduce + residual +
// RMSNorm (+ MXFP8) of the rows each CTA owns.  With peers->mc (the NVLS
// buffer's multicast address) CTA c stores its rows only into this rank's
// own input slot, rank c % world sums them through the switch
// (multimem.ld_reduce) and broadcasts the sum (multimem.st), and every
// rank's CTA c normalises the broadcast rows.  Push mode with chunks > 1: each
// row owner's columns are pushed by `chunks` CTAs and reduced by the first.
int b200_ar_fused_norm(const void* x, const int* pair_row, int K, const void* add, int T, int hidden,
                       const ArPeers* peers, uint32_t* epoch, uint32_t* ticket, float* residual, const float* w,
                       float eps, void* y, uint8_t* q, uint8_t* sf, uint32_t* err, cudaStream_t st,
                       int chunks = 1);
int b200_moe_combine_push(const void* y, const int* pair_row, int T, int K, int hidden, const void* add,
                          const ArPeers* peers, const uint32_t* epoch, uint32_t* ticket, int nctas, cudaStream_t st);
// NVLS all-reduce + residual + RMSNorm (+ MXFP8): waits for every rank's
// push (`expected` arrivals each), sums this rank's share of the rows with
// multimem.ld_reduce and broadcasts it with multimem.st, waits for every
// rank's share, then the row epilogue of b200_ar_reduce_norm on the sum.
int b200_nvls_ar_norm(int T, int hidden, const ArPeers* peers, uint32_t* epoch, uint32_t* ticket, int expected,
                      float* residual, const float* w, float eps, void* y, uint8_t* q, uint8_t* sf, uint32_t* err,
                      cudaStream_t st);
// Owner side of the combine fused into the experts' FC2 epilogue: waits for
// every rank's arrival, then per own token row t: sum over k (ids[t][k] >= 0,
// in k order) of comb[p][t][k] + add[t] (shared expert, optional) + residual,
// RMSNorm (+ MXFP8) as b200_ar_reduce_norm.
int b200_ep_comb_reduce_norm(int T_r, int hidden, int K, const int* ids, const void* add, const ArPeers* peers,
                             uint32_t* epoch, uint32_t* ticket, float* residual, const float* w, float eps, void* y,
                             uint8_t* q, uint8_t* sf, uint32_t* err, cudaStream_t st);
// DeepSeek-V4 sublayer boundary under TP: sum of the pushed partials y (push
// protocol) fused with the hyper-connection post X <- post y + comb^T X
// (hc = 4 bf16 streams [T, 4, D], in place) and the row sum of squares.
int b200_ar_hc_post(int T, int D, const ArPeers* peers, uint32_t* epoch, uint32_t* ticket, int expected, void* X,
                    const float* post, const float* comb, float* sumsq, uint32_t* err, cudaStream_t st);

// ---------------------------------------------------------------------------
// Expert-parallel dispatch buffer (symmetric, identical layout on every rank):
//   [0, 256)              uint32 arrival counters cnt[2][kArMaxRanks]
//   [kEpRegionOff + p * par_bytes, ...)   parity-p region:
//       q   [rows_p, hidden] bytes       rows_p = round_up(world * max_t, 128);
//                                        MXFP8 rows use all of it, NVFP4 half
//       sf  [rows_p * hidden / 16]       UE8M0 per 32 (MXFP8) or e4m3 per 16
//                                        (NVFP4), tcgen05 scale layout
//       ids int32 [world * max_t, K]     (-1 = no expert / padded token)
//       w   fp32  [world * max_t, K]
//       g   fp32  [world * max_t]        NVFP4 per-row global scale
// Row (src, t) of a step with T_step tokens per rank is src * T_step + t.
constexpr int64_t kEpRegionOff = 1024;

struct EpPeers {
  uint8_t* base[kArMaxRanks];
  int rank;
  int world;
  int max_t;
  int hidden;
  int K;
  int64_t par_bytes, off_sf, off_ids, off_w, off_g;
};

inline int64_t ep_round(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

inline void ep_layout(int world, int max_t, int hidden, int K, int64_t* par_bytes, int64_t* off_sf, int64_t* off_ids,
                      int64_t* off_w, int64_t* off_g) {
  const int64_t rows = (int64_t)world * max_t;
  const int64_t rows_p = ep_round(rows, 128);
  *off_sf = ep_round(rows_p * hidden, 1024);
  *off_ids = ep_round(*off_sf + rows_p * hidden / 16, 1024);
  *off_w = ep_round(*off_ids + rows * K * 4, 1024);
  *off_g = ep_round(*off_w + rows * K * 4, 1024);
  *par_bytes = ep_round(*off_g + rows * 4, 1024);
}

inline int64_t ep_buffer_bytes(int world, int max_t, int hidden, int K) {
  int64_t pb, a, b, c, d;
  ep_layout(world, max_t, hidden, K, &pb, &a, &b, &c, &d);
  return kEpRegionOff + 2 * pb;
}

// Dispatch: token t of this rank (T_r valid of T_step rows) goes, with its
// routing, to every rank that owns one of its experts (routing rows go to
// every rank, so receivers see -1 for tokens they do not serve).
// fp4 = 1: q / sf / g are NVFP4 rows (hidden / 2 bytes, e4m3 per 16, global g).
int b200_ep_dispatch(const uint8_t* q, const uint8_t* sf, const float* g, int fp4, const int* ids, const float* w,
                     int T_r, int T_step, int experts_per_rank, const EpPeers* peers, const uint32_t* epoch,
                     uint32_t* ticket, cudaStream_t st,
                     int peer_pull = 0);
// Routing layout over the received world * T_step tokens (waits for every
// rank's dispatch; bounded).  release = 1 (no ep_gather follows: the expert
// GEMM reads the received rows in place): also frees the parity (counters to
// zero, epoch + 1), so the consumer finds the rows at parity (epoch + 1) & 1.
// row_pair (optional): sorted row -> pair index (token * K + k), for the
// combine fused into the experts' FC2 epilogue.
int b200_ep_align(const EpPeers* peers, int T_step, int first, int E, int* seg_start, int* seg_count, int* row_token,
                  float* row_weight, int* pair_row, int* total_rows, int bn1, int* ttile1, int bn2, int* ttile2,
                  uint32_t* epoch, uint32_t* err, int release, cudaStream_t st, int* row_pair = nullptr);
// Gather received rows into the expert-sorted operand; the last CTA frees
// the parity (counters to zero, epoch + 1).
int b200_ep_gather(const EpPeers* peers, int T_step, const int* pair_row, int fp4, uint8_t* dq, uint8_t* dsf, float* dg,
                   uint32_t* epoch, uint32_t* ticket, cudaStream_t st);
// Combine + reduce-scatter: each received token's partial over this rank's
// experts goes to its owner's all-reduce slot; `add` (this rank's shared
// expert output for its own T_r tokens) joins the rows this rank owns.
int b200_ep_combine_rs(const void* y, const int* pair_row, int T_step, int T_r, int K, int hidden, const void* add,
                       const ArPeers* ar, const uint32_t* ar_epoch, uint32_t* ar_ticket, int nctas, cudaStream_t st);
