// DeepSeek-V4-family kernels: mHC residual-stream mixing, Engram lookups,
// MQA query / key preparation with a rope tail inside the latent row, the
// attention-sink + inverse-RoPE output fix-up, and the E5 routed-expert prune.
//
//   hc_post        X'_c = post_c * y + sum_r comb[r][c] X_r over the hc
//                  residual streams (bf16, in place) + the row sum of squares
//                  of X' (the RMS of the next coefficients).
//   hc_pre         coefficients from the raw mixes (X_flat . fn^T, computed
//                  by the tcgen05 GEMM in bf16 hi/mid/lo parts): sigmoid pre,
//                  2*sigmoid post, row-softmax + Sinkhorn comb on 16 lanes;
//                  then the sublayer input RMSNorm(sum_c pre_c X_c) * w as
//                  MXFP8 and/or bf16 / fp32.  Head mode: pre only.
//   hc_mean        mean over the streams (draft-model taps).
//   hc_embed       first layer: every stream = the embedding row (+ sum sq).
//   engram_hash    n-gram hash ids per token from the batch and a per-slot
//                  token cache (the token at each KV slot), which it updates.
//   engram_gather  one warp per lookup: 256 e4m3 bytes + 8 UE8M0 scales of a
//                  host-memory row (mapped, read over the host link) -> bf16;
//                  rows outside this rank's shard give zeros.
//   engram_gate    per token: a_c = sigmoid(clamp(<rmsnorm(X_c) q_w,
//                  rmsnorm(k) k_w> / sqrt(D))), X_c += a_c v.
//   kv_store_v4    RMSNorm of the latent row, RoPE on its tail, e4m3 into the
//                  paged cache row (the row's 64 rope-key bytes stay zero).
//   mqa_q_prep     RoPE on each head's tail + per-(token, head) e4m3 scale.
//   attn_fixup     o *= 1 / (1 + 2^(sink log2e - lse)); inverse RoPE of the
//                  tail at the query position.
//   e5_prune       one CTA: histogram of picks, per-row candidate runs
//                  (lightest first), drop experts whose every pick is a
//                  candidate.
//
// Reference parity: sk_unit.cu:1-15 / mhc_unit.cu:1-12 (mHC stats +
// coefficients), hq_unit.cu:1-10 (combine + norm + MXFP8), fin.py:218-246
// (post), eg_gather.cu:1-8 (Engram rows), qr_unit.cu / ro_unit.cu:73 (rope,
// inverse rope tail), route_e5.cu:4-12 (E5), aux.py (stream means).  All
// arithmetic here is our own (sums in fixed thread / warp order).
#include <cuda_fp8.h>

#include "../common/ptx.cuh"
#include "../comm/comm_dev.cuh"
#include "elementwise.h"
#include "row_util.cuh"

namespace b200 {
namespace v4 {

using ew::block_sum;
using ew::load8;
using ew::quant8;
using ew::store8_bf16;
using ew::store8_f32;

constexpr int kThreads = 256;
constexpr int kHC = 4;
constexpr int kMaxIt = 4;    // rows up to 256 * 8 * 4 = 8192 elements
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float sigmoidf(float x) { return 1.f / (1.f + expf(-x)); }

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16(v)); }

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) hc_post_kernel(__nv_bfloat16* X, const __nv_bfloat16* y, int64_t ldy,
                                                           const float* post, const float* comb, int D,
                                                           float* sumsq) {
  __shared__ float red[32];
  __shared__ float cf[kHC * kHC + kHC];
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int t = blockIdx.x;
  if (threadIdx.x < kHC * kHC) cf[threadIdx.x] = __ldcg(comb + (int64_t)t * kHC * kHC + threadIdx.x);
  if (threadIdx.x < kHC) cf[kHC * kHC + threadIdx.x] = __ldcg(post + (int64_t)t * kHC + threadIdx.x);
  __syncthreads();
  __nv_bfloat16* xt = X + (int64_t)t * kHC * D;
  const __nv_bfloat16* yt = y + (int64_t)t * ldy;
  float ss = 0.f;
  for (int v = threadIdx.x * 8; v < D; v += kThreads * 8) {
    float yv[8], xr[kHC][8];
    load8(yt + v, yv);
#pragma unroll
    for (int r = 0; r < kHC; ++r) load8(xt + (int64_t)r * D + v, xr[r]);
#pragma unroll
    for (int c = 0; c < kHC; ++c) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float a = cf[kHC * kHC + c] * yv[i];
#pragma unroll
        for (int r = 0; r < kHC; ++r) a = fmaf(cf[r * kHC + c], xr[r][i], a);
        o[i] = bf16_round(a);
        ss = fmaf(o[i], o[i], ss);
      }
      store8_bf16(xt + (int64_t)c * D + v, o);
    }
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) sumsq[t] = ss;
}

// ---------------------------------------------------------------------------
// Tensor-parallel all-reduce fused with hc_post (the sublayer boundary of the
// V4 family under TP): every rank pushed its partial sublayer output y into
// recv[p][rank] of every rank (P2P stores by ar_push or the o-projection's
// GEMM epilogue, one arrival per source); each CTA waits (bounded) for the
// arrivals, sums the world partials in rank order (fp32, rounded to bf16 like
// the unfused all-reduce's output) and applies hc_post to its row.  The last
// CTA (ticket) zeroes the parity's counters and advances the epoch, as the
// push reduction does.  Replaces NCCL all-reduce + hc_post (two launches and
// a global round trip of y); fin.py:1-20 fuses the same boundary on TP2.
__global__ void __launch_bounds__(kThreads) ar_hc_post_kernel(int D, ArPeers peers, uint32_t* epoch,
                                                              uint32_t* ticket, uint32_t expected,
                                                              __nv_bfloat16* X, const float* post, const float* comb,
                                                              float* sumsq, uint32_t* err) {
  __shared__ float red[32];
  __shared__ float cf[kHC * kHC + kHC];
  __shared__ int ok_s;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int p = (*epoch) & 1;
  uint8_t* mine = peers.base[peers.rank];
  const bool ok = comm::wait_arrivals(mine, p, peers.world, expected, err, &ok_s);
  const int t = blockIdx.x;
  if (threadIdx.x < kHC * kHC) cf[threadIdx.x] = __ldcg(comb + (int64_t)t * kHC * kHC + threadIdx.x);
  if (threadIdx.x < kHC) cf[kHC * kHC + threadIdx.x] = __ldcg(post + (int64_t)t * kHC + threadIdx.x);
  __syncthreads();
  float ss = 0.f;
  if (ok) {
    __nv_bfloat16* xt = X + (int64_t)t * kHC * D;
    const __nv_bfloat16* y0 = comm::recv_slot(mine, p, 0, peers.world, peers.max_t, D) + (int64_t)t * D;
    const int64_t sstride = (int64_t)peers.max_t * D;
    for (int v = threadIdx.x * 8; v < D; v += kThreads * 8) {
      float yv[8], xr[kHC][8];
#pragma unroll
      for (int i = 0; i < 8; ++i) yv[i] = 0.f;
      for (int src = 0; src < peers.world; ++src) {
        const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(y0 + src * sstride + v));
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          yv[2 * i] += f.x;
          yv[2 * i + 1] += f.y;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) yv[i] = bf16_round(yv[i]);
#pragma unroll
      for (int r = 0; r < kHC; ++r) load8(xt + (int64_t)r * D + v, xr[r]);
#pragma unroll
      for (int c = 0; c < kHC; ++c) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float a = cf[kHC * kHC + c] * yv[i];
#pragma unroll
          for (int r = 0; r < kHC; ++r) a = fmaf(cf[r * kHC + c], xr[r][i], a);
          o[i] = bf16_round(a);
          ss = fmaf(o[i], o[i], ss);
        }
        store8_bf16(xt + (int64_t)c * D + v, o);
      }
    }
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) sumsq[t] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t k = atomicAdd(ticket, 1u);
    if (k == gridDim.x - 1) {
      uint32_t* cnt = comm::counters(mine, p);
      for (int src = 0; src < peers.world; ++src) atomicExch(cnt + src, 0u);
      *ticket = 0u;
      __threadfence();
      atomicAdd(epoch, 1u);
    }
  }
}

// ---------------------------------------------------------------------------
// Compressed sparse attention: the compressor.
//   gate_store     g[t] (the compressor's gate logit, a column of the qkv
//                  GEMM output) -> gate[slot of row t].
//   compress       one CTA per token row; rows whose position p completes a
//                  block (p + 1 = 0 mod r) write block j = p / r: weights
//                  softmax_k(gate[slot_k] + bias[k]) over its r positions, the
//                  compressed latent row sum_k w_k kv[slot_k] (e4m3, the
//                  cache's scale) and the compressed indexer key sum_k w_k
//                  ik[slot_k] (e4m3 with its own scale amax / 448).  A block
//                  lives in one page: its row is page * (page / r) + offset.
// Separate launches: a block's other positions may be rows of the same step.
__global__ void gate_store_kernel(const __nv_bfloat16* g, int64_t ld, int gf32, const int64_t* slots, int T,
                                  float* gate) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float v = gf32 ? reinterpret_cast<const float*>(g)[(int64_t)t * ld] : __bfloat162float(g[(int64_t)t * ld]);
  gate[slots[t]] = v;
}

__device__ __forceinline__ float e4m3_to_f(uint8_t b) {
  __nv_fp8_e4m3 f;
  f.__x = b;
  return float(f);
}

__global__ void __launch_bounds__(128) compress_kernel(const int* pos, const int* q_seq, const int* bt, int bt_stride,
                                                       int page, int r, const float* gate, const float* bias,
                                                       const uint8_t* kv, int kvd, float kv_scale,
                                                       const uint8_t* ik, const float* iks, int ikd, uint8_t* ckv,
                                                       uint8_t* cik, float* cis) {
  __shared__ float w_s[8];
  __shared__ int64_t slot_s[8];
  __shared__ float red[4];
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int t = blockIdx.x;
  const int p = pos[t];
  if ((p + 1) % r) return;                       // uniform per CTA
  const int b = q_seq[t];
  const int p0 = p + 1 - r;
  if (threadIdx.x < r) {
    const int q = p0 + threadIdx.x;
    slot_s[threadIdx.x] = (int64_t)__ldcg(bt + (int64_t)b * bt_stride + q / page) * page + q % page;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    float g[8];
    for (int k = 0; k < r; ++k) {
      g[k] = __ldcg(gate + slot_s[k]) + bias[k];
      m = fmaxf(m, g[k]);
    }
    float sum = 0.f;
    for (int k = 0; k < r; ++k) {
      g[k] = __expf(g[k] - m);
      sum += g[k];
    }
    for (int k = 0; k < r; ++k) w_s[k] = g[k] / sum;
  }
  __syncthreads();
  const int cpage = page / r;
  const int64_t crow = (int64_t)__ldcg(bt + (int64_t)b * bt_stride + p0 / page) * cpage + (p0 % page) / r;
  // compressed latent row: 8 bytes per thread (the weighted mean keeps the cache's scale)
  for (int c = threadIdx.x * 8; c < kvd; c += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int k = 0; k < r; ++k) {
      const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(kv + slot_s[k] * kvd + c));
      const uint8_t* bb = reinterpret_cast<const uint8_t*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(w_s[k], e4m3_to_f(bb[i]), acc[i]);
    }
    uint2 outv;
    uint16_t* o16 = reinterpret_cast<uint16_t*>(&outv);
#pragma unroll
    for (int i = 0; i < 4; ++i) o16[i] = f2_to_e4m3x2(acc[2 * i], acc[2 * i + 1]);
    *reinterpret_cast<uint2*>(ckv + crow * kvd + c) = outv;
  }
  // compressed indexer key: 8 values per thread, one e4m3 scale per row
  const int c = threadIdx.x * 8;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  float amax = 0.f;
  if (c < ikd) {
    for (int k = 0; k < r; ++k) {
      const float sk = __ldcg(iks + slot_s[k]) * w_s[k];
      const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(ik + slot_s[k] * ikd + c));
      const uint8_t* bb = reinterpret_cast<const uint8_t*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(sk, e4m3_to_f(bb[i]), acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(acc[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / sc;
  if (c < ikd) {
    uint2 outv;
    uint16_t* o16 = reinterpret_cast<uint16_t*>(&outv);
#pragma unroll
    for (int i = 0; i < 4; ++i) o16[i] = f2_to_e4m3x2(acc[2 * i] * inv, acc[2 * i + 1] * inv);
    *reinterpret_cast<uint2*>(cik + crow * ikd + c) = outv;
  }
  if (threadIdx.x == 0) cis[crow] = sc;
}

// ---------------------------------------------------------------------------
// Coefficients of one row from its raw mixes (mix(j) = X_flat . fn[j]), run
// by the 32 lanes of one warp: sigmoid pre -> pre_s[4]; mode 0 also
// 2*sigmoid post -> post_row[4] and the row-softmax + Sinkhorn comb on 16
// lanes (mirrored on lanes 16-31) -> comb_row[16] (written when the row
// pointers are non-null).
template <class Mix>
__device__ __forceinline__ void hc_coeffs_warp(Mix mix, float rs, const float* scale, const float* base, int mode,
                                               int iters, float eps, float* pre_s, float* post_row,
                                               float* comb_row) {
  const int ln = threadIdx.x & 31, l = threadIdx.x & 15;
  if (l < kHC) {
    const float pre = sigmoidf(scale[0] * rs * mix(l) + base[l]) + eps;
    if (ln < kHC) pre_s[l] = pre;
    if (mode == 0 && ln < kHC && post_row)
      post_row[l] = 2.f * sigmoidf(scale[1] * rs * mix(kHC + l) + base[kHC + l]);
  }
  if (mode == 0) {
    // lane l: comb[r][c], r = l / 4, c = l % 4; row peers differ in lane
    // bits 0-1, column peers in bits 2-3
    float m = scale[2] * rs * mix(2 * kHC + l) + base[2 * kHC + l];
    float mx = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    m = expf(m - mx);
    float s = m + __shfl_xor_sync(0xffffffffu, m, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    m = m / s + eps;
    for (int it = 0; it < iters; ++it) {
      if (it > 0) {
        float rsum = m + __shfl_xor_sync(0xffffffffu, m, 1);
        rsum += __shfl_xor_sync(0xffffffffu, rsum, 2);
        m = m / (rsum + eps);
      }
      float csum = m + __shfl_xor_sync(0xffffffffu, m, 4);
      csum += __shfl_xor_sync(0xffffffffu, csum, 8);
      m = m / (csum + eps);
    }
    if (ln < 16 && comb_row) comb_row[l] = m;
  }
}

// raw: row t holds `parts` partial mix vectors, part p at column p * pstride
// (their sum is X_flat . fn^T).  mode 0: sublayer (pre / post / comb), mode 1:
// head (pre only).  Outputs: post [T, 4], comb [T, 16] (mode 0); h as MXFP8
// (q, sf) and / or bf16 hb / fp32 hf rows [T, D].
__global__ void __launch_bounds__(kThreads) hc_pre_kernel(const float* raw, int ldr, int parts, int pstride,
                                                          const float* sumsq, const float* scale, const float* base,
                                                          int mode, int iters, float eps, float inv_width,
                                                          const __nv_bfloat16* X, int D, const float* norm_w,
                                                          float norm_eps, float* post_out, float* comb_out,
                                                          uint8_t* q, uint8_t* sf, __nv_bfloat16* hb, float* hf) {
  __shared__ float red[32];
  __shared__ float pre_s[kHC];
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int t = blockIdx.x;
  if (threadIdx.x < 32) {
    const float rs = 1.f / sqrtf(__ldcg(sumsq + t) * inv_width + eps);
    auto mix = [&](int j) {
      float a = 0.f;
      for (int p = 0; p < parts; ++p) a += __ldcg(raw + (int64_t)t * ldr + p * pstride + j);
      return a;
    };
    hc_coeffs_warp(mix, rs, scale, base, mode, iters, eps, pre_s, mode == 0 ? post_out + (int64_t)t * kHC : nullptr,
                   mode == 0 ? comb_out + (int64_t)t * kHC * kHC : nullptr);
  }
  __syncthreads();
  float p[kHC];
#pragma unroll
  for (int c = 0; c < kHC; ++c) p[c] = pre_s[c];
  const __nv_bfloat16* xt = X + (int64_t)t * kHC * D;
  float h[kMaxIt][8];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < kMaxIt; ++it) {
    const int v = (threadIdx.x + it * kThreads) * 8;
    if (v < D) {
      float xr[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[it][i] = 0.f;
#pragma unroll
      for (int c = 0; c < kHC; ++c) {
        load8(xt + (int64_t)c * D + v, xr);
#pragma unroll
        for (int i = 0; i < 8; ++i) h[it][i] = fmaf(p[c], xr[i], h[it][i]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(h[it][i], h[it][i], ss);
    }
  }
  ss = block_sum(ss, red);
  const float rstd = 1.f / sqrtf(ss / D + norm_eps);
  const int kb = D / 32;
#pragma unroll
  for (int it = 0; it < kMaxIt; ++it) {
    const int v = (threadIdx.x + it * kThreads) * 8;
    if (v >= D) continue;      // D % 32 == 0: a 32-block's 4 lanes agree
    float y[8], w[8];
    load8(norm_w + v, w);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = h[it][i] * rstd * w[i];
    if (hb) store8_bf16(hb + (int64_t)t * D + v, y);
    if (hf) store8_f32(hf + (int64_t)t * D + v, y);
    if (q) quant8(y, q + (int64_t)t * D + v, sf, t, v, kb, true);
  }
}

// ---------------------------------------------------------------------------
// The whole hyper-connection boundary in one kernel: hc_post of the previous
// sublayer's output (when y is given), the raw mixes X_flat . fn^T in fp32 on
// the CUDA cores, the coefficients, and the next sublayer's input
// RMSNorm(sum_c pre_c X_c) * w.  A CTA owns kBRows rows and D / C columns of
// every stream; the C CTAs of a thread-block cluster cover a row group's
// columns and sum their partial mixes and sums of squares in rank order
// through distributed shared memory, so every CTA derives the same
// coefficients.  Each CTA reads its slice of fn (M x 4 x D/C fp32) once for
// all kBRows rows: a warp takes three mix rows m, its lanes stride the slice
// by float4, and every fn load feeds kBRows dot products against the rows
// staged in shared memory.  Decode-sized batches; long prefill chunks keep
// the tcgen05 stats GEMM.  Replaces hc_post + memset + stats GEMM + hc_pre
// (four launches).  Sums run in fixed thread / warp / rank order.
constexpr int kBThreads = 256;
constexpr int kBWarps = kBThreads / 32;
constexpr int kBRows = 8;          // rows per CTA (one warp each for the coefficients)
constexpr int kBMaxM = 24;
constexpr int kBMPerWarp = kBMaxM / kBWarps;   // 3
static_assert(kBRows == kBWarps, "one warp per row for the coefficients");

__global__ void __launch_bounds__(kBThreads) hc_boundary_kernel(
    __nv_bfloat16* X, int T, int D, int C, const __nv_bfloat16* y, int64_t ldy, const float* post_in,
    const float* comb_in, const float* fn, int M, const float* scale, const float* base, int mode, int iters,
    float eps, float inv_width, const float* norm_w, float norm_eps, float* post_out, float* comb_out, uint8_t* q,
    uint8_t* sf, __nv_bfloat16* hb, float* hf) {
  extern __shared__ __align__(16) float xs[];       // [kBRows][kHC][Dq] updated streams of this CTA's columns
  __shared__ float part[kBRows][kBMaxM + 2];        // partial mixes [M], sum sq of X, sum sq of h
  __shared__ float tot[kBRows][kBMaxM + 1];
  __shared__ float wsum[kBWarps][kBRows];
  __shared__ float cf[kBRows][kHC * kHC + kHC];
  __shared__ float pre_s[kBRows][kHC];
  __shared__ float rstd_s[kBRows];
  const int rank = int(cluster_ctarank());
  const int Dq = D / C, d0 = rank * Dq;
  const int t0 = blockIdx.y * kBRows;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vpr = Dq / 8;                          // 8-column vectors per row and stream
  const int items = kBRows * vpr;
  pdl_wait();
  if (tid == 0) pdl_launch_dependents();
  if (y) {
    for (int i = tid; i < kBRows * (kHC * kHC + kHC); i += kBThreads) {
      const int r = i / (kHC * kHC + kHC), j = i % (kHC * kHC + kHC), t = t0 + r;
      cf[r][j] = t < T ? (j < kHC * kHC ? __ldcg(comb_in + (int64_t)t * kHC * kHC + j)
                                        : __ldcg(post_in + (int64_t)t * kHC + j - kHC * kHC))
                       : 0.f;
    }
    __syncthreads();
  }
  // 1. hc_post on this CTA's columns (in place); fp32 copies in shared memory
  float ssx[kBRows];
#pragma unroll
  for (int r = 0; r < kBRows; ++r) ssx[r] = 0.f;
  for (int i = tid; i < items; i += kBThreads) {
    const int r = i / vpr, v = (i % vpr) * 8, t = t0 + r;
    float xr[kHC][8];
    if (t < T) {
      __nv_bfloat16* xt = X + (int64_t)t * kHC * D + d0;
#pragma unroll
      for (int c = 0; c < kHC; ++c) load8(xt + (int64_t)c * D + v, xr[c]);
      if (y) {
        float yv[8], o[kHC][8];
        load8(y + (int64_t)t * ldy + d0 + v, yv);
#pragma unroll
        for (int c = 0; c < kHC; ++c) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float a = cf[r][kHC * kHC + c] * yv[e];
#pragma unroll
            for (int rr = 0; rr < kHC; ++rr) a = fmaf(cf[r][rr * kHC + c], xr[rr][e], a);
            o[c][e] = bf16_round(a);
          }
        }
#pragma unroll
        for (int c = 0; c < kHC; ++c) {
          store8_bf16(xt + (int64_t)c * D + v, o[c]);
#pragma unroll
          for (int e = 0; e < 8; ++e) xr[c][e] = o[c][e];
        }
      }
    } else {
#pragma unroll
      for (int c = 0; c < kHC; ++c)
#pragma unroll
        for (int e = 0; e < 8; ++e) xr[c][e] = 0.f;
    }
    float s2 = 0.f;
#pragma unroll
    for (int c = 0; c < kHC; ++c) {
      float* dst = xs + ((int64_t)r * kHC + c) * Dq + v;
      *reinterpret_cast<float4*>(dst) = make_float4(xr[c][0], xr[c][1], xr[c][2], xr[c][3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(xr[c][4], xr[c][5], xr[c][6], xr[c][7]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s2 = fmaf(xr[c][e], xr[c][e], s2);
    }
#pragma unroll
    for (int rr = 0; rr < kBRows; ++rr) ssx[rr] += (rr == r) ? s2 : 0.f;
  }
#pragma unroll
  for (int r = 0; r < kBRows; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssx[r] += __shfl_xor_sync(0xffffffffu, ssx[r], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kBRows; ++r) wsum[warp][r] = ssx[r];
  }
  __syncthreads();
  if (tid < kBRows) {
    float a = 0.f;
    for (int w = 0; w < kBWarps; ++w) a += wsum[w][tid];
    part[tid][kBMaxM] = a;
  }
  // 2. partial mixes: warp w takes m = w, w + 8, w + 16; lanes stride the
  // CTA's 4 x Dq columns by float4; each fn load serves all kBRows rows
  {
    float acc[kBMPerWarp][kBRows];
#pragma unroll
    for (int j = 0; j < kBMPerWarp; ++j)
#pragma unroll
      for (int r = 0; r < kBRows; ++r) acc[j][r] = 0.f;
    const int64_t K = (int64_t)kHC * D;
    const int ks = kHC * Dq;
    // unrolled: the fn loads of several column steps are in flight together
#pragma unroll 5
    for (int k = lane * 4; k < ks; k += 128) {
      const int c = k / Dq, d = k % Dq;            // Dq % 4 == 0: a float4 never straddles streams
      const float* f = fn + (int64_t)c * D + d0 + d;
      float4 fw[kBMPerWarp];
#pragma unroll
      for (int j = 0; j < kBMPerWarp; ++j) {
        const int m = warp + j * kBWarps;
        fw[j] = m < M ? *reinterpret_cast<const float4*>(f + m * K) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int r = 0; r < kBRows; ++r) {
        const float4 xv = *reinterpret_cast<const float4*>(xs + ((int64_t)r * kHC + c) * Dq + d);
#pragma unroll
        for (int j = 0; j < kBMPerWarp; ++j)
          acc[j][r] = fmaf(xv.x, fw[j].x, fmaf(xv.y, fw[j].y, fmaf(xv.z, fw[j].z, fmaf(xv.w, fw[j].w, acc[j][r]))));
      }
    }
#pragma unroll
    for (int j = 0; j < kBMPerWarp; ++j) {
#pragma unroll
      for (int r = 0; r < kBRows; ++r) {
        float a = acc[j][r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        const int m = warp + j * kBWarps;
        if (lane == 0 && m < M) part[r][m] = a;
      }
    }
  }
  // 3. the cluster's partials summed in rank order (the same in every CTA)
  cluster_sync();
  for (int i = tid; i < kBRows * (kBMaxM + 1); i += kBThreads) {
    const int r = i / (kBMaxM + 1), j = i % (kBMaxM + 1);
    if (j < M || j == kBMaxM) {
      const uint32_t a = smem_u32(&part[r][j]);
      float sum = 0.f;
      for (int rr = 0; rr < C; ++rr) sum += ld_dsmem_f32(mapa_shared(a, rr));
      tot[r][j] = sum;
    }
  }
  __syncthreads();
  {
    const int r = warp, t = t0 + r;               // one warp per row (kBRows == kBWarps)
    if (t < T) {
      const float rs = 1.f / sqrtf(tot[r][kBMaxM] * inv_width + eps);
      const bool w0 = rank == 0 && mode == 0;
      hc_coeffs_warp([&](int j) { return tot[r][j]; }, rs, scale, base, mode, iters, eps, pre_s[r],
                     w0 ? post_out + (int64_t)t * kHC : nullptr, w0 ? comb_out + (int64_t)t * kHC * kHC : nullptr);
    } else if (lane < kHC) {
      pre_s[r][lane] = 0.f;
    }
  }
  __syncthreads();
  // 4. h = sum_c pre_c X_c on this CTA's columns; per-row sums of squares over the cluster
  float ssh[kBRows];
#pragma unroll
  for (int r = 0; r < kBRows; ++r) ssh[r] = 0.f;
  for (int i = tid; i < items; i += kBThreads) {
    const int r = i / vpr, v = (i % vpr) * 8;
    float s2 = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float h = 0.f;
#pragma unroll
      for (int c = 0; c < kHC; ++c) h = fmaf(pre_s[r][c], xs[((int64_t)r * kHC + c) * Dq + v + e], h);
      s2 = fmaf(h, h, s2);
    }
#pragma unroll
    for (int rr = 0; rr < kBRows; ++rr) ssh[rr] += (rr == r) ? s2 : 0.f;
  }
#pragma unroll
  for (int r = 0; r < kBRows; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssh[r] += __shfl_xor_sync(0xffffffffu, ssh[r], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kBRows; ++r) wsum[warp][r] = ssh[r];
  }
  __syncthreads();
  if (tid < kBRows) {
    float a = 0.f;
    for (int w = 0; w < kBWarps; ++w) a += wsum[w][tid];
    part[tid][kBMaxM + 1] = a;
  }
  cluster_sync();
  if (tid < kBRows) {
    const uint32_t a = smem_u32(&part[tid][kBMaxM + 1]);
    float sum = 0.f;
    for (int rr = 0; rr < C; ++rr) sum += ld_dsmem_f32(mapa_shared(a, rr));
    rstd_s[tid] = 1.f / sqrtf(sum / D + norm_eps);
  }
  // the last reads of other CTAs' shared memory are done after this barrier
  cluster_sync();
  // 5. RMSNorm * w -> bf16 / fp32 / MXFP8.  A uniform trip count: quant8's
  // 4-lane amax exchange needs the whole warp; vpr % 4 == 0 keeps a 32-column
  // block's four lanes on one row.
  const int kb = D / 32;
  const int nit = (items + kBThreads - 1) / kBThreads;
  for (int it = 0; it < nit; ++it) {
    const int i = it * kBThreads + tid;
    const int r = i / vpr, v = (i % vpr) * 8, t = t0 + r;
    const bool ok = i < items && t < T;
    float yv[8];
    if (ok) {
      float w8[8];
      load8(norm_w + d0 + v, w8);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float h = 0.f;
#pragma unroll
        for (int c = 0; c < kHC; ++c) h = fmaf(pre_s[r][c], xs[((int64_t)r * kHC + c) * Dq + v + e], h);
        yv[e] = h * rstd_s[r] * w8[e];
      }
      if (hb) store8_bf16(hb + (int64_t)t * D + d0 + v, yv);
      if (hf) store8_f32(hf + (int64_t)t * D + d0 + v, yv);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) yv[e] = 0.f;
    }
    if (q) quant8(yv, q + (int64_t)(ok ? t : 0) * D + d0 + v, sf, ok ? t : 0, d0 + v, kb, ok);
  }
}

__global__ void __launch_bounds__(kThreads) hc_mean_kernel(const __nv_bfloat16* X, int D, __nv_bfloat16* out) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int t = blockIdx.x;
  for (int v = threadIdx.x * 8; v < D; v += kThreads * 8) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, x[8];
#pragma unroll
    for (int c = 0; c < kHC; ++c) {
      load8(X + ((int64_t)t * kHC + c) * D + v, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] += x[i];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] *= 1.f / kHC;
    store8_bf16(out + (int64_t)t * D + v, a);
  }
}

// ---------------------------------------------------------------------------
// Engram
constexpr int kEngramDim = 256;
constexpr int kMaxNgram = 8;

__global__ void engram_hash_kernel(const int* ids, const int* pos, const int* q_seq, const int* block_table,
                                   int bt_stride, const int64_t* out_slots, int page_size, int* tok_cache, int T,
                                   int heads, int per_head, int max_n, const unsigned long long* mults, int* out) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const int p = __ldcg(pos + t), b = __ldcg(q_seq + t);
  long long ctx[kMaxNgram];
#pragma unroll
  for (int i = 0; i < kMaxNgram; ++i) {
    long long tok = -1;
    const int pp = p - i;
    if (i < max_n && pp >= 0) {
      if (i == 0) {
        tok = __ldcg(ids + t);
      } else if (t - i >= 0 && __ldcg(q_seq + t - i) == b && __ldcg(pos + t - i) == pp) {
        tok = __ldcg(ids + t - i);          // predecessor in this batch
      } else {
        const int page = __ldcg(block_table + (int64_t)b * bt_stride + pp / page_size);
        tok = __ldcg(tok_cache + (int64_t)page * page_size + pp % page_size);
      }
    }
    ctx[i] = tok;
  }
  const int span = max_n >= 2 ? max_n - 1 : 1;
  for (int j = 0; j < heads; ++j) {
    const int n = max_n >= 2 ? 2 + j % span : 1;
    const unsigned long long m = mults[j];
    unsigned long long h = 0ull;
    for (int i = 0; i < n; ++i) {
      const unsigned long long v = ctx[i] >= 0 ? (unsigned long long)(ctx[i] + 1) : 0ull;
      h = (h ^ v) * m;
    }
    out[(int64_t)t * heads + j] = j * per_head + int((h >> 32) % (unsigned long long)per_head);
  }
  // this token's own slot (its successors in later steps read it)
  tok_cache[__ldcg(out_slots + t)] = __ldcg(ids + t);
}

__global__ void engram_gather_kernel(const uint8_t* table, const uint8_t* scale, const int* ids, int n, int row_lo,
                                     int row_hi, __nv_bfloat16* out) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= n) return;
  const int id = __ldcg(ids + w);
  const bool own = id >= row_lo && id < row_hi;
  uint2 raw = make_uint2(0u, 0u);
  uint32_t e = 0u;
  if (own) {
    const int64_t r = id - row_lo;
    raw = *reinterpret_cast<const uint2*>(table + r * kEngramDim + lane * 8);
    e = scale[r * (kEngramDim / 32) + lane / 4];
  }
  // UE8M0: 2^(e - 127) built from the exponent bits (e = 0: 2^-127)
  const float s = e == 0u ? __uint_as_float(0x00400000u) : __uint_as_float(e << 23);
  const uint8_t* by = reinterpret_cast<const uint8_t*>(&raw);
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    __nv_fp8_e4m3 f;
    f.__x = by[i];
    v[i] = own ? float(f) * s : 0.f;
  }
  store8_bf16(out + (int64_t)w * kEngramDim + lane * 8, v);
}

__global__ void __launch_bounds__(kThreads) engram_gate_kernel(__nv_bfloat16* X, int D, const void* kv, int kv_f32,
                                                               int64_t ldkv, const float* q_w, const float* k_w,
                                                               float eps, float clampv, float* sumsq) {
  __shared__ float red[32];
  __shared__ float gate[kHC];
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int t = blockIdx.x;
  __nv_bfloat16* xt = X + (int64_t)t * kHC * D;
  float ssk = 0.f, ssx[kHC], dot[kHC];
#pragma unroll
  for (int c = 0; c < kHC; ++c) ssx[c] = dot[c] = 0.f;
  for (int v = threadIdx.x * 8; v < D; v += kThreads * 8) {
    float k[8], qw[8], kw[8], x[8];
    if (kv_f32) load8(reinterpret_cast<const float*>(kv) + t * ldkv + v, k);
    else load8(reinterpret_cast<const __nv_bfloat16*>(kv) + t * ldkv + v, k);
    load8(q_w + v, qw);
    load8(k_w + v, kw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ssk = fmaf(k[i], k[i], ssk);
      k[i] *= qw[i] * kw[i];
    }
#pragma unroll
    for (int c = 0; c < kHC; ++c) {
      load8(xt + (int64_t)c * D + v, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ssx[c] = fmaf(x[i], x[i], ssx[c]);
        dot[c] = fmaf(x[i], k[i], dot[c]);
      }
    }
  }
  ssk = block_sum(ssk, red);
#pragma unroll
  for (int c = 0; c < kHC; ++c) {
    ssx[c] = block_sum(ssx[c], red);
    dot[c] = block_sum(dot[c], red);
  }
  if (threadIdx.x < kHC) {
    const int c = threadIdx.x;
    const float rk = 1.f / sqrtf(ssk / D + eps), rx = 1.f / sqrtf(ssx[c] / D + eps);
    const float z = fminf(fmaxf(dot[c] * rk * rx / sqrtf(float(D)), -clampv), clampv);
    gate[c] = sigmoidf(z);
  }
  __syncthreads();
  float ss = 0.f;
  for (int v = threadIdx.x * 8; v < D; v += kThreads * 8) {
    float val[8], x[8];
    if (kv_f32) load8(reinterpret_cast<const float*>(kv) + t * ldkv + D + v, val);
    else load8(reinterpret_cast<const __nv_bfloat16*>(kv) + t * ldkv + D + v, val);
#pragma unroll
    for (int c = 0; c < kHC; ++c) {
      load8(xt + (int64_t)c * D + v, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x[i] = bf16_round(fmaf(gate[c], val[i], x[i]));
        ss = fmaf(x[i], x[i], ss);
      }
      store8_bf16(xt + (int64_t)c * D + v, x);
    }
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) sumsq[t] = ss;
}

// first layer's streams: every stream = the token's embedding row
__global__ void __launch_bounds__(kThreads) hc_embed_kernel(const __nv_bfloat16* embed, const int* ids, int D,
                                                            __nv_bfloat16* X, float* sumsq) {
  __shared__ float red[32];
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int t = blockIdx.x;
  const __nv_bfloat16* e = embed + (int64_t)__ldcg(ids + t) * D;
  float ss = 0.f;
  for (int v = threadIdx.x * 8; v < D; v += kThreads * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(e + v);
    float x[8];
    load8(e + v, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
    for (int c = 0; c < kHC; ++c) *reinterpret_cast<uint4*>(X + ((int64_t)t * kHC + c) * D + v) = raw;
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) sumsq[t] = ss * kHC;
}

// ---------------------------------------------------------------------------
// MQA key / query preparation and the attention output fix-up
constexpr int kRow = 576;    // cache / query row bytes of the latent attention kernel

__global__ void __launch_bounds__(128) kv_store_v4_kernel(const void* kv, int f32, int64_t ld, int L, int rd,
                                                          const float* w, float eps, const int* pos,
                                                          const float* table, const int64_t* slots, uint8_t* cache,
                                                          float inv_scale) {
  __shared__ float red[32];
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int t = blockIdx.x;
  const int per = L / 128;     // 4 consecutive elements per thread at L = 512 (pairs stay in a thread)
  float v[8];
  float ss = 0.f;
  for (int i = 0; i < per; ++i) {
    const int j = threadIdx.x * per + i;
    v[i] = f32 ? reinterpret_cast<const float*>(kv)[t * ld + j]
               : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(kv)[t * ld + j]);
    ss = fmaf(v[i], v[i], ss);
  }
  ss = ew::block_sum(ss, red);
  const float rstd = 1.f / sqrtf(ss / L + eps);
  const int p = __ldcg(pos + t);
  const int tail = L - rd;
  for (int i = 0; i < per; ++i) v[i] *= rstd * w[threadIdx.x * per + i];
  for (int i = 0; i < per; i += 2) {
    const int j = threadIdx.x * per + i;
    if (j >= tail) {
      const int pi = (j - tail) >> 1;
      const float c = table[(int64_t)p * rd + pi], s = table[(int64_t)p * rd + rd / 2 + pi];
      const float x0 = v[i], x1 = v[i + 1];
      v[i] = x0 * c - x1 * s;
      v[i + 1] = x0 * s + x1 * c;
    }
  }
  uint8_t* row = cache + __ldcg(slots + t) * kRow;
  for (int i = 0; i < per; i += 2) {
    const uint16_t b2 = f2_to_e4m3x2(v[i] * inv_scale, v[i + 1] * inv_scale);
    *reinterpret_cast<uint16_t*>(row + threadIdx.x * per + i) = b2;
  }
  for (int j = L + threadIdx.x; j < kRow; j += 128) row[j] = 0;
}

// one warp per (token, head); 16 consecutive elements per lane (L = 512)
// q8 / qs hold Hq >= H heads per token (extra heads stay as the caller set
// them: zero queries that pad H to the attention kernel's head block)
__global__ void mqa_q_prep_kernel(const __nv_bfloat16* q, int64_t qt, int64_t qh, int T, int H, int Hq, int rd,
                                  const int* pos, const float* table, uint8_t* q8, float* qs) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= T * H) return;
  const int t = w / H, h = w - t * H;
  constexpr int L = 512, E = 16;
  const __nv_bfloat16* src = q + t * qt + h * qh + lane * E;
  float v[E];
  ew::load8(src, *reinterpret_cast<float(*)[8]>(v));
  ew::load8(src + 8, *reinterpret_cast<float(*)[8]>(v + 8));
  const int tail = L - rd, p = __ldcg(pos + t);
  if (lane * E >= tail) {
#pragma unroll
    for (int i = 0; i < E; i += 2) {
      const int pi = (lane * E + i - tail) >> 1;
      const float c = table[(int64_t)p * rd + pi], s = table[(int64_t)p * rd + rd / 2 + pi];
      const float x0 = v[i], x1 = v[i + 1];
      v[i] = x0 * c - x1 * s;
      v[i + 1] = x0 * s + x1 * c;
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / sc;
  const int64_t wq = (int64_t)t * Hq + h;
  uint8_t* dst = q8 + wq * kRow;
  uint32_t packed[E / 4];
#pragma unroll
  for (int i = 0; i < E; i += 4) {
    const uint32_t lo = f2_to_e4m3x2(v[i] * inv, v[i + 1] * inv), hi = f2_to_e4m3x2(v[i + 2] * inv, v[i + 3] * inv);
    packed[i / 4] = lo | (hi << 16);
  }
  *reinterpret_cast<uint4*>(dst + lane * E) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  reinterpret_cast<uint16_t*>(dst + L)[lane] = 0;      // no separate rope key: zero query part
  if (lane == 0) qs[wq] = sc;
}

__global__ void attn_fixup_kernel(__nv_bfloat16* o, int T, int H, const float* lse, const float* sink, int rd,
                                  const int* pos, const float* table) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= T * H) return;
  const int t = w / H, h = w - t * H;
  constexpr int L = 512, E = 16;
  float f = 1.f;
  if (sink) {
    const float l = __ldcg(lse + w);
    f = l == -INFINITY ? 0.f : 1.f / (1.f + exp2f(sink[h] * kLog2e - l));
  }
  __nv_bfloat16* row = o + (int64_t)w * L + lane * E;
  float v[E];
  ew::load8(row, *reinterpret_cast<float(*)[8]>(v));
  ew::load8(row + 8, *reinterpret_cast<float(*)[8]>(v + 8));
#pragma unroll
  for (int i = 0; i < E; ++i) v[i] *= f;
  const int tail = L - rd, p = __ldcg(pos + t);
  if (lane * E >= tail) {
#pragma unroll
    for (int i = 0; i < E; i += 2) {
      const int pi = (lane * E + i - tail) >> 1;
      const float c = table[(int64_t)p * rd + pi], s = table[(int64_t)p * rd + rd / 2 + pi];
      const float x0 = v[i], x1 = v[i + 1];
      v[i] = x0 * c + x1 * s;           // rotation by -angle
      v[i + 1] = -x0 * s + x1 * c;
    }
  }
  ew::store8_bf16(row, *reinterpret_cast<float(*)[8]>(v));
  ew::store8_bf16(row + 8, *reinterpret_cast<float(*)[8]>(v + 8));
}

// ---------------------------------------------------------------------------
constexpr int kPruneMaxK = 16;

__global__ void e5_prune_kernel(int* ids, float* w, int T, int K, int E, float budget, int max_count) {
  extern __shared__ int sh[];
  int* cnt = sh;
  int* keep = sh + E;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = keep[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < T * K; i += blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    int id[kPruneMaxK], ord[kPruneMaxK];
    float wt[kPruneMaxK];
    float mass = 0.f;
    for (int k = 0; k < K; ++k) {
      id[k] = ids[t * K + k];
      wt[k] = w[t * K + k];
      if (id[k] >= 0) mass += wt[k];
      ord[k] = k;
    }
    // (weight, slot) ascending: insertion sort, stable on equal weights
    for (int a = 1; a < K; ++a) {
      const int x = ord[a];
      int b = a - 1;
      while (b >= 0 && wt[ord[b]] > wt[x]) {
        ord[b + 1] = ord[b];
        --b;
      }
      ord[b + 1] = x;
    }
    float run = 0.f;
    const float lim = budget * mass;
    for (int a = 0; a < K; ++a) {
      const int k = ord[a];
      const int e = id[k];
      if (e < 0 || e >= E) continue;
      bool cand = false;
      if (cnt[e] <= max_count) {
        run += wt[k];
        cand = run <= lim;
      }
      if (!cand) keep[e] = 1;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < T * K; i += blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E && !keep[e]) {
      ids[i] = -1;
      w[i] = 0.f;
    }
  }
}

}  // namespace v4
}  // namespace b200

using namespace b200::v4;

int b200_hc_post(void* X, const void* y, int64_t ldy, const float* post, const float* comb, int T, int hc, int D,
                 float* sumsq, cudaStream_t st) {
  if (T <= 0) return 0;
  if (hc != kHC || D % 8 || ldy % 8) return -1;
  b200::launch_pdl(hc_post_kernel, dim3(T), dim3(kThreads), 0, st, reinterpret_cast<__nv_bfloat16*>(X),
                   reinterpret_cast<const __nv_bfloat16*>(y), ldy, post, comb, D, sumsq);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_ar_hc_post(int T, int D, const ArPeers* peers, uint32_t* epoch, uint32_t* ticket, int expected, void* X,
                    const float* post, const float* comb, float* sumsq, uint32_t* err, cudaStream_t st) {
  if (T <= 0) return 0;
  if (D % 8 || T > peers->max_t || peers->mc || expected <= 0) return -1;
  b200::launch_pdl(b200::v4::ar_hc_post_kernel, dim3(T), dim3(b200::v4::kThreads), 0, st, D, *peers, epoch, ticket,
                   (uint32_t)expected, reinterpret_cast<__nv_bfloat16*>(X), post, comb, sumsq, err);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_compress_store(const void* g, int64_t ld, int gf32, const int64_t* slots, const int* pos, const int* q_seq,
                        const int* bt, int bt_stride, int page, int r, int T, float* gate, const float* bias,
                        const uint8_t* kv, int kvd, float kv_scale, const uint8_t* ik, const float* iks, int ikd,
                        uint8_t* ckv, uint8_t* cik, float* cis, cudaStream_t st) {
  if (T <= 0) return 0;
  if (r < 2 || r > 8 || page % r || kvd % 8 || ikd % 8 || ikd > 128 * 8) return -1;
  b200::launch_pdl(b200::v4::gate_store_kernel, dim3((T + 127) / 128), dim3(128), 0, st,
                   reinterpret_cast<const __nv_bfloat16*>(g), ld, gf32, slots, T, gate);
  b200::launch_pdl(b200::v4::compress_kernel, dim3(T), dim3(128), 0, st, pos, q_seq, bt, bt_stride, page, r,
                   (const float*)gate, bias, kv, kvd, kv_scale, ik, iks, ikd, ckv, cik, cis);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_hc_pre(const float* raw, int ldr, int parts, int pstride, const float* sumsq, const float* scale,
                const float* base, int mode, int iters, float eps, float inv_width, const void* X, int T, int hc,
                int D, const float* norm_w, float norm_eps, float* post, float* comb, uint8_t* q, uint8_t* sf,
                void* hb, float* hf, cudaStream_t st) {
  if (T <= 0) return 0;
  // D % 256: a 32-column block never straddles an active and an idle warp
  if (hc != kHC || D % 256 || D > kThreads * 8 * kMaxIt || (mode == 0 && (!post || !comb))) return -1;
  b200::launch_pdl(hc_pre_kernel, dim3(T), dim3(kThreads), 0, st, raw, ldr, parts, pstride, sumsq, scale, base, mode,
                   iters, eps, inv_width, reinterpret_cast<const __nv_bfloat16*>(X), D, norm_w, norm_eps, post, comb,
                   q, sf, reinterpret_cast<__nv_bfloat16*>(hb), hf);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_hc_boundary(void* X, int T, int hc, int D, const void* y, int64_t ldy, const float* post_in,
                     const float* comb_in, const float* fn, int M, const float* scale, const float* base, int mode,
                     int iters, float eps, float inv_width, const float* norm_w, float norm_eps, float* post,
                     float* comb, uint8_t* q, uint8_t* sf, void* hb, float* hf, cudaStream_t st) {
  using namespace b200::v4;
  if (T <= 0) return 0;
  if (hc != kHC || M > kBMaxM || M < kHC || (mode == 0 && (!post || !comb || M < 2 * kHC + kHC * kHC))) return -1;
  if (y && (!post_in || !comb_in)) return -1;
  // C CTAs per row group: columns per CTA a multiple of 32 (quant blocks on
  // one CTA, whole float4s per stream), the rows' fp32 copies in shared memory
  // (16-CTA clusters, a non-portable size the B200 supports, halve each
  // CTA's slice of fn and of the rows; 8 where the attribute is refused)
  auto kern = hc_boundary_kernel;
  const bool c16 =
      cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
  if (!c16) cudaGetLastError();
  int C = 0;
  for (int c = c16 ? 16 : 8; c >= 1; c >>= 1)
    if (D % (32 * c) == 0 && D / c >= 256 && size_t(kBRows) * kHC * (D / c) * sizeof(float) <= 160 * 1024) {
      C = c;
      break;
    }
  if (C == 0 || (reinterpret_cast<uintptr_t>(fn) & 15)) return -2;
  const int Dq = D / C;
  const size_t smem = size_t(kBRows) * kHC * Dq * sizeof(float);
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, (T + kBRows - 1) / kBRows);
  cfg.blockDim = dim3(kBThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = b200::pdl_enabled() ? 2 : 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<__nv_bfloat16*>(X), T, D, C,
                                             reinterpret_cast<const __nv_bfloat16*>(y), ldy, post_in, comb_in, fn, M,
                                             scale, base, mode, iters, eps, inv_width, norm_w, norm_eps, post, comb, q,
                                             sf, reinterpret_cast<__nv_bfloat16*>(hb), hf);
  return err == cudaSuccess ? 0 : 1000 + int(err);
}

int b200_hc_mean(const void* X, int T, int hc, int D, void* out, cudaStream_t st) {
  if (T <= 0) return 0;
  if (hc != kHC || D % 8) return -1;
  b200::launch_pdl(hc_mean_kernel, dim3(T), dim3(kThreads), 0, st, reinterpret_cast<const __nv_bfloat16*>(X), D,
                   reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_engram_hash(const int* ids, const int* pos, const int* q_seq, const int* block_table, int bt_stride,
                     const int64_t* out_slots, int page_size, int* tok_cache, int T, int heads, int per_head,
                     int max_n, const unsigned long long* mults, int* out, cudaStream_t st) {
  if (T <= 0) return 0;
  if (max_n < 1 || max_n > kMaxNgram || heads <= 0 || per_head <= 0) return -1;
  b200::launch_pdl(engram_hash_kernel, dim3((T + 127) / 128), dim3(128), 0, st, ids, pos, q_seq, block_table,
                   bt_stride, out_slots, page_size, tok_cache, T, heads, per_head, max_n, mults, out);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_engram_gather(const uint8_t* table, const uint8_t* scale, const int* ids, int n, int row_lo, int row_hi,
                       void* out, cudaStream_t st) {
  if (n <= 0) return 0;
  b200::launch_pdl(engram_gather_kernel, dim3((n * 32 + 255) / 256), dim3(256), 0, st, table, scale, ids, n, row_lo,
                   row_hi, reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_engram_gate(void* X, int T, int hc, int D, const void* kv, int kv_f32, int64_t ldkv, const float* q_w,
                     const float* k_w, float eps, float clampv, float* sumsq, cudaStream_t st) {
  if (T <= 0) return 0;
  if (hc != kHC || D % 8 || ldkv % 8 || !sumsq) return -1;
  b200::launch_pdl(engram_gate_kernel, dim3(T), dim3(kThreads), 0, st, reinterpret_cast<__nv_bfloat16*>(X), D, kv,
                   kv_f32, ldkv, q_w, k_w, eps, clampv, sumsq);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_hc_embed(const void* embed, const int* ids, int T, int hc, int D, void* X, float* sumsq, cudaStream_t st) {
  if (T <= 0) return 0;
  if (hc != kHC || D % 8) return -1;
  b200::launch_pdl(hc_embed_kernel, dim3(T), dim3(kThreads), 0, st, reinterpret_cast<const __nv_bfloat16*>(embed),
                   ids, D, reinterpret_cast<__nv_bfloat16*>(X), sumsq);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_kv_store_v4(const void* kv, int f32, int64_t ld, int T, int L, int rd, const float* w, float eps,
                     const int* pos, const float* table, const int64_t* slots, uint8_t* cache, float kv_scale,
                     cudaStream_t st) {
  if (T <= 0) return 0;
  if (L != 512 || rd % 4 || rd > L) return -1;
  b200::launch_pdl(kv_store_v4_kernel, dim3(T), dim3(128), 0, st, kv, f32, ld, L, rd, w, eps, pos, table, slots,
                   cache, 1.f / kv_scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_mqa_q_prep(const void* q, int64_t qt, int64_t qh, int T, int H, int Hq, int rd, const int* pos,
                    const float* table, uint8_t* q8, float* qs, cudaStream_t st) {
  if (T <= 0) return 0;
  if (rd % 16 || rd > 512 || qt % 8 || qh % 8 || Hq < H) return -1;
  const int warps = T * H;
  b200::launch_pdl(mqa_q_prep_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, st,
                   reinterpret_cast<const __nv_bfloat16*>(q), qt, qh, T, H, Hq, rd, pos, table, q8, qs);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_attn_fixup(void* o, int T, int H, const float* lse, const float* sink, int rd, const int* pos,
                    const float* table, cudaStream_t st) {
  if (T <= 0) return 0;
  if (rd % 16 || rd > 512 || (sink && !lse)) return -1;
  const int warps = T * H;
  b200::launch_pdl(attn_fixup_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, st,
                   reinterpret_cast<__nv_bfloat16*>(o), T, H, lse, sink, rd, pos, table);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_e5_prune(int* ids, float* w, int T, int K, int E, float budget, int max_count, cudaStream_t st) {
  if (T <= 0) return 0;
  if (K > kPruneMaxK || E <= 0) return -1;
  b200::launch_pdl(e5_prune_kernel, dim3(1), dim3(1024), 2 * E * sizeof(int), st, ids, w, T, K, E, budget, max_count);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
