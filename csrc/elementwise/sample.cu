// Sampling over a vocab-parallel LM head without gathering the logits.
//
//   lm_candidates (one CTA per row, 1024 threads) over this rank's logits
//       shard [B, n]: the row max m and sum s = sum exp((x - m) / T) (T = the
//       row's temperature, 1 for greedy rows), and the Kc largest logits as
//       (value, global token id) candidates (radix select).  With peers, the
//       Kc + 1 entries go straight into every rank's receive slot over NVLink
//       and the last CTA publishes (the same push protocol as the fused
//       all-reduce); else into a local buffer.
//   sample_final (one CTA per row) waits for every rank's candidates
//       (bounded), sorts the world * Kc candidates (value desc, id asc),
//       forms the exact full-vocabulary softmax normaliser from the per-rank
//       (m, s) pairs, applies top-k / top-p like the reference sampler and
//       draws with the row's uniform; greedy rows take the largest logit
//       (lowest id on ties).
//
// Exact for greedy rows and whenever each shard's part of the kept set fits
// in its Kc candidates (Kc = 64 here: top_k <= 64 always qualifies).
//
// Reference parity: the reference's LGP lever (lgp.py:81-150) pulls the peer
// logit shard over NVLink into fp32 full logits before stock sampling; this
// design moves only the candidates.
#include "../common/radix_select.cuh"
#include "../comm/comm_dev.cuh"
#include "elementwise.h"

namespace b200 {
namespace smp {

constexpr int kMaxCand = 512;          // world * Kc

__device__ __forceinline__ float ld_logit(const void* p, int64_t i, int f32) {
  return f32 ? __ldcg(reinterpret_cast<const float*>(p) + i)
             : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// Entry layout per row (Kc + 1 uint2): [0] = (row max, sum of exps) as float
// bits, [1 + j] = (candidate logit bits, global token id).
__global__ void __launch_bounds__(rsel::kThreads) lm_candidates_kernel(const void* logits, int f32, int64_t ld, int n,
                                                                        int Kc, int vocab_off, const float* temperature,
                                                                        uint2* out, ArPeers peers, const uint32_t* epoch,
                                                                        uint32_t* ticket) {
  __shared__ rsel::Smem sm;
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t row = (int64_t)b * ld;
  auto load = [&](int i) { return ld_logit(logits, row + i, f32); };
  // row max
  float m = -INFINITY;
  for (int i = tid; i < n; i += rsel::kThreads) m = fmaxf(m, load(i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) red[tid >> 5] = m;
  __syncthreads();
  m = -INFINITY;
#pragma unroll
  for (int w = 0; w < rsel::kThreads / 32; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  const float T = temperature[b] > 0.f ? temperature[b] : 1.f;
  const float inv_t = 1.f / T;
  float s = 0.f;
  for (int i = tid; i < n; i += rsel::kThreads) s += __expf((load(i) - m) * inv_t);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((tid & 31) == 0) red[tid >> 5] = s;
  __syncthreads();
  s = 0.f;
#pragma unroll
  for (int w = 0; w < rsel::kThreads / 32; ++w) s += red[w];
  const int p = peers.world > 0 ? ((*epoch) & 1) : 0;
  const int stride = Kc + 1;
  auto put = [&](int j, uint2 v) {
    if (peers.world > 0) {
      for (int q = 0; q < peers.world; ++q) {
        uint2* dst = reinterpret_cast<uint2*>(comm::recv_slot(peers.base[q], p, peers.rank, peers.world, peers.max_t,
                                                              peers.hidden));
        dst[(int64_t)b * stride + j] = v;
      }
    } else {
      out[(int64_t)b * stride + j] = v;
    }
  };
  if (tid == 0) put(0, make_uint2(__float_as_uint(m), __float_as_uint(s)));
  if (n <= Kc) {
    for (int j = tid; j < Kc; j += rsel::kThreads)
      put(1 + j, j < n ? make_uint2(__float_as_uint(load(j)), uint32_t(vocab_off + j))
                       : make_uint2(__float_as_uint(-INFINITY), 0xFFFFFFFFu));
  } else {
    rsel::select_topk(load, n, Kc, sm, [&](int slot, int i) {
      put(1 + slot, make_uint2(__float_as_uint(load(i)), uint32_t(vocab_off + i)));
    });
  }
  if (peers.world > 0) comm::publish_push(peers.base, peers.world, peers.rank, p, ticket);
}

__global__ void __launch_bounds__(256) sample_final_kernel(const uint2* cand, int Kc, int world, ArPeers peers,
                                                            uint32_t* epoch, uint32_t* ticket, const float* temperature,
                                                            const float* top_p, const int* top_k,
                                                            const float* uniform, int64_t* tokens, uint32_t* err) {
  __shared__ float sv[kMaxCand];
  __shared__ int si[kMaxCand];
  __shared__ float sm_m[8], sm_s[8];
  __shared__ int ok_s;
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  const bool fused = peers.world > 0;
  const int p = fused ? ((*epoch) & 1) : 0;
  uint8_t* mine = fused ? peers.base[peers.rank] : nullptr;
  bool ok = true;
  if (fused) ok = comm::wait_arrivals(mine, p, peers.world, 1u, err, &ok_s);
  const int stride = Kc + 1;
  const int C = world * Kc;
  int P2 = 1;
  while (P2 < C) P2 <<= 1;
  for (int i = tid; i < P2; i += blockDim.x) {
    float v = -INFINITY;
    int id = 0x7FFFFFFF;
    if (i < C && ok) {
      const int r = i / Kc, j = i - r * Kc;
      const uint2* src = fused ? reinterpret_cast<const uint2*>(
                                     comm::recv_slot(mine, p, r, peers.world, peers.max_t, peers.hidden))
                               : cand + (int64_t)r * gridDim.x * stride;
      const uint2 e = __ldcg(src + (int64_t)b * stride + 1 + j);
      v = __uint_as_float(e.x);
      id = e.y == 0xFFFFFFFFu ? 0x7FFFFFFF : int(e.y);
    }
    sv[i] = v;
    si[i] = id;
  }
  if (tid < world && ok) {
    const uint2* src = fused ? reinterpret_cast<const uint2*>(
                                   comm::recv_slot(mine, p, tid, peers.world, peers.max_t, peers.hidden))
                             : cand + (int64_t)tid * gridDim.x * stride;
    const uint2 e = __ldcg(src + (int64_t)b * stride);
    sm_m[tid] = __uint_as_float(e.x);
    sm_s[tid] = __uint_as_float(e.y);
  }
  __syncthreads();
  // bitonic sort: value descending, token id ascending on ties
  for (int k = 2; k <= P2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < P2; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const bool desc = (i & k) == 0;
          const bool i_first = sv[i] > sv[l] || (sv[i] == sv[l] && si[i] < si[l]);
          if (i_first != desc) {
            const float tv = sv[i]; sv[i] = sv[l]; sv[l] = tv;
            const int ti = si[i]; si[i] = si[l]; si[l] = ti;
          }
        }
      }
      __syncthreads();
    }
  }
  if (tid == 0) {
    int64_t tok = si[0];
    const float T = temperature[b];
    if (ok && T > 0.f) {
      const float inv_t = 1.f / T;
      float M = -INFINITY;
      for (int r = 0; r < world; ++r) M = fmaxf(M, sm_m[r]);
      float Z = 0.f;
      for (int r = 0; r < world; ++r) Z += sm_s[r] * __expf((sm_m[r] - M) * inv_t);
      const int kk = top_k[b] > 0 ? min(top_k[b], C) : C;
      const float tp = top_p[b];
      // kept prefix: top-k, then top-p on the full-vocabulary probabilities
      float cum = 0.f, kept = 0.f;
      int nk = 0;
      for (int i = 0; i < kk; ++i) {
        if (sv[i] == -INFINITY) break;
        const float pi = __expf((sv[i] - M) * inv_t) / Z;
        if (cum >= tp) break;
        cum += pi;
        kept += pi;
        ++nk;
      }
      const float target = uniform[b] * kept;
      float acc = 0.f;
      tok = si[nk > 0 ? nk - 1 : 0];
      for (int i = 0; i < nk; ++i) {
        acc += __expf((sv[i] - M) * inv_t) / Z;
        if (acc >= target) {
          tok = si[i];
          break;
        }
      }
    }
    tokens[b] = ok ? tok : -1;
  }
  if (fused) {
    // completion: the last CTA frees this parity (counters, epoch)
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const uint32_t t = atomicAdd(ticket, 1u);
      if (t == gridDim.x - 1) {
        uint32_t* cnt = comm::counters(mine, p);
        for (int r = 0; r < peers.world; ++r) atomicExch(cnt + r, 0u);
        *ticket = 0u;
        __threadfence();
        atomicAdd(epoch, 1u);
      }
    }
  }
}

}  // namespace smp
}  // namespace b200

int b200_lm_candidates(const void* logits, int f32, int64_t ld, int B, int n, int Kc, int vocab_off,
                       const float* temperature, void* out, const ArPeers* peers, const uint32_t* epoch,
                       uint32_t* ticket, cudaStream_t st) {
  if (B <= 0) return 0;
  if (Kc <= 0 || Kc > 64) return -1;
  ArPeers none{};
  const ArPeers& pp = peers ? *peers : none;
  if (peers && ((int64_t)B * (Kc + 1) * 8 > (int64_t)peers->max_t * peers->hidden * 2)) return -2;
  b200::launch_pdl(b200::smp::lm_candidates_kernel, dim3(B), dim3(b200::rsel::kThreads), 0, st, logits, f32, ld, n,
                   Kc, vocab_off, temperature, reinterpret_cast<uint2*>(out), pp, epoch, ticket);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_sample_final(const void* cand, int B, int Kc, int world, const ArPeers* peers, uint32_t* epoch,
                      uint32_t* ticket, const float* temperature, const float* top_p, const int* top_k,
                      const float* uniform, int64_t* tokens, uint32_t* err, cudaStream_t st) {
  if (B <= 0) return 0;
  if (world * Kc > b200::smp::kMaxCand || world > 8) return -1;
  ArPeers none{};
  const ArPeers& pp = peers ? *peers : none;
  b200::launch_pdl(b200::smp::sample_final_kernel, dim3(B), dim3(256), 0, st, reinterpret_cast<const uint2*>(cand), Kc,
                   world, pp, epoch, ticket, temperature, top_p, top_k, uniform, tokens, err);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
