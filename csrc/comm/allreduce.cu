// Fused tensor-parallel all-reduce + residual add + RMSNorm + MXFP8 quant
// over NVLink peer memory (one process per GPU, buffers from torch symmetric
// memory).
//
// Symmetric buffer layout (identical on every rank, bytes from its base):
//   [0, 256)                     uint32 arrival counters cnt[2][kMaxRanks]
//   [kRecvOff, ...)              bf16 recv[2][world][max_t][hidden]
// Two parities alternate between consecutive all-reduces (parity = epoch & 1,
// epoch a device counter every rank advances in the same order), so a rank
// never overwrites a slot a slower peer is still reading.
//
//   push (one kernel, or a GEMM / MoE-combine epilogue): rank r P2P-stores its
//        partial rows into recv[p][r] of every rank, then each CTA publishes
//        with a system-scope fence + one atomic increment of cnt[p][r] on
//        every rank.
//   reduce: each CTA waits (bounded by %globaltimer) until cnt[p][q] == the
//        pushers' CTA count for all q, sums recv[p][0..W) in rank order (so
//        every rank produces bitwise identical rows), adds the fp32 residual
//        in place, RMSNorm, and writes bf16 and/or MXFP8 outputs.  The last
//        CTA (ticket) zeroes cnt[p][*] and advances the epoch.
//
// Ordering argument for slot reuse: rank r's push at epoch e+2 is stream-
// ordered after its reduce at e+1, which waited for every peer's push at
// e+1, which each peer issued after finishing its own reduce at e.
//
// Reference parity: the reference's FIN push plane (fin.py:384, 16-byte
// relaxed stores + Lamport markers, unbounded polls at fin.py:459-471) and
// EPA epilogue push (epa.py:795, epa_gemm.py:1849-1890); here every poll is
// bounded and reports an error code instead of hanging.
#include "../common/ptx.cuh"
#include "comm_dev.cuh"
#include <algorithm>

namespace b200 {
namespace comm {

constexpr int kThreads = 256;
constexpr int kMaxIt = 8;     // hidden <= 256 * 8 * 8 = 16384

__device__ __forceinline__ int64_t sf_off(int row, int kblock, int kb_total) {
  const int rb = row >> 7, r = row & 127, kc = kblock >> 2, c = kblock & 3;
  return ((int64_t)(rb * (kb_total >> 2) + kc) << 9) + ((r & 31) << 4) + ((r >> 5) << 2) + c;
}

__device__ __forceinline__ void publish_push(const ArPeers& peers, int parity, uint32_t* ticket) {
  publish_push(peers.base, peers.world, peers.rank, parity, ticket);
}


// Row epilogue shared by the push, NVLS and expert-combine reductions: v =
// sum of the nsrc bf16 rows src0 + row * row_stride + i * src_stride (in
// index order; source i skipped when ids_row[i] < 0) + add_row (optional) +
// residual (updated in place, fp32); RMSNorm; bf16 y and / or MXFP8 q + sf
// (tcgen05 scale layout).  One CTA of kThreads per row; `red` is >= 32
// floats of shared memory.
__device__ __forceinline__ void row_add_norm_quant(int row, int hidden, const __nv_bfloat16* src0, int64_t src_stride,
                                                   int nsrc, int64_t row_stride, const int* ids_row,
                                                   const __nv_bfloat16* add_row, float* residual,
                                                   const float* __restrict__ w, float eps, __nv_bfloat16* y,
                                                   uint8_t* q, uint8_t* sf, float* red) {
  const int units = hidden >> 3;
  {
    float v[kMaxIt][8];
    float ss = 0.f;
#pragma unroll
    for (int it = 0; it < kMaxIt; ++it) {
      const int u = it * kThreads + threadIdx.x;
      if (u < units) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[it][i] = 0.f;
        for (int src = 0; src < nsrc; ++src) {
          if (ids_row && __ldcg(ids_row + src) < 0) continue;
          const __nv_bfloat16* s = src0 + src * src_stride + (int64_t)row * row_stride;
          const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(s + u * 8));
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            v[it][2 * i] += f.x;
            v[it][2 * i + 1] += f.y;
          }
        }
        if (add_row) {
          const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(add_row + u * 8));
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            v[it][2 * i] += f.x;
            v[it][2 * i + 1] += f.y;
          }
        }
        float* rp = residual + (int64_t)row * hidden + u * 8;
        const float4 r0 = *reinterpret_cast<const float4*>(rp);
        const float4 r1 = *reinterpret_cast<const float4*>(rp + 4);
        v[it][0] += r0.x; v[it][1] += r0.y; v[it][2] += r0.z; v[it][3] += r0.w;
        v[it][4] += r1.x; v[it][5] += r1.y; v[it][6] += r1.z; v[it][7] += r1.w;
        *reinterpret_cast<float4*>(rp) = make_float4(v[it][0], v[it][1], v[it][2], v[it][3]);
        *reinterpret_cast<float4*>(rp + 4) = make_float4(v[it][4], v[it][5], v[it][6], v[it][7]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[it][i] * v[it][i];
      }
    }
    // block reduction of the sum of squares
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float s2 = threadIdx.x < (kThreads >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      if (threadIdx.x == 0) red[0] = s2;
    }
    __syncthreads();
    const float rs = rsqrtf(red[0] / float(hidden) + eps);
    const int kb_total = hidden >> 5;
#pragma unroll
    for (int it = 0; it < kMaxIt; ++it) {
      if (it * kThreads >= units) break;
      const int u = it * kThreads + threadIdx.x;
      const bool valid = u < units;
      float o[8];
      if (valid) {
        const float4 w0 = *reinterpret_cast<const float4*>(w + u * 8);
        const float4 w1 = *reinterpret_cast<const float4*>(w + u * 8 + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[it][i] * rs * wv[i];
        if (y) {
          uint4 outv;
          __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&outv);
#pragma unroll
          for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
          *reinterpret_cast<uint4*>(y + (int64_t)row * hidden + u * 8) = outv;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0.f;
      }
      if (q) {
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(o[i]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const int e = ceil_log2_bits(amax * (1.0f / 448.0f));
        const float inv = exp2_int(-e);
        uint2 packed;
        uint16_t* o16 = reinterpret_cast<uint16_t*>(&packed);
#pragma unroll
        for (int i = 0; i < 4; ++i) o16[i] = f2_to_e4m3x2(o[2 * i] * inv, o[2 * i + 1] * inv);
        if (valid) {
          *reinterpret_cast<uint2*>(q + (int64_t)row * hidden + u * 8) = packed;
          if ((u & 3) == 0) sf[sf_off(row, (u * 8) >> 5, kb_total)] = uint8_t(e + 127);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) ar_push_kernel(const __nv_bfloat16* __restrict__ x, int T, int hidden,
                                                           ArPeers peers, const uint32_t* epoch, uint32_t* ticket) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();   // e.g. the next GEMM prefetches weights during our wait
  const int p = (*epoch) & 1;
  const int64_t n16 = (int64_t)T * hidden / 8;       // 16-byte vectors
  const int64_t per = (n16 + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = blockIdx.x * per;
  const int64_t v1 = min(n16, v0 + per);
  const uint4* src = reinterpret_cast<const uint4*>(x);
  for (int q = 0; q < push_dests(peers); ++q) {
    uint4* dst = reinterpret_cast<uint4*>(push_slot(peers, q, p, hidden));
    for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) dst[v] = src[v];
  }
  publish_push(peers, p, ticket);
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) ar_reduce_norm_kernel(
    int T, int hidden, ArPeers peers, uint32_t* epoch, uint32_t* ticket, uint32_t expected, float* residual,
    const float* __restrict__ w, float eps, __nv_bfloat16* y, uint8_t* q, uint8_t* sf, uint32_t* err) {
  __shared__ float red[32];
  __shared__ int ok_s;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();   // e.g. the next GEMM prefetches weights during our wait
  const int p = (*epoch) & 1;
  uint8_t* mine = peers.base[peers.rank];
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint32_t* cnt = counters(mine, p);
    const uint64_t t0 = globaltimer_ns();
    for (int src = 0; src < peers.world && ok; ++src) {
      while (ld_acquire_sys(cnt + src) < expected) {
        if (globaltimer_ns() - t0 > kWaitBudgetNs) {
          atomicExch(err, kErrPeerTimeout);
          ok = 0;
          break;
        }
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  if (ok_s && blockIdx.x < T)
    row_add_norm_quant(blockIdx.x, hidden, recv_slot(mine, p, 0, peers.world, peers.max_t, hidden),
                       (int64_t)peers.max_t * hidden, peers.world, hidden, nullptr, nullptr, residual, w, eps, y, q,
                       sf, red);
  // completion: the last CTA resets this parity's counters and advances the epoch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(ticket, 1u);
    if (t == gridDim.x - 1) {
      uint32_t* cnt = counters(mine, p);
      for (int src = 0; src < peers.world; ++src) atomicExch(cnt + src, 0u);
      *ticket = 0u;
      __threadfence();
      atomicAdd(epoch, 1u);
    }
  }
}

}  // namespace comm
}  // namespace b200

int b200_ar_push(const void* x, int T, int hidden, const ArPeers* peers, const uint32_t* epoch, uint32_t* ticket,
                 int nctas, cudaStream_t st) {
  if (T <= 0) return 0;
  if (T > peers->max_t || hidden % 8 || peers->world > kArMaxRanks || nctas <= 0) return -1;
  b200::launch_pdl(b200::comm::ar_push_kernel, dim3(nctas), dim3(b200::comm::kThreads), 0, st, reinterpret_cast<const __nv_bfloat16*>(x), T,
                                                                      hidden, *peers, epoch, ticket);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_ar_reduce_norm(int T, int hidden, const ArPeers* peers, uint32_t* epoch, uint32_t* ticket, int push_ctas,
                        float* residual, const float* w, float eps, void* y, uint8_t* q, uint8_t* sf, uint32_t* err,
                        cudaStream_t st) {
  if (T <= 0) return 0;
  if (T > peers->max_t || hidden % 32 || hidden > b200::comm::kThreads * 8 * b200::comm::kMaxIt) return -1;
  b200::launch_pdl(b200::comm::ar_reduce_norm_kernel, dim3(T), dim3(b200::comm::kThreads), 0, st, 
      T, hidden, *peers, epoch, ticket, (uint32_t)push_ctas, residual, w, eps,
      reinterpret_cast<__nv_bfloat16*>(y), q, sf, err);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

// ---------------------------------------------------------------------------
// MoE combine fused with the all-reduce push: for token t, the rank-partial
// sum over its local experts' weighted rows y[pair_row[t, j]] plus the
// shared-expert partial add[t] goes straight into recv[p][rank][t] of every
// rank.  grid: `nctas` CTAs over the tokens.
namespace b200 {
namespace comm {
// One-kernel push all-reduce (+ MoE combine) + residual + RMSNorm (+ MXFP8)
// for decode-sized steps.  CTA c of G owns rows c, c + G, ... (the same grid
// on every rank): it stores its rows' partial - x, or for the MoE the sum of
// the token's local expert rows y[pair_row] plus the shared-expert row - into
// recv[p][rank] of every rank, raises cta_cnt[p][c] on every rank
// (red.release.sys after a system fence), waits (bounded) until all ranks
// raised its own cta_cnt[p][c], then sums the world partials of its rows in
// rank order and runs the row epilogue.  Rows meet only their own CTAs, so
// no grid-wide publish sits between the stores and the reduction, and one
// launch replaces the push + reduce pair.  The last CTA (ticket) zeroes this
// parity's CTA counters and advances the epoch (parity reuse is two
// all-reduces away, as for the two-kernel protocol).
template <bool COMBINE>
__global__ void __launch_bounds__(kThreads) ar_fused_norm_kernel(
    const __nv_bfloat16* __restrict__ x, const int* __restrict__ pair_row, int K, const __nv_bfloat16* __restrict__ add,
    int T, int hidden, ArPeers peers, uint32_t* epoch, uint32_t* ticket, float* residual, const float* __restrict__ w,
    float eps, __nv_bfloat16* y, uint8_t* q, uint8_t* sf, uint32_t* err, int S) {
  // S CTAs per row owner: CTA b pushes column chunk b % S of the rows of
  // owner c = b / S; every chunk CTA raises the owner's flag, and the chunk-0
  // CTA waits for world * S arrivals and reduces the whole rows.
  __shared__ float red[32];
  __shared__ int ok_s;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int p = (*epoch) & 1;
  const int c = blockIdx.x / S, chunk = blockIdx.x % S;
  const int G = gridDim.x / S;
  uint8_t* mine = peers.base[peers.rank];
  const int units = hidden >> 3;
  const int u_per = (units + S - 1) / S;
  const int u0 = chunk * u_per, u1 = min(units, u0 + u_per);
  for (int t = c; t < T; t += G) {
    for (int u = u0 + threadIdx.x; u < u1; u += kThreads) {
      uint4 outv;
      if constexpr (COMBINE) {
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        for (int j = 0; j < K; ++j) {
          const int r = __ldcg(pair_row + t * K + j);
          if (r < 0) continue;
          const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(x + (int64_t)r * hidden) + u);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
          }
        }
        if (add) {
          const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(add + (int64_t)t * hidden) + u);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
          }
        }
        __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&outv);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      } else {
        outv = __ldcg(reinterpret_cast<const uint4*>(x + (int64_t)t * hidden) + u);
      }
      for (int d = 0; d < peers.world; ++d) {
        __nv_bfloat16* dst = recv_slot(peers.base[d], p, peers.rank, peers.world, peers.max_t, hidden);
        *reinterpret_cast<uint4*>(dst + (int64_t)t * hidden + u * 8) = outv;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int d = 0; d < peers.world; ++d)
      asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(cta_counters(peers.base[d], p) + c), "r"(1u)
                   : "memory");
    int ok = 1;
    if (chunk == 0) {
      const uint32_t* cnt = cta_counters(mine, p) + c;
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(cnt) < (uint32_t)(peers.world * S)) {
        if (globaltimer_ns() - t0 > kWaitBudgetNs) {
          atomicExch(err, kErrPeerTimeout);
          ok = 0;
          break;
        }
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  if (ok_s && chunk == 0) {
    for (int t = c; t < T; t += G) {
      row_add_norm_quant(t, hidden, recv_slot(mine, p, 0, peers.world, peers.max_t, hidden),
                         (int64_t)peers.max_t * hidden, peers.world, hidden, nullptr, nullptr, residual, w, eps, y, q,
                         sf, red);
      __syncthreads();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t tk = atomicAdd(ticket, 1u);
    if (tk == gridDim.x - 1) {
      uint32_t* cnt = cta_counters(mine, p);
      for (int i = 0; i < G; ++i) atomicExch(cnt + i, 0u);
      *ticket = 0u;
      __threadfence();
      atomicAdd(epoch, 1u);
    }
  }
}

__global__ void __launch_bounds__(kThreads) moe_combine_push_kernel(const __nv_bfloat16* __restrict__ y,
                                                                     const int* __restrict__ pair_row, int T, int K,
                                                                     int hidden, const __nv_bfloat16* __restrict__ add,
                                                                     ArPeers peers, const uint32_t* epoch, uint32_t* ticket) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();   // e.g. the next GEMM prefetches weights during our wait
  const int p = (*epoch) & 1;
  const int vec_per_row = hidden / 8;
  const int64_t nvec = (int64_t)T * vec_per_row;
  const int64_t per = (nvec + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = blockIdx.x * per, v1 = min(nvec, v0 + per);
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const int t = int(v / vec_per_row);
    const int c = int(v - (int64_t)t * vec_per_row) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < K; ++j) {
      const int r = __ldcg(pair_row + t * K + j);
      if (r < 0) continue;
      const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(y + (int64_t)r * hidden + c));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    if (add) {
      const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(add + (int64_t)t * hidden + c));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    uint4 outv;
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&outv);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
    for (int q = 0; q < push_dests(peers); ++q) {
      __nv_bfloat16* dst = push_slot(peers, q, p, hidden);
      *reinterpret_cast<uint4*>(dst + (int64_t)t * hidden + c) = outv;
    }
  }
  publish_push(peers, p, ticket);
}
}  // namespace comm
}  // namespace b200

int b200_moe_combine_push(const void* y, const int* pair_row, int T, int K, int hidden, const void* add,
                          const ArPeers* peers, const uint32_t* epoch, uint32_t* ticket, int nctas, cudaStream_t st) {
  if (T <= 0) return 0;
  if (T > peers->max_t || hidden % 8 || nctas <= 0) return -1;
  b200::launch_pdl(b200::comm::moe_combine_push_kernel, dim3(nctas), dim3(b200::comm::kThreads), 0, st, 
      reinterpret_cast<const __nv_bfloat16*>(y), pair_row, T, K, hidden, reinterpret_cast<const __nv_bfloat16*>(add),
      *peers, epoch, ticket);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

// ---------------------------------------------------------------------------
// NVLS all-reduce + residual + RMSNorm (+ MXFP8), one kernel of
// G = min(T, kNvlsMaxCtas) CTAs, all co-resident (step 3 waits for every CTA
// of every rank, so the grid never exceeds one CTA per SM).
//
//   1. wait until every rank's pusher published its arrival for this parity
//      (the pushers stored their partial only into their own in[p] slot);
//   2. this rank's share of the 16-byte vectors of the T x hidden sum:
//      multimem.ld_reduce (the switch adds the same vector of every rank's
//      in[p], fp32 accumulation) -> multimem.st into out[p] of every rank;
//   3. each CTA publishes its share (P2P release increment of cnt_out[p][me]
//      on every rank) and waits until every rank's G CTAs did;
//   4. row epilogue on out[p] (local reads), as in the push reduction; CTA c
//      takes rows c, c + G, ...
// Bytes over NVLink per rank: one multicast read and one multicast write of
// 1/world of the rows, versus (world - 1) full copies for the push.  Every
// rank reads the same sums, so the outputs are identical on every rank.
// Slot reuse follows the push protocol's argument: a rank pushes parity p
// again only after its reduction of the other parity, which waited for every
// rank's step 3 of this one.  The last CTA (ticket) zeroes both counter rows
// of the parity and advances the epoch.
namespace b200 {
namespace comm {

constexpr int kNvlsMaxCtas = 148;

__device__ __forceinline__ void mm_ld_reduce_bf16x8(const void* mc, uint4& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(mc) : "memory");
}
__device__ __forceinline__ void mm_st_b128(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};"
               :: "l"(mc), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__global__ void __launch_bounds__(kThreads) nvls_ar_norm_kernel(
    int T, int hidden, ArPeers peers, uint32_t* epoch, uint32_t* ticket, uint32_t expected, float* residual,
    const float* __restrict__ w, float eps, __nv_bfloat16* y, uint8_t* q, uint8_t* sf, uint32_t* err) {
  __shared__ float red[32];
  __shared__ int ok_s;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int p = (*epoch) & 1;
  uint8_t* mine = peers.base[peers.rank];
  const int64_t slot = (int64_t)peers.max_t * hidden;                 // elements per slot
  const int64_t in_off = kArRecvOff + (int64_t)p * slot * 2;           // bytes
  const int64_t out_off = kArRecvOff + (int64_t)(2 + p) * slot * 2;
  // 1. every rank's partial is in its in[p]
  bool ok = wait_arrivals(mine, p, peers.world, expected, err, &ok_s);
  // 2. this rank's share of the sum, broadcast through the switch
  if (ok) {
    const int64_t nvec = (int64_t)T * hidden / 8;
    const int64_t per_rank = (nvec + peers.world - 1) / peers.world;
    const int64_t r0 = peers.rank * per_rank, r1 = min(nvec, r0 + per_rank);
    const int64_t per_cta = (r1 - r0 + gridDim.x - 1) / gridDim.x;
    const int64_t c0 = r0 + blockIdx.x * per_cta, c1 = min(r1, c0 + per_cta);
    const uint4* in_mc = reinterpret_cast<const uint4*>(peers.mc + in_off);
    uint4* out_mc = reinterpret_cast<uint4*>(peers.mc + out_off);
    for (int64_t v = c0 + threadIdx.x; v < c1; v += blockDim.x) {
      uint4 s;
      mm_ld_reduce_bf16x8(in_mc + v, s);
      mm_st_b128(out_mc + v, s);
    }
  }
  // 3. publish this CTA's share on every rank, then wait for all shares
  __syncthreads();
  if (threadIdx.x == 0 && ok) {
    __threadfence_system();
    for (int d = 0; d < peers.world; ++d)
      asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(counters2(peers.base[d], p) + peers.rank), "r"(1u)
                   : "memory");
  }
  if (threadIdx.x == 0) {
    int ok2 = ok ? 1 : 0;
    const uint32_t* cnt = counters2(mine, p);
    const uint64_t t0 = globaltimer_ns();
    for (int src = 0; src < peers.world && ok2; ++src) {
      while (ld_acquire_sys(cnt + src) < (uint32_t)gridDim.x) {
        if (globaltimer_ns() - t0 > kWaitBudgetNs) {
          atomicExch(err, kErrPeerTimeout);
          ok2 = 0;
          break;
        }
      }
    }
    ok_s = ok2;
  }
  __syncthreads();
  // 4. row epilogue on the broadcast sum
  if (ok_s)
    for (int row = blockIdx.x; row < T; row += gridDim.x) {
      row_add_norm_quant(row, hidden, reinterpret_cast<const __nv_bfloat16*>(mine + out_off), 0, 1, hidden, nullptr,
                         nullptr, residual, w, eps, y, q, sf, red);
      __syncthreads();                  // `red` is reused by the next row
    }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(ticket, 1u);
    if (t == gridDim.x - 1) {
      uint32_t* cnt = counters(mine, p);
      uint32_t* cnt2 = counters2(mine, p);
      for (int src = 0; src < peers.world; ++src) {
        atomicExch(cnt + src, 0u);
        atomicExch(cnt2 + src, 0u);
      }
      *ticket = 0u;
      __threadfence();
      atomicAdd(epoch, 1u);
    }
  }
}

// One-kernel NVLS all-reduce (+ MoE combine) + residual + RMSNorm (+ MXFP8).
// CTA c of G owns rows c, c + G, ... on every rank and rank c % world
// reduces them: every rank's CTA c stores its rows' partial into its own
// in[p] (local stores), raises cta_cnt[p][c] on the reducer; the reducer's
// CTA c waits for all world arrivals, sums the rows through the switch
// (multimem.ld_reduce over in[p]) and broadcasts the sums into every rank's
// out[p] (multimem.st), then raises cta_cnt2[p][c] on every rank; every
// rank's CTA c waits for that flag and runs the row epilogue on out[p].
// Only per-CTA flags, one launch; each rank's memory is read once per row
// through the switch and the sums cross NVLink once.  The last CTA (ticket)
// zeroes this parity's flags and advances the epoch.
template <bool COMBINE>
__global__ void __launch_bounds__(kThreads) nvls_fused_norm_kernel(
    const __nv_bfloat16* __restrict__ x, const int* __restrict__ pair_row, int K, const __nv_bfloat16* __restrict__ add,
    int T, int hidden, ArPeers peers, uint32_t* epoch, uint32_t* ticket, float* residual, const float* __restrict__ w,
    float eps, __nv_bfloat16* y, uint8_t* q, uint8_t* sf, uint32_t* err) {
  __shared__ float red[32];
  __shared__ int ok_s;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int p = (*epoch) & 1;
  const int G = gridDim.x, c = blockIdx.x;
  const int reducer = c % peers.world;
  uint8_t* mine = peers.base[peers.rank];
  const int64_t slot = (int64_t)peers.max_t * hidden;                 // elements per slot
  const int64_t in_off = kArRecvOff + (int64_t)p * slot * 2;           // bytes
  const int64_t out_off = kArRecvOff + (int64_t)(2 + p) * slot * 2;
  const int units = hidden >> 3;
  __nv_bfloat16* in_mine = reinterpret_cast<__nv_bfloat16*>(mine + in_off);
  // 1. this CTA's rows of the partial into this rank's own input slot
  for (int t = c; t < T; t += G) {
    for (int u = threadIdx.x; u < units; u += kThreads) {
      uint4 outv;
      if constexpr (COMBINE) {
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        for (int j = 0; j < K; ++j) {
          const int r = __ldcg(pair_row + t * K + j);
          if (r < 0) continue;
          const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(x + (int64_t)r * hidden) + u);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
          }
        }
        if (add) {
          const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(add + (int64_t)t * hidden) + u);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
          }
        }
        __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&outv);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      } else {
        outv = __ldcg(reinterpret_cast<const uint4*>(x + (int64_t)t * hidden) + u);
      }
      *reinterpret_cast<uint4*>(in_mine + (int64_t)t * hidden + u * 8) = outv;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(cta_counters(peers.base[reducer], p) + c), "r"(1u)
                 : "memory");
  }
  // 2. the reducer sums the rows through the switch and broadcasts them
  int ok = 1;
  if (peers.rank == reducer) {
    if (threadIdx.x == 0) {
      const uint32_t* cnt = cta_counters(mine, p) + c;
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(cnt) < (uint32_t)peers.world) {
        if (globaltimer_ns() - t0 > kWaitBudgetNs) {
          atomicExch(err, kErrPeerTimeout);
          ok = 0;
          break;
        }
      }
      ok_s = ok;
    }
    __syncthreads();
    ok = ok_s;
    if (ok) {
      const uint4* in_mc = reinterpret_cast<const uint4*>(peers.mc + in_off);
      uint4* out_mc = reinterpret_cast<uint4*>(peers.mc + out_off);
      for (int t = c; t < T; t += G)
        for (int u = threadIdx.x; u < units; u += kThreads) {
          const int64_t v = (int64_t)t * units + u;
          uint4 s;
          mm_ld_reduce_bf16x8(in_mc + v, s);
          mm_st_b128(out_mc + v, s);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && ok) {
      __threadfence_system();
      for (int d = 0; d < peers.world; ++d)
        asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(cta_counters2(peers.base[d], p) + c), "r"(1u)
                     : "memory");
    }
  }
  // 3. wait for this CTA's broadcast rows, then the row epilogue
  if (threadIdx.x == 0) {
    int ok2 = 1;
    const uint32_t* cnt = cta_counters2(mine, p) + c;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(cnt) < 1u) {
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        atomicExch(err, kErrPeerTimeout);
        ok2 = 0;
        break;
      }
    }
    ok_s = ok2;
  }
  __syncthreads();
  if (ok_s)
    for (int t = c; t < T; t += G) {
      row_add_norm_quant(t, hidden, reinterpret_cast<const __nv_bfloat16*>(mine + out_off), 0, 1, hidden, nullptr,
                         nullptr, residual, w, eps, y, q, sf, red);
      __syncthreads();
    }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t tk = atomicAdd(ticket, 1u);
    if (tk == (uint32_t)G - 1) {
      uint32_t* c1 = cta_counters(mine, p);
      uint32_t* c2 = cta_counters2(mine, p);
      for (int i = 0; i < G; ++i) {
        atomicExch(c1 + i, 0u);
        atomicExch(c2 + i, 0u);
      }
      *ticket = 0u;
      __threadfence();
      atomicAdd(epoch, 1u);
    }
  }
}

}  // namespace comm
}  // namespace b200

int b200_nvls_ar_norm(int T, int hidden, const ArPeers* peers, uint32_t* epoch, uint32_t* ticket, int expected,
                      float* residual, const float* w, float eps, void* y, uint8_t* q, uint8_t* sf, uint32_t* err,
                      cudaStream_t st) {
  if (T <= 0) return 0;
  if (!peers->mc || T > peers->max_t || hidden % 32 || hidden > b200::comm::kThreads * 8 * b200::comm::kMaxIt ||
      peers->world > kArMaxRanks || expected <= 0)
    return -1;
  const int G = T < b200::comm::kNvlsMaxCtas ? T : b200::comm::kNvlsMaxCtas;
  b200::launch_pdl(b200::comm::nvls_ar_norm_kernel, dim3(G), dim3(b200::comm::kThreads), 0, st, T, hidden, *peers,
                   epoch, ticket, (uint32_t)expected, residual, w, eps, reinterpret_cast<__nv_bfloat16*>(y), q, sf,
                   err);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

// ---------------------------------------------------------------------------
// Owner side of the expert-parallel combine fused into the experts' FC2
// epilogue (moe_fused.cu): every rank stored the weighted output row of each
// pair (t, k) it served straight into comb[p][t][k] of t's owner and
// published one arrival.  One CTA per own token row: wait (bounded) for every
// rank's arrival, sum the row's K pair rows in k order (pairs whose expert id
// is < 0 were pruned / padded and are skipped) + the shared-expert row, add
// the residual, RMSNorm (+ MXFP8).  The last CTA zeroes the parity's
// counters and advances the epoch (the push reduction's protocol).
namespace b200 {
namespace comm {
__global__ void __launch_bounds__(kThreads) ep_comb_reduce_norm_kernel(
    int T_r, int hidden, int K, const int* __restrict__ ids, const __nv_bfloat16* __restrict__ add, ArPeers peers,
    uint32_t* epoch, uint32_t* ticket, float* residual, const float* __restrict__ w, float eps, __nv_bfloat16* y,
    uint8_t* q, uint8_t* sf, uint32_t* err) {
  __shared__ float red[32];
  __shared__ int ok_s;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int p = (*epoch) & 1;
  uint8_t* mine = peers.base[peers.rank];
  const bool ok = wait_arrivals(mine, p, peers.world, 1u, err, &ok_s);
  const int row = blockIdx.x;
  if (ok && row < T_r) {
    const __nv_bfloat16* comb = reinterpret_cast<const __nv_bfloat16*>(
        mine + ep_combine_off(peers.world, peers.max_t, hidden) + (int64_t)p * peers.max_t * K * hidden * 2);
    row_add_norm_quant(row, hidden, comb, hidden, K, (int64_t)K * hidden, ids + (int64_t)row * K,
                       add ? add + (int64_t)row * hidden : nullptr, residual, w, eps, y, q, sf, red);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(ticket, 1u);
    if (t == gridDim.x - 1) {
      uint32_t* cnt = counters(mine, p);
      for (int src = 0; src < peers.world; ++src) atomicExch(cnt + src, 0u);
      *ticket = 0u;
      __threadfence();
      atomicAdd(epoch, 1u);
    }
  }
}
}  // namespace comm
}  // namespace b200

int b200_ep_comb_reduce_norm(int T_r, int hidden, int K, const int* ids, const void* add, const ArPeers* peers,
                             uint32_t* epoch, uint32_t* ticket, float* residual, const float* w, float eps, void* y,
                             uint8_t* q, uint8_t* sf, uint32_t* err, cudaStream_t st) {
  if (T_r <= 0) return 0;
  if (T_r > peers->max_t || hidden % 32 || hidden > b200::comm::kThreads * 8 * b200::comm::kMaxIt || K <= 0)
    return -1;
  b200::launch_pdl(b200::comm::ep_comb_reduce_norm_kernel, dim3(T_r), dim3(b200::comm::kThreads), 0, st, T_r, hidden,
                   K, ids, reinterpret_cast<const __nv_bfloat16*>(add), *peers, epoch, ticket, residual, w, eps,
                   reinterpret_cast<__nv_bfloat16*>(y), q, sf, err);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_ar_fused_norm(const void* x, const int* pair_row, int K, const void* add, int T, int hidden,
                       const ArPeers* peers, uint32_t* epoch, uint32_t* ticket, float* residual, const float* w,
                       float eps, void* y, uint8_t* q, uint8_t* sf, uint32_t* err, cudaStream_t st, int chunks) {
  if (T <= 0) return 0;
  if (T > peers->max_t || hidden % 32 || hidden > b200::comm::kThreads * 8 * b200::comm::kMaxIt ||
      (pair_row && K <= 0) || chunks < 1 || chunks > 8)
    return -1;
  const int G = std::min(T, std::min(148, kArMaxCtas));
  const int S = peers->mc ? 1 : chunks;       // the NVLS variant keeps one CTA per row owner
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto* ab = reinterpret_cast<const __nv_bfloat16*>(add);
  auto* yb = reinterpret_cast<__nv_bfloat16*>(y);
  if (peers->mc) {
    if (pair_row)
      b200::launch_pdl(b200::comm::nvls_fused_norm_kernel<true>, dim3(G), dim3(b200::comm::kThreads), 0, st, xb,
                       pair_row, K, ab, T, hidden, *peers, epoch, ticket, residual, w, eps, yb, q, sf, err);
    else
      b200::launch_pdl(b200::comm::nvls_fused_norm_kernel<false>, dim3(G), dim3(b200::comm::kThreads), 0, st, xb,
                       (const int*)nullptr, 0, (const __nv_bfloat16*)nullptr, T, hidden, *peers, epoch, ticket,
                       residual, w, eps, yb, q, sf, err);
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
  }
  if (pair_row)
    b200::launch_pdl(b200::comm::ar_fused_norm_kernel<true>, dim3(G * S), dim3(b200::comm::kThreads), 0, st, xb,
                     pair_row, K, ab, T, hidden, *peers, epoch, ticket, residual, w, eps, yb, q, sf, err, S);
  else
    b200::launch_pdl(b200::comm::ar_fused_norm_kernel<false>, dim3(G * S), dim3(b200::comm::kThreads), 0, st, xb,
                     (const int*)nullptr, 0, (const __nv_bfloat16*)nullptr, T, hidden, *peers, epoch, ticket, residual,
                     w, eps, yb, q, sf, err, S);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
