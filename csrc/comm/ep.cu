// Expert-parallel MoE over NVLink peer memory (DP attention + EP experts).
//
// Each rank serves its own tokens in attention; the MoE boundary moves them
// to the ranks owning their experts and brings the weighted expert outputs
// back, with no host round trip and no NCCL call:
//
//   ep_dispatch   (one CTA per local token row) after the router: P2P-stores
//                 the token's MXFP8 row (e4m3 + scale words) into the
//                 dispatch buffer of every rank that owns one of its top-k
//                 experts, and its routing row (ids, weights) into every
//                 rank's buffer; the last CTA publishes one arrival per rank.
//   ep_align      (one CTA) waits, bounded, for every rank's arrival, then
//                 builds the grouped-GEMM routing layout over all received
//                 rows (experts outside this rank's range are skipped).
//   ep_gather     copies the received rows into the expert-sorted operand of
//                 the grouped FC1 GEMM; its last CTA frees the parity.  With
//                 the fused expert kernel this step disappears: its producer
//                 warp reads each sorted row straight from the dispatch
//                 buffer (cp.async, 128B-swizzled into the operand tile) and
//                 ep_align frees the parity instead (release = 1).
//   ep_combine_rs after FC2 (whose epilogue already applied the routing
//                 weights): sums each received token's rows over this rank's
//                 experts and stores the partial straight into the owner
//                 rank's all-reduce slot (reduce-scatter); the owner's
//                 ar_reduce_norm sums the world partials in rank order, adds
//                 the residual, RMSNorm and MXFP8 - one fused kernel.
//
// Two parities alternate (device epoch advanced by ep_gather or ep_align), as in the
// tensor-parallel all-reduce: a rank pushes into parity p again only after
// its reduce-scatter of the previous layer, which waited for every peer's
// combine, which each peer issued after its gather had released p.
//
// Reference parity: the reference runs EP through SGLang's a2a backends
// (moe_fwd.py:355-382, fork_loop.py:151-158) and fuses only the TP finalize
// (fin.py:384); this path is our own design.
#include "../elementwise/moe_layout.cuh"
#include "comm_dev.cuh"

namespace b200 {
namespace ep {

constexpr int kThreads = 128;

__device__ __forceinline__ uint8_t* region(const EpPeers& P, int q, int parity) {
  return P.base[q] + kEpRegionOff + parity * P.par_bytes;
}

__global__ void __launch_bounds__(kThreads) ep_dispatch_kernel(const uint8_t* __restrict__ q,
                                                                const uint8_t* __restrict__ sf,
                                                                const float* __restrict__ g, int fp4,
                                                                const int* __restrict__ ids,
                                                                const float* __restrict__ w, int T_r, int T_step,
                                                                int experts_per_rank, EpPeers P, const uint32_t* epoch,
                                                                uint32_t* ticket, int peer_pull) {
  __shared__ uint32_t mask_s;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int p = (*epoch) & 1;
  const int t = blockIdx.x;
  const bool valid = t < T_r;
  const int K = P.K;
  const int row = P.rank * T_step + t;
  if (threadIdx.x < 32) {
    uint32_t m = 0;
    for (int k = threadIdx.x; k < K; k += 32) {
      const int id = valid ? __ldcg(ids + t * K + k) : -1;
      if (id >= 0) m |= 1u << (id / experts_per_rank);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m |= __shfl_xor_sync(0xffffffffu, m, o);
    if (threadIdx.x == 0) mask_s = m;
  }
  __syncthreads();
  const uint32_t mask = mask_s;
  const int row_bytes = fp4 ? P.hidden / 2 : P.hidden;
  const int kb = fp4 ? P.hidden / 16 : P.hidden / 32;   // scale columns
  const int words = kb / 4;                 // 4 scale bytes (4 k-blocks) per word
  for (int d = 0; d < P.world; ++d) {
    uint8_t* reg = region(P, d, p);
    int* did = reinterpret_cast<int*>(reg + P.off_ids);
    float* dw = reinterpret_cast<float*>(reg + P.off_w);
    for (int k = threadIdx.x; k < K; k += kThreads) {
      did[(int64_t)row * K + k] = valid ? __ldcg(ids + t * K + k) : -1;
      dw[(int64_t)row * K + k] = valid ? __ldcg(w + t * K + k) : 0.f;
    }
    // peer pull: the row stays in this rank's own region (row t), read there
    // by the owners' expert kernels over NVLink; otherwise it is stored into
    // every owner's region (row = rank * T_step + t)
    const bool here = peer_pull ? (d == P.rank && mask != 0u) : ((mask >> d) & 1u) != 0u;
    if (!here) continue;
    const int drow = peer_pull ? t : row;
    const uint4* src = reinterpret_cast<const uint4*>(q + (int64_t)t * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(reg + (int64_t)drow * row_bytes);
    for (int i = threadIdx.x; i < row_bytes / 16; i += kThreads) dst[i] = __ldcg(src + i);
    if (fp4 && threadIdx.x == 0) reinterpret_cast<float*>(reg + P.off_g)[drow] = __ldcg(g + t);
    uint8_t* dsf = reg + P.off_sf;
    for (int c = threadIdx.x; c < words; c += kThreads) {
      const uint32_t v = *reinterpret_cast<const uint32_t*>(sf + moe::sf_offset(t, 4 * c, kb));
      *reinterpret_cast<uint32_t*>(dsf + moe::sf_offset(drow, 4 * c, kb)) = v;
    }
  }
  comm::publish_push(P.base, P.world, P.rank, p, ticket);
}

__global__ void __launch_bounds__(1024) ep_align_kernel(EpPeers P, int T_step, int first, int E, int* seg_start,
                                                        int* seg_count, int* row_token, float* row_weight,
                                                        int* pair_row, int* total_rows, int bn1, int* ttile1, int bn2,
                                                        int* ttile2, uint32_t* epoch, uint32_t* err, int release,
                                                        int* row_pair) {
  extern __shared__ int sh[];
  __shared__ int ok_s;
  pdl_wait();
  pdl_launch_dependents();
  const int p = (*epoch) & 1;
  uint8_t* mine = P.base[P.rank];
  const bool ok = comm::wait_arrivals(mine, p, P.world, 1u, err, &ok_s);
  uint8_t* reg = region(P, P.rank, p);
  // On a timeout the layout is built over zero tokens (every pair unrouted),
  // so the GEMMs run empty and the error word tells the host.
  const int T = ok ? P.world * T_step : 0;
  if (!ok)
    for (int i = threadIdx.x; i < P.world * T_step * P.K; i += blockDim.x) pair_row[i] = -1;
  moe::moe_align_body(reinterpret_cast<const int*>(reg + P.off_ids), reinterpret_cast<const float*>(reg + P.off_w), T,
                      P.K, first, E, seg_start, seg_count, row_token, row_weight, pair_row, total_rows, bn1, ttile1, bn2,
                      ttile2, sh, row_pair);
  if (release) {
    // every thread read the epoch above; the rows stay in place for the
    // expert GEMM of this layer, and the next push into parity p comes two
    // layers on, after this rank's reduce-scatter of the next layer
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t* cnt = comm::counters(mine, p);
      for (int s = 0; s < P.world; ++s) atomicExch(cnt + s, 0u);
      __threadfence();
      atomicAdd(epoch, 1u);
    }
  }
}

__global__ void __launch_bounds__(kThreads) ep_gather_kernel(EpPeers P, int T_step, const int* pair_row, int fp4,
                                                              uint8_t* dq, uint8_t* dsf, float* dg, uint32_t* epoch,
                                                              uint32_t* ticket) {
  pdl_wait();
  pdl_launch_dependents();
  const int p = (*epoch) & 1;
  const int i = blockIdx.x;
  uint8_t* mine = P.base[P.rank];
  const uint8_t* reg = region(P, P.rank, p);
  const int r = __ldcg(pair_row + i);
  if (r >= 0) {
    const int t = i / P.K;
    if (fp4) {
      const int rb = P.hidden / 2, nb = P.hidden / 16;
      const uint4* s = reinterpret_cast<const uint4*>(reg + (int64_t)t * rb);
      uint4* d = reinterpret_cast<uint4*>(dq + (int64_t)r * rb);
      for (int j = threadIdx.x; j < rb / 16; j += blockDim.x) d[j] = __ldcg(s + j);
      for (int b = threadIdx.x; b < nb; b += blockDim.x)
        dsf[moe::sf_offset(r, b, nb)] = __ldcg(reg + P.off_sf + moe::sf_offset(t, b, nb));
      if (threadIdx.x == 0) dg[r] = __ldcg(reinterpret_cast<const float*>(reg + P.off_g) + t);
    } else {
      moe::moe_gather_pair(reg, reg + P.off_sf, t, r, P.hidden, dq, dsf);
    }
  }
  // completion: the last CTA frees this parity for the dispatch two layers on
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(ticket, 1u);
    if (prev == gridDim.x - 1) {
      uint32_t* cnt = comm::counters(mine, p);
      for (int s = 0; s < P.world; ++s) atomicExch(cnt + s, 0u);
      *ticket = 0u;
      __threadfence();
      atomicAdd(epoch, 1u);
    }
  }
}

__global__ void __launch_bounds__(256) ep_combine_rs_kernel(const __nv_bfloat16* __restrict__ y,
                                                             const int* __restrict__ pair_row, int T_step, int T_r,
                                                             int K, int hidden, const __nv_bfloat16* __restrict__ add,
                                                             ArPeers A, const uint32_t* epoch, uint32_t* ticket) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int p = (*epoch) & 1;
  const int vec_per_row = hidden / 8;
  const int64_t nvec = (int64_t)A.world * T_step * vec_per_row;
  const int64_t per = (nvec + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = blockIdx.x * per, v1 = min(nvec, v0 + per);
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const int g = int(v / vec_per_row);
    const int c = int(v - (int64_t)g * vec_per_row) * 8;
    const int owner = g / T_step, t = g - owner * T_step;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < K; ++j) {
      const int r = __ldcg(pair_row + (int64_t)g * K + j);
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
    if (add && owner == A.rank && t < T_r) {
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
    __nv_bfloat16* dst = comm::recv_slot(A.base[owner], p, A.rank, A.world, A.max_t, hidden);
    *reinterpret_cast<uint4*>(dst + (int64_t)t * hidden + c) = outv;
  }
  comm::publish_push(A.base, A.world, A.rank, p, ticket);
}

}  // namespace ep
}  // namespace b200

int b200_ep_dispatch(const uint8_t* q, const uint8_t* sf, const float* g, int fp4, const int* ids, const float* w,
                     int T_r, int T_step, int experts_per_rank, const EpPeers* peers, const uint32_t* epoch,
                     uint32_t* ticket, cudaStream_t st, int peer_pull) {
  if (T_step <= 0 || T_r > T_step || T_step > peers->max_t || peers->world > kArMaxRanks || peers->hidden % 128 ||
      experts_per_rank <= 0 || (fp4 && !g))
    return -1;
  b200::launch_pdl(b200::ep::ep_dispatch_kernel, dim3(T_step), dim3(b200::ep::kThreads), 0, st, q, sf, g, fp4, ids, w,
                   T_r, T_step, experts_per_rank, *peers, epoch, ticket, peer_pull);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_ep_align(const EpPeers* peers, int T_step, int first, int E, int* seg_start, int* seg_count, int* row_token,
                  float* row_weight, int* pair_row, int* total_rows, int bn1, int* ttile1, int bn2, int* ttile2,
                  uint32_t* epoch, uint32_t* err, int release, cudaStream_t st, int* row_pair) {
  if (T_step <= 0 || T_step > peers->max_t) return -1;
  b200::launch_pdl(b200::ep::ep_align_kernel, dim3(1), dim3(1024), 3 * E * sizeof(int), st, *peers, T_step, first, E,
                   seg_start, seg_count, row_token, row_weight, pair_row, total_rows, bn1 > 0 ? bn1 : 128, ttile1,
                   bn2 > 0 ? bn2 : 128, ttile2, epoch, err, release, row_pair);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_ep_gather(const EpPeers* peers, int T_step, const int* pair_row, int fp4, uint8_t* dq, uint8_t* dsf, float* dg,
                   uint32_t* epoch, uint32_t* ticket, cudaStream_t st) {
  if (T_step <= 0 || T_step > peers->max_t || (fp4 && !dg)) return -1;
  const int npairs = peers->world * T_step * peers->K;
  b200::launch_pdl(b200::ep::ep_gather_kernel, dim3(npairs), dim3(b200::ep::kThreads), 0, st, *peers, T_step, pair_row,
                   fp4, dq, dsf, dg, epoch, ticket);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_ep_combine_rs(const void* y, const int* pair_row, int T_step, int T_r, int K, int hidden, const void* add,
                       const ArPeers* ar, const uint32_t* ar_epoch, uint32_t* ar_ticket, int nctas, cudaStream_t st) {
  if (T_step <= 0 || T_step > ar->max_t || hidden % 8 || nctas <= 0) return -1;
  b200::launch_pdl(b200::ep::ep_combine_rs_kernel, dim3(nctas), dim3(256), 0, st,
                   reinterpret_cast<const __nv_bfloat16*>(y), pair_row, T_step, T_r, K, hidden,
                   reinterpret_cast<const __nv_bfloat16*>(add), *ar, ar_epoch, ar_ticket);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
