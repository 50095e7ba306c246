// Block-wide top-K selection by radix select (one CTA of 1024 threads per
// row), shared by the sparse-attention indexer and the sampler.
//
// Four passes of 8-bit digits over an order-preserving uint32 key of each
// float find the key of the K-th largest value (smem histogram; lanes that
// hit the same bin combine their increments, since one row's values crowd
// into a few exponent bins).  An order-preserving compaction then emits the
// K selected positions in ascending order - every value above the
// threshold plus the first ties at it - so the result is deterministic.
#pragma once
#include "ptx.cuh"

namespace b200 {
namespace rsel {

constexpr int kThreads = 1024;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive block scan over kThreads threads; returns this thread's prefix
// and writes the block total to *total.
__device__ __forceinline__ int block_excl_scan(int v, int* warp_buf, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_buf[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int w = warp_buf[lane];
    int z = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, z, o);
      if (lane >= o) z += y;
    }
    warp_buf[lane] = z - w;
    if (lane == 31) *total = z;
  }
  __syncthreads();
  const int r = warp_buf[warp] + x - v;
  __syncthreads();
  return r;
}

struct Smem {
  int hist[256];
  int warp_buf[32];
  int total, bin, rem;
};

// Selects the K largest of load(0..n-1) (requires n > K) and calls
// emit(slot, i) for each, slot = 0..K-1 in ascending i.  All threads of the
// block must call it.
template <class Load, class Emit>
__device__ __forceinline__ void select_topk(Load load, int n, int K, Smem& sm, Emit emit) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, mask = 0;
  int remaining = K;
  for (int d = 3; d >= 0; --d) {
    const int shift = 8 * d;
    for (int i = tid; i < 256; i += kThreads) sm.hist[i] = 0;
    __syncthreads();
    for (int i0 = 0; i0 < n; i0 += kThreads) {
      const int i = i0 + tid;
      int bin = -1;
      if (i < n) {
        const uint32_t u = order_key(load(i));
        if ((u & mask) == prefix) bin = (u >> shift) & 255;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (bin >= 0 && (tid & 31) == __ffs(peers) - 1) atomicAdd(&sm.hist[bin], __popc(peers));
    }
    __syncthreads();
    if (tid < 32) {
      // lane l owns bins 255-8l .. 248-8l (descending)
      int c[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = sm.hist[255 - 8 * tid - j];
        sum += c[j];
      }
      int incl = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (tid >= off) incl += y;
      }
      const int above = incl - sum;
      if (above < remaining && remaining <= incl) {
        int acc = above;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (acc < remaining && remaining <= acc + c[j]) {
            sm.bin = 255 - 8 * tid - j;
            sm.rem = remaining - acc;
          }
          acc += c[j];
        }
      }
    }
    __syncthreads();
    prefix |= uint32_t(sm.bin) << shift;
    mask |= 0xFFu << shift;
    remaining = sm.rem;
    __syncthreads();
  }
  // prefix = key of the K-th largest value
  const int per = (n + kThreads - 1) / kThreads;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  int gt = 0, eq = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t u = order_key(load(i));
    gt += u > prefix;
    eq += u == prefix;
  }
  const int eq_before = block_excl_scan(eq, sm.warp_buf, &sm.total);
  const int take_eq = max(0, min(eq, remaining - eq_before));
  int off = block_excl_scan(gt + take_eq, sm.warp_buf, &sm.total);
  int taken = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t u = order_key(load(i));
    if (u > prefix || (u == prefix && taken < take_eq)) {
      if (u == prefix) ++taken;
      if (off < K) emit(off, i);
      ++off;
    }
  }
}

// ---------------------------------------------------------------------------
// Cluster-wide top-K.  A row is split over the C CTAs (C <= 8) of one
// thread-block cluster; each CTA keeps its contiguous slice's keys in shared
// memory, so the four digit passes read shared memory instead of L2.  After
// each pass's local histogram, one cluster barrier makes every CTA's
// histogram visible and each CTA sums the C histograms through distributed
// shared memory and finds the same digit on its own (histograms alternate
// between two buffers, so the next pass zeroes a buffer nobody still reads).
// The compaction offsets each CTA's output by the counts of the ranks before
// it: K positions in ascending order, ties taken lowest index first - the
// same result as select_topk.
struct ClusterSmem {
  int hist[2][256];
  int tot[256];
  int warp_buf[32];
  int total;
  int cnt[2];      // values above / at the threshold in this CTA's slice
  int bin, rem, off, eq_pre;
};

__device__ __forceinline__ int ld_dsmem_s32(uint32_t cluster_addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// keys: this CTA's slice (order keys), m of them, first at row index `base`.
// All threads of all CTAs of the cluster must call it; emit(slot, i) gets
// the row index i = base + local index.
template <class Emit>
__device__ __forceinline__ void cluster_select_topk(const uint32_t* keys, int m, int base, int K, int C, int rank,
                                                    ClusterSmem& sm, Emit emit) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, mask = 0;
  int remaining = K;
  for (int d = 3; d >= 0; --d) {
    const int shift = 8 * d;
    int* h = sm.hist[d & 1];
    for (int i = tid; i < 256; i += kThreads) h[i] = 0;
    __syncthreads();
    for (int i0 = 0; i0 < m; i0 += kThreads) {
      const int i = i0 + tid;
      int bin = -1;
      if (i < m) {
        const uint32_t u = keys[i];
        if ((u & mask) == prefix) bin = (u >> shift) & 255;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (bin >= 0 && (tid & 31) == __ffs(peers) - 1) atomicAdd(&h[bin], __popc(peers));
    }
    cluster_sync();
    for (int i = tid; i < 256; i += kThreads) {
      const uint32_t a = smem_u32(&h[i]);
      int sum = 0;
      for (int r = 0; r < C; ++r) sum += ld_dsmem_s32(mapa_shared(a, r));
      sm.tot[i] = sum;
    }
    __syncthreads();
    if (tid < 32) {
      int c[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = sm.tot[255 - 8 * tid - j];
        sum += c[j];
      }
      int incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += y;
      }
      const int above = incl - sum;
      if (above < remaining && remaining <= incl) {
        int acc = above;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (acc < remaining && remaining <= acc + c[j]) {
            sm.bin = 255 - 8 * tid - j;
            sm.rem = remaining - acc;
          }
          acc += c[j];
        }
      }
    }
    __syncthreads();
    prefix |= uint32_t(sm.bin) << shift;
    mask |= 0xFFu << shift;
    remaining = sm.rem;
  }
  const int per = (m + kThreads - 1) / kThreads;
  const int lo = min(m, tid * per), hi = min(m, lo + per);
  int gt = 0, eq = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t u = keys[i];
    gt += u > prefix;
    eq += u == prefix;
  }
  const int eq_before = block_excl_scan(eq, sm.warp_buf, &sm.total);
  const int eq_cta = sm.total;
  block_excl_scan(gt, sm.warp_buf, &sm.total);
  const int gt_cta = sm.total;
  if (tid == 0) {
    sm.cnt[0] = gt_cta;
    sm.cnt[1] = eq_cta;
  }
  cluster_sync();
  if (tid == 0) {
    int off = 0, e = 0;
    for (int r = 0; r < rank; ++r) {
      const int g = ld_dsmem_s32(mapa_shared(smem_u32(&sm.cnt[0]), r));
      const int q = ld_dsmem_s32(mapa_shared(smem_u32(&sm.cnt[1]), r));
      off += g + max(0, min(q, remaining - e));
      e += q;
    }
    sm.off = off;
    sm.eq_pre = e;
  }
  // the last reads of other CTAs' shared memory are done: after this barrier
  // any CTA may finish
  cluster_sync();
  const int take_eq = max(0, min(eq, remaining - (sm.eq_pre + eq_before)));
  int off = sm.off + block_excl_scan(gt + take_eq, sm.warp_buf, &sm.total);
  int taken = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t u = keys[i];
    if (u > prefix || (u == prefix && taken < take_eq)) {
      if (u == prefix) ++taken;
      if (off < K) emit(off, base + i);
      ++off;
    }
  }
}

}  // namespace rsel
}  // namespace b200
