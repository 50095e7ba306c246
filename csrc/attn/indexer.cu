// Lightning indexer for sparse MLA (DeepSeek-V3.2 style), sm_100a.
//
//   score[t, s] = k_scale[s] * sum_h w'[t, h] * relu(q8[t, h] . k8[s])
//   topk[t]     = the min(K, n) cache positions with the largest scores
//
// q8 / k8 are e4m3 with one fp32 scale per (token, head) / per cached token;
// the query scale is folded into the head weight (relu(a x) = a relu(x) for
// a > 0), so the tensor cores see plain e4m3 x e4m3 products.
//
// Kernels:
//   ix_k_store   LayerNorm + RoPE + e4m3 quantisation of the new keys into the
//                paged indexer cache (one warp per token).
//   ix_q_quant   RoPE + per-(token, head) e4m3 quantisation of the queries and
//                the folded head weights (one warp per (token, head)).
//   ix_score     tcgen05: S^T[128 keys, 64 heads] = K . Q^T per 128-key tile
//                (keys are the MMA M, heads the N), double-buffered in TMEM;
//                the epilogue warps apply relu, the head weights and the key
//                scale and write one fp32 score per key.  Grid = (query,
//                key split) so decode batches still cover the SMs.
//   topk_select  radix select of the K largest scores per query (4 passes of
//                8-bit digits over an smem histogram), then an order-
//                preserving compaction: the output lists positions in
//                ascending order, ties at the threshold resolved towards
//                lower positions, so results are deterministic.
//
// Reference parity: the reference calls DeepGEMM's prefill indexer and the
// serving fork's top-k (ix.py:5-18, ct.py:8-14); these kernels are our own.
#include "../common/ptx.cuh"
#include "../common/radix_select.cuh"
#include <algorithm>

#include "attn.h"

namespace b200 {
namespace ix {

constexpr int kD = 128;          // indexer head dim (bytes per e4m3 key)
// cache pages hold 64 token rows (compressed key caches 64 / r rows, same page ids)
constexpr int kTile = 128;       // keys per MMA tile
constexpr int kThreads = 192;
constexpr int kStages = 4;

__device__ __forceinline__ float ld_val(const void* p, int64_t i, int f32) {
  return f32 ? reinterpret_cast<const float*>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Rotates lane-held pairs (x0, x1) and (x2, x3) = dims 4l..4l+3 when they lie
// inside the first R (rope) dims; table row = [cos(R/2) | sin(R/2)].
__device__ __forceinline__ void rope4(float (&x)[4], int lane, int R, const float* trow) {
  if (4 * lane >= R) return;
  const int half = R >> 1;
#pragma unroll
  for (int pr = 0; pr < 2; ++pr) {
    const int j = 2 * lane + pr;
    const float c = trow[j], s = trow[half + j];
    const float a = x[2 * pr], b = x[2 * pr + 1];
    x[2 * pr] = a * c - b * s;
    x[2 * pr + 1] = a * s + b * c;
  }
}

__global__ void ix_k_store_kernel(const void* k, int f32, int64_t ld, int T, const float* ln_w, const float* ln_b,
                                  float eps, const int* pos, const float* table, int R, const int64_t* slots,
                                  uint8_t* cache, float* scale) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  if (w >= T) return;
  float x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = ld_val(k, (int64_t)w * ld + 4 * lane + i, f32);
  const float mean = warp_sum(x[0] + x[1] + x[2] + x[3]) * (1.f / kD);
  float vs = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) vs += (x[i] - mean) * (x[i] - mean);
  const float rs = rsqrtf(warp_sum(vs) * (1.f / kD) + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = (x[i] - mean) * rs * ln_w[4 * lane + i] + ln_b[4 * lane + i];
  rope4(x, lane, R, table + (int64_t)pos[w] * R);
  float am = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
  am = fmaxf(warp_max(am), 1e-12f);
  const float s = am / 448.f;
  const float inv = 1.f / s;
  const int64_t slot = slots[w];
  const uint32_t lo = f2_to_e4m3x2(x[0] * inv, x[1] * inv), hi = f2_to_e4m3x2(x[2] * inv, x[3] * inv);
  *reinterpret_cast<uint32_t*>(cache + slot * kD + 4 * lane) = lo | (hi << 16);
  if (lane == 0) scale[slot] = s;
}

__global__ void ix_q_quant_kernel(const void* q, int q_f32, int64_t ldq, const void* wraw, int w_f32, int64_t ldw,
                                  int T, int NH, float w_factor, const int* pos, const float* table, int R,
                                  uint8_t* q8, float* wq) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  if (w >= T * NH) return;
  const int t = w / NH, h = w - t * NH;
  float x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = ld_val(q, (int64_t)t * ldq + h * kD + 4 * lane + i, q_f32);
  rope4(x, lane, R, table + (int64_t)pos[t] * R);
  float am = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
  am = warp_max(am);
  const float s = am > 0.f ? am / 448.f : 1.f;
  const float inv = 1.f / s;
  const uint32_t lo = f2_to_e4m3x2(x[0] * inv, x[1] * inv), hi = f2_to_e4m3x2(x[2] * inv, x[3] * inv);
  *reinterpret_cast<uint32_t*>(q8 + (int64_t)w * kD + 4 * lane) = lo | (hi << 16);
  if (lane == 0) wq[w] = ld_val(wraw, (int64_t)t * ldw + h, w_f32) * w_factor * s;
}

// ----------------------------------------------------------------------------
// ix_score: tcgen05 scores
// ----------------------------------------------------------------------------
template <int NH>
struct ScoreSmem {
  static constexpr int kQ = NH * kD;                   // e4m3 [NH x 128], 128B swizzle
  static constexpr int kK = kTile * kD;                // 16 KB per stage
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = ((kQ + 1023) / 1024) * 1024;
  static constexpr int kOffW = kOffK + kStages * kK;   // fp32 head weights
  static constexpr int kOffBar = kOffW + NH * 4;
  static constexpr int kBytes = kOffBar + 256 + 1024;
  static constexpr int kTmemCols = 2 * NH <= 32 ? 32 : 2 * NH <= 64 ? 64 : 2 * NH <= 128 ? 128 : 256;
};

struct ScoreParams {
  const float* wq;          // [T, NH]
  const float* k_scale;     // [slots]
  const int* block_table;
  int bt_stride;
  const int* q_seq;
  const int* q_pos;
  int page;                 // key rows per cache page (64; 64 / r for compressed keys)
  int nsplit;
  float* scores;            // [T, ld]
  int64_t ld;
  uint32_t* err;
};

template <int NH>
__global__ void __launch_bounds__(kThreads, 1)
ix_score_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k, ScoreParams p) {
  using S = ScoreSmem<NH>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm + S::kOffQ;
  uint8_t* sK = sm + S::kOffK;
  float* sW = reinterpret_cast<float*>(sm + S::kOffW);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* k_full = bars;                  // [kStages]
  uint64_t* k_empty = bars + kStages;       // [kStages]
  uint64_t* q_full = bars + 2 * kStages;
  uint64_t* acc_full = q_full + 1;          // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = warp_id(), lane = lane_id();
  const int t = blockIdx.x, split = blockIdx.y;
  pdl_wait();
  pdl_launch_dependents();
  const int b = p.q_seq[t];
  const int n = p.q_pos[t] + 1;
  const int chunk = (((n + p.nsplit - 1) / p.nsplit) + kTile - 1) / kTile * kTile;
  const int k_lo = split * chunk;
  const int k_hi = min(n, k_lo + chunk);
  const int nt = k_hi > k_lo ? (k_hi - k_lo + kTile - 1) / kTile : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < NH; i += kThreads) sW[i] = p.wq[(int64_t)t * NH + i];
  if (warp == 1) {
    tmem_alloc(tmem_holder, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0 && nt > 0) {
      mbar_arrive_expect_tx(q_full, S::kQ);
      tma_load_2d(sQ, &tm_q, q_full, 0, t * NH);
      for (int i = 0; i < nt; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(&k_empty[s], ((i / kStages) - 1) & 1, p.err)) break;
        mbar_arrive_expect_tx(&k_full[s], S::kK);
        const int tok0 = k_lo + i * kTile;
        for (int pg = 0; pg < kTile / p.page; ++pg) {
          const int tk = tok0 + pg * p.page;
          const int page = tk < n ? p.block_table[(int64_t)b * p.bt_stride + tk / p.page] : 0;
          tma_load_2d(sK + s * S::kK + pg * p.page * kD, &tm_k, &k_full[s], 0, page * p.page);
        }
      }
    }
  } else if (warp == 1) {
    const uint32_t idesc = idesc_f8(128, NH, false, false);
    bool ok = nt > 0 && mbar_wait(q_full, 0, p.err);
    for (int i = 0; ok && i < nt; ++i) {
      const int s = i % kStages;
      const int a = i & 1;
      if (!mbar_wait(&k_full[s], (i / kStages) & 1, p.err)) break;
      if (i >= 2 && !mbar_wait(&acc_empty[a], ((i >> 1) - 1) & 1, p.err)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t kb = smem_u32(sK + s * S::kK), qb = smem_u32(sQ);
#pragma unroll
        for (int kk = 0; kk < kD / 32; ++kk)
          mma_f8(tmem + a * NH, desc_kmajor_sw128(kb + kk * 32), desc_kmajor_sw128(qb + kk * 32), idesc, kk > 0 ? 1u : 0u);
        mma_commit(&k_empty[s]);
        mma_commit(&acc_full[a]);
      }
      __syncwarp();
    }
  } else {
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    for (int i = 0; i < nt; ++i) {
      const int a = i & 1;
      if (!mbar_wait(&acc_full[a], (i >> 1) & 1, p.err)) break;
      tc_fence_after();
      const uint32_t base = tmem + a * NH + (uint32_t(sub * 32) << 16);
      float acc = 0.f;
#pragma unroll
      for (int c0 = 0; c0 < NH; c0 += 16) {
        uint32_t r[16];
        tmem_ld_x16(base + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) acc += fmaxf(__uint_as_float(r[j]), 0.f) * sW[c0 + j];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      const int key = k_lo + i * kTile + row;
      if (key < k_hi) {
        const int64_t slot = (int64_t)p.block_table[(int64_t)b * p.bt_stride + key / p.page] * p.page + key % p.page;
        p.scores[(int64_t)t * p.ld + key] = acc * p.k_scale[slot];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// ----------------------------------------------------------------------------
// topk_select
// ----------------------------------------------------------------------------
constexpr int kTopkThreads = rsel::kThreads;

__global__ void __launch_bounds__(kTopkThreads)
topk_select_kernel(const float* scores, int64_t ld, const int* q_pos, int K, int* out) {
  __shared__ rsel::Smem sm;
  const int t = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  const int n = q_pos[t] + 1;
  int* o = out + (int64_t)t * K;
  if (n <= K) {
    for (int i = threadIdx.x; i < K; i += kTopkThreads) o[i] = i < n ? i : -1;
    return;
  }
  const float* sc = scores + (int64_t)t * ld;
  rsel::select_topk([&](int i) { return __ldcg(sc + i); }, n, K, sm, [&](int slot, int i) { o[slot] = i; });
}

// Cluster variant: grid (C, T), one cluster of C CTAs per row; each CTA
// stages its slice of at most `cap` scores as order keys in shared memory.
// Rows longer than C * cap (a bound the host sized from the longest row it
// knows of) fall back to the one-CTA select over global memory.
__global__ void __launch_bounds__(kTopkThreads)
topk_cluster_kernel(const float* scores, int64_t ld, const int* q_pos, int K, int C, int cap, int* out) {
  extern __shared__ __align__(16) uint32_t keys[];
  __shared__ rsel::ClusterSmem sm;
  __shared__ rsel::Smem sm1;
  const int t = blockIdx.y;
  const int rank = int(cluster_ctarank());
  pdl_wait();
  pdl_launch_dependents();
  const int n = q_pos[t] + 1;          // uniform over the cluster: early exits skip no barrier
  int* o = out + (int64_t)t * K;
  const float* sc = scores + (int64_t)t * ld;
  if (n <= K) {
    if (rank == 0)
      for (int i = threadIdx.x; i < K; i += kTopkThreads) o[i] = i < n ? i : -1;
    return;
  }
  const int chunk = (n + C - 1) / C;
  if (chunk > cap) {
    if (rank == 0)
      rsel::select_topk([&](int i) { return __ldcg(sc + i); }, n, K, sm1, [&](int slot, int i) { o[slot] = i; });
    return;
  }
  const int lo = rank * chunk;
  const int m = max(0, min(n, lo + chunk) - lo);
  for (int i = threadIdx.x; i < m; i += kTopkThreads) keys[i] = rsel::order_key(__ldcg(sc + lo + i));
  __syncthreads();
  rsel::cluster_select_topk(keys, m, lo, K, C, rank, sm, [&](int slot, int i) { o[slot] = i; });
}

// ----------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

static int map_rows128(CUtensorMap* m, const void* base, int64_t rows, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kD};
  cuuint32_t box[2] = {(cuuint32_t)kD, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

}  // namespace ix
}  // namespace b200

int b200_ix_k_store(const void* k, int f32, int64_t ld, int T, const float* ln_w, const float* ln_b, float eps,
                    const int* pos, const float* table, int R, const int64_t* slots, uint8_t* cache, float* scale,
                    cudaStream_t st) {
  if (T <= 0) return 0;
  if (R > 64 || (R & 3)) return -1;
  b200::launch_pdl(b200::ix::ix_k_store_kernel, dim3((T * 32 + 127) / 128), dim3(128), 0, st, k, f32, ld, T, ln_w,
                   ln_b, eps, pos, table, R, slots, cache, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_ix_q_quant(const void* q, int q_f32, int64_t ldq, const void* wraw, int w_f32, int64_t ldw, int T, int NH,
                    float w_factor, const int* pos, const float* table, int R, uint8_t* q8, float* wq, cudaStream_t st) {
  if (T <= 0) return 0;
  if (R > 64 || (R & 3)) return -1;
  b200::launch_pdl(b200::ix::ix_q_quant_kernel, dim3((T * NH * 32 + 127) / 128), dim3(128), 0, st, q, q_f32, ldq,
                   wraw, w_f32, ldw, T, NH, w_factor, pos, table, R, q8, wq);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_ix_score(const uint8_t* q8, const float* wq, int T, int NH, const uint8_t* k_cache, int64_t cache_rows,
                  const float* k_scale, const int* block_table, int bt_stride, const int* q_seq, const int* q_pos,
                  int page_size, int nsplit, float* scores, int64_t ld, uint32_t* err, cudaStream_t st) {
  using namespace b200::ix;
  if (T <= 0) return 0;
  // page_size: key rows per page (64; 32 / 16 / 8 for keys compressed 2x /
  // 4x / 8x, paged with the same page ids); a 128-key tile loads 128 /
  // page_size boxes, each a whole number of 1 KB swizzle atoms
  if (page_size < 8 || 64 % page_size || NH != 64 || nsplit < 1) return -1;
  using S = ScoreSmem<64>;
  CUtensorMap mq, mk;
  if (map_rows128(&mq, q8, (int64_t)T * NH, NH)) return -2;
  if (map_rows128(&mk, k_cache, cache_rows, page_size)) return -3;
  ScoreParams p{};
  p.page = page_size;
  p.wq = wq;
  p.k_scale = k_scale;
  p.block_table = block_table;
  p.bt_stride = bt_stride;
  p.q_seq = q_seq;
  p.q_pos = q_pos;
  p.nsplit = nsplit;
  p.scores = scores;
  p.ld = ld;
  p.err = err;
  auto kern = ix_score_kernel<64>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
  b200::launch_pdl(kern, dim3(T, nsplit), dim3(kThreads), S::kBytes, st, mq, mk, p);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_topk_select(const float* scores, int64_t ld, const int* q_pos, int T, int K, int* out, cudaStream_t st,
                     int max_n) {
  if (T <= 0) return 0;
  if (K <= 0) return -1;
  // cluster of C CTAs per row, about 4K scores (16 KB of keys) each
  constexpr int kMaxC = 8, kPerCta = 4096, kMaxSmem = 200 * 1024;
  const int C = std::min(kMaxC, std::max(1, (max_n + kPerCta - 1) / kPerCta));
  const int cap = ((max_n + C - 1) / C + 3) & ~3;
  if (max_n <= K || C < 2 || cap * 4 > kMaxSmem) {
    b200::launch_pdl(b200::ix::topk_select_kernel, dim3(T), dim3(b200::ix::kTopkThreads), 0, st, scores, ld, q_pos,
                     K, out);
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
  }
  auto kern = b200::ix::topk_cluster_kernel;
  const size_t smem = size_t(cap) * 4;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, T);
  cfg.blockDim = dim3(b200::ix::kTopkThreads);
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
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, scores, ld, q_pos, K, C, cap, out);
  return err == cudaSuccess ? 0 : 1000 + int(err);
}
