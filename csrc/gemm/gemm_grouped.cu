// Persistent grouped MXFP8 GEMM for the routed experts (sm_100a, tcgen05).
//
// One CTA per SM walks a device-built tile list: tile w covers weight rows
// [128 n, 128 n + 128) of expert e and sorted token rows [seg_start[e] +
// BN tt, +BN).  The producer warp streams k-tiles continuously across the
// CTA's tiles (no pipeline drain between tiles, weights fetched with an L2
// evict-first hint), the MMA warp accumulates into one of two TMEM buffers,
// and the four epilogue warps drain the other buffer meanwhile.
//
//   FC1 (kEpiSwiglu):       h = mxfp8(silu(x Wg^T) * (x Wu^T))   gate/up tiles in
//                           two TMEM column ranges, one warp = one 32-channel
//                           scale block
//   FC2 (kEpiWeightedBf16): y[r] = bf16(routing_weight[r] * (h Wd^T)[r])
//
// NVFP4 variant (FP4 = true, kind::mxf4nvf4 with 16-element e4m3 scales):
// the same 128-byte k-tiles now hold 256 e2m1 elements (4 MMAs of K = 64),
// each MMA reads its own 512-byte scale chunk (4 per k-tile and operand,
// staged through a 4-slot TMEM ring), the epilogue applies the fp32 global
// scales (per expert x per token row), and FC1 requantizes its SwiGLU output
// to NVFP4 (16-channel blocks = 16 lanes of an epilogue warp).
//
// The tile list comes from the routing-layout kernel: ttile_off[e] is the
// prefix sum over experts of ceil(count_e / BN).  All waits are bounded.
//
// Reference parity: routed experts run FlashInfer trtllm-gen NVFP4 FC1/FC2
// kernels in the reference (mo.py:19-40, moet.py:5-12, rr.py:1-15).
#include "../common/ptx.cuh"
#include "gemm_mxf8.h"

namespace b200 {
namespace ggemm {

constexpr int kThreads = 192;
constexpr int kTileM = 128;
constexpr int kTileK = 128;
constexpr int kSf = 512;

template <int BN, int EPI, bool FP4>
struct Cfg {
  static constexpr int kA = (EPI == kEpiSwiglu) ? 2 : 1;
  static constexpr int kSfK = FP4 ? 4 * kSf : kSf;          // scale bytes per 128 rows per k-tile
  static constexpr int kLoadBytes = kA * kTileM * kTileK + BN * kTileK + kA * kSfK + kSfK;   // TMA bytes per stage
  static constexpr int kStageBytes = kLoadBytes + kSfK;   // + padding after the activation scale chunks
  static constexpr int kAcc = kA * BN;                      // columns per accumulator buffer
  static constexpr int kSlotCols = FP4 ? 16 * kA + 16 : 4 * kA + 4;   // scale columns per stage
  // Two accumulator buffers (the epilogue drains one while the MMAs fill the
  // other) when they leave TMEM room for four scale slots; the wide prefill
  // tiles (FC1 gate + up at 128 tokens, FC2 at 256) keep one.
  static constexpr int kBufs = (2 * kAcc + 4 * kSlotCols <= 512) ? 2 : 1;
  // Stages bounded by shared memory and by TMEM (one scale slot per stage, so
  // a slot is rewritten only after its stage's MMAs released the stage).
  static constexpr int kStagesSmem = (208 * 1024) / kStageBytes;
  static constexpr int kStagesTmem = (512 - kBufs * kAcc) / kSlotCols;
  static constexpr int kStages0 = kStagesSmem < kStagesTmem ? kStagesSmem : kStagesTmem;
  static constexpr int kStages = kStages0 > 16 ? 16 : kStages0;
  static constexpr int kSfSlots = kStages;
  static constexpr int kSfCols = kSfSlots * kSlotCols;
  static constexpr int kNeed = kBufs * kAcc + kSfCols;
  static constexpr int kTmemCols = kNeed <= 32 ? 32 : kNeed <= 64 ? 64 : kNeed <= 128 ? 128 : kNeed <= 256 ? 256 : 512;
  static_assert(kNeed <= 512, "TMEM budget");
  static_assert(kStages >= 2, "pipeline depth");
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 512;
};

struct Params {
  const uint8_t* sfa;
  int64_t sfa_estride;
  const uint8_t* sfb;
  int nw;                    // weight rows per expert (FC1: 2*inter, FC2: hidden)
  int n_tiles;               // output-row tiles per expert (FC1: inter/128, FC2: hidden/128)
  int k;
  int E;
  const int* seg_start;
  const int* seg_count;
  const int* ttile_off;      // [E+1]
  void* out;
  int ldo;
  uint8_t* q_out;
  uint8_t* sf_out;
  int ldq;
  int inter;
  const float* row_weight;
  uint32_t* err;
  const float* w_g;          // NVFP4: per-expert global scale
  const float* x_g;          // NVFP4: per-row activation global scale (or null)
  float x_g_const;
  float out_g;               // NVFP4 FC1: global scale of the requantized output
  int a_tiled;               // weights stored as contiguous 128 x 128-byte tiles (3-D tensor map)
};

__device__ __forceinline__ int64_t sf_offset(int row, int kblock, int kb_total) {
  const int rb = row >> 7, r = row & 127, kc = kblock >> 2, c = kblock & 3;
  return ((int64_t)(rb * (kb_total >> 2) + kc) << 9) + ((r & 31) << 4) + ((r >> 5) << 2) + c;
}

// Work tile: expert e, output-row tile tile_n, token tile tt of that expert.
struct Tile {
  int e, tile_n, tt, rows;
};


// Tiles are ordered (expert, token tile) major, output-row tile minor, so
// CTAs running at the same time share the expert's activation rows in L2.
// The routing layout (tile offsets, segment starts / counts) is staged in
// shared memory once per CTA: sm_lay[0..E] = ttile_off, [E+1..2E] =
// seg_start, [2E+1..3E] = seg_count.
constexpr int kMaxExperts = 512;   // local experts per GPU (V4.1-Flash: 384 on one GPU)
__device__ __forceinline__ Tile map_tile(const Params& p, const int* lay, int w) {
  Tile t;
  const int ttg = w / p.n_tiles;
  t.tile_n = w - ttg * p.n_tiles;
  int lo = 0, hi = p.E;   // e with ttile_off[e] <= ttg < ttile_off[e+1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (lay[mid] <= ttg) lo = mid; else hi = mid;
  }
  t.e = lo;
  t.tt = ttg - lay[lo];
  t.rows = lay[2 * p.E + 1 + lo];
  return t;
}

template <int BN, int EPI, bool FP4>
__global__ void __launch_bounds__(kThreads, 1)
grouped_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, Params p) {
  using C = Cfg<BN, EPI, FP4>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::kStages * C::kA * kTileM * kTileK;
  uint8_t* sSFA = sB + C::kStages * BN * kTileK;
  uint8_t* sSFB = sSFA + C::kStages * C::kA * C::kSfK;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + C::kStages * 2 * C::kSfK);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;    // [2]
  uint64_t* acc_empty = acc_full + 2;         // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
  __shared__ int lay[3 * kMaxExperts + 1];

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t tmem_sf = tmem + C::kBufs * C::kAcc;

  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();   // dependents wait for this grid's completion
  for (int i = threadIdx.x; i <= p.E; i += blockDim.x) lay[i] = __ldcg(p.ttile_off + i);
  for (int i = threadIdx.x; i < p.E; i += blockDim.x) {
    lay[p.E + 1 + i] = __ldcg(p.seg_start + i);
    lay[2 * p.E + 1 + i] = __ldcg(p.seg_count + i);
  }
  __syncthreads();
  const int total = lay[p.E] * p.n_tiles;
  const int kbytes = FP4 ? p.k / 2 : p.k;      // operand bytes per row
  const int nk = kbytes / kTileK;
  const int kc_total = FP4 ? p.k / 64 : p.k / kTileK;   // 512-byte sf chunks per 128 rows
  constexpr int kChunksPerTile = FP4 ? 4 : 1;

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      constexpr uint32_t bytes = C::kLoadBytes;
      int it = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < total; w += gridDim.x) {
        const Tile t = map_tile(p, lay, w);
        const int e = t.e;
        const int a_row = e * p.nw + t.tile_n * kTileM;
        const int b_row = lay[p.E + 1 + e] + t.tt * BN;
        const uint8_t* sfa_e = p.sfa + (int64_t)e * p.sfa_estride;
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % C::kStages;
          if (it >= C::kStages && !mbar_wait(&empty[s], ((it / C::kStages) - 1) & 1, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], bytes);
          uint8_t* a_dst = sA + (size_t)s * C::kA * kTileM * kTileK;
          if (p.a_tiled) {
            // tile (row block, k-tile) = one contiguous 16 KB block
            tma_load_3d_hint(a_dst, &tm_a, &full[s], 0, 0, (a_row >> 7) * nk + kt, pol_w);
            if (EPI == kEpiSwiglu)
              tma_load_3d_hint(a_dst + kTileM * kTileK, &tm_a, &full[s], 0, 0, ((a_row + p.inter) >> 7) * nk + kt,
                               pol_w);
          } else {
            tma_load_2d_hint(a_dst, &tm_a, &full[s], kt * kTileK, a_row, pol_w);
            if (EPI == kEpiSwiglu)
              tma_load_2d_hint(a_dst + kTileM * kTileK, &tm_a, &full[s], kt * kTileK, a_row + p.inter, pol_w);
          }
          tma_load_2d_hint(sB + (size_t)s * BN * kTileK, &tm_b, &full[s], kt * kTileK, b_row, pol_x);
          uint8_t* sfa_dst = sSFA + (size_t)s * C::kA * C::kSfK;
          const int kc0 = kt * kChunksPerTile;
          bulk_load_hint(sfa_dst, sfa_e + ((int64_t)(t.tile_n * kc_total + kc0) << 9), C::kSfK, &full[s], pol_w);
          if (EPI == kEpiSwiglu) {
            const int rb_up = (p.inter + t.tile_n * kTileM) >> 7;
            bulk_load_hint(sfa_dst + C::kSfK, sfa_e + ((int64_t)(rb_up * kc_total + kc0) << 9), C::kSfK, &full[s],
                           pol_w);
          }
          bulk_load_hint(sSFB + (size_t)s * 2 * C::kSfK, p.sfb + ((int64_t)((b_row >> 7) * kc_total + kc0) << 9),
                         C::kSfK, &full[s], pol_x);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    int it = 0, c = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < total; w += gridDim.x, ++c) {
      const Tile t = map_tile(p, lay, w);
      const int b_row = lay[p.E + 1 + t.e] + t.tt * BN;
      const int buf = c % C::kBufs;
      if (c >= C::kBufs && !mbar_wait(&acc_empty[buf], ((c / C::kBufs) - 1) & 1, p.err)) { ok = false; break; }
      tc_fence_after();
      const uint32_t acc = tmem + buf * C::kAcc;
      for (int kt = 0; kt < nk; ++kt, ++it) {
        const int s = it % C::kStages;
        if (!mbar_wait(&full[s], (it / C::kStages) & 1, p.err)) { ok = false; break; }
        tc_fence_after();
        // Activation scales of this token tile: rows o..o+BN-1 of the
        // 128-row scale chunk (o = b_row % 128).  When o != 0 the warp
        // repacks them into a tile-local chunk (row j -> line j % 32, byte
        // group j / 32) so the MMA always reads scales at the base column.
        const int o = b_row & 127;
        uint8_t* sfb_stage = sSFB + (size_t)s * 2 * C::kSfK;
        if (o != 0) {
          for (int ch = 0; ch < kChunksPerTile; ++ch)
            for (int j = lane; j < BN; j += 32) {
              const int r = o + j;
              const uint32_t v =
                  *reinterpret_cast<const uint32_t*>(sfb_stage + ch * kSf + (r & 31) * 16 + (r >> 5) * 4);
              *reinterpret_cast<uint32_t*>(sfb_stage + C::kSfK + ch * kSf + (j & 31) * 16 + (j >> 5) * 4) = v;
            }
          fence_proxy_async_smem();
          __syncwarp();
        }
        if (lane == 0) {
          const uint32_t sf_a = tmem_sf + (it % C::kSfSlots) * C::kSlotCols;
          const uint32_t sf_b = sf_a + 4 * kChunksPerTile * C::kA;
          const uint8_t* sfa_src = sSFA + (size_t)s * C::kA * C::kSfK;
          const uint8_t* sfb_src = sfb_stage + (o != 0 ? C::kSfK : 0);
          for (int a = 0; a < C::kA; ++a)
            for (int ch = 0; ch < kChunksPerTile; ++ch)
              tmem_cp_32x128b_x4(sf_a + 4 * (a * kChunksPerTile + ch),
                                 smem_desc(smem_u32(sfa_src + a * C::kSfK + ch * kSf), 0, 128, 0));
          for (int ch = 0; ch < kChunksPerTile; ++ch)
            tmem_cp_32x128b_x4(sf_b + 4 * ch, smem_desc(smem_u32(sfb_src + ch * kSf), 0, 128, 0));
          const uint32_t a_base = smem_u32(sA + (size_t)s * C::kA * kTileM * kTileK);
          const uint32_t b_base = smem_u32(sB + (size_t)s * BN * kTileK);
          for (int kk = 0; kk < kTileK / 32; ++kk) {
            const uint64_t bdesc = desc_kmajor_sw128(b_base + kk * 32);
            const uint32_t accf = (kt > 0 || kk > 0) ? 1u : 0u;
            for (int a = 0; a < C::kA; ++a) {
              const uint64_t adesc = desc_kmajor_sw128(a_base + a * kTileM * kTileK + kk * 32);
              if constexpr (FP4) {
                // MMA kk (64 elements) reads scale chunk kk: its own 4 columns
                mma_nvf4(acc + a * BN, adesc, bdesc, idesc_nvf4(kTileM, BN),
                         sf_a + 4 * (a * kChunksPerTile + kk), sf_b + 4 * kk, accf);
              } else {
                mma_mxf8(acc + a * BN, adesc, bdesc, idesc_mxf8(kTileM, BN, kk, kk),
                         (sf_a + 4 * a) | (uint32_t(kk) << 30), sf_b | (uint32_t(kk) << 30), accf);
              }
            }
          }
          mma_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (ok && lane == 0) mma_commit(&acc_full[buf]);
      __syncwarp();
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    const int sub = warp & 3;
    const int tid = threadIdx.x - 64;
    int c = 0;
    const int kb_out = p.ldq / 32;
    for (int w = blockIdx.x; w < total; w += gridDim.x, ++c) {
      const Tile t = map_tile(p, lay, w);
      const int buf = c % C::kBufs;
      if (!mbar_wait(&acc_full[buf], (c / C::kBufs) & 1, p.err)) break;
      tc_fence_after();
      const int b_row = lay[p.E + 1 + t.e] + t.tt * BN;
      const int tmax = t.rows - t.tt * BN;
      const int wrow = t.tile_n * kTileM + sub * 32 + lane;
      const uint32_t lane_addr = tmem + buf * C::kAcc + (uint32_t(sub * 32) << 16);
      const float wg = FP4 ? __ldcg(p.w_g + t.e) : 1.f;
      if constexpr (FP4 && EPI == kEpiSwiglu) {
        // h = silu(g) * u with both scaled by the global scales; NVFP4 out:
        // one 16-channel block per half-warp, two channels per byte.
        const float inv_og = 1.f / p.out_g;
        const int kb16 = p.inter / 16;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t g[16], u[16];
          tmem_ld_x16(lane_addr + c0, g);
          tmem_ld_x16(lane_addr + BN + c0, u);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int orow = b_row + c0 + j;
            const float sc = wg * (p.x_g ? __ldcg(p.x_g + orow) : p.x_g_const);
            const float gv = __uint_as_float(g[j]) * sc;
            const float h = gv / (1.0f + __expf(-gv)) * (__uint_as_float(u[j]) * sc);
            float amax = fabsf(h);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const uint16_t s2 = f2_to_e4m3x2(amax * (1.f / 6.f) * inv_og, 0.f);
            __nv_fp8_e4m3 s8;
            s8.__x = uint8_t(s2 & 0xFF);
            const float sf = float(s8);
            const float v = sf > 0.f ? h * inv_og / sf : 0.f;
            const float vn = __shfl_down_sync(0xffffffffu, v, 1);
            if (c0 + j < tmax) {
              if ((lane & 1) == 0) p.q_out[(int64_t)orow * (p.ldq / 2) + (wrow >> 1)] = uint8_t(f2_to_e2m1x2(v, vn));
              if ((lane & 15) == 0) p.sf_out[sf_offset(orow, wrow >> 4, kb16)] = uint8_t(s2 & 0xFF);
            }
          }
        }
      } else if constexpr (EPI == kEpiSwiglu) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t g[16], u[16];
          tmem_ld_x16(lane_addr + c0, g);
          tmem_ld_x16(lane_addr + BN + c0, u);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float gv = __uint_as_float(g[j]);
            const float h = gv / (1.0f + __expf(-gv)) * __uint_as_float(u[j]);
            float amax = fabsf(h);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const int ex = ceil_log2_bits(amax * (1.0f / 448.0f));
            if (c0 + j < tmax) {
              const int orow = b_row + c0 + j;
              p.q_out[(int64_t)orow * p.ldq + wrow] = uint8_t(f2_to_e4m3x2(h * exp2_int(-ex), 0.f) & 0xFF);
              if (lane == 0) p.sf_out[sf_offset(orow, wrow >> 5, kb_out)] = uint8_t(ex + 127);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld_x16(lane_addr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (c0 + j < tmax) {
              const int orow = b_row + c0 + j;
              float v = __uint_as_float(r[j]) * __ldcg(p.row_weight + orow);
              if (FP4) v *= wg * (p.x_g ? __ldcg(p.x_g + orow) : p.x_g_const);
              reinterpret_cast<__nv_bfloat16*>(p.out)[(int64_t)orow * p.ldo + wrow] = __float2bfloat16(v);
            }
          }
        }
      }
      tc_fence_before();
      named_barrier(1, 128);
      if (tid == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encoder() {
  static EncodeTiledFn enc = nullptr;
  if (!enc) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    enc = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return enc;
}

// Tiled weights: [blocks][128 rows][128 bytes] with blocks = rows/128 * cols/128.
static int map_u8_tiled(CUtensorMap* m, const void* base, int64_t rows, int64_t cols) {
  EncodeTiledFn enc = encoder();
  if (!enc) return -1;
  cuuint64_t dims[3] = {128u, 128u, (cuuint64_t)((rows / 128) * (cols / 128))};
  cuuint64_t strides[2] = {128u, 128u * 128u};
  cuuint32_t box[3] = {128u, 128u, 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

static int map_u8(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn enc = encoder();
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

template <int BN, int EPI, bool FP4>
static int launch(const GroupedArgs& a, cudaStream_t st) {
  using C = Cfg<BN, EPI, FP4>;
  CUtensorMap ma, mb;
  const int kbytes = FP4 ? a.k / 2 : a.k;
  if (a.a_tiled ? map_u8_tiled(&ma, a.w, (int64_t)a.E * a.nw, kbytes)
                : map_u8(&ma, a.w, (int64_t)a.E * a.nw, kbytes, kTileM))
    return -2;
  if (map_u8(&mb, a.x, a.x_rows, kbytes, BN)) return -3;
  Params p{};
  p.sfa = a.w_sf;
  p.sfa_estride = a.w_sf_estride;
  p.sfb = a.x_sf;
  p.nw = a.nw;
  p.n_tiles = (EPI == kEpiSwiglu ? a.inter : a.nw) / kTileM;
  p.k = a.k;
  p.E = a.E;
  p.seg_start = a.seg_start;
  p.seg_count = a.seg_count;
  p.ttile_off = a.ttile_off;
  p.out = a.out;
  p.ldo = a.ldo;
  p.q_out = a.q_out;
  p.sf_out = a.sf_out;
  p.ldq = a.ldq;
  p.inter = a.inter;
  p.row_weight = a.row_weight;
  p.err = a.err;
  p.w_g = a.w_g;
  p.x_g = a.x_g;
  p.x_g_const = a.x_g_const;
  p.out_g = a.out_g;
  p.a_tiled = a.a_tiled;
  auto kern = grouped_kernel<BN, EPI, FP4>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.num_ctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (a.pdl && b200::pdl_enabled()) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, ma, mb, p) == cudaSuccess ? 0 : 1;
}

template <int EPI, bool FP4>
static int launch_bn(const GroupedArgs& a, cudaStream_t st) {
  switch (a.bn) {
    case 16: return launch<16, EPI, FP4>(a, st);
    case 32: return launch<32, EPI, FP4>(a, st);
    case 64: return launch<64, EPI, FP4>(a, st);
    case 128: return launch<128, EPI, FP4>(a, st);
  }
  return -4;
}

}  // namespace ggemm
}  // namespace b200

int b200_gemm_grouped(const GroupedArgs* a, cudaStream_t st) {
  using namespace b200::ggemm;
  if (a->k % 128 || a->nw % 128 || a->num_ctas <= 0 || a->E > b200::ggemm::kMaxExperts) return -1;
  if (a->fp4) {
    if (a->k % 256 || !a->w_g || (a->epi == kEpiSwiglu && (a->out_g <= 0.f || a->inter % 128))) return -1;
    if (a->epi == kEpiSwiglu) return launch_bn<kEpiSwiglu, true>(*a, st);
    if (a->epi == kEpiWeightedBf16) return launch_bn<kEpiWeightedBf16, true>(*a, st);
    return -5;
  }
  if (a->epi == kEpiSwiglu) return launch_bn<kEpiSwiglu, false>(*a, st);
  if (a->epi == kEpiWeightedBf16) return launch_bn<kEpiWeightedBf16, false>(*a, st);
  return -5;
}
