// Batched bf16 GEMM on tcgen05 (sm_100a) for the MLA weight absorptions,
// weight-stationary "swap-AB" like the MXFP8 GEMM:
//
//   D^T[b][M, T] = A[b][M, K] . X[b][T, K]^T      (A: per-head weight, X: tokens)
//
// with 128-row weight tiles as the MMA M, the tokens as N (BN = 16..128),
// kind::f16 MMAs (bf16 in, fp32 accumulate in TMEM), 3-D TMA boxes so X may be
// any strided view (a head's slice of a projection output).  Epilogues:
//
//   kBf16Store   out[t * ot + b * ob + m] = bf16(acc)
//   kQPrep       absorb_q fused with the attention's query prep: one CTA
//                holds all four 128-row tiles of the 512-dim latent of its
//                head, so per (token, head) it applies RoPE to the un-rotated
//                rope part, takes the amax over the 576 values and writes the
//                e4m3 query + fp32 scale the MLA kernel consumes;
//   kMxfp8Rows   absorb_o fused with the output projection's MXFP8 quant:
//                batch b's M rows are columns [M b, M b + M) of the output
//                projection's operand row (V3: value absorption per head,
//                M = 128; V4: grouped low-rank wo_a per head group, M = rank);
//                a warp's 32 lanes are one UE8M0 block.
//
// Warp roles: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 2-5
// epilogue.  All waits are bounded.
//
// Reference parity: the reference runs the weight absorptions as DeepGEMM
// fp8 einsums / strided cuBLAS bmm (fork_attn.py:482-513, rt.py:20-40).
#include "../common/ptx.cuh"
#include "gemm_mxf8.h"

namespace b200 {
namespace bgemm {

constexpr int kThreads = 192;
constexpr int kTileM = 128;
constexpr int kTileKB = 128;      // bytes of K per stage (64 bf16)
constexpr int kStages = 4;

enum : int { kBf16Store = 0, kQPrep = 1, kMxfp8Rows = 2, kF32Atomic = 3 };

template <int BN, int MT>
struct Cfg {
  static constexpr int kA = kTileM * kTileKB;        // 16 KB
  static constexpr int kB = BN * kTileKB;
  static constexpr int kStage = kA + kB;
  static constexpr int kAcc = MT * BN;
  static constexpr int kTmemCols = kAcc <= 32 ? 32 : kAcc <= 64 ? 64 : kAcc <= 128 ? 128 : kAcc <= 256 ? 256 : 512;
  static_assert(kAcc <= 512, "TMEM");
  static constexpr int kRope = BN * 64 * 4 + BN * 4;  // roped q_pe (fp32) + per-token amax
  static constexpr int kSmem = kStages * kStage + kRope + 1024 + 256;
};

struct Params {
  int T, K, M;               // tokens, reduction, weight rows per batch (M = MT * 128 per CTA)
  // kBf16Store
  __nv_bfloat16* out;
  int64_t ot, ob;
  // kQPrep
  const __nv_bfloat16* q_pe; // un-rotated rope part, strided [T, B, 64]
  int64_t pe_t, pe_b;
  const int* pos;
  const float* table;        // [P, 64] cos | sin
  uint8_t* q8;               // e4m3 [T, B, 576]
  float* qs;                 // [T, B]
  int B;
  // kMxfp8Rows
  uint8_t* q;                // e4m3 [T, B * 128]
  uint8_t* sf;               // tcgen05 scale layout, K = B * 128
  // kF32Atomic (split-K): out_f32[t * ot + m] += partial over this CTA's k-range
  float* out_f32;
  int splits;
  uint32_t* err;
};

__device__ __forceinline__ int64_t sf_offset(int row, int kblock, int kb_total) {
  const int rb = row >> 7, r = row & 127, kc = kblock >> 2, c = kblock & 3;
  return ((int64_t)(rb * (kb_total >> 2) + kc) << 9) + ((r & 31) << 4) + ((r >> 5) << 2) + c;
}

template <int BN, int MT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
bf16_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_x, Params p) {
  using C = Cfg<BN, MT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = sm;
  uint8_t* sB = sA + kStages * C::kA;
  float* sRope = reinterpret_cast<float*>(sB + kStages * C::kB);     // [BN][64]
  float* sRmax = sRope + BN * 64;                                     // [BN] (float bits via atomicMax)
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sRope) + C::kRope);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_full + 1);
  __shared__ float red[4][16];

  const int warp = warp_id(), lane = lane_id();
  const int b = blockIdx.x;               // batch (head)
  const int t0 = blockIdx.y * BN;         // first token
  const int split = blockIdx.z % p.splits;
  const int m0 = (blockIdx.z / p.splits) * MT;   // first 128-row tile
  const int nk_all = p.K * 2 / kTileKB;
  const int nk_per = (nk_all + p.splits - 1) / p.splits;
  const int k_lo = split * nk_per;
  const int nk = max(0, min(nk_all, k_lo + nk_per) - k_lo);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int iters = MT * nk;

  if (warp == 0) {
    if (lane == 0) {
      // weights are constants: the first stages load before the PDL wait
      const uint64_t pol_w = policy_evict_first();
      for (int i = 0; i < iters; ++i) {
        const int s = i % kStages;
        const int mt = i / nk, kt = i - mt * nk;
        if (i >= kStages && !mbar_wait(&empty[s], ((i / kStages) - 1) & 1, p.err)) break;
        mbar_arrive_expect_tx(&full[s], C::kStage);
        tma_load_3d_hint(sA + s * C::kA, &tm_a, &full[s], (k_lo + kt) * (kTileKB / 2), (m0 + mt) * kTileM, b, pol_w);
        if (i == 0) pdl_wait();
        tma_load_3d(sB + s * C::kB, &tm_x, &full[s], (k_lo + kt) * (kTileKB / 2), t0, b);
      }
      if (iters == 0) pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    const uint32_t idesc = idesc_bf16(kTileM, BN, false, false);
    bool ok = true;
    for (int i = 0; ok && i < iters; ++i) {
      const int s = i % kStages;
      const int mt = i / nk, kt = i - mt * nk;
      if (!mbar_wait(&full[s], (i / kStages) & 1, p.err)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t a = smem_u32(sA + s * C::kA), x = smem_u32(sB + s * C::kB);
#pragma unroll
        for (int kk = 0; kk < kTileKB / 32; ++kk)
          mma_bf16(tmem + mt * BN, desc_kmajor_sw128(a + kk * 32), desc_kmajor_sw128(x + kk * 32), idesc,
                   (kt > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (ok && lane == 0) mma_commit(acc_full);
    __syncwarp();
  } else {
    pdl_wait();
    if (threadIdx.x == 64) pdl_launch_dependents();
    const int sub = warp & 3;
    const int tid = threadIdx.x - 64;
    if constexpr (EPI == kQPrep) {
      // RoPE of the rope part while the MMAs run
      for (int i = tid; i < BN; i += 128) sRmax[i] = 0.f;
      named_barrier(1, 128);
      for (int i = tid; i < BN * 32; i += 128) {
        const int j = i >> 5, pr = i & 31, t = t0 + j;
        float y0 = 0.f, y1 = 0.f;
        if (t < p.T) {
          const __nv_bfloat16* r = p.q_pe + (int64_t)t * p.pe_t + (int64_t)b * p.pe_b;
          const float x0 = __bfloat162float(r[2 * pr]), x1 = __bfloat162float(r[2 * pr + 1]);
          const float* tr = p.table + (int64_t)p.pos[t] * 64;
          const float c = tr[pr], sn = tr[32 + pr];
          y0 = x0 * c - x1 * sn;
          y1 = x0 * sn + x1 * c;
        }
        sRope[j * 64 + 2 * pr] = y0;
        sRope[j * 64 + 2 * pr + 1] = y1;
        atomicMax(reinterpret_cast<int*>(sRmax + j), __float_as_int(fmaxf(fabsf(y0), fabsf(y1))));
      }
      named_barrier(1, 128);
    }
    const bool ok = iters > 0 && mbar_wait(acc_full, 0, p.err);
    tc_fence_after();
    if (ok) {
      const uint32_t lane_addr = tmem + (uint32_t(sub * 32) << 16);
      const int rl = sub * 32 + lane;              // row within a 128-row tile
      if constexpr (EPI == kF32Atomic) {
#pragma unroll 1
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 16) {
            uint32_t r[16];
            tmem_ld_x16(lane_addr + mt * BN + c0, r);
            tmem_ld_wait();
            const int m = (m0 + mt) * kTileM + rl;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int t = t0 + c0 + j;
              if (t < p.T) atomicAdd(p.out_f32 + (int64_t)t * p.ot + (int64_t)b * p.ob + m, __uint_as_float(r[j]));
            }
          }
      } else if constexpr (EPI == kBf16Store) {
#pragma unroll 1
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 16) {
            uint32_t r[16];
            tmem_ld_x16(lane_addr + mt * BN + c0, r);
            tmem_ld_wait();
            const int m = (m0 + mt) * kTileM + rl;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int t = t0 + c0 + j;
              if (t < p.T) p.out[(int64_t)t * p.ot + (int64_t)b * p.ob + m] = __float2bfloat16(__uint_as_float(r[j]));
            }
          }
      } else if constexpr (EPI == kMxfp8Rows) {
        const int kb = p.B * p.M / 32;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld_x16(lane_addr + c0, r);
          tmem_ld_wait();
          const int col = b * p.M + m0 * kTileM + rl;   // output-projection operand column
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float v = __uint_as_float(r[j]);
            float amax = fabsf(v);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const int ex = ceil_log2_bits(amax * (1.0f / 448.0f));
            const int t = t0 + c0 + j;
            if (t < p.T) {
              p.q[(int64_t)t * p.B * p.M + col] = uint8_t(f2_to_e4m3x2(v * exp2_int(-ex), 0.f) & 0xFF);
              if (lane == 0) p.sf[sf_offset(t, col >> 5, kb)] = uint8_t(ex + 127);
            }
          }
        }
      } else {   // kQPrep: MT == 4, the whole 512-dim latent of this head
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[4][16];
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) tmem_ld_x16(lane_addr + mt * BN + c0, r[mt]);
          tmem_ld_wait();
          // per-token amax over the 512 latent values (+ the rope part)
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float a = 0.f;
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) a = fmaxf(a, fabsf(__uint_as_float(r[mt][j])));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
            if (lane == 0) red[sub][j] = a;
          }
          named_barrier(1, 128);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int t = t0 + c0 + j;
            const float amax = fmaxf(fmaxf(fmaxf(red[0][j], red[1][j]), fmaxf(red[2][j], red[3][j])),
                                     sRmax[c0 + j]);
            const float sc = amax > 0.f ? amax / 448.f : 1.f;
            const float inv = 1.f / sc;
            if (t < p.T) {
              uint8_t* dst = p.q8 + ((int64_t)t * p.B + b) * 576;
#pragma unroll
              for (int mt = 0; mt < 4; ++mt)
                dst[mt * kTileM + rl] = uint8_t(f2_to_e4m3x2(__uint_as_float(r[mt][j]) * inv, 0.f) & 0xFF);
              if (tid < 32) {
                const float* ro = sRope + (c0 + j) * 64;
                *reinterpret_cast<uint16_t*>(dst + 512 + 2 * tid) = f2_to_e4m3x2(ro[2 * tid] * inv,
                                                                               ro[2 * tid + 1] * inv);
              }
              if (tid == 32) p.qs[(int64_t)t * p.B + b] = sc;
            }
          }
          named_barrier(1, 128);
        }
      }
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

// bf16 view [B][R][K] with element strides (row, batch); box 64 x box_rows x 1.
static int map3(CUtensorMap* m, const void* base, int64_t K, int64_t R, int64_t B, int64_t rs, int64_t bs,
                int box_rows) {
  EncodeTiledFn enc = encoder();
  if (!enc) return -1;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)R, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)rs * 2, (cuuint64_t)bs * 2};
  cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

template <int BN, int MT, int EPI>
static int launch(const Bf16GemmArgs& a, const Params& p, cudaStream_t st) {
  using C = Cfg<BN, MT>;
  CUtensorMap ma, mx;
  if (map3(&ma, a.w, a.K, a.M, a.B, a.K, (int64_t)a.M * a.K, kTileM)) return -2;
  if (map3(&mx, a.x, a.K, a.T, a.B, a.x_ts, a.x_bs, BN)) return -3;
  auto kern = bf16_gemm_kernel<BN, MT, EPI>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  const dim3 grid(a.B, (a.T + BN - 1) / BN, a.M / kTileM / MT * p.splits);
  b200::launch_pdl(kern, grid, dim3(kThreads), C::kSmem, st, ma, mx, p);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

template <int EPI, int MT>
static int launch_bn(const Bf16GemmArgs& a, const Params& p, cudaStream_t st) {
  if (a.T <= 16) return launch<16, MT, EPI>(a, p, st);
  if (a.T <= 32) return launch<32, MT, EPI>(a, p, st);
  if (a.T <= 64) return launch<64, MT, EPI>(a, p, st);
  return launch<128, MT, EPI>(a, p, st);
}

}  // namespace bgemm
}  // namespace b200

int b200_bf16_gemm(const Bf16GemmArgs* a, cudaStream_t st) {
  using namespace b200::bgemm;
  if (a->T <= 0) return 0;
  if (a->M % kTileM || a->K % 64 || a->B <= 0 || (a->x_ts % 8) || (a->x_bs % 8)) return -1;
  Params p{};
  p.T = a->T;
  p.K = a->K;
  p.M = a->M;
  p.B = a->B;
  p.err = a->err;
  p.splits = a->splits > 0 ? a->splits : 1;
  if (a->epi != kF32Atomic && p.splits != 1) return -1;
  switch (a->epi) {
    case kBf16Store:
      p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
      p.ot = a->out_ts;
      p.ob = a->out_bs;
      return launch_bn<kBf16Store, 1>(*a, p, st);
    case kQPrep:
      if (a->M != 512 || !a->q_pe) return -1;
      p.q_pe = reinterpret_cast<const __nv_bfloat16*>(a->q_pe);
      p.pe_t = a->pe_ts;
      p.pe_b = a->pe_bs;
      p.pos = a->pos;
      p.table = a->table;
      p.q8 = a->q8;
      p.qs = a->qs;
      return launch_bn<kQPrep, 4>(*a, p, st);
    case kF32Atomic:
      p.out_f32 = reinterpret_cast<float*>(a->out);
      p.ot = a->out_ts;
      p.ob = a->out_bs;
      return launch_bn<kF32Atomic, 1>(*a, p, st);
    case kMxfp8Rows:
      p.q = a->q;
      p.sf = a->sf;
      return launch_bn<kMxfp8Rows, 1>(*a, p, st);
  }
  return -5;
}
