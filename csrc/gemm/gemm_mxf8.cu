// MXFP8 block-scaled GEMM on tcgen05 (sm_100a), weight-stationary "swap-AB":
//
//   D^T[Nw, T] = W[Nw, K] . X[T, K]^T     (W e4m3, X e4m3, UE8M0 per 32 along K)
//
// The weight matrix is the 128-row MMA operand A (one 128-row tile per CTA),
// the tokens are the MMA's N dimension (BN = 16..256), so decode batches of a
// few tokens still issue full-rate MMAs while the kernel streams weights.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator +
// single-thread MMA issuer, warps 2-5 = epilogue (each reads the 32 TMEM lanes
// of its subpartition).  Per pipeline stage (K = 128): the A tile (128 x 128
// bytes, 128B-swizzled), the B tile (BN x 128 bytes), and the scale factors
// as 512-byte sf128x4 chunks fetched with 1-D bulk copies and moved into
// TMEM with tcgen05.cp.  Each CTA loads its own tiles (no cluster sharing).
//
// Epilogues: bf16 store, fp32 atomic accumulate (split-K), fused SwiGLU +
// MXFP8 requant (gate and up tiles accumulate into two TMEM column ranges;
// a warp's 32 lanes are 32 consecutive intermediate channels = one scale
// block), and a routing-weighted bf16 store for MoE down projections.
//
// Grouped mode (MoE): blockIdx.z = local expert; rows of X are sorted by
// expert with each expert's segment starting at a 128-aligned row offset.
//
// Reference parity: the reference's dense MXFP8 GEMM is the FlashInfer
// CuTe-DSL kernel (pws_gemm.py:124, dt.py) with cluster-shared TMA loads;
// routed experts use trtllm-gen kernels (mo.py:19-40).
#include "../common/ptx.cuh"
#include "gemm_mxf8.h"
#include "../comm/comm.h"

namespace b200 {
namespace gemm {

constexpr int kThreads = 192;
constexpr int kTileM = 128;
constexpr int kTileK = 128;
constexpr int kSfChunk = 512;

template <int BN, int EPI>
struct Cfg {
  static constexpr bool kGateUp = (EPI == kEpiSwiglu || EPI == kEpiClusterSwiglu);
  static constexpr int kA = kGateUp ? 2 : 1;                     // A tiles per stage
  static constexpr int kBChunks = (BN + 127) / 128;               // SF chunks for B
  static constexpr int kLoadBytes = kA * kTileM * kTileK + BN * kTileK + kA * kSfChunk + kBChunks * kSfChunk;
  static constexpr int kStageBytes = kLoadBytes + kSfChunk;   // + a repack chunk for the activation scales
  static constexpr int kStages0 = (200 * 1024) / kStageBytes;
  // Split-K cluster kernels stream few k-tiles per CTA: 4 stages keep two
  // CTAs resident per SM (and twice as many clusters) instead of one.
  static constexpr bool kCluster = (EPI == kEpiClusterSplit || EPI == kEpiClusterPush || EPI == kEpiClusterSwiglu);
  static constexpr int kStagesCap = kCluster ? (kGateUp ? 3 : 4) : 12;
  static constexpr int kStages = kStages0 > kStagesCap ? kStagesCap : kStages0;
  static constexpr int kAccCols = kA * BN;
  static constexpr int kSfColsA = 4 * kA;
  static constexpr int kSfColsB = 4 * kBChunks;
  static constexpr int kSfCols = kStages * (kSfColsA + kSfColsB);
  static constexpr int kTmemNeed = kAccCols + kSfCols;
  static constexpr int kTmemCols = kTmemNeed <= 32 ? 32 : kTmemNeed <= 64 ? 64 : kTmemNeed <= 128 ? 128
                                   : kTmemNeed <= 256 ? 256 : 512;
  static_assert(kTmemNeed <= 512, "TMEM budget");
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

struct Params {
  const uint8_t* sfa;        // weights' packed scales (grouped: per-expert stride sfa_estride)
  const uint8_t* sfb;        // activations' packed scales (row blocks over the sorted rows)
  int64_t sfa_estride;       // bytes between experts' scale blocks
  int nw;                    // weight rows per expert (multiple of 128)
  int t;                     // tokens (dense) / total sorted rows (grouped)
  int k;                     // reduction dim (multiple of 128)
  int k_tiles_per_split;     // split-K slice length in k tiles
  // grouped
  const int* seg_start;      // [E] first sorted row of expert e (128-aligned)
  const int* seg_count;      // [E] rows of expert e
  // outputs
  void* out;                 // bf16 [rows, ldo] or fp32 [rows, ldo]
  int ldo;
  // swiglu epilogue: quantized output + packed scales over the same rows
  uint8_t* q_out;            // e4m3 [rows, nw/2 .. ] row-major, ld = ldq
  uint8_t* sf_out;           // packed sf128x4 for q_out (K = ldq)
  int ldq;
  int inter;                 // rows of the up block offset inside W (gate at 0, up at inter)
  // weighted store (MoE down): per sorted row weight
  const float* row_weight;
  uint32_t* err;
  ArPeers peers;             // kEpiClusterPush
  const uint32_t* ar_epoch;
  uint32_t* ar_ticket;
};

// Byte offset of the scale byte for (row, kblock) inside a packed sf128x4
// tensor whose K spans kb_total 32-blocks.
__device__ __forceinline__ int64_t sf_offset(int row, int kblock, int kb_total) {
  const int rb = row >> 7, r = row & 127, kc = kblock >> 2, c = kblock & 3;
  return ((int64_t)(rb * (kb_total >> 2) + kc) << 9) + ((r & 31) << 4) + ((r >> 5) << 2) + c;
}

template <int BN, int EPI, bool GROUPED>
__global__ void __launch_bounds__(kThreads, 1)
gemm_mxf8_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, Params p) {
  using C = Cfg<BN, EPI>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                                                    // [S][kA][128*128]
  uint8_t* sB = sA + C::kStages * C::kA * kTileM * kTileK;               // [S][BN*128]
  uint8_t* sSFA = sB + C::kStages * BN * kTileK;                          // [S][kA][512]
  uint8_t* sSFB = sSFA + C::kStages * C::kA * kSfChunk;                   // [S][kBChunks][512]
  uint8_t* sRep = sSFB + C::kStages * C::kBChunks * kSfChunk;                  // [S][512] repacked scales
  uint64_t* full = reinterpret_cast<uint64_t*>(sRep + C::kStages * kSfChunk);
  uint64_t* empty = full + C::kStages;
  uint64_t* accbar = empty + C::kStages;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accbar + 1);

  const int warp = warp_id(), lane = lane_id();
  const int tile_n = blockIdx.x;
  const int tile_t = blockIdx.y;
  const int e = GROUPED ? blockIdx.z : 0;
  const int split = GROUPED ? 0 : blockIdx.z;

  // Programmatic dependent launch: let the next kernel start its prologue
  // now (it waits for this grid's completion before touching our outputs).
  if (threadIdx.x == 0) pdl_launch_dependents();
  // Grouped mode reads the routing layout the previous kernel wrote.
  if (GROUPED) pdl_wait();
  int row0, rows;
  if (GROUPED) {
    row0 = p.seg_start[e];
    rows = p.seg_count[e];
  } else {
    row0 = 0;
    rows = p.t;
  }
  if (tile_t * BN >= rows) return;   // uniform across the CTA: nothing to do
  const int kt0 = split * p.k_tiles_per_split;
  int nk = p.k / kTileK - kt0;
  if (nk > p.k_tiles_per_split) nk = p.k_tiles_per_split;
  if (nk < 0) nk = 0;
  // A cluster's CTAs must all reach its barriers: an empty split stays and
  // contributes zeros.
  if (nk == 0 && !C::kCluster) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accbar, 1);
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
  const uint32_t tmem_acc = tmem;
  const uint32_t tmem_sf = tmem + C::kAccCols;

  // Weight rows of this tile inside the (stacked) weight matrix.
  const int a_row = e * p.nw + tile_n * kTileM;
  const int b_row = row0 + tile_t * BN;
  const int kb_total = p.k / 32;

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      constexpr uint32_t bytes = C::kLoadBytes;
      const uint8_t* sfa_e = p.sfa + (GROUPED ? (int64_t)e * p.sfa_estride : 0);
      const int kc_total = kb_total / 4;
      // Weights never depend on the previous kernel: the first stages' weight
      // tiles are in flight before griddepcontrol.wait, activations after it.
      auto load_a = [&](int i) {
        const int s = i % C::kStages;
        const int kt = kt0 + i;
        mbar_arrive_expect_tx(&full[s], bytes);
        uint8_t* a_dst = sA + (size_t)s * C::kA * kTileM * kTileK;
        tma_load_2d(a_dst, &tm_a, &full[s], kt * kTileK, a_row);
        if (C::kGateUp) tma_load_2d(a_dst + kTileM * kTileK, &tm_a, &full[s], kt * kTileK, a_row + p.inter);
        uint8_t* sfa_dst = sSFA + (size_t)s * C::kA * kSfChunk;
        bulk_load(sfa_dst, sfa_e + ((int64_t)(tile_n * kc_total + kt) << 9), kSfChunk, &full[s]);
        if (C::kGateUp) {
          const int rb_up = (p.inter + tile_n * kTileM) >> 7;
          bulk_load(sfa_dst + kSfChunk, sfa_e + ((int64_t)(rb_up * kc_total + kt) << 9), kSfChunk, &full[s]);
        }
      };
      auto load_b = [&](int i) {
        const int s = i % C::kStages;
        const int kt = kt0 + i;
        tma_load_2d(sB + (size_t)s * BN * kTileK, &tm_b, &full[s], kt * kTileK, b_row);
        for (int c = 0; c < C::kBChunks; ++c) {
          const int rb = (b_row >> 7) + c;
          bulk_load(sSFB + ((size_t)s * C::kBChunks + c) * kSfChunk,
                    p.sfb + ((int64_t)(rb * kc_total + kt) << 9), kSfChunk, &full[s]);
        }
      };
      const int pre = nk < C::kStages ? nk : C::kStages;
      for (int i = 0; i < pre; ++i) load_a(i);
      if (!GROUPED) pdl_wait();
      for (int i = 0; i < pre; ++i) load_b(i);
      for (int i = pre; i < nk; ++i) {
        const int s = i % C::kStages;
        if (!mbar_wait(&empty[s], ((i / C::kStages) - 1) & 1, p.err)) break;
        load_a(i);
        load_b(i);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      if (!mbar_wait(&full[s], (i / C::kStages) & 1, p.err)) { ok = false; break; }
      tc_fence_after();
      // Token tiles of BN <= 128 rows may start at row o = b_row % 128 of a
      // scale chunk: repack rows o..o+BN-1 into a tile-local chunk so the
      // MMA reads the activation scales at the base TMEM column.
      const int o = b_row & 127;
      if (BN <= 128 && o != 0) {
        const uint8_t* src = sSFB + (size_t)s * C::kBChunks * kSfChunk;
        uint8_t* dst = sRep + (size_t)s * kSfChunk;
        for (int j = lane; j < BN; j += 32) {
          const int r = o + j;
          *reinterpret_cast<uint32_t*>(dst + (j & 31) * 16 + (j >> 5) * 4) =
              *reinterpret_cast<const uint32_t*>(src + (r & 31) * 16 + (r >> 5) * 4);
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (lane == 0) {
        const uint32_t sf_a = tmem_sf + s * (C::kSfColsA + C::kSfColsB);
        const uint32_t sf_b = sf_a + C::kSfColsA;
        const uint8_t* sfa_src = sSFA + (size_t)s * C::kA * kSfChunk;
        for (int a = 0; a < C::kA; ++a)
          tmem_cp_32x128b_x4(sf_a + 4 * a, smem_desc(smem_u32(sfa_src + a * kSfChunk), 0, 128, 0));
        if (BN <= 128 && o != 0) {
          tmem_cp_32x128b_x4(sf_b, smem_desc(smem_u32(sRep + (size_t)s * kSfChunk), 0, 128, 0));
        } else {
          for (int c = 0; c < C::kBChunks; ++c)
            tmem_cp_32x128b_x4(sf_b + 4 * c,
                               smem_desc(smem_u32(sSFB + ((size_t)s * C::kBChunks + c) * kSfChunk), 0, 128, 0));
        }
        const uint32_t a_base = smem_u32(sA + (size_t)s * C::kA * kTileM * kTileK);
        const uint32_t b_base = smem_u32(sB + (size_t)s * BN * kTileK);
        for (int kk = 0; kk < kTileK / 32; ++kk) {
          const uint64_t bdesc = desc_kmajor_sw128(b_base + kk * 32);
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          for (int a = 0; a < C::kA; ++a) {
            const uint64_t adesc = desc_kmajor_sw128(a_base + a * kTileM * kTileK + kk * 32);
            const uint32_t idesc = idesc_mxf8(kTileM, BN, kk, kk);
            mma_mxf8(tmem_acc + a * BN, adesc, bdesc, idesc, (sf_a + 4 * a) | (uint32_t(kk) << 30),
                     sf_b | (uint32_t(kk) << 30), acc);
          }
        }
        mma_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (lane == 0) {
      if (ok) mma_commit(accbar);
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ------------------------------
    const int sub = warp & 3;                        // TMEM subpartition of this warp
    const int wrow = tile_n * kTileM + sub * 32 + lane;   // weight row (output column)
    const bool ok = mbar_wait(accbar, 0, p.err);
    tc_fence_after();
    if (ok) {
      const uint32_t lane_addr = tmem_acc + (uint32_t(sub * 32) << 16);
      const int tmax = rows - tile_t * BN;           // valid token columns in this tile
      if (EPI == kEpiClusterSplit || EPI == kEpiClusterPush || EPI == kEpiClusterSwiglu) {
        // stage this split's partial tile: red[row][kA*BN+1] over the (drained) A stages
        float* red = reinterpret_cast<float*>(sA);
        const int row = sub * 32 + lane;
        constexpr int kW = C::kA * BN + 1;
#pragma unroll 1
        for (int c0 = 0; c0 < C::kA * BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld_x16(lane_addr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) red[row * kW + c0 + j] = nk > 0 ? __uint_as_float(r[j]) : 0.f;
        }
      } else if (EPI == kEpiStoreBf16 || EPI == kEpiAtomicF32 || EPI == kEpiWeightedBf16) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld_x16(lane_addr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tcol = c0 + j;
            if (tcol < tmax) {
              const int orow = b_row + tcol;
              float v = __uint_as_float(r[j]);
              if (EPI == kEpiAtomicF32) {
                atomicAdd(reinterpret_cast<float*>(p.out) + (int64_t)orow * p.ldo + wrow, v);
              } else {
                if (EPI == kEpiWeightedBf16) v *= p.row_weight[orow];
                reinterpret_cast<__nv_bfloat16*>(p.out)[(int64_t)orow * p.ldo + wrow] = __float2bfloat16(v);
              }
            }
          }
        }
      } else if (EPI == kEpiSwiglu) {
        // gate accum at [0, BN), up accum at [BN, 2BN); this thread's channel
        // is wrow (0..inter); one warp covers one 32-channel scale block.
        const int ch = wrow;
        const int kb_out = p.ldq / 32;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t g[16], u[16];
          tmem_ld_x16(lane_addr + c0, g);
          tmem_ld_x16(lane_addr + BN + c0, u);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float gv = __uint_as_float(g[j]);
            const float uv = __uint_as_float(u[j]);
            const float h = gv / (1.0f + __expf(-gv)) * uv;
            float amax = fabsf(h);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const int ex = ceil_log2_bits(amax * (1.0f / 448.0f));
            const float inv = exp2_int(-ex);
            const int tcol = c0 + j;
            if (tcol < tmax) {
              const int orow = b_row + tcol;
              const uint16_t q2 = f2_to_e4m3x2(h * inv, 0.f);
              p.q_out[(int64_t)orow * p.ldq + ch] = uint8_t(q2 & 0xFF);
              if (lane == 0) p.sf_out[sf_offset(orow, ch >> 5, kb_out)] = uint8_t(ex + 127);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (EPI == kEpiClusterSplit || EPI == kEpiClusterPush || EPI == kEpiClusterSwiglu) {
    // Every split of this output tile has staged its partial; CTA `rank`
    // sums rows [rank*RPC, (rank+1)*RPC) of the tile across the cluster.
    // kEpiClusterPush stores the sums into recv[parity][my rank] of every
    // rank (P2P over NVLink, 16-byte stores) and then publishes with one
    // counter increment per rank, so the all-reduce transfer overlaps the
    // remaining tiles.  kEpiClusterSwiglu applies SwiGLU to the summed gate
    // and up rows and requantizes to MXFP8 (one warp = one 32-channel block).
    constexpr int kW = C::kA * BN + 1;
    const int parity = (EPI == kEpiClusterPush) ? int(__ldcg(p.ar_epoch) & 1u) : 0;
    cluster_sync();
    const int S = gridDim.z;
    const uint32_t rank = cluster_ctarank();
    const int rpc = kTileM / S;
    const uint32_t red_local = smem_u32(sA);
    const int tmax = rows - tile_t * BN;
    if constexpr (EPI == kEpiClusterSwiglu) {
      // work item = (token column, 32-channel block), spread over the
      // cluster's warps (any split count: a block may belong to any rank)
      constexpr int kBlocks = kTileM / 32;
      constexpr int kWarps = kThreads / 32;
      for (int wi = int(rank) * kWarps + warp; wi < BN * kBlocks; wi += S * kWarps) {
        const int col = wi / kBlocks;
        if (col >= tmax) continue;                     // uniform per warp
        const int rr = (wi % kBlocks) * 32 + lane;
        float g = 0.f, u = 0.f;
        for (int q = 0; q < S; ++q) {
          g += ld_dsmem_f32(mapa_shared(red_local + (uint32_t)(rr * kW + col) * 4u, q));
          u += ld_dsmem_f32(mapa_shared(red_local + (uint32_t)(rr * kW + BN + col) * 4u, q));
        }
        const float h = g / (1.0f + __expf(-g)) * u;
        float amax = fabsf(h);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const int ex = ceil_log2_bits(amax * (1.0f / 448.0f));
        const int orow = b_row + col;
        const int ch = tile_n * kTileM + rr;
        p.q_out[(int64_t)orow * p.ldq + ch] = uint8_t(f2_to_e4m3x2(h * exp2_int(-ex), 0.f) & 0xFF);
        if (lane == 0) p.sf_out[sf_offset(orow, ch >> 5, p.ldq / 32)] = uint8_t(ex + 127);
      }
    } else {
      // 8 consecutive output channels per work item -> one 16-byte store
      const int groups = rpc / 8;
      for (int i = threadIdx.x; i < groups * BN; i += kThreads) {
        const int col = i / groups;
        if (col >= tmax) continue;
        const int rr0 = rank * rpc + (i % groups) * 8;
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int q = 0; q < S; ++q) {
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += ld_dsmem_f32(mapa_shared(red_local + (uint32_t)((rr0 + j) * kW + col) * 4u, q));
        }
        uint4 v;
        __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) h2[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
        const int64_t oi = (int64_t)(b_row + col) * p.ldo + tile_n * kTileM + rr0;
        if constexpr (EPI == kEpiClusterPush) {
          // push mode: recv[parity][my rank] of every rank; NVLS mode (mc set):
          // only this rank's own input slot in[parity]
          const int nd = p.peers.mc ? 1 : p.peers.world;
          for (int dst = 0; dst < nd; ++dst) {
            __nv_bfloat16* slot =
                p.peers.mc ? reinterpret_cast<__nv_bfloat16*>(p.peers.base[p.peers.rank] + kArRecvOff) +
                                 (int64_t)parity * p.peers.max_t * p.ldo
                           : reinterpret_cast<__nv_bfloat16*>(p.peers.base[dst] + kArRecvOff) +
                                 ((int64_t)(parity * p.peers.world + p.peers.rank) * p.peers.max_t) * p.ldo;
            *reinterpret_cast<uint4*>(slot + oi) = v;
          }
        } else {
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + oi) = v;
        }
      }
    }
    if constexpr (EPI == kEpiClusterPush) {
      // every CTA fences + takes a ticket; the last publishes once per rank
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t prev = atomicAdd(p.ar_ticket, 1u);
        if (prev == gridDim.x * gridDim.y * gridDim.z - 1) {
          __threadfence_system();
          *p.ar_ticket = 0u;
          for (int dst = 0; dst < p.peers.world; ++dst) {
            uint32_t* cnt = reinterpret_cast<uint32_t*>(p.peers.base[dst]) + parity * kArMaxRanks + p.peers.rank;
            asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(cnt), "r"(1u) : "memory");
          }
        }
      }
    }
    cluster_sync();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D byte matrix [rows, cols] (row stride ld bytes), box [box_rows, 128], 128B swizzle.
int make_map_u8(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

template <int BN, int EPI, bool GROUPED>
static int launch_t(const GemmArgs& a, cudaStream_t st) {
  using C = Cfg<BN, EPI>;
  CUtensorMap ma, mb;
  const int64_t a_rows = GROUPED ? (int64_t)a.num_experts * a.nw : (int64_t)a.nw_total;
  if (make_map_u8(&ma, a.w, a_rows, a.k, a.k, kTileM)) return -1;
  if (make_map_u8(&mb, a.x, a.x_rows, a.k, a.k, BN)) return -2;
  Params p{};
  p.sfa = a.w_sf;
  p.sfb = a.x_sf;
  p.sfa_estride = a.w_sf_estride;
  p.nw = a.nw;
  p.t = a.t;
  p.k = a.k;
  const int ktiles = a.k / kTileK;
  const int splits = a.splits > 0 ? a.splits : 1;
  p.k_tiles_per_split = (ktiles + splits - 1) / splits;
  p.seg_start = a.seg_start;
  p.seg_count = a.seg_count;
  p.out = a.out;
  p.ldo = a.ldo;
  p.q_out = a.q_out;
  p.sf_out = a.sf_out;
  p.ldq = a.ldq;
  p.inter = a.inter;
  p.row_weight = a.row_weight;
  p.err = a.err;
  if (EPI == kEpiClusterPush) {
    p.peers = *reinterpret_cast<const ArPeers*>(a.ar_peers);
    p.ar_epoch = a.ar_epoch;
    p.ar_ticket = a.ar_ticket;
  }
  auto kern = gemm_mxf8_kernel<BN, EPI, GROUPED>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  dim3 grid;
  grid.x = (C::kGateUp ? a.inter : a.nw) / kTileM;
  grid.y = GROUPED ? (a.max_rows_per_expert + BN - 1) / BN : (a.t + BN - 1) / BN;
  grid.z = GROUPED ? a.num_experts : splits;
  if (grid.y == 0) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (a.pdl && b200::pdl_enabled()) ? 1 : 0;
  int nattr = 1;
  if (C::kCluster) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = grid.z;
    nattr = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kern, ma, mb, p);
  return err == cudaSuccess ? 0 : 1000 + int(err);
}

template <int EPI, bool GROUPED>
static int launch_bn(const GemmArgs& a, cudaStream_t st) {
  const int t = GROUPED ? a.max_rows_per_expert : a.t;
  if (t <= 16) return launch_t<16, EPI, GROUPED>(a, st);
  if (t <= 32) return launch_t<32, EPI, GROUPED>(a, st);
  if (t <= 64) return launch_t<64, EPI, GROUPED>(a, st);
  if constexpr (EPI == kEpiSwiglu || EPI == kEpiClusterSwiglu) {
    return launch_t<128, EPI, GROUPED>(a, st);
  } else {
    if (t <= 128) return launch_t<128, EPI, GROUPED>(a, st);
    return launch_t<256, EPI, GROUPED>(a, st);
  }
}

}  // namespace gemm
}  // namespace b200

int b200_gemm_mxf8(const GemmArgs* a, cudaStream_t st) {
  using namespace b200::gemm;
  const bool g = a->num_experts > 0;
  switch (a->epi) {
    case kEpiStoreBf16: return g ? launch_bn<kEpiStoreBf16, true>(*a, st) : launch_bn<kEpiStoreBf16, false>(*a, st);
    case kEpiAtomicF32: return g ? -10 : launch_bn<kEpiAtomicF32, false>(*a, st);
    case kEpiSwiglu: return g ? launch_bn<kEpiSwiglu, true>(*a, st) : launch_bn<kEpiSwiglu, false>(*a, st);
    case kEpiWeightedBf16: return g ? launch_bn<kEpiWeightedBf16, true>(*a, st) : -11;
    case kEpiClusterSplit:
      if (g || a->splits < 2 || a->splits > 8 || (128 % a->splits) != 0 || a->t > 128) return -13;
      return launch_bn<kEpiClusterSplit, false>(*a, st);
    case kEpiClusterPush:
      if (g || a->splits < 2 || a->splits > 8 || (128 % a->splits) != 0 || a->t > 128 || !a->ar_peers) return -14;
      return launch_bn<kEpiClusterPush, false>(*a, st);
    case kEpiClusterSwiglu:
      if (g || a->splits < 2 || a->splits > 8 || a->t > 128 || a->inter % 128) return -15;
      return launch_bn<kEpiClusterSwiglu, false>(*a, st);
  }
  return -12;
}
