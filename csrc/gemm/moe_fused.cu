// Fused persistent MoE expert GEMMs (sm_100a, tcgen05): FC1 and FC2 of the
// routed experts in ONE launch.
//
//   FC1 unit  (expert e, token tile tt, row tile n):  h = quant(silu(x Wg^T) *
//             (x Wu^T)) for 128 intermediate channels (gate and up tiles in
//             two TMEM column ranges), written to the FC2 operand buffer;
//   FC2 unit  (expert e, token tile tt, row-tile pair p): y = routing_weight
//             * (h Wd^T) for 256 hidden rows (two 128-row weight tiles share
//             the stage layout and TMEM accumulators of FC1's gate / up).
//
// With the two GEMMs in separate launches the second waits for the first's
// last tile wave, which at 32 experts per GPU leaves most SMs idle for the
// last ~20% of FC1.  Here every CTA grabs work units in order from a global
// counter (FC1 units first, then FC2), and an FC2 unit of expert e starts as
// soon as all FC1 units of e are done (per-expert completion counters,
// release / acquire, bounded wait), so FC2 tiles fill FC1's tail.  Grabbing
// in order makes the dependency wait deadlock-free: every FC1 unit an FC2
// unit waits for was taken earlier by a running CTA whose warps do not wait
// on anything but their own pipeline.
//
// Warp roles as in the grouped GEMM (producer, MMA issuer + TMEM owner, four
// epilogue warps); the producer publishes each grabbed unit to the other
// roles through a 4-entry shared-memory ring.  The last CTA to finish resets
// the counters, so the launch is graph-replayable.  All waits are bounded.
#include "../common/ptx.cuh"
#include "gemm_mxf8.h"
#include "../comm/comm.h"

namespace b200 {
namespace moef {

constexpr int kThreads = 192;
constexpr int kTileM = 128;
constexpr int kTileK = 128;
constexpr int kSf = 512;
constexpr int kRing = 4;
constexpr int kMaxExperts = 512;   // local experts per GPU (V4.1-Flash: 384 on one GPU)

template <int BN, bool FP4>
struct Cfg {
  static constexpr int kSfK = FP4 ? 4 * kSf : kSf;          // scale bytes per 128 rows per k-tile
  static constexpr int kLoadBytes = 2 * kTileM * kTileK + BN * kTileK + 2 * kSfK + kSfK;
  static constexpr int kStageBytes = kLoadBytes + kSfK;     // + activation-scale repack area
  static constexpr int kAcc = 2 * BN;
  static constexpr int kSlotCols = FP4 ? 48 : 12;
  static constexpr int kStagesSmem = (200 * 1024) / kStageBytes;
  static constexpr int kStagesTmem = (512 - 2 * kAcc) / kSlotCols;
  static constexpr int kStages0 = kStagesSmem < kStagesTmem ? kStagesSmem : kStagesTmem;
  static constexpr int kStages = kStages0 > 16 ? 16 : kStages0;
  static constexpr int kSfCols = kStages * kSlotCols;
  static constexpr int kNeed = 2 * kAcc + kSfCols;
  static constexpr int kTmemCols = kNeed <= 32 ? 32 : kNeed <= 64 ? 64 : kNeed <= 128 ? 128 : kNeed <= 256 ? 256 : 512;
  static_assert(kNeed <= 512 && kStages >= 2, "TMEM / pipeline budget");
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 1024;
};

struct Params {
  const uint8_t* sfa1;
  int64_t sfa1_estride;
  const uint8_t* sfb1;
  const uint8_t* sfa2;
  int64_t sfa2_estride;
  uint8_t* hq;               // FC1 output = FC2 activation operand [rows, inter] (bytes: inter or inter/2)
  uint8_t* hq_sf;
  __nv_bfloat16* y;          // FC2 output [rows, hidden]
  int ldy;
  int hidden, inter, E;
  const int* seg_start;
  const int* seg_count;
  const int* ttile_off;
  const float* row_weight;
  const float* x_g;          // NVFP4: FC1 input global scale per sorted row
  const float* w1_g;         // NVFP4: per-expert global scales
  const float* w2_g;
  float out_g;               // NVFP4: global scale of h (FC1 output / FC2 input)
  int* work;                 // [0] next unit, [1] finished CTAs
  int* fc1_done;             // [E] finished FC1 units per expert
  uint32_t* err;
  int a_tiled;
  // pull mode: FC1 activation rows straight from their source buffers
  int pull;
  const uint8_t* src_q[8];
  const uint8_t* src_sf[8];
  const float* src_g[8];
  int src_rows;
  const int* row_token;
  // sources in a two-parity buffer: every source pointer moves by
  // ((*src_epoch + src_epoch_add) & 1) * src_par_bytes (null: fixed sources)
  const uint32_t* src_epoch;
  int src_epoch_add;
  int64_t src_par_bytes;
  // expert-parallel combine in the FC2 epilogue (MoeFusedArgs)
  const int* c_row_pair;
  int c_K, c_T_step;
  uint8_t* c_base[8];
  int c_rank, c_world, c_max_t;
  int64_t c_off;
  const uint32_t* c_epoch;
};

__device__ __forceinline__ int64_t sf_offset(int row, int kblock, int kb_total) {
  const int rb = row >> 7, r = row & 127, kc = kblock >> 2, c = kblock & 3;
  return ((int64_t)(rb * (kb_total >> 2) + kc) << 9) + ((r & 31) << 4) + ((r >> 5) << 2) + c;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

struct Unit {
  bool fc1;
  int e, tt, n;        // n: FC1 row tile or FC2 row-tile pair
  int rows;            // tokens of expert e
};

// lay[0..E] = token-tile prefix, [E+1..2E] seg_start, [2E+1..3E] seg_count
__device__ __forceinline__ Unit decode(int u, int U1, int n1, int n2, const int* lay, int E) {
  Unit d;
  int ttg;
  if (u < U1) {
    d.fc1 = true;
    ttg = u / n1;
    d.n = u - ttg * n1;
  } else {
    d.fc1 = false;
    const int v = u - U1;
    ttg = v / n2;
    d.n = v - ttg * n2;
  }
  int lo = 0, hi = E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (lay[mid] <= ttg) lo = mid; else hi = mid;
  }
  d.e = lo;
  d.tt = ttg - lay[lo];
  d.rows = lay[2 * E + 1 + lo];
  return d;
}

template <int BN, bool FP4>
__global__ void __launch_bounds__(kThreads, 1)
moe_fused_kernel(const __grid_constant__ CUtensorMap tm_w1, const __grid_constant__ CUtensorMap tm_x,
                 const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_h, Params p) {
  using C = Cfg<BN, FP4>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::kStages * 2 * kTileM * kTileK;
  uint8_t* sSFA = sB + C::kStages * BN * kTileK;
  uint8_t* sSFB = sSFA + C::kStages * 2 * C::kSfK;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + C::kStages * 2 * C::kSfK);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;    // [2]
  uint64_t* acc_empty = acc_full + 2;         // [2]
  uint64_t* tq_full = acc_empty + 2;          // [kRing]
  uint64_t* tq_empty = tq_full + kRing;       // [kRing]
  int* tile_q = reinterpret_cast<int*>(tq_empty + kRing);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tile_q + kRing);
  __shared__ int lay[3 * kMaxExperts + 1];
  // pull mode: the current FC1 unit's row sources, resolved once per unit
  // (row address, scale base, row index in its source; null = padding row)
  __shared__ const uint8_t* pull_q[BN];
  __shared__ const uint8_t* pull_sf[BN];
  __shared__ int pull_row[BN];

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      // pull mode: lane 0's expect-tx arrival + one per producer lane after its copies
      mbar_init(&full[s], p.pull ? 33 : 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 1);
    }
    for (int r = 0; r < kRing; ++r) {
      mbar_init(&tq_full[r], 1);
      mbar_init(&tq_empty[r], 2);      // MMA warp + epilogue warpgroup
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tm_w1);
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_w2);
    prefetch_tensormap(&tm_h);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t tmem_sf = tmem + 2 * C::kAcc;

  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int E = p.E;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) lay[i] = __ldcg(p.ttile_off + i);
  for (int i = threadIdx.x; i < E; i += blockDim.x) {
    lay[E + 1 + i] = __ldcg(p.seg_start + i);
    lay[2 * E + 1 + i] = __ldcg(p.seg_count + i);
  }
  __syncthreads();
  const int n1 = p.inter / kTileM;          // FC1 row tiles
  const int n2 = p.hidden / (2 * kTileM);   // FC2 row-tile pairs
  const int U1 = lay[E] * n1;
  const int U = U1 + lay[E] * n2;
  const int kb1 = FP4 ? p.hidden / 2 : p.hidden;    // operand bytes per row
  const int kb2 = FP4 ? p.inter / 2 : p.inter;
  const int kct1 = FP4 ? p.hidden / 64 : p.hidden / kTileK;   // sf chunks per 128 rows
  const int kct2 = FP4 ? p.inter / 64 : p.inter / kTileK;
  constexpr int kChunksPerTile = FP4 ? 4 : 1;

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    // Lane 0 grabs units and issues the TMA loads of the weights (and, unless
    // pulling, of the activations); in pull mode every lane also gathers the
    // FC1 activation rows of the stage with 16-byte cp.async (P2P for peer
    // rows) into the 128B-swizzled tile, plus their scale words.
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const int kbq1 = FP4 ? p.hidden / 16 : p.hidden / 32;     // activation scale columns
  const int64_t par_off =
      p.src_epoch ? (int64_t)((__ldcg(p.src_epoch) + (uint32_t)p.src_epoch_add) & 1u) * p.src_par_bytes : 0;
    int it = 0;
    for (int q = 0;; ++q) {
      const int slot = q % kRing;
      if (q >= kRing && !__all_sync(0xffffffffu, mbar_wait(&tq_empty[slot], ((q / kRing) - 1) & 1, p.err))) break;
      int u = 0;
      if (lane == 0) {
        u = atomicAdd(p.work, 1);
        if (u >= U) u = -1;
        tile_q[slot] = u;
        mbar_arrive(&tq_full[slot]);
      }
      u = __shfl_sync(0xffffffffu, u, 0);
      if (u < 0) break;
      const Unit d = decode(u, U1, n1, n2, lay, E);
      const int b_row = lay[E + 1 + d.e] + d.tt * BN;
      const bool pulled = p.pull && d.fc1;
      int nk, a_row0, a_row1, kct;
      const CUtensorMap *ma, *mb;
      const uint8_t *sfa, *sfb;
      if (d.fc1) {
        nk = kb1 / kTileK;
        a_row0 = d.e * 2 * p.inter + d.n * kTileM;
        a_row1 = a_row0 + p.inter;
        ma = &tm_w1;
        mb = &tm_x;
        sfa = p.sfa1 + (int64_t)d.e * p.sfa1_estride;
        sfb = p.sfb1;
        kct = kct1;
      } else {
        if (lane == 0) {
          // the expert's FC1 output must be complete (bounded wait; skipped
          // once any wait of this launch has given up, so a failed launch
          // ends after one deadline instead of one per unit)
          const int need = n1 * (lay[d.e + 1] - lay[d.e]);
          const uint64_t t0 = globaltimer_ns();
          while (ld_acquire_gpu(p.fc1_done + d.e) < need && *reinterpret_cast<volatile uint32_t*>(p.err) == 0) {
            if (globaltimer_ns() - t0 > kWaitBudgetNs) {
              atomicExch(p.err, kErrDepTimeout);
              break;
            }
          }
          fence_proxy_async_global();
        }
        __syncwarp();
        nk = kb2 / kTileK;
        a_row0 = d.e * p.hidden + d.n * 2 * kTileM;
        a_row1 = a_row0 + kTileM;
        ma = &tm_w2;
        mb = &tm_h;
        sfa = p.sfa2 + (int64_t)d.e * p.sfa2_estride;
        sfb = p.hq_sf;
        kct = kct2;
      }
      const int rb0 = (a_row0 - d.e * (d.fc1 ? 2 * p.inter : p.hidden)) >> 7;
      const int rb1 = (a_row1 - d.e * (d.fc1 ? 2 * p.inter : p.hidden)) >> 7;
      const int tmax = d.rows - d.tt * BN;
      if (pulled) {
        __syncwarp();
        for (int j = lane; j < BN; j += 32) {
          const uint8_t *rq = nullptr, *rs = nullptr;
          int lr = 0;
          if (j < tmax) {
            const int g = __ldcg(p.row_token + b_row + j);
            const int sr = g / p.src_rows;
            lr = g - sr * p.src_rows;
            rq = p.src_q[sr] + par_off + (int64_t)lr * kb1;
            rs = p.src_sf[sr] + par_off;
          }
          pull_q[j] = rq;
          pull_sf[j] = rs;
          pull_row[j] = lr;
        }
        __syncwarp();
      }
      bool ok = true;
      for (int kt = 0; kt < nk; ++kt, ++it) {
        const int s = it % C::kStages;
        if (it >= C::kStages &&
            !__all_sync(0xffffffffu, mbar_wait(&empty[s], ((it / C::kStages) - 1) & 1, p.err))) {
          ok = false;
          break;
        }
        uint8_t* sfb_dst = sSFB + (size_t)s * 2 * C::kSfK;
        const int kc0 = kt * kChunksPerTile;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], pulled ? C::kLoadBytes - BN * kTileK - C::kSfK : C::kLoadBytes);
          uint8_t* a_dst = sA + (size_t)s * 2 * kTileM * kTileK;
          if (p.a_tiled) {
            tma_load_3d_hint(a_dst, ma, &full[s], 0, 0, (a_row0 >> 7) * nk + kt, pol_w);
            tma_load_3d_hint(a_dst + kTileM * kTileK, ma, &full[s], 0, 0, (a_row1 >> 7) * nk + kt, pol_w);
          } else {
            tma_load_2d_hint(a_dst, ma, &full[s], kt * kTileK, a_row0, pol_w);
            tma_load_2d_hint(a_dst + kTileM * kTileK, ma, &full[s], kt * kTileK, a_row1, pol_w);
          }
          uint8_t* sfa_dst = sSFA + (size_t)s * 2 * C::kSfK;
          bulk_load_hint(sfa_dst, sfa + ((int64_t)(rb0 * kct + kc0) << 9), C::kSfK, &full[s], pol_w);
          bulk_load_hint(sfa_dst + C::kSfK, sfa + ((int64_t)(rb1 * kct + kc0) << 9), C::kSfK, &full[s], pol_w);
          if (!pulled) {
            tma_load_2d_hint(sB + (size_t)s * BN * kTileK, mb, &full[s], kt * kTileK, b_row, pol_x);
            bulk_load_hint(sfb_dst, sfb + ((int64_t)((b_row >> 7) * kct + kc0) << 9), C::kSfK, &full[s], pol_x);
          }
        }
        if (p.pull) {
          if (pulled) {
            const uint32_t bdst = smem_u32(sB + (size_t)s * BN * kTileK);
#pragma unroll
            for (int i = 0; i < BN / 4; ++i) {
              const int j = (lane >> 3) + 4 * i, c = lane & 7;
              const uint8_t* rq = pull_q[j];
              cp_async_16(bdst + j * kTileK + ((c ^ (j & 7)) << 4), rq ? rq + kt * kTileK + c * 16 : p.src_q[0],
                          rq ? 16u : 0u);
            }
            const uint32_t sdst = smem_u32(sfb_dst);
            for (int idx = lane; idx < BN * kChunksPerTile; idx += 32) {
              const int j = idx / kChunksPerTile, ch = idx - j * kChunksPerTile;
              const uint8_t* rs = pull_sf[j];
              cp_async_4(sdst + ch * kSf + (j & 31) * 16 + (j >> 5) * 4,
                         rs ? rs + sf_offset(pull_row[j], 4 * (kc0 + ch), kbq1) : p.src_sf[0], rs ? 4u : 0u);
            }
            // each lane's arrival fires when its copies have landed; the MMA
            // thread fences them into the async proxy after its wait
            cp_async_mbar_arrive_noinc(&full[s]);
          } else {
            mbar_arrive(&full[s]);
          }
        }
      }
      if (!ok) break;
    }
    if (p.pull) cp_async_wait_all();   // nothing lands after this warp has left (error exits)
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    int it = 0;
    for (int q = 0;; ++q) {
      const int slot = q % kRing;
      if (!mbar_wait(&tq_full[slot], (q / kRing) & 1, p.err)) break;
      const int u = tile_q[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&tq_empty[slot]);
      if (u < 0) break;
      const Unit d = decode(u, U1, n1, n2, lay, E);
      const int b_row = lay[E + 1 + d.e] + d.tt * BN;
      const int nk = (d.fc1 ? kb1 : kb2) / kTileK;
      const int buf = q & 1;
      if (q >= 2 && !mbar_wait(&acc_empty[buf], ((q >> 1) - 1) & 1, p.err)) break;
      tc_fence_after();
      const uint32_t acc = tmem + buf * C::kAcc;
      bool ok = true;
      for (int kt = 0; kt < nk; ++kt, ++it) {
        const int s = it % C::kStages;
        if (!mbar_wait(&full[s], (it / C::kStages) & 1, p.err)) { ok = false; break; }
        tc_fence_after();
        if (p.pull && d.fc1) fence_proxy_async_smem();   // cp.async (generic proxy) rows -> tcgen05 reads
        const int o = (p.pull && d.fc1) ? 0 : (b_row & 127);   // pulled rows sit at tile-local positions
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
          const uint32_t sf_a = tmem_sf + s * C::kSlotCols;
          const uint32_t sf_b = sf_a + 4 * kChunksPerTile * 2;
          const uint8_t* sfa_src = sSFA + (size_t)s * 2 * C::kSfK;
          const uint8_t* sfb_src = sfb_stage + (o != 0 ? C::kSfK : 0);
          for (int a = 0; a < 2; ++a)
            for (int ch = 0; ch < kChunksPerTile; ++ch)
              tmem_cp_32x128b_x4(sf_a + 4 * (a * kChunksPerTile + ch),
                                 smem_desc(smem_u32(sfa_src + a * C::kSfK + ch * kSf), 0, 128, 0));
          for (int ch = 0; ch < kChunksPerTile; ++ch)
            tmem_cp_32x128b_x4(sf_b + 4 * ch, smem_desc(smem_u32(sfb_src + ch * kSf), 0, 128, 0));
          const uint32_t a_base = smem_u32(sA + (size_t)s * 2 * kTileM * kTileK);
          const uint32_t b_base = smem_u32(sB + (size_t)s * BN * kTileK);
          for (int kk = 0; kk < kTileK / 32; ++kk) {
            const uint64_t bdesc = desc_kmajor_sw128(b_base + kk * 32);
            const uint32_t accf = (kt > 0 || kk > 0) ? 1u : 0u;
            for (int a = 0; a < 2; ++a) {
              const uint64_t adesc = desc_kmajor_sw128(a_base + a * kTileM * kTileK + kk * 32);
              if constexpr (FP4) {
                mma_nvf4(acc + a * BN, adesc, bdesc, idesc_nvf4(kTileM, BN), sf_a + 4 * (a * kChunksPerTile + kk),
                         sf_b + 4 * kk, accf);
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
      if (!ok) break;
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    const int sub = warp & 3;
    const int tid = threadIdx.x - 64;
    const int kbq = FP4 ? p.inter / 16 : p.inter / 32;   // scale columns of h
    const int64_t g_off =
        p.src_epoch ? (int64_t)((__ldcg(p.src_epoch) + (uint32_t)p.src_epoch_add) & 1u) * p.src_par_bytes : 0;
    for (int q = 0;; ++q) {
      const int slot = q % kRing;
      if (!mbar_wait(&tq_full[slot], (q / kRing) & 1, p.err)) break;
      const int u = tile_q[slot];
      named_barrier(1, 128);
      if (tid == 0) mbar_arrive(&tq_empty[slot]);
      if (u < 0) break;
      const Unit d = decode(u, U1, n1, n2, lay, E);
      const int buf = q & 1;
      if (!mbar_wait(&acc_full[buf], (q >> 1) & 1, p.err)) break;
      tc_fence_after();
      const int b_row = lay[E + 1 + d.e] + d.tt * BN;
      const int tmax = d.rows - d.tt * BN;
      const uint32_t lane_addr = tmem + buf * C::kAcc + (uint32_t(sub * 32) << 16);
      if (d.fc1) {
        const int wrow = d.n * kTileM + sub * 32 + lane;     // intermediate channel
        const float wg = FP4 ? __ldcg(p.w1_g + d.e) : 1.f;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t g[16], uu[16];
          tmem_ld_x16(lane_addr + c0, g);
          tmem_ld_x16(lane_addr + BN + c0, uu);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int orow = b_row + c0 + j;
            if constexpr (FP4) {
              float xg = 0.f;
              if (p.pull) {
                // padding rows of the segment have no token (row_token unset)
                if (c0 + j < tmax) {
                  const int gi = __ldcg(p.row_token + orow);
                  const int sr = gi / p.src_rows;
                  xg = __ldcg(reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(p.src_g[sr]) + g_off) +
                              (gi - sr * p.src_rows));
                }
              } else {
                xg = __ldcg(p.x_g + orow);
              }
              const float sc = wg * xg;
              const float gv = __uint_as_float(g[j]) * sc;
              const float h = gv / (1.0f + __expf(-gv)) * (__uint_as_float(uu[j]) * sc);
              float amax = fabsf(h);
#pragma unroll
              for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
              const float inv_og = 1.f / p.out_g;
              const uint16_t s2 = f2_to_e4m3x2(amax * (1.f / 6.f) * inv_og, 0.f);
              __nv_fp8_e4m3 s8;
              s8.__x = uint8_t(s2 & 0xFF);
              const float sf = float(s8);
              const float v = sf > 0.f ? h * inv_og / sf : 0.f;
              const float vn = __shfl_down_sync(0xffffffffu, v, 1);
              if (c0 + j < tmax) {
                if ((lane & 1) == 0) p.hq[(int64_t)orow * (p.inter / 2) + (wrow >> 1)] = uint8_t(f2_to_e2m1x2(v, vn));
                if ((lane & 15) == 0) p.hq_sf[sf_offset(orow, wrow >> 4, kbq)] = uint8_t(s2 & 0xFF);
              }
            } else {
              const float gv = __uint_as_float(g[j]);
              const float h = gv / (1.0f + __expf(-gv)) * __uint_as_float(uu[j]);
              float amax = fabsf(h);
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
              const int ex = ceil_log2_bits(amax * (1.0f / 448.0f));
              if (c0 + j < tmax) {
                p.hq[(int64_t)orow * p.inter + wrow] = uint8_t(f2_to_e4m3x2(h * exp2_int(-ex), 0.f) & 0xFF);
                if (lane == 0) p.hq_sf[sf_offset(orow, wrow >> 5, kbq)] = uint8_t(ex + 127);
              }
            }
          }
        }
      } else {
        const float wg = FP4 ? __ldcg(p.w2_g + d.e) * p.out_g : 1.f;
        const int cpar = p.c_row_pair ? int(__ldcg(p.c_epoch) & 1u) : 0;
#pragma unroll 1
        for (int a = 0; a < 2; ++a) {
          const int wrow = d.n * 2 * kTileM + a * kTileM + sub * 32 + lane;   // hidden row
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 16) {
            uint32_t r[16];
            tmem_ld_x16(lane_addr + a * BN + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (c0 + j < tmax) {
                const int orow = b_row + c0 + j;
                const float v = __uint_as_float(r[j]) * __ldcg(p.row_weight + orow) * wg;
                if (p.c_row_pair) {
                  // pair (token, k) -> its owner's combine slot [parity][row there][k] (P2P store)
                  const int pair = __ldcg(p.c_row_pair + orow);
                  const int tok = pair / p.c_K;
                  const int kk = pair - tok * p.c_K;
                  const int dst = tok / p.c_T_step;
                  const int tl = tok - dst * p.c_T_step;
                  __nv_bfloat16* slot = reinterpret_cast<__nv_bfloat16*>(p.c_base[dst] + p.c_off) +
                                        (((int64_t)cpar * p.c_max_t + tl) * p.c_K + kk) * p.hidden;
                  slot[wrow] = __float2bfloat16(v);
                } else {
                  p.y[(int64_t)orow * p.ldy + wrow] = __float2bfloat16(v);
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      named_barrier(1, 128);
      if (tid == 0) {
        if (d.fc1) {
          // publish this FC1 unit: its h rows are visible to TMA loads of
          // other CTAs (generic -> async proxy, then release)
          __threadfence();
          fence_proxy_async_global();
          atomicAdd(p.fc1_done + d.e, 1);
        }
        mbar_arrive(&acc_empty[buf]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  // the last CTA resets the work counters (graph replays start from zero);
  // with the combine fused in, it also publishes this rank's arrival on every
  // rank (each CTA's system-scope fence orders its peer stores first)
  if (threadIdx.x == 0) {
    if (p.c_row_pair) __threadfence_system();
    else __threadfence();
    const int prev = atomicAdd(p.work + 1, 1);
    if (prev == gridDim.x - 1) {
      for (int e = 0; e < E; ++e) p.fc1_done[e] = 0;
      p.work[0] = 0;
      __threadfence();
      p.work[1] = 0;
      if (p.c_row_pair) {
        __threadfence_system();
        const int par = int(__ldcg(p.c_epoch) & 1u);
        for (int q = 0; q < p.c_world; ++q)
          asm volatile("red.release.sys.global.add.u32 [%0], %1;"
                       ::"l"(reinterpret_cast<uint32_t*>(p.c_base[q]) + par * kArMaxRanks + p.c_rank), "r"(1u)
                       : "memory");
      }
    }
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

static int map2d(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
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

static int map_tiled(CUtensorMap* m, const void* base, int64_t rows, int64_t cols) {
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

template <int BN, bool FP4>
static int launch(const MoeFusedArgs& a, cudaStream_t st) {
  using C = Cfg<BN, FP4>;
  const int kb1 = FP4 ? a.hidden / 2 : a.hidden, kb2 = FP4 ? a.inter / 2 : a.inter;
  CUtensorMap m1, mx, m2, mh;
  const int64_t r1 = (int64_t)a.E * 2 * a.inter, r2 = (int64_t)a.E * a.hidden;
  if (a.a_tiled ? map_tiled(&m1, a.w13, r1, kb1) : map2d(&m1, a.w13, r1, kb1, kTileM)) return -2;
  if (a.a_tiled ? map_tiled(&m2, a.w2, r2, kb2) : map2d(&m2, a.w2, r2, kb2, kTileM)) return -2;
  if (map2d(&mx, a.pull ? a.hq : a.x, a.rows, a.pull ? kb2 : kb1, BN)) return -3;   // unused when pulling
  if (map2d(&mh, a.hq, a.rows, kb2, BN)) return -3;
  Params p{};
  p.sfa1 = a.w13_sf;
  p.sfa1_estride = a.w13_sf_estride;
  p.sfb1 = a.x_sf;
  p.sfa2 = a.w2_sf;
  p.sfa2_estride = a.w2_sf_estride;
  p.hq = a.hq;
  p.hq_sf = a.hq_sf;
  p.y = reinterpret_cast<__nv_bfloat16*>(a.y);
  p.ldy = a.ldy;
  p.hidden = a.hidden;
  p.inter = a.inter;
  p.E = a.E;
  p.seg_start = a.seg_start;
  p.seg_count = a.seg_count;
  p.ttile_off = a.ttile_off;
  p.row_weight = a.row_weight;
  p.x_g = a.x_g;
  p.w1_g = a.w1_g;
  p.w2_g = a.w2_g;
  p.out_g = a.out_g;
  p.work = a.work;
  p.fc1_done = a.fc1_done;
  p.err = a.err;
  p.a_tiled = a.a_tiled;
  p.pull = a.pull;
  for (int i = 0; i < 8; ++i) {
    p.src_q[i] = a.src_q[i];
    p.src_sf[i] = a.src_sf[i];
    p.src_g[i] = a.src_g[i];
  }
  p.src_rows = a.src_rows;
  p.row_token = a.row_token;
  p.c_row_pair = a.c_row_pair;
  p.c_K = a.c_K;
  p.c_T_step = a.c_T_step;
  for (int i = 0; i < 8; ++i) p.c_base[i] = a.c_base[i];
  p.c_rank = a.c_rank;
  p.c_world = a.c_world;
  p.c_max_t = a.c_max_t;
  p.c_off = a.c_off;
  p.c_epoch = a.c_epoch;
  p.src_epoch = a.src_epoch;
  p.src_epoch_add = a.src_epoch_add;
  p.src_par_bytes = a.src_par_bytes;
  auto kern = moe_fused_kernel<BN, FP4>;
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
  return cudaLaunchKernelEx(&cfg, kern, m1, mx, m2, mh, p) == cudaSuccess ? 0 : 1;
}

template <bool FP4>
static int launch_bn(const MoeFusedArgs& a, cudaStream_t st) {
  switch (a.bn) {
    case 16: return launch<16, FP4>(a, st);
    case 32: return launch<32, FP4>(a, st);
    case 64: return launch<64, FP4>(a, st);
  }
  return -4;
}

}  // namespace moef
}  // namespace b200

int b200_moe_fused(const MoeFusedArgs* a, cudaStream_t st) {
  using namespace b200::moef;
  if (a->E > kMaxExperts || a->E <= 0 || a->num_ctas <= 0 || a->hidden % 256 || a->inter % 128 || !a->work ||
      !a->fc1_done)
    return -1;
  if (a->pull && (a->src_rows <= 0 || !a->row_token || !a->src_q[0] || !a->src_sf[0])) return -1;
  if (a->c_row_pair && (a->c_K <= 0 || a->c_T_step <= 0 || a->c_world < 1 || a->c_world > 8 || !a->c_epoch ||
                        a->c_T_step > a->c_max_t))
    return -1;
  if (a->fp4) {
    if (a->hidden % 256 || a->inter % 256 || !a->w1_g || !a->w2_g || (!a->x_g && !a->pull) ||
        (a->pull && !a->src_g[0]) || a->out_g <= 0.f)
      return -1;
    return launch_bn<true>(*a, st);
  }
  return launch_bn<false>(*a, st);
}
