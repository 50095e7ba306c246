// Absorbed MLA decode attention on tcgen05 over the paged e4m3 latent cache.
//
// Work item = (query token t, group of HB heads, KV split s).  Per 128-token
// KV tile (two 64-token pages fetched by TMA: four 128-byte latent boxes with
// 128B swizzle + one 64-byte rope box with 64B swizzle):
//
//   MMA1  S^T[128 tok, HB] = K[128 tok, 576] . Q[HB, 576]^T      (kind::f8f6f4)
//   softmax warps: S^T -> registers (thread = token row x half of the
//         heads); head-wise tile max by a butterfly over the warp plus one
//         shared-memory exchange between the four warps of a column half;
//         per-head running max in the log2 domain, raised only when a tile
//         exceeds it by more than 8 (so P = 2^(x - m) <= 256 fits e4m3 and O
//         rarely needs a rescale); P written from registers as e4m3 into the
//         MMA2 B operand (MN-major); the softmax denominators accumulate per
//         thread and are reduced once, in the epilogue
//   MMA2  O^T[512, HB] += V^T[512, 128 tok] . P^T[128 tok, HB]    (4 x M=128)
//
// KV tokens are the MMA's M (128) dimension and heads the N dimension, so a
// tensor-parallel rank with 16 heads still issues M=128 MMAs.  O^T lives in
// TMEM for the whole split; the epilogue normalises by the running sum and
// writes bf16 (or a partial + log-sum-exp for the split merge).
//
// Warp roles (320 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2-9 softmax / correction / epilogue (two warps per TMEM
// subpartition, each owning half of the head columns: the per-tile softmax
// is the kernel's critical path, one named barrier per tile).  All waits
// bounded.
//
// Sparse variant (SPARSE = true): the query attends only to the cache
// positions in its top-k list (-1 = unused entry).  The KV rows of a tile are
// then scattered over pages; TMA tile::gather4 loads (this GPU's cache, no
// multicast) bring four rows per instruction into the same 128B / 64B
// swizzled layout the dense boxes produce, so the MMA descriptors are shared
// with the dense path and the stage completes on its transaction bytes.
//
// Reference parity: the reference's own sparse-MLA decode kernel `bsx`
// (ro_unit.cu:480; c36s SPA design ro_unit.cu:136-172) uses the same
// transposed S^T / O^T arrangement with e4m3 P; this kernel is written from
// the PTX ISA, not from that code.
#include "../common/ptx.cuh"
#include "attn.h"

namespace b200 {
namespace mla {

constexpr int kSmThreads = 256;      // softmax / epilogue threads (warps 2-9)
constexpr int kThreads = 64 + kSmThreads;
constexpr int kTile = 128;          // KV tokens per tile
constexpr int kPage = 64;           // tokens per KV page (one TMA box height)
constexpr int kL = 512;             // latent
constexpr int kR = 64;              // rope
constexpr int kD = kL + kR;         // bytes per cached token
constexpr int kStages = 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThresh = 8.0f;

template <int HB>
struct Smem {
  static constexpr int kQLat = 4 * HB * 128;            // 4 latent boxes [HB x 128B]
  static constexpr int kQRope = HB * 64;                // rope box [HB x 64B]
  static constexpr int kKVLat = 4 * kTile * 128;        // 64 KB
  static constexpr int kKVRope = kTile * 64;            // 8 KB
  static constexpr int kKVStage = kKVLat + kKVRope;     // 72 KB
  static constexpr int kP = kTile * HB;                 // e4m3 P^T
  static constexpr int kOffQ = 0;
  static constexpr int kOffKV = ((kQLat + kQRope + 1023) / 1024) * 1024;
  static constexpr int kOffP = kOffKV + kStages * kKVStage;
  static constexpr int kPPad = ((kP + 127) / 128) * 128;
  // P^T double-buffered (softmax of tile i overlaps MMA2 of tile i - 1) when
  // it fits next to two KV stages; 64-head groups keep one buffer.
  static constexpr int kRed = 2 * 2 * 4 * (HB / 2) * 4;  // [parity][half][warp][HB/2] fp32 partial maxima
  static constexpr int kPB = (kOffP + 2 * kPPad + kRed + 256 + 1024 <= 227 * 1024) ? 2 : 1;
  static constexpr int kOffS = kOffP + kPB * kPPad;
  static constexpr int kOffRed = kOffS;
  static constexpr int kOffHead = kOffRed + kRed;
  static constexpr int kOffBar = kOffHead;
  static constexpr int kBytes = kOffBar + 256 + 1024;
  static_assert(kBytes <= 227 * 1024, "shared memory");
  static constexpr int kTmemS = 0;                      // 2 x HB columns
  static constexpr int kTmemO = 2 * HB;                 // 4 x HB columns
  static constexpr int kTmemNeed = 6 * HB;
  static constexpr int kTmemCols = kTmemNeed <= 32 ? 32 : kTmemNeed <= 64 ? 64 : kTmemNeed <= 128 ? 128
                                   : kTmemNeed <= 256 ? 256 : 512;
};

struct Params {
  const int* block_table;
  int bt_stride;
  const int* q_seq;
  const int* q_pos;
  const float* q_scale;      // [T, H]
  int H;
  int nsplit;
  int split_tokens;          // KV tokens per split (multiple of 128)
  float qk_factor;           // sm_scale * kv_scale * log2(e)
  float kv_scale;
  __nv_bfloat16* out;        // [T, H, 512] when nsplit == 1
  float* part_o;             // [nsplit, T, H, 512] when nsplit > 1
  float* part_lse;           // [nsplit, T, H]
  float* lse_out;            // [T, H] log2-domain log-sum-exp of the scaled scores (optional)
  uint32_t* err;
  const uint8_t* cache;      // e4m3 [rows, 576] (sparse gathers)
  const int* topk;           // [T, topk_n] cache positions, -1 = none (sparse)
  int topk_n;
  int ratio2;                // compressed rows (entries >= kMlaCompFlag) in the second cache, 0 = none
};

__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Column reduction of N values per lane over the warp's 32 lanes (max, or
// sum when MX is false) in N - 1 + 5 - log2(N) shuffles: at each step the
// lanes split the remaining columns in two halves, keep one and send the
// other to their partner; afterwards lane l holds column l >> (5 - log2 N)
// in v[0].  Compile-time sizes keep every index static (registers only).
template <int N, int OFF, bool MX>
__device__ __forceinline__ void col_reduce(float* v, int lane) {
  if constexpr (OFF >= 1) {
    if constexpr (N > 1) {
      const bool upper = (lane & OFF) != 0;
#pragma unroll
      for (int j = 0; j < N / 2; ++j) {
        const float give = upper ? v[j] : v[j + N / 2];
        const float keep = upper ? v[j + N / 2] : v[j];
        const float got = __shfl_xor_sync(0xffffffffu, give, OFF);
        v[j] = MX ? fmaxf(keep, got) : keep + got;
      }
      col_reduce<N / 2, OFF / 2, MX>(v, lane);
    } else {
      const float got = __shfl_xor_sync(0xffffffffu, v[0], OFF);
      v[0] = MX ? fmaxf(v[0], got) : v[0] + got;
      col_reduce<1, OFF / 2, MX>(v, lane);
    }
  }
}

template <int HB, bool SPARSE>
__global__ void __launch_bounds__(kThreads, 1)
mla_tc_kernel(const __grid_constant__ CUtensorMap tm_q_lat, const __grid_constant__ CUtensorMap tm_q_rope,
              const __grid_constant__ CUtensorMap tm_kv_lat, const __grid_constant__ CUtensorMap tm_kv_rope,
              const __grid_constant__ CUtensorMap tm_c_lat, const __grid_constant__ CUtensorMap tm_c_rope,
              Params p) {
  using S = Smem<HB>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm + S::kOffQ;
  uint8_t* sKV = sm + S::kOffKV;
  uint8_t* sP = sm + S::kOffP;
  float* sRed = reinterpret_cast<float*>(sm + S::kOffRed);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kOffBar);
  uint64_t* kv_full = bars;              // [2]
  uint64_t* kv_empty = bars + 2;         // [2]
  uint64_t* q_full = bars + 4;
  uint64_t* s_full = bars + 5;           // [2]
  uint64_t* s_free = bars + 7;           // [2]
  uint64_t* p_full = bars + 9;           // [2] P^T buffer (i & 1) written
  uint64_t* o_done = bars + 11;          // [2] MMA2 of tile i (i & 1) complete
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 13);

  const int warp = warp_id(), lane = lane_id();
  const int t = blockIdx.x;
  const int h0 = blockIdx.y * HB;
  const int split = blockIdx.z;

  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  const int b = p.q_seq[t];
  const int n = p.q_pos[t] + 1;
  // Keys: cache positions [0, n) (dense) or the first min(topk_n, n) entries
  // of the query's top-k list (sparse).  Keys per split adapt to this
  // query's own length (graph-safe).
  const int nk = SPARSE ? min(p.topk_n, n) : n;
  const int chunk = (((nk + p.nsplit - 1) / p.nsplit) + kTile - 1) / kTile * kTile;
  const int k_lo = split * chunk;
  const int k_hi = min(nk, k_lo + chunk);
  const int nt = k_hi > k_lo ? (k_hi - k_lo + kTile - 1) / kTile : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kSmThreads / 32);    // one arrival per softmax warp
    }
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], kSmThreads / 32);    // one arrival per softmax warp
      mbar_init(&o_done[i], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (SPARSE && nt > 0) {
      // Sparse rows are gathered by TMA (tile::gather4: four cache rows of one
      // 128-byte latent column box, or of the 64-byte rope box, per
      // instruction, into the same swizzled layout the dense boxes produce).
      // Lane l resolves rows 4l..4l+3 of the tile to cache rows and issues
      // their five gathers; lane 0 posts the stage's byte count first.  Rows
      // with no entry read the sequence's position 0 (always written) and are
      // masked to -inf by the softmax.  Completion is tracked by the stage's
      // transaction bytes, so the producer never waits for its own copies.
      if (lane == 0) {
        const int qrow = t * p.H + h0;
        mbar_arrive_expect_tx(q_full, S::kQLat + S::kQRope);
        for (int c = 0; c < 4; ++c) tma_load_2d(sQ + c * HB * 128, &tm_q_lat, q_full, c * 128, qrow);
        tma_load_2d(sQ + S::kQLat, &tm_q_rope, q_full, kL, qrow);
      }
      __syncwarp();
      const int* list = p.topk + (int64_t)t * p.topk_n;
      const int64_t row0 = (int64_t)__ldcg(p.block_table + (int64_t)b * p.bt_stride) * kPage;   // position 0
      for (int i = 0; i < nt; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(&kv_empty[s], ((i / kStages) - 1) & 1, p.err)) break;
        uint8_t* dst = sKV + s * S::kKVStage;
        const int tok0 = k_lo + i * kTile;
        if (lane == 0) mbar_arrive_expect_tx(&kv_full[s], S::kKVStage);
        __syncwarp();
        int ent[4], rows[4];
        bool comp = false;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int j = tok0 + 4 * lane + m;                 // list entry of tile row 4 lane + m
          ent[m] = j < k_hi ? __ldcg(list + j) : -1;
          comp |= (p.ratio2 > 0 && ent[m] >= kMlaCompFlag);
        }
        // a group of four entries reads one cache: compressed blocks (entries
        // >= kMlaCompFlag; the selection keeps them in groups of four after
        // the window) or full-resolution positions; a group's empty entries
        // read that cache's first row and are masked by the softmax
        const int cpage = comp ? kPage / p.ratio2 : kPage;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          if (comp) {
            const int jb = ent[m] >= kMlaCompFlag ? ent[m] - kMlaCompFlag : 0;
            const int q0 = jb * p.ratio2;
            rows[m] = __ldcg(p.block_table + (int64_t)b * p.bt_stride + q0 / kPage) * cpage + (q0 % kPage) / p.ratio2;
          } else {
            rows[m] = (ent[m] >= 0 && ent[m] < n)
                          ? __ldcg(p.block_table + (int64_t)b * p.bt_stride + ent[m] / kPage) * kPage + ent[m] % kPage
                          : int(row0);
          }
        }
        const CUtensorMap* ml = comp ? &tm_c_lat : &tm_kv_lat;
        const CUtensorMap* mr = comp ? &tm_c_rope : &tm_kv_rope;
#pragma unroll
        for (int c = 0; c < 4; ++c)                          // latent: 4 boxes of 128 B
          tma_gather4(dst + c * kTile * 128 + 4 * lane * 128, ml, &kv_full[s], c * 128, rows);
        tma_gather4(dst + S::kKVLat + 4 * lane * 64, mr, &kv_full[s], kL, rows);
      }
    } else if (!SPARSE && nt > 0) {
      // The warp reads the split's page ids 32 at a time (lane l holds the
      // page of logical page lp0 + 32 w + l) ahead of the tiles that use
      // them, so no block-table load sits between a stage's release and its
      // next TMA issue; lane 0 issues the loads.
      if (lane == 0) {
        const int qrow = t * p.H + h0;
        mbar_arrive_expect_tx(q_full, S::kQLat + S::kQRope);
        for (int c = 0; c < 4; ++c) tma_load_2d(sQ + c * HB * 128, &tm_q_lat, q_full, c * 128, qrow);
        tma_load_2d(sQ + S::kQLat, &tm_q_rope, q_full, kL, qrow);
      }
      const int* btr = p.block_table + (int64_t)b * p.bt_stride;
      const int lp0 = k_lo / kPage;                  // k_lo is a multiple of the 128-token tile
      int pg_reg = 0;
      for (int i = 0; i < nt; ++i) {
        const int s = i % kStages;
        if ((i & 15) == 0) {                         // 16 tiles = 32 pages per window
          const int lp = lp0 + 2 * i + lane;
          pg_reg = (lp * kPage < n) ? __ldcg(btr + lp) : 0;     // past the end: the scratch page 0
        }
        int okw = 1;
        if (lane == 0 && i >= kStages && !mbar_wait(&kv_empty[s], ((i / kStages) - 1) & 1, p.err)) okw = 0;
        if (!__shfl_sync(0xffffffffu, okw, 0)) break;
        const int pa = __shfl_sync(0xffffffffu, pg_reg, (2 * i) & 31);
        const int pb = __shfl_sync(0xffffffffu, pg_reg, (2 * i + 1) & 31);
        if (lane == 0) {
          mbar_arrive_expect_tx(&kv_full[s], S::kKVStage);
          uint8_t* dst = sKV + s * S::kKVStage;
          for (int pg = 0; pg < 2; ++pg) {
            const int row = (pg ? pb : pa) * kPage;
            for (int c = 0; c < 4; ++c)
              tma_load_2d(dst + c * kTile * 128 + pg * kPage * 128, &tm_kv_lat, &kv_full[s], c * 128, row);
            tma_load_2d(dst + S::kKVLat + pg * kPage * 64, &tm_kv_rope, &kv_full[s], kL, row);
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    const uint32_t idesc1 = idesc_f8(128, HB, false, false);
    const uint32_t idesc2 = idesc_f8(128, HB, true, true);
    bool ok = nt > 0 && mbar_wait(q_full, 0, p.err);
    auto mma2 = [&](int i) -> bool {
      if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1, p.err)) return false;
      tc_fence_after();
      if (lane == 0) {
        const int s = i % kStages;
        const uint32_t kv = smem_u32(sKV + s * S::kKVStage);
        const uint32_t pb = smem_u32(sP + (i % S::kPB) * S::kPPad);
        for (int c = 0; c < 4; ++c) {
          for (int kk = 0; kk < kTile / 32; ++kk) {
            // A = V^T: MN-major SW128, 8-token groups 1024 B apart
            const uint64_t ad = smem_desc(kv + c * kTile * 128 + kk * 32 * 128, 0, 1024, 2);
            // B = P^T: MN-major no swizzle; core matrix = 8 tokens x 16 heads
            const uint64_t bd = smem_desc(pb + kk * 4 * (HB / 16) * 128, (HB / 16) * 128, 128, 0);
            mma_f8(tmem + S::kTmemO + c * HB, ad, bd, idesc2, (i > 0 || kk > 0) ? 1u : 0u);
          }
        }
        mma_commit(&o_done[i & 1]);
        mma_commit(&kv_empty[s]);
      }
      __syncwarp();
      return true;
    };
    for (int i = 0; ok && i < nt; ++i) {
      const int s = i % kStages;
      if (!mbar_wait(&kv_full[s], (i / kStages) & 1, p.err)) { ok = false; break; }
      if (i >= 2 && !mbar_wait(&s_free[i & 1], ((i >> 1) - 1) & 1, p.err)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t kv = smem_u32(sKV + s * S::kKVStage);
        const uint32_t q = smem_u32(sQ);
        const uint32_t d = tmem + S::kTmemS + (i & 1) * HB;
        int step = 0;
        for (int c = 0; c < 4; ++c)
          for (int kk = 0; kk < 4; ++kk, ++step)
            mma_f8(d, desc_kmajor_sw128(kv + c * kTile * 128 + kk * 32), desc_kmajor_sw128(q + c * HB * 128 + kk * 32),
                   idesc1, step > 0 ? 1u : 0u);
        for (int kk = 0; kk < 2; ++kk)
          mma_f8(d, smem_desc(kv + S::kKVLat + kk * 32, 16, 512, 4), smem_desc(q + S::kQLat + kk * 32, 16, 512, 4),
                 idesc1, 1u);
        mma_commit(&s_full[i & 1]);
      }
      __syncwarp();
      if (i >= 1 && !mma2(i - 1)) { ok = false; break; }
    }
    if (ok && nt > 0) mma2(nt - 1);
  } else {
    // ---------------------- softmax / correction / epilogue ----------------------
    // Thread = one token row of the tile (TMEM lane) x NC = HB/2 head columns
    // held in registers: warps 2-5 take heads [0, NC), warps 6-9 [NC, HB).
    // Per tile: the head-wise tile max is reduced in registers (butterfly over
    // the warp) and across the four warps of a column half through shared
    // memory (the tile's only named barrier); P is written straight from
    // registers into the MMA2 operand; the softmax denominator accumulates
    // per thread (its rows) and is reduced once at the end.
    constexpr int NC = HB / 2;
    constexpr int kLogNC = NC == 8 ? 3 : NC == 16 ? 4 : 5;
    const int sub = warp & 3;                    // TMEM subpartition
    const int half = (warp - 2) >> 2;            // column half
    const int hc0 = half * NC;
    const int row = sub * 32 + lane;             // token row of S^T / latent row of O^T
    const int wslot = (warp - 2) & 3;            // this warp's slot among the 4 of its half
    const int mycol = lane >> (5 - kLogNC);      // column whose max / sum this lane holds after a reduction
    float fac[NC], m[NC], lrow[NC];
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      fac[j] = p.q_scale[(int64_t)t * p.H + h0 + hc0 + j] * p.qk_factor;
      m[j] = -INFINITY;
      lrow[j] = 0.f;
    }
    // sRed: [2 tile parities][2 halves][4 warps][NC] partial maxima.
    // A wait that runs out of time clears `ok`; the warp then skips its
    // remaining waits but keeps taking part in every named barrier, so the
    // eight warps never disagree on the barrier count.
    bool ok = true;
    for (int i = 0; i < nt; ++i) {
      const int tok0 = k_lo + i * kTile;
      // the row's list entry is loaded before the wait for S (it does not depend on it)
      int pos = 0;
      if (SPARSE && tok0 + row < k_hi) pos = __ldcg(p.topk + (int64_t)t * p.topk_n + tok0 + row);
      if (ok && !mbar_wait(&s_full[i & 1], (i >> 1) & 1, p.err)) ok = false;
      tc_fence_after();
      float x[NC];
      {
        const uint32_t base = tmem + S::kTmemS + (i & 1) * HB + hc0 + (uint32_t(sub * 32) << 16);
#pragma unroll
        for (int c0 = 0; c0 < NC; c0 += 8) {
          uint32_t r[8];
          tmem_ld_x8(base + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) x[c0 + j] = __uint_as_float(r[j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[i & 1]);      // this warp's S^T columns are read
      bool valid = tok0 + row < k_hi;
      if (SPARSE && valid) valid = (pos >= 0 && pos < n) || (p.ratio2 > 0 && pos >= kMlaCompFlag);
      float v[NC];
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        x[j] = valid ? x[j] * fac[j] : -INFINITY;
        v[j] = x[j];
      }
      // butterfly max over the warp's 32 rows: lane ends with column `mycol`
      col_reduce<NC, 16, true>(v, lane);
      float* red = sRed + ((i & 1) * 2 + half) * 4 * NC;
      if ((lane & ((32 >> kLogNC) - 1)) == 0) red[wslot * NC + mycol] = v[0];
      named_bar(1, kSmThreads);
      // new running max (raised lazily: only when a tile exceeds it by more
      // than kRescaleThresh, so P = 2^(x - m) <= 256 fits e4m3)
      bool changed = false;
      float alpha[NC];
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        const float mt = fmaxf(fmaxf(red[j], red[NC + j]), fmaxf(red[2 * NC + j], red[3 * NC + j]));
        alpha[j] = 1.f;
        if (mt > m[j] + kRescaleThresh || (m[j] == -INFINITY && mt != -INFINITY)) {
          alpha[j] = (m[j] == -INFINITY) ? 0.f : exp2f(m[j] - mt);
          if (m[j] != -INFINITY) changed = true;
          m[j] = mt;
        }
      }
      // P^T buffer (i % kPB) was last read by MMA2 of tile i - kPB
      if (ok && i >= S::kPB && !mbar_wait(&o_done[(i - S::kPB) & 1], ((i - S::kPB) >> 1) & 1, p.err)) ok = false;
      uint8_t* sPi = sP + (i % S::kPB) * S::kPPad;
      // P = 2^(x - m) as e4m3 into the MN-major core-matrix layout
      // [k group row/8][n chunk h/16][8 x 16]; the row sum uses the quantized P
#pragma unroll
      for (int c0 = 0; c0 < NC; c0 += 16) {
        constexpr int W16 = NC < 16 ? NC : 16;
        uint32_t pk[W16 / 4];
#pragma unroll
        for (int j = 0; j < W16; j += 2) {
          const int a = c0 + j;
          const float p0 = (x[a] == -INFINITY) ? 0.f : exp2f(x[a] - m[a]);
          const float p1 = (x[a + 1] == -INFINITY) ? 0.f : exp2f(x[a + 1] - m[a + 1]);
          const uint16_t q2 = f2_to_e4m3x2(p0, p1);
          __nv_fp8_e4m3 f0, f1;
          f0.__x = uint8_t(q2 & 0xFF);
          f1.__x = uint8_t(q2 >> 8);
          lrow[a] = lrow[a] * alpha[a] + float(f0);
          lrow[a + 1] = lrow[a + 1] * alpha[a + 1] + float(f1);
          if ((j & 2) == 0) pk[j >> 2] = q2;
          else pk[j >> 2] |= uint32_t(q2) << 16;
        }
        const int h = hc0 + c0;
        uint8_t* dstp = sPi + (row >> 3) * (HB / 16) * 128 + (h >> 4) * 128 + (row & 7) * 16 + (h & 15);
        if constexpr (W16 == 16) {
          *reinterpret_cast<uint4*>(dstp) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        } else {
          *reinterpret_cast<uint2*>(dstp) = make_uint2(pk[0], pk[1]);
        }
      }
      // rescale this warp's O^T columns whose max moved (rare): after MMA2 of tile i - 1
      if (__any_sync(0xffffffffu, changed) && i >= 1 && ok) {
        if (!mbar_wait(&o_done[(i - 1) & 1], ((i - 1) >> 1) & 1, p.err)) ok = false;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const uint32_t ob = tmem + S::kTmemO + c * HB + hc0 + (uint32_t(sub * 32) << 16);
#pragma unroll
          for (int c0 = 0; c0 < NC; c0 += 8) {
            uint32_t r[8];
            tmem_ld_x8(ob + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 8; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha[c0 + j]);
            tmem_st_x8(ob + c0, r);
          }
        }
        tmem_st_wait();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[i & 1]);      // this warp's P rows (and O^T rescale) are done
    }
    // softmax denominators: sum of lrow over the 128 rows, per head
    float l[NC];
    {
      float v[NC];
#pragma unroll
      for (int j = 0; j < NC; ++j) v[j] = lrow[j];
      col_reduce<NC, 16, false>(v, lane);
      named_bar(1, kSmThreads);                        // every warp is past its last tile's max exchange
      float* red = sRed + half * 4 * NC;
      if ((lane & ((32 >> kLogNC) - 1)) == 0) red[wslot * NC + mycol] = v[0];
      named_bar(1, kSmThreads);
#pragma unroll
      for (int j = 0; j < NC; ++j) l[j] = (red[j] + red[NC + j]) + (red[2 * NC + j] + red[3 * NC + j]);
    }
    // epilogue: O^T (lane = latent row within block c, column = head)
    if (nt > 0 && ok && mbar_wait(&o_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, p.err)) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const uint32_t ob = tmem + S::kTmemO + c * HB + hc0 + (uint32_t(sub * 32) << 16);
        const int d = c * 128 + row;
#pragma unroll
        for (int c0 = 0; c0 < NC; c0 += 8) {
          uint32_t r[8];
          tmem_ld_x8(ob + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int h = hc0 + c0 + j;
            const float lj = l[c0 + j];
            const float o = lj > 0.f ? __uint_as_float(r[j]) * p.kv_scale / lj : 0.f;
            const int64_t oi = ((int64_t)t * p.H + h0 + h) * kL + d;
            if (p.nsplit == 1) {
              p.out[oi] = __float2bfloat16(o);
            } else {
              p.part_o[(int64_t)split * ((int64_t)gridDim.x * p.H * kL) + oi] = o;
            }
          }
        }
      }
      if (sub == 0 && lane < NC && (p.nsplit > 1 || p.lse_out)) {
        // lane j of warp (sub 0) of each half writes head hc0 + j
        float lj = 0.f, mj = -INFINITY;
#pragma unroll
        for (int j = 0; j < NC; ++j)
          if (j == lane) { lj = l[j]; mj = m[j]; }
        const float v = lj > 0.f ? mj + log2f(lj) : -INFINITY;
        const int h = hc0 + lane;
        if (p.nsplit > 1) p.part_lse[(int64_t)split * gridDim.x * p.H + (int64_t)t * p.H + h0 + h] = v;
        else p.lse_out[(int64_t)t * p.H + h0 + h] = v;
      }
    } else if (sub == 0 && lane < NC && (p.nsplit > 1 || p.lse_out)) {
      // empty split
      const int h = hc0 + lane;
      if (p.nsplit > 1) p.part_lse[(int64_t)split * gridDim.x * p.H + (int64_t)t * p.H + h0 + h] = -INFINITY;
      else p.lse_out[(int64_t)t * p.H + h0 + h] = -INFINITY;
    }
    const int tid = threadIdx.x - 64;
    if (nt == 0 && p.nsplit == 1) {
      for (int e = tid; e < HB * kL; e += kSmThreads)
        p.out[((int64_t)t * p.H + h0) * kL + e] = __float2bfloat16(0.f);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// Merge split partials: out = sum_s 2^(lse_s - M) o_s / sum_s 2^(lse_s - M).
__global__ void mla_merge_kernel(const float* part_o, const float* part_lse, int nsplit, int TH, __nv_bfloat16* out,
                                 float* lse_out) {
  const int th = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_lse[(int64_t)s * TH + th]);
  float w[16];
  float den = 0.f;
  for (int s = 0; s < nsplit && s < 16; ++s) {
    const float l = part_lse[(int64_t)s * TH + th];
    w[s] = (l == -INFINITY) ? 0.f : exp2f(l - M);
    den += w[s];
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  if (lse_out && threadIdx.x == 0) lse_out[th] = den > 0.f ? M + log2f(den) : -INFINITY;
  for (int d = threadIdx.x; d < kL; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < nsplit && s < 16; ++s)
      if (w[s] != 0.f) acc += w[s] * part_o[((int64_t)s * TH + th) * kL + d];
    out[(int64_t)th * kL + d] = __float2bfloat16(acc * inv);
  }
}

// q_abs [T,H,512] bf16 + q_pe [T,H,64] bf16 -> e4m3 [T,H,576] with a per-(t,h) fp32 scale.
__global__ void q_quant_kernel(const __nv_bfloat16* q_abs, const __nv_bfloat16* q_pe, int TH, uint8_t* q8, float* qs) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  if (w >= TH) return;
  const __nv_bfloat16* a = q_abs + (int64_t)w * kL;
  const __nv_bfloat16* r = q_pe + (int64_t)w * kR;
  float v[18];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __bfloat162float(a[lane + 32 * i]);
  v[16] = __bfloat162float(r[lane]);
  v[17] = __bfloat162float(r[lane + 32]);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 18; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / sc;
  uint8_t* dst = q8 + (int64_t)w * kD;
#pragma unroll
  for (int i = 0; i < 16; ++i) dst[lane + 32 * i] = uint8_t(f2_to_e4m3x2(v[i] * inv, 0.f) & 0xFF);
  dst[kL + lane] = uint8_t(f2_to_e4m3x2(v[16] * inv, 0.f) & 0xFF);
  dst[kL + lane + 32] = uint8_t(f2_to_e4m3x2(v[17] * inv, 0.f) & 0xFF);
  if (lane == 0) qs[w] = sc;
}

// q_abs (strided [T,H,512] bf16, e.g. the head-major batched-GEMM output) and
// the un-rotated rope part q_pe (strided [T,H,64]) -> RoPE on q_pe, then e4m3
// [T,H,576] with a per-(t,h) fp32 scale: one warp per (token, head).
__global__ void q_prep_kernel(const __nv_bfloat16* q_abs, int64_t qa_t, int64_t qa_h, const __nv_bfloat16* q_pe,
                              int64_t qp_t, int64_t qp_h, int T, int H, const int* pos, const float* table,
                              uint8_t* q8, float* qs) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  if (w >= T * H) return;
  const int t = w / H, h = w - t * H;
  const __nv_bfloat16* a = q_abs + (int64_t)t * qa_t + (int64_t)h * qa_h;
  const __nv_bfloat16* r = q_pe + (int64_t)t * qp_t + (int64_t)h * qp_h;
  float v[18];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __bfloat162float(a[lane + 32 * i]);
  {
    // rope pair (2 lane, 2 lane + 1) at frequency lane; table row = cos(32) | sin(32)
    const float x0 = __bfloat162float(r[2 * lane]), x1 = __bfloat162float(r[2 * lane + 1]);
    const float* tr = table + (int64_t)pos[t] * kR;
    const float c = tr[lane], sn = tr[kR / 2 + lane];
    v[16] = x0 * c - x1 * sn;
    v[17] = x0 * sn + x1 * c;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 18; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / sc;
  uint8_t* dst = q8 + (int64_t)w * kD;
#pragma unroll
  for (int i = 0; i < 16; ++i) dst[lane + 32 * i] = uint8_t(f2_to_e4m3x2(v[i] * inv, 0.f) & 0xFF);
  *reinterpret_cast<uint16_t*>(dst + kL + 2 * lane) = f2_to_e4m3x2(v[16] * inv, v[17] * inv);
  if (lane == 0) qs[w] = sc;
}

// ---------------------------------------------------------------------------
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

static int map2d(CUtensorMap* m, const void* base, int64_t rows, int box_rows, int box_cols, CUtensorMapSwizzle sw) {
  cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kD};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

template <int HB, bool SPARSE>
static int launch(const MlaTcArgs& a, cudaStream_t st) {
  using S = Smem<HB>;
  CUtensorMap mql, mqr, mkl, mkr;
  const int64_t qrows = (int64_t)a.T * a.H;
  if (map2d(&mql, a.q8, qrows, HB, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return -2;
  if (map2d(&mqr, a.q8, qrows, HB, 64, CU_TENSOR_MAP_SWIZZLE_64B)) return -3;
  // dense: one 64-row page per box; sparse: one-row boxes for tile::gather4
  const int kv_box_rows = SPARSE ? 1 : kPage;
  if (map2d(&mkl, a.cache, a.cache_rows, kv_box_rows, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return -4;
  if (map2d(&mkr, a.cache, a.cache_rows, kv_box_rows, 64, CU_TENSOR_MAP_SWIZZLE_64B)) return -5;
  // compressed rows (sparse only; otherwise the maps repeat the main cache's, unused)
  CUtensorMap mcl = mkl, mcr = mkr;
  if (SPARSE && a.cache2 && a.ratio2 > 0) {
    if (map2d(&mcl, a.cache2, a.cache2_rows, 1, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return -7;
    if (map2d(&mcr, a.cache2, a.cache2_rows, 1, 64, CU_TENSOR_MAP_SWIZZLE_64B)) return -8;
  }
  Params p{};
  p.block_table = a.block_table;
  p.bt_stride = a.bt_stride;
  p.q_seq = a.q_seq;
  p.q_pos = a.q_pos;
  p.q_scale = a.q_scale;
  p.H = a.H;
  p.nsplit = a.nsplit;
  p.split_tokens = a.split_tokens;
  p.qk_factor = a.sm_scale * a.kv_scale * kLog2e;
  p.kv_scale = a.kv_scale;
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.part_o = a.part_o;
  p.part_lse = a.part_lse;
  p.lse_out = a.lse_out;
  p.err = a.err;
  p.cache = a.cache;
  p.topk = a.topk;
  p.topk_n = a.topk_n;
  p.ratio2 = (SPARSE && a.cache2) ? a.ratio2 : 0;
  auto kern = mla_tc_kernel<HB, SPARSE>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
  dim3 grid(a.T, a.H / HB, a.nsplit);
  b200::launch_pdl(kern, dim3(grid), dim3(kThreads), S::kBytes, st, mql, mqr, mkl, mkr, mcl, mcr, p);
  if (cudaGetLastError() != cudaSuccess) return 1;
  if (a.nsplit > 1) {
    b200::launch_pdl(mla_merge_kernel, dim3(a.T * a.H), dim3(128), 0, st, a.part_o, a.part_lse, a.nsplit, a.T * a.H,
                                                 reinterpret_cast<__nv_bfloat16*>(a.out), a.lse_out);
    if (cudaGetLastError() != cudaSuccess) return 2;
  }
  return 0;
}

}  // namespace mla
}  // namespace b200

int b200_mla_q_quant(const void* q_abs, const void* q_pe, int TH, uint8_t* q8, float* qs, cudaStream_t st) {
  if (TH <= 0) return 0;
  b200::launch_pdl(b200::mla::q_quant_kernel, dim3((TH * 32 + 127) / 128), dim3(128), 0, st, 
      reinterpret_cast<const __nv_bfloat16*>(q_abs), reinterpret_cast<const __nv_bfloat16*>(q_pe), TH, q8, qs);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_mla_q_prep(const void* q_abs, int64_t qa_t, int64_t qa_h, const void* q_pe, int64_t qp_t, int64_t qp_h, int T,
                    int H, const int* pos, const float* table, uint8_t* q8, float* qs, cudaStream_t st) {
  if (T * H <= 0) return 0;
  b200::launch_pdl(b200::mla::q_prep_kernel, dim3((T * H * 32 + 127) / 128), dim3(128), 0, st,
                   reinterpret_cast<const __nv_bfloat16*>(q_abs), qa_t, qa_h,
                   reinterpret_cast<const __nv_bfloat16*>(q_pe), qp_t, qp_h, T, H, pos, table, q8, qs);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_mla_tc(const MlaTcArgs* a, cudaStream_t st) {
  using namespace b200::mla;
  if (a->T <= 0) return 0;
  if (a->page_size != kPage || a->nsplit < 1 || a->nsplit > 16) return -1;
  const int hb = a->hb ? a->hb : (a->H % 64 == 0 ? 64 : a->H % 32 == 0 ? 32 : 16);
  if (a->H % hb != 0) return -6;
  if (a->topk != nullptr) {
    if (a->topk_n <= 0) return -1;
    if (hb == 64) return launch<64, true>(*a, st);
    if (hb == 32) return launch<32, true>(*a, st);
    if (hb == 16) return launch<16, true>(*a, st);
    return -6;
  }
  if (hb == 64) return launch<64, false>(*a, st);
  if (hb == 32) return launch<32, false>(*a, st);
  if (hb == 16) return launch<16, false>(*a, st);
  return -6;
}

// ===========================================================================
// Allocation-free MLA decode entry point.
//
// For callers that must not allocate device memory themselves: a host
// runtime that has already handed all of HBM to its own pool (weights + KV
// cache reserved up front), or one that cannot afford the device-wide
// synchronisation that cudaMalloc / cudaFree may cause in the middle of
// serving.  The caller passes inputs and the output; the kernel's scratch
// (quantised queries, per-split partial outputs and log-sum-exps) lives in
// the fixed device arrays below.
//
// Limits: T * H <= kNoAllocMaxRows query rows and nsplit * T * H <=
// kNoAllocMaxPartRows split partials; larger requests are rejected with
// B200_NOALLOC_ERR_TOO_LARGE.  The arrays total about 10.8 MB and every GPU
// that loads this library keeps them until the process exits.  All calls
// share them: two calls whose kernels overlap on the GPU (different streams,
// or different host threads) race on the scratch and give wrong results.
// Nothing in the scratch needs to start at zero: each call writes every
// element it later reads.  The first call on a device looks up the arrays'
// device addresses (cudaGetSymbolAddress) with that device current; make
// that first call before any stream capture.  The stream passed must belong
// to the current device (checked: a stream of another device is rejected).
//
// Errors inside the kernels (a bounded mbarrier wait that ran out of time)
// set bits in a status word that also lives in the library (sticky across
// calls, zero at load).  b200_mla_decode_noalloc_status reads it after the
// stream's work and clears it, so a caller can tell a timed-out decode from
// a good one without allocating anything.
// ===========================================================================
#include <mutex>

namespace {
constexpr int kNoAllocMaxRows = 4096;                  // T * H
constexpr int kNoAllocMaxPartRows = 4096;              // nsplit * T * H
static __device__ __align__(256) uint8_t g_noalloc_q8[kNoAllocMaxRows * 576];
static __device__ __align__(256) float g_noalloc_qscale[kNoAllocMaxRows];
static __device__ __align__(256) float g_noalloc_part_o[kNoAllocMaxPartRows * 512];
static __device__ __align__(256) float g_noalloc_part_lse[kNoAllocMaxPartRows];
static __device__ __align__(256) uint32_t g_noalloc_err;   // kernel status bits (sticky until read)

constexpr int kMaxDevices = 64;
struct NoAllocScratch {
  bool ready = false;
  uint8_t* q8 = nullptr;
  float* qscale = nullptr;
  float* part_o = nullptr;
  float* part_lse = nullptr;
  uint32_t* err = nullptr;
};
NoAllocScratch g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

int noalloc_setup(int dev) {
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  NoAllocScratch& s = g_scratch[dev];
  if (s.ready) return 0;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.q8), g_noalloc_q8) != cudaSuccess) return -1;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.qscale), g_noalloc_qscale) != cudaSuccess) return -1;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.part_o), g_noalloc_part_o) != cudaSuccess) return -1;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.part_lse), g_noalloc_part_lse) != cudaSuccess) return -1;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.err), g_noalloc_err) != cudaSuccess) return -1;
  s.ready = true;
  return 0;
}
}  // namespace

extern "C" __attribute__((visibility("default"))) int b200_mla_decode_noalloc(
    const void* q_abs, const void* q_pe, int T, int H, const void* kv_cache, long long cache_rows,
    const int* block_table, int bt_stride, const int* q_seq, const int* q_pos, int page_size, float sm_scale,
    float kv_scale, int nsplit, void* out, cudaStream_t stream) {
  if (T <= 0 || H <= 0 || nsplit < 1 || nsplit > 16 || page_size != b200::mla::kPage || (H % 16) != 0 ||
      !q_abs || !q_pe || !kv_cache || !block_table || !q_seq || !q_pos || !out)
    return B200_NOALLOC_ERR_BAD_ARG;
  if ((long long)T * H > kNoAllocMaxRows || (long long)nsplit * T * H > kNoAllocMaxPartRows)
    return B200_NOALLOC_ERR_TOO_LARGE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return B200_NOALLOC_ERR_SETUP;
  if (stream != nullptr) {                 // the scratch addresses are the current device's
    int sdev = -1;
    if (cudaStreamGetDevice(stream, &sdev) != cudaSuccess || sdev != dev) return B200_NOALLOC_ERR_BAD_ARG;
  }
  if (noalloc_setup(dev) != 0) return B200_NOALLOC_ERR_SETUP;
  const NoAllocScratch& s = g_scratch[dev];
  if (b200_mla_q_quant(q_abs, q_pe, T * H, s.q8, s.qscale, stream) != 0) return B200_NOALLOC_ERR_LAUNCH;
  MlaTcArgs a{};
  a.q8 = s.q8;
  a.q_scale = s.qscale;
  a.cache = reinterpret_cast<const uint8_t*>(kv_cache);
  a.cache_rows = cache_rows;
  a.block_table = block_table;
  a.bt_stride = bt_stride;
  a.q_seq = q_seq;
  a.q_pos = q_pos;
  a.T = T;
  a.H = H;
  a.page_size = page_size;
  a.nsplit = nsplit;
  a.sm_scale = sm_scale;
  a.kv_scale = kv_scale;
  a.out = out;
  a.part_o = s.part_o;
  a.part_lse = s.part_lse;
  a.err = s.err;
  return b200_mla_tc(&a, stream) == 0 ? 0 : B200_NOALLOC_ERR_LAUNCH;
}

// Waits for `stream`, copies the kernels' status word of the current device
// into *status (0 = every call since the last read finished its waits) and
// clears it.  No allocation: one copy to the caller's host word, one memset.
extern "C" __attribute__((visibility("default"))) int b200_mla_decode_noalloc_status(cudaStream_t stream,
                                                                                    unsigned int* status) {
  if (!status) return B200_NOALLOC_ERR_BAD_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return B200_NOALLOC_ERR_SETUP;
  if (noalloc_setup(dev) != 0) return B200_NOALLOC_ERR_SETUP;
  uint32_t* e = g_scratch[dev].err;
  if (cudaMemcpyAsync(status, e, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaMemsetAsync(e, 0, sizeof(uint32_t), stream) != cudaSuccess || cudaStreamSynchronize(stream) != cudaSuccess)
    return B200_NOALLOC_ERR_LAUNCH;
  return 0;
}

extern "C" __attribute__((visibility("default"))) const char* b200_mla_decode_noalloc_error(int code) {
  switch (code) {
    case 0: return "ok";
    case B200_NOALLOC_ERR_BAD_ARG:
      return "bad argument (null pointer, T/H <= 0, H not a multiple of 16, nsplit outside 1..16, page size != 64, "
             "or a stream of another device than the current one)";
    case B200_NOALLOC_ERR_TOO_LARGE:
      return "request exceeds the static scratch: need T*H <= 4096 and nsplit*T*H <= 4096";
    case B200_NOALLOC_ERR_SETUP: return "could not look up the scratch arrays' device addresses";
    case B200_NOALLOC_ERR_LAUNCH: return "kernel launch failed";
  }
  return "unknown error";
}
