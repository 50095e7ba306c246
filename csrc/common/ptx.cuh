// Hand-written PTX wrappers for sm_100a: mbarriers, TMA (tiled and 1-D bulk
// loads, never cluster-broadcast), tcgen05 (TMEM alloc, MMA, commit, loads,
// scale-factor copies), PDL and bounded waits.
//
// Every wait in this project is bounded: spin loops give up after a
// %globaltimer deadline, record an error code in a device word the host
// checks, and return, so a protocol bug cannot hang a shared GPU.
#pragma once
#include <cstdlib>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#define B200_DEVICE __device__ __forceinline__

namespace b200 {

// ---------------------------------------------------------------------------
// misc
// ---------------------------------------------------------------------------
B200_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

B200_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

B200_DEVICE bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

B200_DEVICE int warp_id() { return threadIdx.x >> 5; }
B200_DEVICE int lane_id() { return threadIdx.x & 31; }

// Programmatic dependent launch.
B200_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
B200_DEVICE void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Error codes written to the device status word.
enum : uint32_t {
  kOk = 0,
  kErrMbarTimeout = 1,
  kErrPeerTimeout = 2,
  kErrBadArg = 3,
  kErrDepTimeout = 4,     // an in-kernel dependency (another CTA's work) did not arrive in time
};

// Wall-clock budget for any single wait inside a kernel (ns).
constexpr uint64_t kWaitBudgetNs = 2000000000ull;  // 2 s

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
B200_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

B200_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

B200_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

B200_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

B200_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

B200_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and sets *err) when the
// budget ran out; callers then skip the remaining work and exit cleanly.
B200_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) {
      if (err) atomicExch(err, kErrMbarTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA / bulk copies (global -> shared, this GPU's memory or a peer's; no
// cluster broadcast anywhere in this project)
// ---------------------------------------------------------------------------
B200_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

B200_DEVICE void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y,
                             int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// TMA gather of four rows (rows[0..3]) of one column box starting at byte
// column x of a 2-D tensor map whose box is one row high (this GPU's memory;
// no cluster broadcast).  The rows land consecutively at smem_dst, swizzled
// by the map's mode like a 4-row box.
B200_DEVICE void tma_gather4(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, const int (&rows)[4]) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(rows[0]),
        "r"(rows[1]), "r"(rows[2]), "r"(rows[3])
      : "memory");
}

// 1-D bulk copy: both addresses 16-byte aligned, bytes a multiple of 16.
B200_DEVICE void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

B200_DEVICE void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor (sm_100 layout):
//   [0,14)  start address >> 4
//   [16,30) leading-dimension byte offset >> 4
//   [32,46) stride-dimension byte offset >> 4
//   [46,48) version = 1
//   [49,52) base offset, [52] LBO mode
//   [61,64) swizzle: 0 none, 2 = 128B, 4 = 64B, 6 = 32B
B200_DEVICE uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t swizzle) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(swizzle & 7) << 61;
  return d;
}

// K-major operand tile whose rows are 128 bytes, TMA-written with 128-byte
// swizzle; 8-row groups are 1024 bytes apart.
B200_DEVICE uint64_t desc_kmajor_sw128(uint32_t saddr) { return smem_desc(saddr, 16, 1024, 2); }

// Instruction descriptor for kind::mxf8f6f4.block_scale, A and B e4m3,
// K-major, UE8M0 scales, f32 accumulate.  sf ids select the scale byte.
__host__ __device__ constexpr uint32_t idesc_mxf8(uint32_t M, uint32_t N, uint32_t sfa_id, uint32_t sfb_id) {
  return (sfb_id & 3u) << 4          // B scale-factor id
         | 0u << 7                   // A format e4m3
         | 0u << 10                  // B format e4m3
         | ((N >> 3) & 0x3Fu) << 17  // N / 8
         | 1u << 23                  // scale format UE8M0
         | ((M >> 4) & 0x1Fu) << 24  // M / 16
         | (sfa_id & 3u) << 29;      // A scale-factor id
}

// Instruction descriptor for kind::mxf4nvf4.block_scale with 16-element
// blocks (NVFP4): A and B e2m1, K-major, UE4M3 scales, f32 accumulate; each
// MMA (K = 64) reads the four scale bytes of its row's 32-bit TMEM word.
__host__ __device__ constexpr uint32_t idesc_nvf4(uint32_t M, uint32_t N) {
  return 1u << 7                     // A format e2m1
         | 1u << 10                  // B format e2m1
         | ((N >> 3) & 0x3Fu) << 17  // N / 8
         | 0u << 23                  // scale format UE4M3
         | ((M >> 4) & 0x1Fu) << 24; // M / 16
}

// Instruction descriptor for kind::f8f6f4 (no block scale): e4m3 x e4m3 -> f32.
__host__ __device__ constexpr uint32_t idesc_f8(uint32_t M, uint32_t N, bool a_mn_major, bool b_mn_major) {
  return 1u << 4                      // D format f32
         | 0u << 7 | 0u << 10         // e4m3, e4m3
         | (a_mn_major ? 1u : 0u) << 15 | (b_mn_major ? 1u : 0u) << 16
         | ((N >> 3) & 0x3Fu) << 17 | ((M >> 4) & 0x1Fu) << 24;
}

// Instruction descriptor for kind::f16 with bf16 inputs, f32 accumulate.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t M, uint32_t N, bool a_mn_major, bool b_mn_major) {
  return 1u << 4 | 1u << 7 | 1u << 10 | (a_mn_major ? 1u : 0u) << 15 | (b_mn_major ? 1u : 0u) << 16 |
         ((N >> 3) & 0x3Fu) << 17 | ((M >> 4) & 0x1Fu) << 24;
}

B200_DEVICE void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
B200_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
B200_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

B200_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
B200_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem) x B(smem), block-scaled with scales in tmem.
B200_DEVICE void mma_mxf8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa_tmem,
                          uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// D(tmem) (+)= A(smem) x B(smem), NVFP4 block-scaled (e2m1, e4m3 scale per 16).
B200_DEVICE void mma_nvf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa_tmem,
                          uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Two floats -> packed e2m1 pair (round to nearest even, saturating): lo in
// bits 0-3, hi in bits 4-7.
B200_DEVICE uint32_t f2_to_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .b8 b;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b, %2, %1;\n\t"
      "cvt.u32.u8 %0, b;\n\t}"
      : "=r"(r) : "f"(lo), "f"(hi));
  return r & 0xFFu;
}

// D(tmem) (+)= A(smem) x B(smem), e4m3 without block scales.
B200_DEVICE void mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(smem) x B(smem), bf16.
B200_DEVICE void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier when all prior tcgen05 ops of this thread complete.
B200_DEVICE void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Copy 32 rows x 16 bytes from shared memory (descriptor) into TMEM lanes
// 0-31, replicated to all four 32-lane subpartitions.
B200_DEVICE void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Each thread of the warp reads 8 consecutive 32-bit columns of its lane.
B200_DEVICE void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
B200_DEVICE void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
B200_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

B200_DEVICE void tmem_st_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
               ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
B200_DEVICE void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// fp8 helpers
// ---------------------------------------------------------------------------
// Two floats -> two e4m3 (round to nearest even, saturating); lo in bits 0-7.
B200_DEVICE uint16_t f2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// ceil(log2(x)) for x > 0 from the float bits; -127 for x == 0.
B200_DEVICE int ceil_log2_bits(float x) {
  const uint32_t b = __float_as_uint(x);
  if ((b & 0x7FFFFFFFu) == 0u) return -127;
  int e = int((b >> 23) & 0xFF) - 127;
  if (b & 0x7FFFFFu) e += 1;
  return e < -127 ? -127 : (e > 127 ? 127 : e);
}

// 2^e as a float for -126 <= e <= 127 (exact).
B200_DEVICE float exp2_int(int e) { return __uint_as_float(uint32_t(e + 127) << 23); }

}  // namespace b200

namespace b200 {
// L2 eviction-priority policies for TMA loads.
B200_DEVICE uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
B200_DEVICE uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
B200_DEVICE void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y,
                                  uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
B200_DEVICE void tma_load_3d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y,
                                  int32_t z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z),
        "l"(policy)
      : "memory");
}
B200_DEVICE void bulk_load_hint(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// 16-byte cp.async (L2-only) with zero fill: src_bytes 0 writes 16 zero bytes.
// Used for row gathers whose rows are too scattered for a tiled TMA box.
B200_DEVICE void cp_async_16(uint32_t smem_dst, const void* gsrc, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_dst), "l"(gsrc), "r"(src_bytes) : "memory");
}
// 4-byte cp.async (L1-allocating) with zero fill (src_bytes 0 writes zeros).
B200_DEVICE void cp_async_4(uint32_t smem_dst, const void* gsrc, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_dst), "l"(gsrc), "r"(src_bytes) : "memory");
}
B200_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
B200_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// The mbarrier gets one arrival (counted in its expected count: .noinc) once
// every cp.async this thread issued before has landed; the producer never
// blocks on its copies.
B200_DEVICE void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
template <int N>
B200_DEVICE void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

B200_DEVICE void named_barrier(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
}  // namespace b200

namespace b200 {
// Thread-block clusters: barrier, rank, distributed shared memory loads.
B200_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
B200_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
B200_DEVICE uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
B200_DEVICE float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}
}  // namespace b200

namespace b200 {
// Launch with programmatic stream serialization: the kernel may start while
// the previous kernel in the stream drains; every kernel of this project
// executes griddepcontrol.wait before it reads its predecessor's outputs or
// writes anything, and triggers its own dependents at entry.
// B200_NO_PDL=1 in the environment launches plainly instead (a diagnostic:
// per-kernel profiles then show each kernel's own duration rather than one
// stretched by an early start).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("B200_NO_PDL");
    return !(e && e[0] == '1');
  }();
  return on;
}
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
}  // namespace b200
