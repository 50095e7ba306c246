// RoPE, latent-KV cache store, sigmoid group-limited router top-k, and the
// MoE dispatch layout (expert segments, row gather, weighted combine).
//
// Reference parity: K9 `q_rope_fp8` (qr_unit.cu:104), K10 `inv_rope_tail`
// (ro_unit.cu:73), K12 `route_e5_kernel` (route_e5.cu:853; here V3's sigmoid
// + group-limited top-k instead of sqrtsoftplus + E5 prune) and the routing
// record it writes for the expert GEMMs (rr.py:1-15).
#include "../common/ptx.cuh"
#include "elementwise.h"
#include "moe_layout.cuh"

namespace b200 {
namespace ew2 {

__device__ __forceinline__ float ld_any(const void* p, int64_t i, int f32) {
  return f32 ? reinterpret_cast<const float*>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// In-place RoPE on x[t, h, 0:d] (interleaved pairs); table [P, d] = cos | sin.
__global__ void rope_kernel(void* x, int f32, int64_t st_t, int64_t st_h, int H, int d, const int* pos,
                            const float* table) {
  const int t = blockIdx.x;
  const int half = d >> 1;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  const int p = pos[t];
  for (int i = threadIdx.x; i < H * half; i += blockDim.x) {
    const int h = i / half, j = i % half;
    const int64_t base = (int64_t)t * st_t + (int64_t)h * st_h + 2 * j;
    const float c = table[(int64_t)p * d + j], s = table[(int64_t)p * d + half + j];
    if (f32) {
      float* xp = reinterpret_cast<float*>(x);
      const float a = xp[base], b = xp[base + 1];
      xp[base] = a * c - b * s;
      xp[base + 1] = a * s + b * c;
    } else {
      __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(x);
      const float a = __bfloat162float(xp[base]), b = __bfloat162float(xp[base + 1]);
      xp[base] = __float2bfloat16(a * c - b * s);
      xp[base + 1] = __float2bfloat16(a * s + b * c);
    }
  }
}

// One warp per token: latent = rmsnorm(kv[:L]) * w, pe = rope(kv[L:L+R]);
// cache[slot] = e4m3([latent | pe] / kv_scale).  L % 32 == 0, R == 64.
__global__ void kv_store_kernel(const void* kv, int f32, int64_t ld, int T, int L, int R, const float* w, float eps,
                                const int* pos, const float* table, const int64_t* slots, uint8_t* cache,
                                float inv_scale) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  if (warp >= T) return;
  const int64_t row = (int64_t)warp * ld;
  float ss = 0.f;
  for (int i = lane; i < L; i += 32) {
    const float v = ld_any(kv, row + i, f32);
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rs = rsqrtf(ss / float(L) + eps);
  uint8_t* dst = cache + slots[warp] * (int64_t)(L + R);
  for (int i = 2 * lane; i < L; i += 64) {
    const float a = ld_any(kv, row + i, f32) * rs * w[i] * inv_scale;
    const float b = ld_any(kv, row + i + 1, f32) * rs * w[i + 1] * inv_scale;
    *reinterpret_cast<uint16_t*>(dst + i) = f2_to_e4m3x2(a, b);
  }
  const int p = pos[warp];
  const int half = R >> 1;
  for (int j = lane; j < half; j += 32) {
    const float a = ld_any(kv, row + L + 2 * j, f32), b = ld_any(kv, row + L + 2 * j + 1, f32);
    const float c = table[(int64_t)p * R + j], s = table[(int64_t)p * R + half + j];
    *reinterpret_cast<uint16_t*>(dst + L + 2 * j) = f2_to_e4m3x2((a * c - b * s) * inv_scale,
                                                                  (a * s + b * c) * inv_scale);
  }
}

// Router: one warp per token over E <= 256 experts (E % 32 == 0).
// scores = sigmoid(logits); choice = scores + bias; group score = sum of the
// top-2 choices in each of G groups; keep the top `topk_group` groups; pick
// the top-k choices among them; weights = scores renormalised * scaling.
// Ties resolve to the lower expert index.
constexpr int kMaxEPerLane = 16;   // up to 512 experts

__global__ void router_kernel(const float* logits, const float* bias, int T, int E, int G, int topk_group, int K,
                              float scaling, int renorm, int scoring, float* w_out, int* id_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  if (warp >= T) return;
  const int per = E / 32;     // experts per lane, contiguous: lane owns [lane*per, lane*per+per)
  float sc[kMaxEPerLane], ch[kMaxEPerLane];
#pragma unroll
  for (int i = 0; i < kMaxEPerLane; ++i) {
    if (i < per) {
      const int e = lane * per + i;
      const float l = logits[(int64_t)warp * E + e];
      // sigmoid (V3) or sqrt(softplus) (V4; softplus(l) = l above 20)
      sc[i] = scoring == 0 ? 1.0f / (1.0f + __expf(-l)) : sqrtf(l > 20.f ? l : log1pf(expf(l)));
      ch[i] = sc[i] + bias[e];
    } else {
      sc[i] = 0.f;
      ch[i] = -INFINITY;
    }
  }
  // group selection: group g covers experts [g*E/G, (g+1)*E/G) = lanes [g*32/G, (g+1)*32/G)
  if (G > 1) {
    const int lanes_per_group = 32 / G;
    float b1 = -INFINITY, b2 = -INFINITY;   // top-2 within this lane
#pragma unroll
    for (int i = 0; i < kMaxEPerLane; ++i) {
      if (i < per) {
        const float v = ch[i];
        if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) b2 = v;
      }
    }
    // merge top-2 across the lanes of the group
    for (int o = 1; o < lanes_per_group; o <<= 1) {
      const float o1 = __shfl_xor_sync(0xffffffffu, b1, o);
      const float o2 = __shfl_xor_sync(0xffffffffu, b2, o);
      const float n1 = fmaxf(b1, o1);
      const float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
      b1 = n1;
      b2 = n2;
    }
    const float gscore = b1 + b2;            // same value on every lane of the group
    const int my_group = lane / lanes_per_group;
    // rank groups: group g is kept if fewer than topk_group groups beat it
    int beat = 0;
    for (int g = 0; g < G; ++g) {
      const float og = __shfl_sync(0xffffffffu, gscore, g * lanes_per_group);
      if (og > gscore || (og == gscore && g < my_group)) ++beat;
    }
    if (beat >= topk_group) {
#pragma unroll
      for (int i = 0; i < kMaxEPerLane; ++i) ch[i] = -INFINITY;
    }
  }
  float wsum = 0.f;
  float wk = 0.f;
  int idk = 0;
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxEPerLane; ++i) {
      if (i < per && ch[i] > best) { best = ch[i]; bi = lane * per + i; }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    const int owner = bi / per;
    float s = 0.f;
    if (lane == owner) {
      const int li = bi - lane * per;
#pragma unroll
      for (int i = 0; i < kMaxEPerLane; ++i)
        if (i == li) { s = sc[i]; ch[i] = -INFINITY; }
    }
    s = __shfl_sync(0xffffffffu, s, owner);
    wsum += s;
    if (lane == k) { wk = s; idk = bi; }
  }
  if (lane < K) {
    const float norm = (renorm && K > 1) ? 1.0f / (wsum + 1e-20f) : 1.0f;
    w_out[(int64_t)warp * K + lane] = wk * norm * scaling;
    id_out[(int64_t)warp * K + lane] = idk;
  }
}

// ---------------------------------------------------------------------------
// MoE dispatch layout for the local experts [first, first + E).
//   seg_count[e]  rows routed to local expert e
//   seg_start[e]  first sorted row of e (128-aligned)
//   row_token[r]  token of sorted row r;  row_weight[r] its routing weight
//   pair_row[t*K+j]  sorted row of (t, j), or -1 if the expert is not local
// One CTA; counts via shared-memory atomics.
// ---------------------------------------------------------------------------
__global__ void moe_align_kernel(const int* ids, const float* w, int T, int K, int first, int E, int* seg_start,
                                 int* seg_count, int* row_token, float* row_weight, int* pair_row, int* total_rows,
                                 int bn1, int* ttile1, int bn2, int* ttile2) {
  extern __shared__ int sh[];
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  moe::moe_align_body(ids, w, T, K, first, E, seg_start, seg_count, row_token, row_weight, pair_row, total_rows, bn1,
                      ttile1, bn2, ttile2, sh);
}
__global__ void moe_gather_kernel(const uint8_t* xq, const uint8_t* xsf, const int* pair_row, int npairs, int K,
                                  int Kd, uint8_t* dq, uint8_t* dsf) {
  const int i = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  if (i >= npairs) return;
  const int r = pair_row[i];
  if (r < 0) return;
  moe::moe_gather_pair(xq, xsf, i / K, r, Kd, dq, dsf);
}

// out[t] = sum_j y[pair_row[t, j]] (+ add[t]): one CTA per token, each
// thread 8 columns at a time with 16-byte loads of all K rows in flight
// (the row ids are read once, before the column loop).
constexpr int kCombMaxK = 16;
__global__ void __launch_bounds__(128) moe_combine_kernel(const __nv_bfloat16* y, const int* pair_row, int T, int K,
                                                          int D, const void* add, int add_f32, void* out,
                                                          int out_f32) {
  const int t = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  int rows[kCombMaxK];
#pragma unroll
  for (int j = 0; j < kCombMaxK; ++j) rows[j] = j < K ? __ldcg(pair_row + (int64_t)t * K + j) : -1;
  for (int v = threadIdx.x; v < D / 8; v += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kCombMaxK; ++j) {
      if (rows[j] < 0) continue;
      const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(y + (int64_t)rows[j] * D) + v);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    const int64_t o = (int64_t)t * D + v * 8;
    if (add) {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += ld_any(add, o + i, add_f32);
    }
    if (out_f32) {
      float* of = reinterpret_cast<float*>(out) + o;
      *reinterpret_cast<float4*>(of) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(of + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      uint4 outv;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&outv);
#pragma unroll
      for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + o) = outv;
    }
  }
}

}  // namespace ew2
}  // namespace b200

using namespace b200::ew2;

int b200_rope(void* x, int f32, int64_t st_t, int64_t st_h, int T, int H, int d, const int* pos, const float* table,
              cudaStream_t st) {
  if (T <= 0) return 0;
  b200::launch_pdl(rope_kernel, dim3(T), dim3(128), 0, st, x, f32, st_t, st_h, H, d, pos, table);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_kv_store(const void* kv, int f32, int64_t ld, int T, int L, int R, const float* w, float eps, const int* pos,
                  const float* table, const int64_t* slots, uint8_t* cache, float kv_scale, cudaStream_t st) {
  if (T <= 0) return 0;
  if (L % 64 != 0) return -1;
  const int threads = 128;
  const int blocks = (T * 32 + threads - 1) / threads;
  b200::launch_pdl(kv_store_kernel, dim3(blocks), dim3(threads), 0, st, kv, f32, ld, T, L, R, w, eps, pos, table, slots, cache, 1.0f / kv_scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_router(const float* logits, const float* bias, int T, int E, int G, int topk_group, int K, float scaling,
                int renorm, int scoring, float* w_out, int* id_out, cudaStream_t st) {
  if (T <= 0) return 0;
  if (E % 32 != 0 || E / 32 > kMaxEPerLane || K > 32 || (G > 1 && (32 % G != 0))) return -1;
  const int threads = 128;
  b200::launch_pdl(router_kernel, dim3((T * 32 + threads - 1) / threads), dim3(threads), 0, st, logits, bias, T, E, G, topk_group, K, scaling,
                                                                       renorm, scoring, w_out, id_out);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_moe_align(const int* ids, const float* w, int T, int K, int first, int E, int* seg_start, int* seg_count,
                   int* row_token, float* row_weight, int* pair_row, int* total_rows, int bn1, int* ttile1, int bn2,
                   int* ttile2, cudaStream_t st) {
  b200::launch_pdl(moe_align_kernel, dim3(1), dim3(1024), 3 * E * sizeof(int), st, ids, w, T, K, first, E, seg_start, seg_count, row_token,
                                                         row_weight, pair_row, total_rows, bn1 > 0 ? bn1 : 128, ttile1,
                                                         bn2 > 0 ? bn2 : 128, ttile2);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_moe_gather(const uint8_t* xq, const uint8_t* xsf, const int* pair_row, int npairs, int K, int Kd, uint8_t* dq,
                    uint8_t* dsf, cudaStream_t st) {
  if (npairs <= 0) return 0;
  b200::launch_pdl(moe_gather_kernel, dim3(npairs), dim3(128), 0, st, xq, xsf, pair_row, npairs, K, Kd, dq, dsf);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_moe_combine(const void* y, const int* pair_row, int T, int K, int D, const void* add, int add_f32, void* out,
                     int out_f32, cudaStream_t st) {
  if (T <= 0) return 0;
  if (K > kCombMaxK || D % 8) return -1;
  b200::launch_pdl(moe_combine_kernel, dim3(T), dim3(128), 0, st, reinterpret_cast<const __nv_bfloat16*>(y), pair_row,
                   T, K, D, add, add_f32, out, out_f32);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
