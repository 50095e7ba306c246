// Absorbed MLA over the paged e4m3 latent cache, CUDA-core version.
//
// One CTA per (query token, group of up to 16 heads).  The query's latent
// (kv_lora) and rope parts stay in shared memory as fp32; the sequence's
// cache is streamed in 64-token chunks (dequantised once per chunk into
// shared memory), scores use an online softmax per head, and the output
// latent accumulates in registers (each thread owns 32 of the 16 x 512
// outputs).  Causal masking by the query's absolute position; an optional
// per-query top-k index list restricts attention (sparse MLA).
//
// This is the correctness path and the fallback for shapes the tcgen05
// kernel does not cover.
#include "../common/ptx.cuh"
#include "attn.h"

namespace b200 {
namespace attn {

constexpr int kHeads = 16;
constexpr int kChunk = 64;
constexpr int kThreads = 256;

template <int L, int R>
__global__ void __launch_bounds__(kThreads) mla_simt_kernel(const __nv_bfloat16* __restrict__ q_abs,
                                                             const __nv_bfloat16* __restrict__ q_pe, int H,
                                                             const uint8_t* __restrict__ cache, float kv_scale,
                                                             const int* __restrict__ block_table, int bt_stride,
                                                             const int* __restrict__ q_seq, const int* __restrict__ q_pos,
                                                             const int* __restrict__ topk, int topk_n, int page_size,
                                                             float sm_scale, __nv_bfloat16* __restrict__ out) {
  constexpr int D = L + R;
  extern __shared__ float sm[];
  float* sq = sm;                        // [kHeads][D]
  float* skv = sq + kHeads * D;          // [kChunk][D]
  float* sp = skv + kChunk * D;          // [kHeads][kChunk]
  float* salpha = sp + kHeads * kChunk;  // [kHeads]
  float* smax = salpha + kHeads;         // [kHeads]
  float* ssum = smax + kHeads;           // [kHeads]

  const int t = blockIdx.x;
  const int h0 = blockIdx.y * kHeads;
  const int nh = min(kHeads, H - h0);
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  const int b = q_seq[t];
  const int n = q_pos[t] + 1;
  const int nkeys = topk ? min(topk_n, n) : n;

  for (int i = threadIdx.x; i < kHeads * D; i += kThreads) {
    const int h = i / D, c = i % D;
    float v = 0.f;
    if (h < nh) {
      v = c < L ? __bfloat162float(q_abs[((int64_t)t * H + h0 + h) * L + c])
                : __bfloat162float(q_pe[((int64_t)t * H + h0 + h) * R + (c - L)]);
    }
    sq[i] = v;
  }
  if (threadIdx.x < kHeads) {
    smax[threadIdx.x] = -INFINITY;
    ssum[threadIdx.x] = 0.f;
  }
  // Output ownership: thread owns head oh = tid / 16, columns oc0 + 16*j.
  const int oh = threadIdx.x / 16;
  const int oc0 = threadIdx.x % 16;
  float acc[L / 16];
#pragma unroll
  for (int j = 0; j < L / 16; ++j) acc[j] = 0.f;
  __syncthreads();

  const float qk_scale = sm_scale * kv_scale;
  for (int base = 0; base < nkeys; base += kChunk) {
    const int cn = min(kChunk, nkeys - base);
    // load + dequantise the chunk
    for (int i = threadIdx.x; i < kChunk * (D / 4); i += kThreads) {
      const int j = i / (D / 4), c4 = i % (D / 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j < cn) {
        int p = base + j;
        if (topk) p = topk[(int64_t)t * topk_n + p];
        if (p >= 0 && p < n) {
          const int page = block_table[(int64_t)b * bt_stride + p / page_size];
          const int64_t slot = (int64_t)page * page_size + p % page_size;
          const uint32_t w = *reinterpret_cast<const uint32_t*>(cache + slot * D + c4 * 4);
          const __nv_fp8x2_e4m3* pr = reinterpret_cast<const __nv_fp8x2_e4m3*>(&w);
          const float2 lo = float2(pr[0]);
          const float2 hi = float2(pr[1]);
          v = make_float4(lo.x, lo.y, hi.x, hi.y);
        } else {
          v = make_float4(NAN, 0.f, 0.f, 0.f);  // marks an invalid slot
        }
      }
      reinterpret_cast<float4*>(skv + j * D)[c4] = v;
    }
    __syncthreads();
    // scores: 16 heads x 64 keys, 4 per thread
    for (int i = threadIdx.x; i < kHeads * kChunk; i += kThreads) {
      const int h = i / kChunk, j = i % kChunk;
      float s = -INFINITY;
      if (h < nh && j < cn && !isnan(skv[j * D])) {
        const float* qa = sq + h * D;
        const float* ka = skv + j * D;
        float d = 0.f;
#pragma unroll 8
        for (int c = 0; c < D; ++c) d += qa[c] * ka[c];
        s = d * qk_scale;
      }
      sp[i] = s;
    }
    __syncthreads();
    // online softmax per head (one warp per 2 heads)
    {
      const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
      for (int h = w; h < kHeads; h += kThreads / 32) {
        float m = fmaxf(sp[h * kChunk + l], sp[h * kChunk + l + 32]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float mold = smax[h];
        const float mnew = fmaxf(mold, m);
        const float e0 = (mnew == -INFINITY) ? 0.f : __expf(sp[h * kChunk + l] - mnew);
        const float e1 = (mnew == -INFINITY) ? 0.f : __expf(sp[h * kChunk + l + 32] - mnew);
        sp[h * kChunk + l] = e0;
        sp[h * kChunk + l + 32] = e1;
        float s = e0 + e1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (l == 0) {
          const float alpha = (mold == -INFINITY) ? 0.f : __expf(mold - mnew);
          salpha[h] = alpha;
          ssum[h] = ssum[h] * alpha + s;
          smax[h] = mnew;
        }
      }
    }
    __syncthreads();
    {
      const float alpha = salpha[oh];
#pragma unroll
      for (int j = 0; j < L / 16; ++j) acc[j] *= alpha;
      for (int k = 0; k < cn; ++k) {
        const float p = sp[oh * kChunk + k];
        if (p != 0.f) {
          const float* v = skv + k * D;
#pragma unroll
          for (int j = 0; j < L / 16; ++j) acc[j] += p * v[oc0 + 16 * j];
        }
      }
    }
    __syncthreads();
  }
  if (oh < nh) {
    const float inv = ssum[oh] > 0.f ? kv_scale / ssum[oh] : 0.f;
#pragma unroll
    for (int j = 0; j < L / 16; ++j)
      out[((int64_t)t * H + h0 + oh) * L + oc0 + 16 * j] = __float2bfloat16(acc[j] * inv);
  }
}

}  // namespace attn
}  // namespace b200

int b200_mla_simt(const void* q_abs, const void* q_pe, int T, int H, int L, int R, const uint8_t* cache,
                  float kv_scale, const int* block_table, int bt_stride, const int* q_seq, const int* q_pos,
                  const int* topk, int topk_n, int page_size, float sm_scale, void* out, cudaStream_t st) {
  using namespace b200::attn;
  if (T <= 0) return 0;
  if (L != 512 || R != 64) return -1;
  constexpr int D = 576;
  const size_t smem = (kHeads * D + kChunk * D + kHeads * kChunk + 3 * kHeads) * sizeof(float);
  auto kern = mla_simt_kernel<512, 64>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(T, (H + kHeads - 1) / kHeads);
  kern<<<grid, kThreads, smem, st>>>(reinterpret_cast<const __nv_bfloat16*>(q_abs),
                                     reinterpret_cast<const __nv_bfloat16*>(q_pe), H, cache, kv_scale, block_table,
                                     bt_stride, q_seq, q_pos, topk, topk_n, page_size, sm_scale,
                                     reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
