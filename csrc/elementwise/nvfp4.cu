// NVFP4 activations for the routed experts (sm_100a).
//
//   nvfp4_quant   bf16 / fp32 rows -> packed e2m1 pairs (low nibble = even
//                 element), one e4m3 scale per 16 elements in the 128-row x
//                 4-column chunk layout the tcgen05 block-scaled MMA copies
//                 into TMEM, and a per-row fp32 global scale
//                 g = amax / (448 * 6) so the e4m3 block scales span the row's
//                 range.  The grouped GEMM's epilogue multiplies each token
//                 column by its g (tokens are the MMA N dimension).
//   moe_gather4   copies routed token rows (data, scales, global scale) into
//                 the expert-sorted operand of the NVFP4 FC1.
//
// Reference parity: the reference quantizes routed-expert inputs to NVFP4 on
// a side stream before FlashInfer's trtllm-gen MoE (nq.py:1-10, mo.py:19-40).
#include "../common/ptx.cuh"
#include "elementwise.h"
#include "moe_layout.cuh"

namespace b200 {
namespace fp4 {

constexpr int kThreads = 256;

__device__ __forceinline__ float ld_any(const void* p, int64_t i, int f32) {
  return f32 ? reinterpret_cast<const float*>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__global__ void __launch_bounds__(kThreads) nvfp4_quant_kernel(const void* x, int f32, int64_t ld, int T, int K,
                                                                uint8_t* q, uint8_t* sf, float* g) {
  __shared__ float red[kThreads / 32];
  const int t = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  if (t >= T) return;
  const int64_t row = (int64_t)t * ld;
  float am = 0.f;
  for (int i = threadIdx.x; i < K; i += kThreads) am = fmaxf(am, fabsf(ld_any(x, row + i, f32)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
  __syncthreads();
  float amax = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const float gt = amax > 0.f ? amax * (1.f / (448.f * 6.f)) : 1.f;
  const float inv_g = 1.f / gt;
  const int nb = K / 16;
  for (int b = threadIdx.x; b < nb; b += kThreads) {
    float v[16];
    float bm = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = ld_any(x, row + b * 16 + i, f32);
      bm = fmaxf(bm, fabsf(v[i]));
    }
    const uint16_t s2 = f2_to_e4m3x2(bm * (1.f / 6.f) * inv_g, 0.f);
    __nv_fp8_e4m3 s8;
    s8.__x = uint8_t(s2 & 0xFF);
    const float sv = float(s8);
    const float mul = sv > 0.f ? inv_g / sv : 0.f;
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w0 |= f2_to_e2m1x2(v[2 * i] * mul, v[2 * i + 1] * mul) << (8 * i);
      w1 |= f2_to_e2m1x2(v[8 + 2 * i] * mul, v[8 + 2 * i + 1] * mul) << (8 * i);
    }
    *reinterpret_cast<uint2*>(q + (int64_t)t * (K / 2) + b * 8) = make_uint2(w0, w1);
    sf[moe::sf_offset(t, b, nb)] = uint8_t(s2 & 0xFF);
  }
  if (threadIdx.x == 0) g[t] = gt;
}

__global__ void moe_gather4_kernel(const uint8_t* xq, const uint8_t* xsf, const float* xg, const int* pair_row,
                                   int npairs, int K, int Kx, uint8_t* dq, uint8_t* dsf, float* dg) {
  const int i = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  if (i >= npairs) return;
  const int r = pair_row[i];
  if (r < 0) return;
  const int t = i / K;
  const uint4* s = reinterpret_cast<const uint4*>(xq + (int64_t)t * (Kx / 2));
  uint4* d = reinterpret_cast<uint4*>(dq + (int64_t)r * (Kx / 2));
  for (int j = threadIdx.x; j < Kx / 32; j += blockDim.x) d[j] = __ldcg(s + j);
  const int nb = Kx / 16;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) dsf[moe::sf_offset(r, b, nb)] = __ldcg(xsf + moe::sf_offset(t, b, nb));
  if (threadIdx.x == 0) dg[r] = __ldcg(xg + t);
}

}  // namespace fp4
}  // namespace b200

int b200_nvfp4_quant(const void* x, int f32, int64_t ld, int T, int K, uint8_t* q, uint8_t* sf, float* g,
                     cudaStream_t st) {
  if (T <= 0) return 0;
  if (K % 64) return -1;
  b200::launch_pdl(b200::fp4::nvfp4_quant_kernel, dim3(T), dim3(b200::fp4::kThreads), 0, st, x, f32, ld, T, K, q, sf,
                   g);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_moe_gather4(const uint8_t* xq, const uint8_t* xsf, const float* xg, const int* pair_row, int npairs, int K,
                     int Kx, uint8_t* dq, uint8_t* dsf, float* dg, cudaStream_t st) {
  if (npairs <= 0) return 0;
  if (Kx % 64) return -1;
  b200::launch_pdl(b200::fp4::moe_gather4_kernel, dim3(npairs), dim3(128), 0, st, xq, xsf, xg, pair_row, npairs, K, Kx,
                   dq, dsf, dg);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
