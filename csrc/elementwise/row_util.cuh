// Row helpers shared by the elementwise kernels: 8-element vector loads and
// stores, MXFP8 quantization of 8 values spread over 4 lanes per 32-block
// (scales in the sf128x4 layout the tcgen05 GEMMs copy into TMEM), and a
// block-wide sum.
#pragma once
#include "../common/ptx.cuh"

namespace b200 {
namespace ew {

__device__ __forceinline__ int64_t sf_off(int row, int kblock, int kb_total) {
  const int rb = row >> 7, r = row & 127, kc = kblock >> 2, c = kblock & 3;
  return ((int64_t)(rb * (kb_total >> 2) + kc) << 9) + ((r & 31) << 4) + ((r >> 5) << 2) + c;
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void store8_bf16(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ void store8_f32(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Quantize 8 values held by this thread as part of a 32-block spread over 4
// consecutive lanes; writes 8 e4m3 bytes and (lane % 4 == 0) the scale byte.
__device__ __forceinline__ void quant8(const float (&v)[8], uint8_t* q, uint8_t* sf_base, int row, int col,
                                       int kb_total, bool valid) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const int e = ceil_log2_bits(amax * (1.0f / 448.0f));
  const float inv = exp2_int(-e);
  uint2 out;
  uint16_t* o16 = reinterpret_cast<uint16_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) o16[i] = f2_to_e4m3x2(v[2 * i] * inv, v[2 * i + 1] * inv);
  if (!valid) return;
  *reinterpret_cast<uint2*>(q) = out;
  if ((col & 31) == 0) sf_base[sf_off(row, col >> 5, kb_total)] = uint8_t(e + 127);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (l == 0) red[0] = s;
  }
  __syncthreads();
  return red[0];
}

}  // namespace ew
}  // namespace b200
