// RMSNorm / residual-add / MXFP8 quantization kernels.
//
// One CTA per row; each thread owns 8 consecutive elements per pass (16-byte
// loads), so 4 neighbouring lanes hold one 32-element scale block and the
// block amax needs two shuffles.  Scales are written straight into the
// sf128x4 layout the tcgen05 GEMM copies into TMEM.
//
// Reference parity: K5 `combine_norm_mxfp8` (hq_unit.cu:170), K8
// `qnorm_mxfp8` (qn_unit.cu:192), K3/K4 MXFP8 quantizers (gq_unit.cu:140,222).
#include "../common/ptx.cuh"
#include "elementwise.h"
#include "row_util.cuh"

namespace b200 {
namespace ew {

constexpr int kThreads = 256;

// ---------------------------------------------------------------------------
// x [rows, K] (+ optional residual add) -> rmsnorm -> {bf16 copy, mxfp8}
//   MODE 0: y = rmsnorm(x)                       (x bf16 or fp32)
//   MODE 1: r = r + x; y = rmsnorm(r)            (x bf16, r fp32 in place)
// Outputs (each optional): y_bf16 [rows, K], q [rows, K] e4m3 + packed sf.
// Rows longer than 256 * 8 * kMaxIt are not supported (K <= 16384).
// ---------------------------------------------------------------------------
constexpr int kMaxIt = 8;

template <typename TX, int MODE>
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const TX* __restrict__ x, int ldx, float* residual,
                                                           const float* __restrict__ w, float eps, int K,
                                                           __nv_bfloat16* y, int ldy, uint8_t* q, uint8_t* sf) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  const int units = K >> 3;
  float v[kMaxIt][8];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < kMaxIt; ++it) {
    const int u = it * kThreads + threadIdx.x;
    if (u < units) {
      load8<TX>(x + (int64_t)row * ldx + u * 8, v[it]);
      if (MODE == 1) {
        float r[8];
        float* rp = residual + (int64_t)row * K + u * 8;
        load8<float>(rp, r);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[it][i] += r[i];
        store8_f32(rp, v[it]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[it][i] * v[it][i];
    }
  }
  const float tot = block_sum(ss, red);
  const float rs = rsqrtf(tot / float(K) + eps);
  const int kb_total = K >> 5;
#pragma unroll
  for (int it = 0; it < kMaxIt; ++it) {
    const int u = it * kThreads + threadIdx.x;
    // all lanes of a warp take part in the shuffles of quant8
    if (it * kThreads >= units) break;
    float o[8];
    if (u < units) {
      const float4 w0 = *reinterpret_cast<const float4*>(w + u * 8);
      const float4 w1 = *reinterpret_cast<const float4*>(w + u * 8 + 4);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[it][i] * rs * wv[i];
      if (y) store8_bf16(y + (int64_t)row * ldy + u * 8, o);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = 0.f;
    }
    if (q) quant8(o, q + (int64_t)row * K + u * 8, sf, row, u * 8, kb_total, u < units);
  }
}

// Plain MXFP8 quantization of x [rows, K] (bf16 or fp32).
// Row k-th element at x[row * ldx + (k / seg) * seg_stride + k % seg]: seg = K
// is a plain row-major matrix; seg < K gathers a row from head-major blocks
// (e.g. [H, T, v] -> row t = concat over h), saving a transpose copy.
template <typename TX>
__global__ void __launch_bounds__(kThreads) quant_kernel(const TX* __restrict__ x, int ldx, int K, int seg,
                                                         int64_t seg_stride, uint8_t* q, uint8_t* sf) {
  const int row = blockIdx.y;
  const int u = blockIdx.x * kThreads + threadIdx.x;
  const int units = K >> 3;
  pdl_wait();
  pdl_launch_dependents();   // dependents wait for this grid before touching its outputs
  float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const int k = u * 8;
  if (u < units) load8<TX>(x + (int64_t)row * ldx + (int64_t)(k / seg) * seg_stride + k % seg, v);
  quant8(v, q + (int64_t)row * K + k, sf, row, k, K >> 5, u < units);
}

}  // namespace ew
}  // namespace b200

using namespace b200::ew;

int b200_rmsnorm(const void* x, int x_is_f32, int ldx, float* residual, const float* w, float eps, int rows, int K,
                 void* y, int ldy, uint8_t* q, uint8_t* sf, cudaStream_t st) {
  if (K % 32 != 0 || K > kThreads * 8 * kMaxIt || rows <= 0) return -1;
  dim3 grid(rows), block(kThreads);
  __nv_bfloat16* yb = reinterpret_cast<__nv_bfloat16*>(y);
  if (residual) {
    b200::launch_pdl(rmsnorm_kernel<__nv_bfloat16, 1>, dim3(grid), dim3(block), 0, st, reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                                              residual, w, eps, K, yb, ldy, q, sf);
  } else if (x_is_f32) {
    b200::launch_pdl(rmsnorm_kernel<float, 0>, dim3(grid), dim3(block), 0, st, reinterpret_cast<const float*>(x), ldx, nullptr, w, eps, K,
                                                      yb, ldy, q, sf);
  } else {
    b200::launch_pdl(rmsnorm_kernel<__nv_bfloat16, 0>, dim3(grid), dim3(block), 0, st, reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                                              nullptr, w, eps, K, yb, ldy, q, sf);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_quant_mxfp8_seg(const void* x, int x_is_f32, int ldx, int rows, int K, int seg, int64_t seg_stride,
                         uint8_t* q, uint8_t* sf, cudaStream_t st) {
  if (K % 128 != 0 || rows <= 0 || seg % 8 != 0 || K % seg != 0) return -1;
  dim3 grid((K / 8 + kThreads - 1) / kThreads, rows), block(kThreads);
  if (x_is_f32)
    b200::launch_pdl(quant_kernel<float>, dim3(grid), dim3(block), 0, st, reinterpret_cast<const float*>(x), ldx, K,
                     seg, seg_stride, q, sf);
  else
    b200::launch_pdl(quant_kernel<__nv_bfloat16>, dim3(grid), dim3(block), 0, st,
                     reinterpret_cast<const __nv_bfloat16*>(x), ldx, K, seg, seg_stride, q, sf);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

int b200_quant_mxfp8(const void* x, int x_is_f32, int ldx, int rows, int K, uint8_t* q, uint8_t* sf,
                     cudaStream_t st) {
  return b200_quant_mxfp8_seg(x, x_is_f32, ldx, rows, K, K, 0, q, sf, st);
}
