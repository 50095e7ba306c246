// Device-side random fill used to initialise large random-weight models at
// HBM speed: a counter-based hash (splitmix64 finaliser) of (seed, index)
// produces 8 bytes per 64-bit word; `and_mask` / `or_mask` shape the bytes
// (e.g. 0xBF keeps e4m3 codes finite with |x| <= 1.875).
#include "../common/ptx.cuh"
#include "elementwise.h"

namespace {
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void fill_bytes_kernel(uint64_t* p, int64_t nwords, uint64_t seed, uint64_t and_mask, uint64_t or_mask) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nwords; i += stride) {
    p[i] = (mix64(seed * 0x100000001B3ull + (uint64_t)i) & and_mask) | or_mask;
  }
}
}  // namespace

int b200_fill_bytes(void* p, int64_t nbytes, uint64_t seed, uint8_t and_mask, uint8_t or_mask, cudaStream_t st) {
  if (nbytes % 8 != 0 || (reinterpret_cast<uintptr_t>(p) & 7)) return -1;
  uint64_t am = 0, om = 0;
  for (int i = 0; i < 8; ++i) {
    am |= (uint64_t)and_mask << (8 * i);
    om |= (uint64_t)or_mask << (8 * i);
  }
  const int64_t nw = nbytes / 8;
  int blocks = (int)((nw + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  fill_bytes_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<uint64_t*>(p), nw, seed, am, om);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
