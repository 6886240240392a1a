// Shared definitions for the ncmorph_b200 CUDA library: status codes, bf16
// conversions with the reference's rounding rule, and launch helpers.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/ncm_cuda.h"

namespace ncm {

// bf16 narrowing with round-to-nearest-even and every NaN mapped to 0x7FC0:
// the rule of ncmorph's bf16_t.from_f32 (packages/bf16/root.zig:17-22),
// which matches PyTorch's float->bfloat16 cast.
__host__ __device__ __forceinline__ uint16_t f32_to_bf16(float f) {
#ifdef __CUDA_ARCH__
  const uint32_t x = __float_as_uint(f);
#else
  uint32_t x;
  __builtin_memcpy(&x, &f, 4);
#endif
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0u;
  return static_cast<uint16_t>((x + 0x7FFFu + ((x >> 16) & 1u)) >> 16);
}

// Exact widening: a bf16 is the top half of an f32 (packages/bf16/root.zig:25-27).
__host__ __device__ __forceinline__ float bf16_to_f32(uint16_t h) {
  const uint32_t x = static_cast<uint32_t>(h) << 16;
#ifdef __CUDA_ARCH__
  return __uint_as_float(x);
#else
  float f;
  __builtin_memcpy(&f, &x, 4);
  return f;
#endif
}

__device__ __forceinline__ float bf16lo(uint32_t pair) { return __uint_as_float(pair << 16); }
__device__ __forceinline__ float bf16hi(uint32_t pair) { return __uint_as_float(pair & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return static_cast<uint32_t>(f32_to_bf16(lo)) | (static_cast<uint32_t>(f32_to_bf16(hi)) << 16);
}

inline int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

}  // namespace ncm

#define NCM_CUDA_TRY(expr)                              \
  do {                                                  \
    cudaError_t _e = (expr);                            \
    if (_e != cudaSuccess) return ncm_set_cuda_error(_e); \
  } while (0)

// Records the CUDA error text for ncm_last_error() and returns NCM_ECUDA.
int ncm_set_cuda_error(cudaError_t e);
// Records a formatted message for ncm_last_error() and returns `status`.
int ncm_fail(int status, const char* fmt, ...);
