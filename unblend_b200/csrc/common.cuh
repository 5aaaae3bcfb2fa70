// Shared helpers for the unblend_b200 CUDA kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/unblend_b200.h"

#define UB_CHECK_LAUNCH()                           \
  do {                                              \
    cudaError_t _e = cudaGetLastError();            \
    if (_e != cudaSuccess) return (int)_e;          \
  } while (0)

#define UB_REQUIRE(cond)                            \
  do {                                              \
    if (!(cond)) return UNBLEND_ERR_INVALID;        \
  } while (0)

namespace ub {

constexpr int kNumSMs = 148;

__device__ __forceinline__ float gelu_erf(float x) {
  // Exact GELU as torch F.gelu(approximate='none'): 0.5 x (1 + erf(x / sqrt(2))).
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// 1 / (1 + 2^(-x log2 e)) with the hardware base-2 exponential and reciprocal
// approximations (about 2 ulp each): four instructions instead of the
// correctly rounded exp and division. Saturates to 0 and 1 at the extremes.
__device__ __forceinline__ float sigmoid_approx(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return r;
}

// Two fp32 FMAs in one instruction (fma.rn.f32x2, sm_100): c + a * b per lane
// pair, each rounded once exactly as fmaf. Halves the issue slots of FMA-bound
// SIMT loops.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(r)
      : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)),
        "l"(*reinterpret_cast<unsigned long long*>(&c)));
  return *reinterpret_cast<float2*>(&r);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline unsigned grid_1d(long long n, int threads, long long cap = 148LL * 16) {
  long long g = (n + threads - 1) / threads;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

}  // namespace ub
