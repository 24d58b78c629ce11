// Shared device helpers for the SQ3.25 / FP4-G16 Mamba-2 kernels (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#ifndef __CUDACC__
#error "common.cuh is CUDA-only"
#endif

namespace sq {

// Status codes shared with include/sq325.h.
enum Status : int {
  kOk = 0, kEInval = 1, kEState = 2, kENonfinite = 3, kECuda = 4, kETimeout = 5, kENomem = 6,
};

// Device-side error word (bitmask) written by kernels whose bounded waits expire
// or whose defensive checks fail.  Read back by the host after synchronisation.
enum DevErr : unsigned {
  kDevTimeoutProducer = 1u, kDevTimeoutMma = 2u, kDevTimeoutEpilogue = 4u, kDevBadArgs = 8u,
};

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// FP8 E4M3FN byte <-> fp32 (exact decode; RNE + satfinite encode).
__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  __nv_fp8_e4m3 v; v.__x = b; return float(v);
}
__device__ __forceinline__ uint8_t f32_to_e4m3(float f) {
  return (uint8_t)__nv_cvt_float_to_fp8(f, __NV_SATFINITE, __NV_E4M3);
}

// Round half away from zero (C round()), restated from its definition.
__device__ __forceinline__ float round_half_away(float q) {
  float a = fabsf(q);
  float r = floorf(a);
  r = (a - r >= 0.5f) ? r + 1.0f : r;
  return copysignf(r, q);
}

// Bounded mbarrier / flag waits: every spin has an iteration limit.
constexpr uint32_t kSpinLimit = 1u << 26;

}  // namespace sq
