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

// Asynchronous 16-byte global -> shared copies (LDGSTS); both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" :: "r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_all;\n" ::: "memory");
}
// Block-cooperative copy of `bytes` (multiple of 16) from global to shared memory.
__device__ __forceinline__ void stage16(void* smem_dst, const void* gsrc, int bytes, int tid, int nthreads) {
  const int n = bytes >> 4;
  for (int i = tid; i < n; i += nthreads)
    cp_async16(reinterpret_cast<char*>(smem_dst) + 16 * i, reinterpret_cast<const char*>(gsrc) + 16 * i);
}

// Bounded mbarrier / flag waits: every spin has an iteration limit.
constexpr uint32_t kSpinLimit = 1u << 26;

// The CUDA error of the calling thread's last failed launch (abi.cu).  Launchers consume
// the runtime's sticky-free launch error with cudaGetLastError(); recording it here lets
// the C-ABI report the real cause instead of "no error".
cudaError_t& last_launch_error();
inline int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return kOk;
  last_launch_error() = e;
  return kECuda;
}

}  // namespace sq
