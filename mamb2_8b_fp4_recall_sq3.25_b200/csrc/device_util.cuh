// Small device helpers shared by the projection, block and decode kernels (sm_100a).
#pragma once
#include "common.cuh"

namespace sq {

// Hardware conversions (sm_100a): four code bytes -> four f16x2 magnitudes*sign
// (element 2i in the low half), and one E4M3 byte -> {v, v} as f16x2.  Both are exact:
// every E2M1 and E4M3 value is representable in fp16.
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n.reg .b8 q0, q1, q2, q3;\nmov.b32 {q0, q1, q2, q3}, %4;\n"
      "cvt.rn.f16x2.e2m1x2 %0, q0;\ncvt.rn.f16x2.e2m1x2 %1, q1;\n"
      "cvt.rn.f16x2.e2m1x2 %2, q2;\ncvt.rn.f16x2.e2m1x2 %3, q3;\n}\n"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3]) : "r"(w));
}
__device__ __forceinline__ uint32_t e4m3_splat_f16x2(uint32_t byte) {
  uint32_t r;
  const uint16_t two = (uint16_t)(byte | (byte << 8));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;\n" : "=r"(r) : "h"(two));
  return r;
}

// Exact decode of one code pair: FP16(FP32(FP32(m*b)*g)).  m*b is exact in fp16 (<= 6
// significant bits, |m*b| <= 2688, >= 2^-10), so HMUL2 gives it exactly; the product with
// the fp32 global scale is then rounded once to fp32 and once to fp16, as the reference.
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 p = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&p);
}
__device__ __forceinline__ uint32_t scale_pair(uint32_t m16x2, uint32_t b16x2, float2 g2) {
  __half2 p = __hmul2(*reinterpret_cast<__half2*>(&m16x2), *reinterpret_cast<__half2*>(&b16x2));
  const float2 f = __fmul2_rn(__half22float2(p), g2);
  __half2 r = __float22half2_rn(f);
  return *reinterpret_cast<uint32_t*>(&r);
}

// D += A . B on the tensor cores: m16n8k16, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

// z * sigmoid(z) in fp32 with the hardware exponential and reciprocal approximations
// (ex2.approx and rcp.approx, a few ulp; torch's silu on the reference side differs from a
// correctly rounded result by a similar amount).  1 + e^-z >= 1, so the reciprocal never
// sees a denormal; e^-z = inf gives 0.
__device__ __forceinline__ float silu_fast(float z) { return z * __fdividef(1.0f, 1.0f + __expf(-z)); }

// Resurface correction and gated-norm input of two adjacent channels of one head:
// y' = fp16(y + fp16(g * fp16(mix))) on half2 (each half2 operation rounds its exact result
// once to fp16, the value the fp32 operation followed by an fp16 rounding gives: products of
// two fp16 values are exact in fp32, and a sum that fp32 must round has operands more than
// 2^13 apart, far from an fp16 rounding boundary), then x = y' * silu(z) in fp32.
__device__ __forceinline__ float2 resurface_pair(uint32_t y2, uint32_t z2, float m0, float m1, __half2 g2, bool has_ad) {
  __half2 yh = *reinterpret_cast<__half2*>(&y2);
  if (has_ad) yh = __hadd2(yh, __hmul2(g2, __floats2half2_rn(m0, m1)));
  const float2 yf = __half22float2(yh);
  const float2 zf = __half22float2(*reinterpret_cast<__half2*>(&z2));
  return make_float2(yf.x * silu_fast(zf.x), yf.y * silu_fast(zf.y));
}

// first-occurrence merge of (value, index) argmax candidates
__device__ __forceinline__ void argmax_merge(float& bv, int& bi, float v2, int i2) {
  if (v2 > bv || (v2 == bv && i2 < bi)) { bv = v2; bi = i2; }
}

}  // namespace sq
