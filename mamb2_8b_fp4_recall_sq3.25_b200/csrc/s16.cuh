// Parameter block of the FP16-state control scan (s16.cu).
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>

namespace sq {

struct S16Params {
  int batch, length, heads, dim, groups;
  const uint16_t* x; long long x_sb, x_st;      // (b,t,h,p) at x + b*x_sb + t*x_st + h*dim + p
  const uint16_t* dt; long long dt_sb, dt_st;   // (b,t,h) at dt + b*dt_sb + t*dt_st + h
  const float* A;                                // [H]
  const uint16_t* B; long long b_sb, b_st;      // (b,t,g,n) at B + b*b_sb + t*b_st + g*128 + n
  const uint16_t* C; long long c_sb, c_st;
  const void* D; int d_is_f32;
  const void* dt_bias; int dt_bias_is_f32;
  uint16_t* state;                               // fp16 [B,H,P,128], updated in place
  uint16_t* y; long long y_sb, y_st;
  float* stats;                                  // optional fp32 [B,H,ceil(P/16),128]
};

int launch_s16_scan(const S16Params& p, cudaStream_t stream);

}  // namespace sq
