// Parameter block of the legacy sq3p25 scan and its straight-through training backward (ste.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sq {

struct SteParams {
  int batch, length, heads, dim, groups;
  const uint16_t* x; long long x_sb, x_st;             // (b,t,h,p) at x + b*x_sb + t*x_st + h*dim + p
  const uint16_t* dt; long long dt_sb, dt_st;          // (b,t,h)
  const float* A;                                      // [H] fp32 (negative)
  const uint16_t* B; long long b_sb, b_st;             // (b,t,g,n) at B + b*b_sb + t*b_st + g*128 + n
  const uint16_t* C; long long c_sb, c_st;
  const void* D; int d_is_f32;
  const void* dt_bias; int dt_bias_is_f32;
  const uint8_t* perm;                                 // [G,128]: 16 INT8 | 64 INT4 | 48 pruned
  // forward: packed state (lo/hi u8[8], q4 u8[32], s8/s4 fp16 per row) and y
  uint8_t* lo; uint8_t* hi; uint8_t* q4; uint16_t* s8; uint16_t* s4;
  uint16_t* y; long long y_sb, y_st;
  // backward (contiguous layouts): upstream dy [B,L,H,P] fp16; dx [B,L,H,P], ddt [B,L,H],
  // db / dc [B,L,G,128] fp32; chunk length and the workspace arrays (bound by the launcher)
  const uint16_t* dy;
  float* dx; float* ddt; float* db; float* dc;
  int chunk, nchunk;
  float* cp; float* hist; float* adj; float* part;
};

int launch_sq3p25_scan(const SteParams& P, cudaStream_t st);
long long ste_workspace_bytes(int batch, int length, int heads, int dim, int chunk);
int launch_ste_backward(SteParams P, void* workspace, cudaStream_t st);

}  // namespace sq
