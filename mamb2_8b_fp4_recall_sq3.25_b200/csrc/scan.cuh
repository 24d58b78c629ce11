// Parameter block of the fused SQ3.25 selective-state-update kernel.
#pragma once
#include <stdint.h>

namespace sq {

// The seven released tier layouts after the latent shift
// (scripts/fp4_zero_predictor_codec_v1.py:28-36 applied to
//  scripts/w4_state_repair_codec_v2.py:22-28).  Index order is part of the C-ABI.
struct LayoutCounts { int n8, n4, nz; const char* name; };
constexpr LayoutCounts kLayouts[7] = {
  {32, 28, 68, "32_32_64"}, {16, 60, 52, "16_64_48"}, {8, 76, 44, "8_80_40"},
  {24, 44, 60, "24_48_56"}, {36, 20, 72, "36_24_68"}, {40, 12, 76, "40_16_72"},
  {44, 4, 80, "44_8_76"},
};

struct ScanParams {
  int batch, length, heads, dim, groups, layout;
  // fp16 activations; element (b,t,h,p) at x + b*x_sb + t*x_st + h*dim + p
  const uint16_t* x; long long x_sb, x_st;
  const uint16_t* dt; long long dt_sb, dt_st;        // (b,t,h) at dt + b*dt_sb + t*dt_st + h
  const float* A;                                      // [H] fp32 (negative)
  const uint16_t* B; long long b_sb, b_st;           // (b,t,g,n) at B + b*b_sb + t*b_st + g*128 + n
  const uint16_t* C; long long c_sb, c_st;
  const void* D; int d_is_f32;                         // [H]
  const void* dt_bias; int dt_bias_is_f32;             // [H]
  const uint8_t* perm;                                 // [G,128]
  const uint16_t* basis;                               // [G,nz,2] fp16
  const uint16_t* latent_scale;                        // [G,2] fp16
  const uint16_t* predictor;                           // [G,n8+n4+2,nz] fp16
  uint8_t* lo; uint8_t* hi; uint8_t* q4; uint8_t* latent; uint16_t* s8; uint16_t* s4;
  uint16_t* y; long long y_sb, y_st;                   // (b,t,h,p) at y + b*y_sb + t*y_st + h*dim + p
  // Optional fused causal conv (mamba2_recall/state_quant.py:283-317).  conv_mode 0: x/B/C
  // are conv outputs.  1: prefill from a reset state (conv_pos == 0) with the conv1d
  // numerics; 2: one-token step (length 1, conv_pos > 0) with the step numerics.  In
  // modes 1/2 x/B/C point at the RAW in_proj xBC columns and the ring below is read
  // (mode 2) and updated with the newest raw columns.
  int conv_mode;
  const uint16_t* conv_w;   // [10240,4] fp16 (tap k multiplies position t-3+k)
  const uint16_t* conv_b;   // [10240]
  uint16_t* conv_cache;     // [B,4,10240] fp16 ring, slot = position % 4
  int conv_pos;             // absolute position of the first token of this call
  long long conv_cache_sb;  // batch stride of the ring (elements)
  // Optional workspace of the two-kernel multi-token path (modes 0/1, 128-thread CTAs):
  // per-(batch, token, group) conv'd B/C, predictor/zero-tier dots and per-head dt/decay,
  // computed once by a prep kernel.  Null pointers select the single fused kernel.
  uint16_t* prep_bc;        // [B][T][G][256] fp16
  float* prep_pv;           // [B][T][G][FP] fp32
  float2* prep_ddt;         // [B][T][H]
};

int launch_scan(const ScanParams& p, cudaStream_t stream);
// Workspace of the two-kernel path (bytes) and the binding of its three arrays into P
// (P.batch/length/groups/layout set); -1 for invalid sizes.
long long scan_prep_bytes(int batch, int length, int heads, int groups, int layout);
long long scan_prep_bytes_any_layout(int batch, int length, int heads, int groups);
void scan_prep_bind(ScanParams& P, void* ws);
int prepare_scan_kernels();

}  // namespace sq
