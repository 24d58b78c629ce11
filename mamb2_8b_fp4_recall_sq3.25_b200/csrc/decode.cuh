// Persistent batch-1 greedy decode: one cooperative kernel per generated token runs the
// whole 56-layer step (embedding, per layer: Block residual + RMSNorm, in_proj, SQ3.25
// scan step with the conv ring, Resurface + gated RMSNorm, out_proj; final norm, lm_head,
// argmax).  Every CTA owns fixed row tiles of every projection and streams them through one
// TMA ring that runs ahead across phase and layer boundaries; three grid barriers per layer.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sq {

struct DecLayer {
  const uint16_t* norm_w;        // [4096] Block RMSNorm weight
  const uint16_t* conv_w;        // [10240, 4]
  const uint16_t* conv_b;        // [10240]
  const float* A;                // [128] fp32 (negative)
  const uint16_t* D;             // [128] fp16
  const uint16_t* dt_bias;       // [128] fp16
  const uint16_t* gnorm_w;       // [8192] gated RMSNorm weight
  const float* in_g;             // in_proj fp32 global scale
  const float* out_g;            // out_proj fp32 global scale
  const uint8_t* perm;           // [8, 128]
  const uint16_t* basis;         // [8, nz, 2]
  const uint16_t* latent_scale;  // [8, 2]
  const uint16_t* predictor;     // [8, n8+n4+2, nz]
  const uint16_t* ad_V;          // Resurface adapter (null when absent)
  const uint16_t* ad_g;
  const uint16_t* ad_w;
  const uint16_t* ad_b;
  uint8_t* lo; uint8_t* hi; uint8_t* q4; uint8_t* latent; uint16_t* s8; uint16_t* s4;   // batch-1 state
  uint16_t* ring;                // [4, 10240] conv ring, slot = position % 4
  int layout;
  int hard;
};

struct DecodeSync { unsigned long long count; int abort, pad; };


struct DecodeParams {
  const DecLayer* layers;        // [n_layer] (device)
  const CUtensorMap* maps;       // [(2 * n_layer + 1) * 2] codes / scales maps (device, 64-B aligned)
  const CUtensorMap* aux_maps;   // [n_layer][2]: adapter V [128][128], gated-norm weights [128][64]; fp16, SWIZZLE_128B
  const uint8_t* head_codes; const uint8_t* head_scales;
  const uint8_t* emb_codes; const uint8_t* emb_scales; const float* emb_g;
  const float* head_g;
  const uint16_t* norm_f;
  uint16_t* h;                   // [4096] out_proj output
  uint16_t* res;                 // [2][4096] residual, ping-pong by layer parity
  uint16_t* zx;                  // [18560] in_proj output
  uint16_t* y;                   // [8192] scan readout
  uint16_t* logits;              // [vocab]
  float* part_v; int* part_i;    // [grid] argmax candidates
  DecodeSync* sync;
  int* err;
  long long* tok;                // [1] token fed to the first step, replaced by every greedy pick
  long long* out_tokens;         // [steps] picks (may be null)
  int n_layer, vocab, pos, steps; // pos: position of the first step's token
  float eps;
  int exact;                     // 1: projections and head with the exactly decoded fp16 weights
};

// Dynamic shared memory of the kernel; decode_grid() = CTAs of one cooperative launch (one
// per SM) or -1 when this device cannot run it; launch_decode_step enqueues one launch that
// runs p.steps greedy token steps.
int decode_smem_bytes();
int prepare_decode_kernel();
int decode_grid();
int launch_decode_step(const DecodeParams& p, int grid, cudaStream_t st);

}  // namespace sq
