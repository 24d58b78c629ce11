// Fused SQ3.25 selective-state update (the production latent codec), sm_100a.
//
// Semantics: scripts/fp4_zero_predictor_codec_v1.py:76-181 (kernel) plus the host
// predictor correction of :221-225, which is folded in here (group dot products in
// shared memory instead of a separate einsum and an HBM round trip of the [B,L,G,F]
// correction tensor).  Optionally the causal depthwise conv of
// mamba2_recall/state_quant.py:283-317 is fused in front (prefill from a reset state,
// or the one-token step), so the kernel reads the raw in_proj columns directly.
//
// Mapping: one thread owns one recurrent row (b,h,p) of 128 coordinates and keeps its
// n8+n4 stored coordinates in registers for the whole call (the zero tier carries no
// state).  A CTA holds `hpc` heads of one B/C group (hpc*dim <= 128 threads).  Tokens are
// processed in chunks of TC: per chunk the CTA publishes the group's B/C values in tier
// order, dt/decay per (token, head), the predictor readout vector cvec (= the reference's
// `correction`) and the five zero-tier dots for all TC tokens, then every thread runs
// the TC recurrence steps on its row with packed fp32x2 arithmetic.  The next chunk's
// raw inputs are copied asynchronously (cp.async) into a shared-memory ring of raw tokens
// while the current one is computed; the same ring carries the conv history, so no input
// or conv state is held in registers across the recurrence.  Packed rows are read once at
// the start and written once at the end of the call.
#include <algorithm>

#include "common.cuh"
#include "scan.cuh"
#include "scan_math.cuh"

namespace sq {

namespace {

constexpr int kTC = 8;         // tokens per chunk
constexpr int kMaxHpc = 8;     // heads per CTA (dim >= 16)

// Shared-memory plan of one CTA (byte offsets; every region 16-byte aligned).
//   ring   R slots of raw inputs per token: x[128] | B[128] | C[128] fp16 (x holds the
//          CTA's own channels, B/C the whole group row in channel order).  Slot of token t
//          (relative to the call, may be negative) = t mod R.  Slots -3..-1 carry the conv
//          history: zeros after a reset (mode 1) or the conv cache (mode 2).
//   T      token tables of one chunk: B/C in tier order (float4 pairs), cvec, conv'd x.
//          Before the first chunk the same bytes stage the raw static tables and packed rows;
//          after the last chunk they stage the repacked rows.
//   dots, dd, pred, basis, perm, conv weights.
template <int N8, int N4, int TC>
struct ScanSmem {
  static constexpr int NZ = 128 - N8 - N4, F = N8 + N4 + 2;
  static constexpr int R = (2 * TC >= TC + 3) ? 2 * TC : 4;     // power of two >= TC + 3 and 2 TC
  static constexpr int kSlotElems = 384;
  static constexpr int a16(int v) { return (v + 15) / 16 * 16; }
  static constexpr int oRawBasis = a16(F * NZ * 2);
  static constexpr int oRawPerm = oRawBasis + a16(NZ * 4);
  static constexpr int oPackStart = oRawPerm + 128;
  static constexpr int kTok = TC * 64 * 16 + TC * 64 * 8 + TC * 128 * 4;
  static constexpr int kT = (kTok > oPackStart + 128 * 52) ? kTok : oPackStart + 128 * 52;
  static constexpr int oRing = 0;
  static constexpr int oT = oRing + R * kSlotElems * 2;
  static constexpr int oDots = oT + kT;
  static constexpr int oDD = oDots + TC * 8 * 4;
  static constexpr int oPred = oDD + TC * kMaxHpc * 2 * 4;
  static constexpr int oBasis = oPred + a16(F * (NZ + 1) * 4);
  static constexpr int oPerm = oBasis + a16(2 * NZ * 4);
  static constexpr int oW = oPerm + 128 * 4;
  static constexpr int kBytes = oW + 3 * 128 * 5 * 4;
};

// Resident CTAs per SM the register budget is sized for: 4 (<= 128 registers) for every
// layout.  The folded multi-token readout (recur_row_fold) keeps one accumulation per pair,
// which leaves room for the widest stored row (84 coordinates) in 128 registers.
template <int N8, int N4>
constexpr int scan_min_blocks() { return 4; }
// The single fused kernel also holds the group dots' staging: 3 CTAs for the widest rows.
template <int N8, int N4>
constexpr int fused_min_blocks() { return N8 + N4 >= 68 ? 3 : 4; }

template <int N8, int N4, int KJ, int MODE, int TC>
__global__ void __launch_bounds__(128, MODE == 2 ? 1 : fused_min_blocks<N8, N4>())   // decode grids are small
ssu_sq325_kernel(const ScanParams P) {
  using L = ScanSmem<N8, N4, TC>;
  constexpr int NZ = L::NZ;
  constexpr int F = L::F;
  constexpr int R = L::R;
  constexpr int SE = L::kSlotElems;
  constexpr int W8 = N8 / 2, W4 = N4 / 2;
  constexpr int NP = (N8 + N4) / 2;            // stored coordinate pairs
  static_assert(N8 % 2 == 0 && N4 % 2 == 0, "tiers are nibble pairs");

  extern __shared__ __align__(16) unsigned char smem[];
  uint16_t* ring = reinterpret_cast<uint16_t*>(smem + L::oRing);
  float4* sP4 = reinterpret_cast<float4*>(smem + L::oT);                  // [TC][64] {b_j,b_j+1,c_j,c_j+1}
  float2* sV2 = reinterpret_cast<float2*>(smem + L::oT + TC * 64 * 16);   // [TC][64] {cvec_j,cvec_j+1}
  float* sX = reinterpret_cast<float*>(smem + L::oT + TC * 64 * 24);      // [TC][128] conv'd own x
  float* sDots = reinterpret_cast<float*>(smem + L::oDots);               // [TC][8]
  float* sDD = reinterpret_cast<float*>(smem + L::oDD);                   // [TC][kMaxHpc][2] (dt, decay)
  float* sPred = reinterpret_cast<float*>(smem + L::oPred);               // [F][NZ+1]
  float* sBasis = reinterpret_cast<float*>(smem + L::oBasis);             // [2][NZ]
  int* sPerm = reinterpret_cast<int*>(smem + L::oPerm);                   // [128]
  float* sW = reinterpret_cast<float*>(smem + L::oW);                     // [3][128][5] x / B / C taps + bias
  float* sPf = reinterpret_cast<float*>(sP4);
  uint16_t* rawPred = reinterpret_cast<uint16_t*>(smem + L::oT);
  uint16_t* rawBasis = reinterpret_cast<uint16_t*>(smem + L::oT + L::oRawBasis);
  uint8_t* rawPerm = smem + L::oT + L::oRawPerm;
  unsigned char* sPack = smem + L::oT + L::oPackStart;

  const int tid = threadIdx.x;
  const int bd = blockDim.x;
  const int dim = P.dim;
  const int hpc = bd / dim;
  const int b = blockIdx.y;
  const int h0 = blockIdx.x * hpc;
  const int hl = tid / dim;
  const int p = tid - hl * dim;
  const int h = h0 + hl;
  const int hpg = P.heads / P.groups;
  const int g = h0 / hpg;
  const bool group_leader = (h0 % hpg) == 0;       // writes the group's B/C conv cache entries
  const long long row0 = ((long long)b * P.heads + h0) * dim;
  const int rows = bd;
  const int kj = KJ;                                // coordinates per thread: 128 / blockDim

  const uint16_t* xb = P.x + (long long)b * P.x_sb + (long long)h0 * dim;
  const uint16_t* Bb = P.B + (long long)b * P.b_sb + g * 128;
  const uint16_t* Cb = P.C + (long long)b * P.c_sb + g * 128;
  // 16-byte asynchronous copies need 16-byte aligned rows; otherwise the raw inputs are
  // staged with element loads (same layout, synchronous).
  const bool vec = ((((uintptr_t)xb | (uintptr_t)Bb | (uintptr_t)Cb) & 15) == 0) &&
                   ((P.x_st | P.b_st | P.c_st) & 7) == 0;
  const int px = bd / 8;                            // 16-byte pieces of x per token
  const int per_tok = px + 32;

  // raw x/B/C of tokens [c0, c0 + nt) into their ring slots
  uint16_t pre_dt = 0;
  auto prefetch = [&](int c0) {
    const int nt = min(TC, P.length - c0);
    for (int i = tid; i < nt * per_tok; i += bd) {
      const int t = i / per_tok, r = i - t * per_tok;
      const long long tt = c0 + t;
      uint16_t* slot = ring + ((c0 + t) & (R - 1)) * SE;
      const uint16_t* src;
      uint16_t* dst;
      if (r < px) { src = xb + tt * P.x_st + r * 8; dst = slot + r * 8; }
      else if (r < px + 16) { src = Bb + tt * P.b_st + (r - px) * 8; dst = slot + 128 + (r - px) * 8; }
      else { src = Cb + tt * P.c_st + (r - px - 16) * 8; dst = slot + 256 + (r - px - 16) * 8; }
      if (vec) cp_async16(dst, src);
      else {
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[e] = src[e];
      }
    }
    if (tid < nt * hpc) {
      const int t = tid / hpc, hh = h0 + tid % hpc;
      pre_dt = P.dt[(long long)b * P.dt_sb + (long long)(c0 + t) * P.dt_st + hh];
    }
  };

  // ---- stage static tables and packed rows with asynchronous 16-byte copies ----
  unsigned char* pLo = sPack;
  unsigned char* pHi = pLo + rows * W8;
  unsigned char* pQ4 = pHi + rows * W8;
  unsigned char* pLat = pQ4 + rows * W4;
  uint16_t* pS8 = reinterpret_cast<uint16_t*>(pLat + rows * 2);
  uint16_t* pS4 = pS8 + rows;
  stage16(rawPred, P.predictor + (long long)g * F * NZ, F * NZ * 2, tid, bd);
  stage16(rawBasis, P.basis + (long long)g * NZ * 2, NZ * 4, tid, bd);
  stage16(rawPerm, P.perm + g * 128, 128, tid, bd);
  stage16(pLo, P.lo + row0 * W8, rows * W8, tid, bd);
  stage16(pHi, P.hi + row0 * W8, rows * W8, tid, bd);
  stage16(pQ4, P.q4 + row0 * W4, rows * W4, tid, bd);
  stage16(pLat, P.latent + row0 * 2, rows * 2, tid, bd);
  stage16(pS8, P.s8 + row0, rows * 2, tid, bd);
  stage16(pS4, P.s4 + row0, rows * 2, tid, bd);
  if (MODE == 2) {
    // conv history: the cache's three previous positions into the slots of tokens -3..-1
    const uint16_t* cache = P.conv_cache + (long long)b * P.conv_cache_sb;
    for (int i = tid; i < 3 * per_tok; i += bd) {
      const int k = i / per_tok, r = i - k * per_tok;
      const uint16_t* cs = cache + ((P.conv_pos - 3 + k) & 3) * 10240;
      uint16_t* slot = ring + ((k - 3) & (R - 1)) * SE;
      if (r < px) cp_async16(slot + r * 8, cs + h0 * dim + r * 8);
      else if (r < px + 16) cp_async16(slot + 128 + (r - px) * 8, cs + 8192 + g * 128 + (r - px) * 8);
      else cp_async16(slot + 256 + (r - px - 16) * 8, cs + 9216 + g * 128 + (r - px - 16) * 8);
    }
  }
  cp_async_wait_all();
  __syncthreads();
  for (int i = tid; i < F * NZ; i += bd) {
    const int f = i / NZ, d = i - f * NZ;
    sPred[f * (NZ + 1) + d] = h2f(rawPred[i]);
  }
  for (int i = tid; i < NZ; i += bd) {
    sBasis[i] = h2f(rawBasis[2 * i + 0]);
    sBasis[NZ + i] = h2f(rawBasis[2 * i + 1]);
  }
  for (int i = tid; i < 128; i += bd) sPerm[i] = rawPerm[i];
  if (MODE == 1) {
    for (int i = tid; i < 3 * SE; i += bd) ring[((i / SE - 3) & (R - 1)) * SE + i % SE] = 0;
  }
  __syncthreads();
  if (MODE != 0) {
    for (int c = tid; c < bd; c += bd) {
      const int ch = h0 * dim + c;
#pragma unroll
      for (int i = 0; i < 4; ++i) sW[c * 5 + i] = h2f(P.conv_w[ch * 4 + i]);
      sW[c * 5 + 4] = h2f(P.conv_b[ch]);
    }
    for (int j = tid; j < 128; j += bd) {
      const int chb = 8192 + g * 128 + sPerm[j], chc = 9216 + g * 128 + sPerm[j];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sW[(128 + j) * 5 + i] = h2f(P.conv_w[chb * 4 + i]);
        sW[(256 + j) * 5 + i] = h2f(P.conv_w[chc * 4 + i]);
      }
      sW[(128 + j) * 5 + 4] = h2f(P.conv_b[chb]);
      sW[(256 + j) * 5 + 4] = h2f(P.conv_b[chc]);
    }
  }
  prefetch(0);

  // ---- decode own row (:81-114) ----
  float S[N8 + N4];
  {
    const float s8 = h2f(pS8[tid]), s4 = h2f(pS4[tid]);
#pragma unroll
    for (int j = 0; j < N8; ++j) {
      int lo = (pLo[tid * W8 + j / 2] >> (4 * (j & 1))) & 15;
      int hi = (pHi[tid * W8 + j / 2] >> (4 * (j & 1))) & 15;
      int ub = (hi << 4) | lo;
      S[j] = (float)(ub - 256 * (ub > 127)) * s8;
    }
#pragma unroll
    for (int j = 0; j < N4; ++j) {
      int nib = (pQ4[tid * W4 + j / 2] >> (4 * (j & 1))) & 15;
      S[N8 + j] = (float)(nib - 16 * (nib > 7)) * s4;
    }
  }
  const float ls0 = h2f(P.latent_scale[g * 2 + 0]), ls1 = h2f(P.latent_scale[g * 2 + 1]);
  const float ils0 = __frcp_rn(ls0), ils1 = __frcp_rn(ls1);
  const float2 ls2 = make_float2(ls0, ls1), nls2 = make_float2(-ls0, -ls1), ils2 = make_float2(ils0, ils1);
  float2 zz = make_float2(e4m3_to_f32(pLat[tid * 2 + 0]) * ls0, e4m3_to_f32(pLat[tid * 2 + 1]) * ls1);
  const float dv = P.d_is_f32 ? reinterpret_cast<const float*>(P.D)[h] : h2f(reinterpret_cast<const uint16_t*>(P.D)[h]);
  const float bias_own = P.dt_bias_is_f32 ? reinterpret_cast<const float*>(P.dt_bias)[h0 + (tid % max(hpc, 1))]
                                          : h2f(reinterpret_cast<const uint16_t*>(P.dt_bias)[h0 + (tid % max(hpc, 1))]);
  const float A_own = P.A[h0 + (tid % max(hpc, 1))];
  float s8 = 0.f, s4 = 0.f;

  for (int c0 = 0; c0 < P.length; c0 += TC) {
    const int nt = min(TC, P.length - c0);
    cp_async_wait_all();
    __syncthreads();                                   // raw chunk landed; previous chunk's tables free
    // -- publish conv'd x, B/C (tier order) and dt/decay for this chunk --
    {
      float w[5];
      const uint16_t* rx = ring + tid;
      float h1 = 0.f, h2 = 0.f, h3 = 0.f;             // raw x at t-3, t-2, t-1
      if (MODE != 0) {
#pragma unroll
        for (int i = 0; i < 5; ++i) w[i] = sW[tid * 5 + i];
        h1 = h2f(rx[((c0 - 3) & (R - 1)) * SE]);
        h2 = h2f(rx[((c0 - 2) & (R - 1)) * SE]);
        h3 = h2f(rx[((c0 - 1) & (R - 1)) * SE]);
      }
#pragma unroll
      for (int t = 0; t < TC; ++t) {
        if (t < nt) {
          const float raw = h2f(rx[((c0 + t) & (R - 1)) * SE]);
          float xv = raw;
          if (MODE == 1) xv = conv_prefill_value(w, h1, h2, h3, raw);
          if (MODE == 2) xv = conv_step_value(w, h1, h2, h3, raw);
          h1 = h2; h2 = h3; h3 = raw;
          sX[t * 128 + tid] = xv;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < KJ; ++k) {
      const int j = tid + k * bd;
      if (k < kj && j < 128) {
        const int n = sPerm[j];
        float wb[5], wc[5];
        float b1 = 0.f, b2 = 0.f, b3 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
        if (MODE != 0) {
#pragma unroll
          for (int i = 0; i < 5; ++i) { wb[i] = sW[(128 + j) * 5 + i]; wc[i] = sW[(256 + j) * 5 + i]; }
          b1 = h2f(ring[((c0 - 3) & (R - 1)) * SE + 128 + n]);
          b2 = h2f(ring[((c0 - 2) & (R - 1)) * SE + 128 + n]);
          b3 = h2f(ring[((c0 - 1) & (R - 1)) * SE + 128 + n]);
          c1 = h2f(ring[((c0 - 3) & (R - 1)) * SE + 256 + n]);
          c2 = h2f(ring[((c0 - 2) & (R - 1)) * SE + 256 + n]);
          c3 = h2f(ring[((c0 - 1) & (R - 1)) * SE + 256 + n]);
        }
#pragma unroll
        for (int t = 0; t < TC; ++t) {
          if (t < nt) {
            const uint16_t* slot = ring + ((c0 + t) & (R - 1)) * SE;
            const float rb = h2f(slot[128 + n]), rc = h2f(slot[256 + n]);
            float bv = rb, cv = rc;
            if (MODE == 1) { bv = conv_prefill_value(wb, b1, b2, b3, rb); cv = conv_prefill_value(wc, c1, c2, c3, rc); }
            if (MODE == 2) { bv = conv_step_value(wb, b1, b2, b3, rb); cv = conv_step_value(wc, c1, c2, c3, rc); }
            b1 = b2; b2 = b3; b3 = rb;
            c1 = c2; c2 = c3; c3 = rc;
            sPf[t * 256 + (j >> 1) * 4 + (j & 1)] = bv;
            sPf[t * 256 + (j >> 1) * 4 + 2 + (j & 1)] = cv;
          }
        }
      }
    }
    if (tid < nt * hpc) {
      const float dtv = softplus_ref(h2f(pre_dt) + bias_own);
      sDD[((tid / hpc) * kMaxHpc + tid % hpc) * 2 + 0] = dtv;
      sDD[((tid / hpc) * kMaxHpc + tid % hpc) * 2 + 1] = expf(A_own * dtv);
    }
    __syncthreads();                                   // tables visible; this chunk's raw slots consumed
    if (c0 + TC < P.length) prefetch(c0 + TC);
    // -- group-level dots for every token of the chunk --
    for (int task = tid; task < nt * (F + 5); task += bd) {
      const int t = task / (F + 5), f = task - t * (F + 5);
      const float* tb = sPf + t * 256;
      float acc0 = 0.f, acc1 = 0.f;
      if (f < F) {
        const float* pr = sPred + f * (NZ + 1);
#pragma unroll 4
        for (int d = 0; d < NZ; d += 2) {
          const int j0 = N8 + N4 + d;                  // even: pairs never straddle
          acc0 = fmaf(tb[(j0 >> 1) * 4 + 2], pr[d], acc0);
          acc1 = fmaf(tb[(j0 >> 1) * 4 + 3], pr[d + 1], acc1);
        }
        const float acc = acc0 + acc1;
        // multi-token modes fold C into the correction vector (recur_row_fold)
        if (f < N8 + N4) reinterpret_cast<float*>(sV2)[t * 128 + f] = MODE == 2 ? acc : tb[(f >> 1) * 4 + 2 + (f & 1)] + acc;
        else sDots[t * 8 + 5 + f - (N8 + N4)] = acc;
      } else if (f == F && MODE != 2) {
        // B.C over all 128 coordinates (the folded readout's current-token term)
#pragma unroll 4
        for (int j0 = 0; j0 < 128; j0 += 2) {
          const float* q = tb + (j0 >> 1) * 4;
          acc0 = fmaf(q[0], q[2], acc0);
          acc1 = fmaf(q[1], q[3], acc1);
        }
        sDots[t * 8 + 0] = acc0 + acc1;
      } else {
        const int k = f - F;   // 0: B.C (zero tier), 1: basis0.C, 2: basis1.C, 3: basis0.B, 4: basis1.B
        const float* us = (k == 0) ? nullptr : sBasis + ((k - 1) & 1) * NZ;
        const int voff = (k >= 3 || k == 0) ? 0 : 2;   // 0 -> B, 2 -> C (within the float4)
#pragma unroll 4
        for (int d = 0; d < NZ; d += 2) {
          const int j0 = N8 + N4 + d;
          const float* q = tb + (j0 >> 1) * 4;
          const float u0 = (k == 0) ? q[0] : us[d], u1 = (k == 0) ? q[1] : us[d + 1];
          const float v0 = (k == 0) ? q[2] : q[voff], v1 = (k == 0) ? q[3] : q[voff + 1];
          acc0 = fmaf(u0, v0, acc0);
          acc1 = fmaf(u1, v1, acc1);
        }
        sDots[t * 8 + k] = acc0 + acc1;
      }
    }
    __syncthreads();                                   // cvec and dots visible

    // -- per-row recurrence, readout and requant (:115-162) for the chunk's tokens --
#pragma unroll 1
    for (int t = 0; t < nt; ++t) {
      const float dtv = sDD[(t * kMaxHpc + hl) * 2 + 0];
      const float dec = sDD[(t * kMaxHpc + hl) * 2 + 1];
      const float x = sX[t * 128 + tid];
      float m8, m4;
      float dots[7];
#pragma unroll
      for (int i = 0; i < 7; ++i) dots[i] = sDots[t * 8 + i];
      TokenScales ts;
      float out;
      if (MODE == 2) {                                 // one-token step: four readout streams
        float ysum, ycorr;
        recur_row4<N8, NP>(S, sP4 + t * 64, sV2 + t * 64, dec, dtv, x, ysum, ycorr, m8, m4);
        out = token_tail_sums(ysum, ycorr, m8, m4, x, dtv, dec, dv, dots, zz, ls2, nls2, ils2, ts);
      } else {                                         // multi-token: folded readout
        const float yacc = recur_row_fold<N8, NP, false, true>(S, sP4 + t * 64, sV2 + t * 64, dec, dtv, x, m8, m4);
        out = token_tail_fold(yacc, m8, m4, x, dtv, dec, dv, dots, zz, ls2, nls2, ils2, ts);
      }
      P.y[(long long)b * P.y_sb + (long long)(c0 + t) * P.y_st + (long long)h * dim + p] = f2h(out);
      // INT8 / INT4 requant (:155-162, scripts/state_ppl_codec_v6.py:52-61)
      s8 = ts.s8; s4 = ts.s4;
      requant_row<N8, NP>(S, ts);
    }
  }

  // ---- conv cache update: raw columns of the newest positions, channel order ----
  if (MODE != 0) {
    uint16_t* cache = P.conv_cache + (long long)b * P.conv_cache_sb;
    const int nwrite = MODE == 2 ? 1 : min(4, P.length);
    for (int i = 0; i < nwrite; ++i) {
      const int t = P.length - 1 - i;                  // relative token
      const int slot = (P.conv_pos + t) & 3;           // absolute position mod 4
      const uint16_t* src = ring + (t & (R - 1)) * SE;
      cache[slot * 10240 + h0 * dim + tid] = src[tid];
      if (group_leader)
        for (int n = tid; n < 128; n += bd) {
          cache[slot * 10240 + 8192 + g * 128 + n] = src[128 + n];
          cache[slot * 10240 + 9216 + g * 128 + n] = src[256 + n];
        }
    }
  }

  // ---- pack once (:163-181) and store coalesced ----
  __syncthreads();
  {
    const float i8 = s8 > 0.f ? __frcp_rn(s8) : 0.f;
    const float i4 = s4 > 0.f ? __frcp_rn(s4) : 0.f;
#pragma unroll
    for (int j = 0; j < N8; j += 2) {
      const int qa = __float2int_rn(div_exact(S[j], s8, i8));
      const int qb = __float2int_rn(div_exact(S[j + 1], s8, i8));
      pLo[tid * W8 + j / 2] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
      pHi[tid * W8 + j / 2] = (unsigned char)(((qa >> 4) & 15) | (((qb >> 4) & 15) << 4));
    }
#pragma unroll
    for (int j = 0; j < N4; j += 2) {
      const int qa = __float2int_rn(div_exact(S[N8 + j], s4, i4));
      const int qb = __float2int_rn(div_exact(S[N8 + j + 1], s4, i4));
      pQ4[tid * W4 + j / 2] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
    }
    pLat[tid * 2 + 0] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.x, ls0, ils0), -448.f), 448.f));
    pLat[tid * 2 + 1] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.y, ls1, ils1), -448.f), 448.f));
    pS8[tid] = f2h(s8);
    pS4[tid] = f2h(s4);
  }
  __syncthreads();
  auto copy_out = [&](unsigned char* dst, const unsigned char* src, int bytes) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = tid; i < bytes / 16; i += bd) d[i] = s[i];
  };
  copy_out(P.lo + row0 * W8, pLo, rows * W8);
  copy_out(P.hi + row0 * W8, pHi, rows * W8);
  copy_out(P.q4 + row0 * W4, pQ4, rows * W4);
  copy_out(P.latent + row0 * 2, pLat, rows * 2);
  copy_out(reinterpret_cast<unsigned char*>(P.s8 + row0), reinterpret_cast<unsigned char*>(pS8), rows * 2);
  copy_out(reinterpret_cast<unsigned char*>(P.s4 + row0), reinterpret_cast<unsigned char*>(pS4), rows * 2);
}

// ============================================================================================
// Two-kernel path for multi-token calls (modes 0 and 1, 64 <= dim, 128 threads per CTA).
//
// scan_prep_kernel does the per-(batch, token, group) work once instead of once per CTA of
// the group: the B/C conv (mode 1), the predictor readout vector cvec, the pcz pair and the
// five zero-tier dots, and dt/decay per head.  Its outputs go to a caller workspace:
//   bc   [B][T][G][256] fp16   conv'd B (tier order) then conv'd C (tier order)
//   pv   [B][T][G][FP]  fp32   C + cvec [0..NS) | pcz0 pcz1 | B.C (all 128), b0.C, b1.C, b0.B,
//                              b1.B | pad   (the folded readout, recur_row_fold)
//   ddt  [B][T][H]      float2 (dt after softplus, exp(A dt))
// ssu_chunk_kernel then streams x (raw in mode 1), bc, pv and ddt through a cp.async ring and
// runs the recurrence with B*dt precomputed per head.  Same arithmetic, operation for
// operation, as the fused kernel above: results are bit-identical.
// ============================================================================================

constexpr int kPrepTokens = 16;   // tokens per prep CTA
constexpr int kChunkTC = 8;       // tokens per chunk in the chunk kernel

template <int N8, int N4>
struct PrepLayout {
  static constexpr int NS = N8 + N4, NZ = 128 - NS, F = NS + 2;
  static constexpr int FP = (F + 5 + 3) / 4 * 4;       // pv floats per (b,t,g), 16-byte rows
};

template <int N8, int N4, int MODE>
__global__ void __launch_bounds__(256)
scan_prep_kernel(const ScanParams P) {
  using PL = PrepLayout<N8, N4>;
  constexpr int NS = PL::NS, NZ = PL::NZ, F = PL::F, FP = PL::FP;
  constexpr int TT = kPrepTokens;
  constexpr int oPred = TT * 256 * 4;
  constexpr int oBasis = oPred + (F * (NZ + 1) * 4 + 15) / 16 * 16;
  constexpr int oPerm = oBasis + (2 * NZ * 4 + 15) / 16 * 16;
  extern __shared__ __align__(16) unsigned char smem[];
  float* sBC = reinterpret_cast<float*>(smem);                       // [TT][256] conv'd B | C (tier order)
  float* sPred = reinterpret_cast<float*>(smem + oPred);             // [F][NZ+1]
  float* sBasis = reinterpret_cast<float*>(smem + oBasis);           // [2][NZ]
  int* sPerm = reinterpret_cast<int*>(smem + oPerm);                 // [128]
  uint16_t* rawPred = reinterpret_cast<uint16_t*>(smem);             // staging in sBC
  uint16_t* rawBasis = rawPred + (F * NZ * 2 + 15) / 16 * 8;
  uint8_t* rawPerm = reinterpret_cast<uint8_t*>(rawBasis + (NZ * 4 + 15) / 16 * 8);

  const int tid = threadIdx.x;
  const int t0 = blockIdx.x * TT, g = blockIdx.y, b = blockIdx.z;
  const int nt = min(TT, P.length - t0);
  stage16(rawPred, P.predictor + (long long)g * F * NZ, F * NZ * 2, tid, 256);
  stage16(rawBasis, P.basis + (long long)g * NZ * 2, NZ * 4, tid, 256);
  stage16(rawPerm, P.perm + g * 128, 128, tid, 256);
  cp_async_wait_all();
  __syncthreads();
  for (int i = tid; i < F * NZ; i += 256) {
    const int f = i / NZ, d = i - f * NZ;
    sPred[f * (NZ + 1) + d] = h2f(rawPred[i]);
  }
  for (int i = tid; i < NZ; i += 256) {
    sBasis[i] = h2f(rawBasis[2 * i + 0]);
    sBasis[NZ + i] = h2f(rawBasis[2 * i + 1]);
  }
  if (tid < 128) sPerm[tid] = rawPerm[tid];
  __syncthreads();

  // ---- B/C of tier coordinate j = tid % 128 (B for tid < 128, C above), conv'd in mode 1 ----
  {
    const int j = tid & 127;
    const bool isC = tid >= 128;
    const int n = sPerm[j];
    const uint16_t* src = (isC ? P.C + (long long)b * P.c_sb : P.B + (long long)b * P.b_sb) + g * 128 + n;
    const long long st = isC ? P.c_st : P.b_st;
    float w[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    float h1 = 0.f, h2 = 0.f, h3 = 0.f;
    if (MODE == 1) {
      const int ch = (isC ? 9216 : 8192) + g * 128 + n;
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = h2f(P.conv_w[ch * 4 + i]);
      w[4] = h2f(P.conv_b[ch]);
      if (t0 >= 3) h1 = h2f(src[(long long)(t0 - 3) * st]);
      if (t0 >= 2) h2 = h2f(src[(long long)(t0 - 2) * st]);
      if (t0 >= 1) h3 = h2f(src[(long long)(t0 - 1) * st]);
    }
    uint16_t* out = P.prep_bc + (((long long)b * P.length + t0) * P.groups + g) * 256 + tid;
    for (int t = 0; t < nt; ++t) {
      const float raw = h2f(src[(long long)(t0 + t) * st]);
      const float v = MODE == 1 ? conv_prefill_value(w, h1, h2, h3, raw) : raw;
      h1 = h2; h2 = h3; h3 = raw;
      sBC[t * 256 + tid] = v;
      out[(long long)t * P.groups * 256] = f2h(v);     // v is an fp16 value: exact
    }
  }
  // ---- dt / decay for the group's heads ----
  {
    const int hpg = P.heads / P.groups;
    for (int i = tid; i < nt * hpg; i += 256) {
      const int t = i / hpg, h = g * hpg + i % hpg;
      const float bias = P.dt_bias_is_f32 ? reinterpret_cast<const float*>(P.dt_bias)[h]
                                          : h2f(reinterpret_cast<const uint16_t*>(P.dt_bias)[h]);
      const float dtv = softplus_ref(h2f(P.dt[(long long)b * P.dt_sb + (long long)(t0 + t) * P.dt_st + h]) + bias);
      P.prep_ddt[((long long)b * P.length + t0 + t) * P.heads + h] = make_float2(dtv, expf(P.A[h] * dtv));
    }
  }
  __syncthreads();
  // ---- group dots (same accumulation order as the fused kernel) ----
  float* pv = P.prep_pv + (((long long)b * P.length + t0) * P.groups + g) * FP;
  for (int task = tid; task < nt * FP; task += 256) {
    const int t = task / FP, f = task - t * FP;
    const float* tb = sBC + t * 256;
    float r = 0.f;
    if (f < F) {
      const float* pr = sPred + f * (NZ + 1);
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 4
      for (int d = 0; d < NZ; d += 2) {
        acc0 = fmaf(tb[128 + NS + d], pr[d], acc0);
        acc1 = fmaf(tb[128 + NS + d + 1], pr[d + 1], acc1);
      }
      r = acc0 + acc1;
      if (f < NS) r = tb[128 + f] + r;                  // C_j + cvec_j (the folded readout)
    } else if (f == F) {
      // B.C over all 128 coordinates, the same order as the fused kernel
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 4
      for (int j0 = 0; j0 < 128; j0 += 2) {
        acc0 = fmaf(tb[j0], tb[128 + j0], acc0);
        acc1 = fmaf(tb[j0 + 1], tb[128 + j0 + 1], acc1);
      }
      r = acc0 + acc1;
    } else if (f < F + 5) {
      const int k = f - F;   // 0: B.C, 1: basis0.C, 2: basis1.C, 3: basis0.B, 4: basis1.B
      const float* us = (k == 0) ? nullptr : sBasis + ((k - 1) & 1) * NZ;
      const int voff = (k >= 3 || k == 0) ? 0 : 128;   // 0 -> B, 128 -> C
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 4
      for (int d = 0; d < NZ; d += 2) {
        const float u0 = (k == 0) ? tb[NS + d] : us[d], u1 = (k == 0) ? tb[NS + d + 1] : us[d + 1];
        const float v0 = (k == 0) ? tb[128 + NS + d] : tb[voff + NS + d];
        const float v1 = (k == 0) ? tb[128 + NS + d + 1] : tb[voff + NS + d + 1];
        acc0 = fmaf(u0, v0, acc0);
        acc1 = fmaf(u1, v1, acc1);
      }
      r = acc0 + acc1;
    }
    pv[(long long)t * P.groups * FP + f] = r;
  }
}

// Shared-memory plan of the chunk kernel (byte offsets, 16-byte aligned regions).
//   ring  R = 2 TC slots per token: raw (mode 1) or conv'd x[128] fp16 | bc[256] fp16 |
//         pv[FP] fp32 | ddt[hpc] float2.  Slot of token t (call-relative, may be negative)
//         = t mod R; slots of tokens -3..-1 hold the x conv history (zeros after a reset).
//   T     sP4 [TC][hpc][64] float4 {B*dt pair, C pair} per head, sX [TC][128] conv'd x;
//         before the first / after the last chunk: the packed rows.
//   W     x conv taps + bias [128][5] fp32.
template <int N8, int N4>
struct ChunkSmem {
  static constexpr int FP = PrepLayout<N8, N4>::FP;
  static constexpr int TC = kChunkTC, R = 2 * kChunkTC;
  static constexpr int oX = 0, oBC = 256, oPV = 768, oDD = 768 + FP * 4;
  static constexpr int kSlot = (oDD + 2 * 8 + 15) / 16 * 16;   // hpc <= 2
  static constexpr int oRing = 0;
  static constexpr int oT = R * kSlot;
  static constexpr int kTok = TC * 2 * 64 * 16 + TC * 128 * 4;
  static constexpr int kT = kTok > 128 * 52 ? kTok : 128 * 52;
  static constexpr int oW = oT + kT;
  static constexpr int kBytes = oW + 128 * 5 * 4;
};

__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gsrc) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" :: "r"(d), "l"(gsrc) : "memory");
}

template <int N8, int N4, int MODE>
__global__ void __launch_bounds__(128, scan_min_blocks<N8, N4>())
ssu_chunk_kernel(const ScanParams P) {
  using L = ChunkSmem<N8, N4>;
  constexpr int NS = N8 + N4, F = NS + 2, FP = L::FP;
  constexpr int TC = L::TC, R = L::R, SB = L::kSlot;
  constexpr int W8 = N8 / 2, W4 = N4 / 2;
  constexpr int NP = NS / 2;
  static_assert(N8 % 2 == 0 && N4 % 2 == 0, "tiers are nibble pairs");

  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* ring = smem + L::oRing;
  float4* sP4 = reinterpret_cast<float4*>(smem + L::oT);                    // [TC][hpc][64]
  float* sX = reinterpret_cast<float*>(smem + L::oT + TC * 2 * 64 * 16);    // [TC][128]
  float* sW = reinterpret_cast<float*>(smem + L::oW);                       // [128][5]
  float* sPf = reinterpret_cast<float*>(sP4);
  unsigned char* sPack = smem + L::oT;

  const int tid = threadIdx.x;
  const int dim = P.dim;
  const int hpc = 128 / dim;
  const int b = blockIdx.y;
  const int h0 = blockIdx.x * hpc;
  const int hl = tid / dim;
  const int p = tid - hl * dim;
  const int h = h0 + hl;
  const int hpg = P.heads / P.groups;
  const int g = h0 / hpg;
  const bool group_leader = (h0 % hpg) == 0;
  const long long row0 = ((long long)b * P.heads + h0) * dim;
  constexpr int rows = 128;

  auto slot_of = [&](int t) { return ring + (t & (R - 1)) * SB; };
  const uint16_t* xb = P.x + (long long)b * P.x_sb + (long long)h0 * dim;
  const bool vec = ((((uintptr_t)xb) & 15) == 0) && (P.x_st & 7) == 0;
  const long long btg = (long long)b * P.length;       // token row base of this batch entry
  constexpr int kPcs = 16 + 16 + FP / 4;               // 16-byte pieces per token (x, B half of bc, pv)

  auto prefetch = [&](int c0) {
    const int nt = min(TC, P.length - c0);
    for (int i = tid; i < nt * (kPcs + hpc); i += 128) {
      const int t = i / (kPcs + hpc), r = i - t * (kPcs + hpc);
      const long long tt = c0 + t;
      unsigned char* slot = slot_of(c0 + t);
      if (r < 16) {
        const uint16_t* src = xb + tt * P.x_st + r * 8;
        uint16_t* dst = reinterpret_cast<uint16_t*>(slot + L::oX) + r * 8;
        if (vec) cp_async16(dst, src);
        else {
#pragma unroll
          for (int e = 0; e < 8; ++e) dst[e] = src[e];
        }
      } else if (r < 32) {
        cp_async16(slot + L::oBC + (r - 16) * 16, P.prep_bc + ((btg + tt) * P.groups + g) * 256 + (r - 16) * 8);
      } else if (r < kPcs) {
        cp_async16(slot + L::oPV + (r - 32) * 16, P.prep_pv + ((btg + tt) * P.groups + g) * FP + (r - 32) * 4);
      } else {
        cp_async8(slot + L::oDD + (r - kPcs) * 8, P.prep_ddt + (btg + tt) * P.heads + h0 + (r - kPcs));
      }
    }
  };

  // ---- stage packed rows; x conv taps; zero history ----
  unsigned char* pLo = sPack;
  unsigned char* pHi = pLo + rows * W8;
  unsigned char* pQ4 = pHi + rows * W8;
  unsigned char* pLat = pQ4 + rows * W4;
  uint16_t* pS8 = reinterpret_cast<uint16_t*>(pLat + rows * 2);
  uint16_t* pS4 = pS8 + rows;
  stage16(pLo, P.lo + row0 * W8, rows * W8, tid, 128);
  stage16(pHi, P.hi + row0 * W8, rows * W8, tid, 128);
  stage16(pQ4, P.q4 + row0 * W4, rows * W4, tid, 128);
  stage16(pLat, P.latent + row0 * 2, rows * 2, tid, 128);
  stage16(pS8, P.s8 + row0, rows * 2, tid, 128);
  stage16(pS4, P.s4 + row0, rows * 2, tid, 128);
  if (MODE == 1) {
    const int ch = h0 * dim + tid;
#pragma unroll
    for (int i = 0; i < 4; ++i) sW[tid * 5 + i] = h2f(P.conv_w[ch * 4 + i]);
    sW[tid * 5 + 4] = h2f(P.conv_b[ch]);
#pragma unroll
    for (int k = -3; k < 0; ++k) reinterpret_cast<uint16_t*>(slot_of(k) + L::oX)[tid] = 0;
  }
  prefetch(0);
  cp_async_wait_all();
  __syncthreads();

  // ---- decode own row (:81-114) ----
  float S[NS];
  {
    const float s8 = h2f(pS8[tid]), s4 = h2f(pS4[tid]);
#pragma unroll
    for (int j = 0; j < N8; ++j) {
      int lo = (pLo[tid * W8 + j / 2] >> (4 * (j & 1))) & 15;
      int hi = (pHi[tid * W8 + j / 2] >> (4 * (j & 1))) & 15;
      int ub = (hi << 4) | lo;
      S[j] = (float)(ub - 256 * (ub > 127)) * s8;
    }
#pragma unroll
    for (int j = 0; j < N4; ++j) {
      int nib = (pQ4[tid * W4 + j / 2] >> (4 * (j & 1))) & 15;
      S[N8 + j] = (float)(nib - 16 * (nib > 7)) * s4;
    }
  }
  const float ls0 = h2f(P.latent_scale[g * 2 + 0]), ls1 = h2f(P.latent_scale[g * 2 + 1]);
  const float ils0 = __frcp_rn(ls0), ils1 = __frcp_rn(ls1);
  const float2 ls2 = make_float2(ls0, ls1), nls2 = make_float2(-ls0, -ls1), ils2 = make_float2(ils0, ils1);
  float2 zz = make_float2(e4m3_to_f32(pLat[tid * 2 + 0]) * ls0, e4m3_to_f32(pLat[tid * 2 + 1]) * ls1);
  const float dv = P.d_is_f32 ? reinterpret_cast<const float*>(P.D)[h] : h2f(reinterpret_cast<const uint16_t*>(P.D)[h]);
  float s8 = 0.f, s4 = 0.f;

  for (int c0 = 0; c0 < P.length; c0 += TC) {
    const int nt = min(TC, P.length - c0);
    cp_async_wait_all();
    __syncthreads();                                   // chunk landed; previous tables (or the
                                                       // packed rows read by the decode) free
    // -- publish conv'd x and, per head, {B*dt, C} pairs in tier order --
    {
      float w[5];
      const uint16_t* rx = reinterpret_cast<const uint16_t*>(ring + L::oX) + tid;
      float h1 = 0.f, h2 = 0.f, h3 = 0.f;
      if (MODE == 1) {
#pragma unroll
        for (int i = 0; i < 5; ++i) w[i] = sW[tid * 5 + i];
        h1 = h2f(rx[((c0 - 3) & (R - 1)) * (SB / 2)]);
        h2 = h2f(rx[((c0 - 2) & (R - 1)) * (SB / 2)]);
        h3 = h2f(rx[((c0 - 1) & (R - 1)) * (SB / 2)]);
      }
      const int j = tid;
#pragma unroll
      for (int t = 0; t < TC; ++t) {
        if (t < nt) {
          const unsigned char* slot = slot_of(c0 + t);
          const float raw = h2f(rx[((c0 + t) & (R - 1)) * (SB / 2)]);
          float xv = raw;
          if (MODE == 1) xv = conv_prefill_value(w, h1, h2, h3, raw);
          h1 = h2; h2 = h3; h3 = raw;
          sX[t * 128 + tid] = xv;
          const uint16_t* bc = reinterpret_cast<const uint16_t*>(slot + L::oBC);
          const float2* dd = reinterpret_cast<const float2*>(slot + L::oDD);
          const float bv = h2f(bc[j]);
          const float cv = j < NS ? reinterpret_cast<const float*>(slot + L::oPV)[j] : 0.f;   // C_j + cvec_j
          for (int hh = 0; hh < hpc; ++hh) {
            float* q = sPf + ((t * hpc + hh) * 64 + (j >> 1)) * 4 + (j & 1);
            q[0] = bv * dd[hh].x;
            q[2] = cv;
          }
        }
      }
    }
    __syncthreads();                                   // tables visible; raw x of the chunk consumed
    if (c0 + TC < P.length) prefetch(c0 + TC);

    // -- per-row recurrence, readout and requant (:115-162) for the chunk's tokens --
#pragma unroll 1
    for (int t = 0; t < nt; ++t) {
      const unsigned char* slot = slot_of(c0 + t);
      const float2 ddv = reinterpret_cast<const float2*>(slot + L::oDD)[hl];
      const float dtv = ddv.x, dec = ddv.y;
      const float x = sX[t * 128 + tid];
      const float4* cp = sP4 + (t * hpc + hl) * 64;
      const float* pv = reinterpret_cast<const float*>(slot + L::oPV);
      float m8, m4;
      const float yacc = recur_row_fold<N8, NP, true, false>(S, cp, nullptr, dec, dtv, x, m8, m4);
      float dots[7];
      {
        const float2 d01 = *reinterpret_cast<const float2*>(pv + F), d23 = *reinterpret_cast<const float2*>(pv + F + 2);
        const float2 pz = *reinterpret_cast<const float2*>(pv + NS);
        dots[0] = d01.x; dots[1] = d01.y; dots[2] = d23.x; dots[3] = d23.y; dots[4] = pv[F + 4];
        dots[5] = pz.x; dots[6] = pz.y;
      }
      TokenScales ts;
      const float out = token_tail_fold(yacc, m8, m4, x, dtv, dec, dv, dots, zz, ls2, nls2, ils2, ts);
      P.y[(long long)b * P.y_sb + (long long)(c0 + t) * P.y_st + (long long)h * dim + p] = f2h(out);
      // INT8 / INT4 requant (:155-162, scripts/state_ppl_codec_v6.py:52-61)
      s8 = ts.s8; s4 = ts.s4;
      requant_row<N8, NP>(S, ts);
    }
  }

  // ---- conv cache update (mode 1): raw columns of the newest positions ----
  if (MODE == 1) {
    uint16_t* cache = P.conv_cache + (long long)b * P.conv_cache_sb;
    const int nwrite = min(4, P.length);
    for (int i = 0; i < nwrite; ++i) {
      const int t = P.length - 1 - i;
      const int cs = (P.conv_pos + t) & 3;
      cache[cs * 10240 + h0 * dim + tid] = reinterpret_cast<const uint16_t*>(slot_of(t) + L::oX)[tid];
      if (group_leader) {
        cache[cs * 10240 + 8192 + g * 128 + tid] = P.B[(long long)b * P.b_sb + (long long)t * P.b_st + g * 128 + tid];
        cache[cs * 10240 + 9216 + g * 128 + tid] = P.C[(long long)b * P.c_sb + (long long)t * P.c_st + g * 128 + tid];
      }
    }
  }

  // ---- pack once (:163-181) and store coalesced ----
  __syncthreads();
  {
    const float i8 = s8 > 0.f ? __frcp_rn(s8) : 0.f;
    const float i4 = s4 > 0.f ? __frcp_rn(s4) : 0.f;
#pragma unroll
    for (int j = 0; j < N8; j += 2) {
      const int qa = __float2int_rn(div_exact(S[j], s8, i8));
      const int qb = __float2int_rn(div_exact(S[j + 1], s8, i8));
      pLo[tid * W8 + j / 2] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
      pHi[tid * W8 + j / 2] = (unsigned char)(((qa >> 4) & 15) | (((qb >> 4) & 15) << 4));
    }
#pragma unroll
    for (int j = 0; j < N4; j += 2) {
      const int qa = __float2int_rn(div_exact(S[N8 + j], s4, i4));
      const int qb = __float2int_rn(div_exact(S[N8 + j + 1], s4, i4));
      pQ4[tid * W4 + j / 2] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
    }
    pLat[tid * 2 + 0] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.x, ls0, ils0), -448.f), 448.f));
    pLat[tid * 2 + 1] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.y, ls1, ils1), -448.f), 448.f));
    pS8[tid] = f2h(s8);
    pS4[tid] = f2h(s4);
  }
  __syncthreads();
  auto copy_out = [&](unsigned char* dst, const unsigned char* src, int bytes) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = tid; i < bytes / 16; i += 128) d[i] = s[i];
  };
  copy_out(P.lo + row0 * W8, pLo, rows * W8);
  copy_out(P.hi + row0 * W8, pHi, rows * W8);
  copy_out(P.q4 + row0 * W4, pQ4, rows * W4);
  copy_out(P.latent + row0 * 2, pLat, rows * 2);
  copy_out(reinterpret_cast<unsigned char*>(P.s8 + row0), reinterpret_cast<unsigned char*>(pS8), rows * 2);
  copy_out(reinterpret_cast<unsigned char*>(P.s4 + row0), reinterpret_cast<unsigned char*>(pS4), rows * 2);
}

template <int N8, int N4, int MODE>
int launch_chunked(const ScanParams& P, bool prepare_only, cudaStream_t stream) {
  using PL = PrepLayout<N8, N4>;
  constexpr int prep_smem = kPrepTokens * 256 * 4 + (PL::F * (PL::NZ + 1) * 4 + 15) / 16 * 16 +
                            (2 * PL::NZ * 4 + 15) / 16 * 16 + 128 * 4;
  constexpr int chunk_smem = ChunkSmem<N8, N4>::kBytes;
  auto kp = scan_prep_kernel<N8, N4, MODE>;
  auto kc = ssu_chunk_kernel<N8, N4, MODE>;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kp, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem) != cudaSuccess ||
        cudaFuncSetAttribute(kc, cudaFuncAttributeMaxDynamicSharedMemorySize, chunk_smem) != cudaSuccess ||
        cudaFuncSetAttribute(kc, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return kECuda;
    attr = true;
  }
  if (prepare_only) return kOk;
  dim3 gp((P.length + kPrepTokens - 1) / kPrepTokens, P.groups, P.batch);
  kp<<<gp, 256, prep_smem, stream>>>(P);
  dim3 gc(P.heads / (128 / P.dim), P.batch);
  kc<<<gc, 128, chunk_smem, stream>>>(P);
  return launch_status();
}

// ============================================================================================
// Half-row chunk kernel (modes 0 and 1, dim 64, batch 1 or 2): the chunk kernel's arithmetic
// with two threads per state row and one head per CTA.  A multi-token call at batch 1 gives
// the one-thread-per-row kernel only 64 CTAs (43% of the SMs) for a long sequential walk over
// the tokens; this kernel runs 128 CTAs whose threads carry half a row each (<= 42 stored
// floats in 72 registers), so each token step is about half as long.  At larger batches the
// row kernel is faster (the token tail runs in both halves: 23% more instructions).
//
// Pair split: with N8/2 and N4/2 even for every released layout, thread half h of a row takes
// the global pairs jp = 2i + h (i = 0..NP/2-1).  Both halves then see the same tier boundary
// (local pair i < N8/4 is INT8), so the instruction stream is identical and only the table
// offset differs.  Half 0 accumulates exactly the chunk kernel's even-pair readout chain and
// half 1 its odd-pair chain; one shuffle adds them (IEEE addition is commutative, so both
// halves form the same sum) and the two halves run the token tail redundantly on identical
// inputs.  Results are bit-identical to ssu_chunk_kernel and ssu_sq325_kernel.
//
// Lane mapping: row r = warp * 16 + (lane & 15), half = lane >> 4; the halves of a row are
// lanes l and l ^ 16 of one warp.
// ============================================================================================

template <int N8, int N4>
struct HalfSmem {
  static constexpr int FP = PrepLayout<N8, N4>::FP;
  static constexpr int TC = kChunkTC, R = 2 * kChunkTC;
  // ring slot: raw (mode 1) or conv'd x[64] fp16 | B in tier order [128] fp16 | pv[FP] fp32 | ddt
  static constexpr int oX = 0, oBC = 128, oPV = 384, oDD = 384 + FP * 4;
  static constexpr int kSlot = (oDD + 8 + 15) / 16 * 16;
  static constexpr int oT = R * kSlot;
  // token tables of one chunk: sP4 [TC][64] float4 {B*dt pair, C + cvec pair}, sX [TC][64];
  // before the first / after the last chunk the packed rows (64 x 52 B)
  static constexpr int kTok = TC * 64 * 16 + TC * 64 * 4;
  static constexpr int kT = kTok > 64 * 52 ? kTok : 64 * 52;
  static constexpr int oW = oT + kT;                  // x conv taps + bias [64][5] fp32
  static constexpr int kBytes = oW + 64 * 5 * 4;
};

template <int N8, int N4, int MODE>
__global__ void __launch_bounds__(128, 7)
ssu_half_kernel(const ScanParams P) {
  using L = HalfSmem<N8, N4>;
  constexpr int NS = N8 + N4, F = NS + 2, FP = L::FP;
  constexpr int TC = L::TC, R = L::R, SB = L::kSlot;
  constexpr int W8 = N8 / 2, W4 = N4 / 2;
  constexpr int NP = NS / 2, NPH = NP / 2;          // pairs per row / per half
  constexpr int P8H = N8 / 4;                       // INT8 pairs per half
  static_assert(N8 % 4 == 0 && N4 % 4 == 0, "each half takes the same tier pattern");
  constexpr int dim = 64, rows = 64;

  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* ring = smem;
  float4* sP4 = reinterpret_cast<float4*>(smem + L::oT);                   // [TC][64]
  float* sX = reinterpret_cast<float*>(smem + L::oT + TC * 64 * 16);       // [TC][64]
  float* sW = reinterpret_cast<float*>(smem + L::oW);                      // [64][5]
  unsigned char* sPack = smem + L::oT;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int half = lane >> 4;
  const int r = (tid >> 5) * 16 + (lane & 15);
  const int h = blockIdx.x, b = blockIdx.y;
  const int hpg = P.heads / P.groups;
  const int g = h / hpg;
  const long long row0 = ((long long)b * P.heads + h) * dim;

  auto slot_of = [&](int t) { return ring + (t & (R - 1)) * SB; };
  const uint16_t* xb = P.x + (long long)b * P.x_sb + (long long)h * dim;
  const bool vec = ((((uintptr_t)xb) & 15) == 0) && (P.x_st & 7) == 0;
  const long long btg = (long long)b * P.length;
  constexpr int kPcs = 8 + 16 + FP / 4;             // 16-byte pieces per token (x, B half of bc, pv)

  auto prefetch = [&](int c0) {
    const int nt = min(TC, P.length - c0);
    for (int i = tid; i < nt * (kPcs + 1); i += 128) {
      const int t = i / (kPcs + 1), q = i - t * (kPcs + 1);
      const long long tt = c0 + t;
      unsigned char* slot = slot_of(c0 + t);
      if (q < 8) {
        const uint16_t* src = xb + tt * P.x_st + q * 8;
        uint16_t* dst = reinterpret_cast<uint16_t*>(slot + L::oX) + q * 8;
        if (vec) cp_async16(dst, src);
        else {
#pragma unroll
          for (int e = 0; e < 8; ++e) dst[e] = src[e];
        }
      } else if (q < 24) {
        cp_async16(slot + L::oBC + (q - 8) * 16, P.prep_bc + ((btg + tt) * P.groups + g) * 256 + (q - 8) * 8);
      } else if (q < kPcs) {
        cp_async16(slot + L::oPV + (q - 24) * 16, P.prep_pv + ((btg + tt) * P.groups + g) * FP + (q - 24) * 4);
      } else {
        cp_async8(slot + L::oDD, P.prep_ddt + (btg + tt) * P.heads + h);
      }
    }
  };

  // ---- stage packed rows; x conv taps; zero history ----
  unsigned char* pLo = sPack;
  unsigned char* pHi = pLo + rows * W8;
  unsigned char* pQ4 = pHi + rows * W8;
  unsigned char* pLat = pQ4 + rows * W4;
  uint16_t* pS8 = reinterpret_cast<uint16_t*>(pLat + rows * 2);
  uint16_t* pS4 = pS8 + rows;
  stage16(pLo, P.lo + row0 * W8, rows * W8, tid, 128);
  stage16(pHi, P.hi + row0 * W8, rows * W8, tid, 128);
  stage16(pQ4, P.q4 + row0 * W4, rows * W4, tid, 128);
  stage16(pLat, P.latent + row0 * 2, rows * 2, tid, 128);
  stage16(pS8, P.s8 + row0, rows * 2, tid, 128);
  stage16(pS4, P.s4 + row0, rows * 2, tid, 128);
  if (MODE == 1 && tid < dim) {
    const int ch = h * dim + tid;
#pragma unroll
    for (int i = 0; i < 4; ++i) sW[tid * 5 + i] = h2f(P.conv_w[ch * 4 + i]);
    sW[tid * 5 + 4] = h2f(P.conv_b[ch]);
#pragma unroll
    for (int k = -3; k < 0; ++k) reinterpret_cast<uint16_t*>(slot_of(k) + L::oX)[tid] = 0;
  }
  prefetch(0);
  cp_async_wait_all();
  __syncthreads();

  // ---- decode this half of the row (:81-114): local pair i = global pair 2i + half ----
  float S[2 * NPH];
  {
    const float s8 = h2f(pS8[r]), s4 = h2f(pS4[r]);
#pragma unroll
    for (int i = 0; i < P8H; ++i) {
      const int jp = 2 * i + half;
      const int lo = pLo[r * W8 + jp], hi = pHi[r * W8 + jp];
      const int ua = ((hi & 15) << 4) | (lo & 15), ub = (hi & 0xF0) | (lo >> 4);
      S[2 * i] = (float)(ua - 256 * (ua > 127)) * s8;
      S[2 * i + 1] = (float)(ub - 256 * (ub > 127)) * s8;
    }
#pragma unroll
    for (int i = P8H; i < NPH; ++i) {
      const int q = pQ4[r * W4 + 2 * (i - P8H) + half];
      const int na = q & 15, nb = q >> 4;
      S[2 * i] = (float)(na - 16 * (na > 7)) * s4;
      S[2 * i + 1] = (float)(nb - 16 * (nb > 7)) * s4;
    }
  }
  const float ls0 = h2f(P.latent_scale[g * 2 + 0]), ls1 = h2f(P.latent_scale[g * 2 + 1]);
  const float ils0 = __frcp_rn(ls0), ils1 = __frcp_rn(ls1);
  const float2 ls2 = make_float2(ls0, ls1), nls2 = make_float2(-ls0, -ls1), ils2 = make_float2(ils0, ils1);
  float2 zz = make_float2(e4m3_to_f32(pLat[r * 2 + 0]) * ls0, e4m3_to_f32(pLat[r * 2 + 1]) * ls1);
  const float dv = P.d_is_f32 ? reinterpret_cast<const float*>(P.D)[h] : h2f(reinterpret_cast<const uint16_t*>(P.D)[h]);
  float s8 = 0.f, s4 = 0.f;
  uint16_t* yrow = P.y + (long long)b * P.y_sb + (long long)h * dim + r;

  for (int c0 = 0; c0 < P.length; c0 += TC) {
    const int nt = min(TC, P.length - c0);
    cp_async_wait_all();
    __syncthreads();                                   // chunk landed; previous tables (or the
                                                       // packed rows read by the decode) free
    // -- conv'd x: channel c = tid % 64, tokens of parity tid / 64 (each token's conv reads
    //    only raw ring values, so the tokens are independent) --
    {
      const int c = tid & 63;
      const uint16_t* rx = reinterpret_cast<const uint16_t*>(ring + L::oX) + c;
      float w[5];
      if (MODE == 1) {
#pragma unroll
        for (int i = 0; i < 5; ++i) w[i] = sW[c * 5 + i];
      }
      for (int t = tid >> 6; t < nt; t += 2) {
        const int tt = c0 + t;
        const float raw = h2f(rx[(tt & (R - 1)) * (SB / 2)]);
        float xv = raw;
        if (MODE == 1)
          xv = conv_prefill_value(w, h2f(rx[((tt - 3) & (R - 1)) * (SB / 2)]), h2f(rx[((tt - 2) & (R - 1)) * (SB / 2)]),
                                  h2f(rx[((tt - 1) & (R - 1)) * (SB / 2)]), raw);
        sX[t * 64 + c] = xv;
      }
    }
    // -- per token and pair: {B*dt pair, C + cvec pair} (one 16-byte store per pair) --
    for (int e = tid; e < nt * 64; e += 128) {
      const int t = e >> 6, jp = e & 63;
      const unsigned char* slot = slot_of(c0 + t);
      const float dtv = reinterpret_cast<const float2*>(slot + L::oDD)->x;
      const __half2 bb = reinterpret_cast<const __half2*>(slot + L::oBC)[jp];
      const float2 bf = __half22float2(bb);
      float2 cc = make_float2(0.f, 0.f);
      if (2 * jp < NS) cc = reinterpret_cast<const float2*>(slot + L::oPV)[jp];      // C_j + cvec_j
      sP4[t * 64 + jp] = make_float4(bf.x * dtv, bf.y * dtv, cc.x, cc.y);
    }
    __syncthreads();                                   // tables visible; raw x of the chunk consumed
    if (c0 + TC < P.length) prefetch(c0 + TC);

    // -- per half-row recurrence, readout and requant (:115-162) for the chunk's tokens --
#pragma unroll 1
    for (int t = 0; t < nt; ++t) {
      const unsigned char* slot = slot_of(c0 + t);
      const float2 ddv = *reinterpret_cast<const float2*>(slot + L::oDD);
      const float dtv = ddv.x, dec = ddv.y;
      const float x = sX[t * 64 + r];
      const float4* cp = sP4 + t * 64 + half;
      const float* pv = reinterpret_cast<const float*>(slot + L::oPV);
      float m8a = 0.f, m8b = 0.f, m4a = 0.f, m4b = 0.f;
      float2 ya = make_float2(0.f, 0.f);
      {
        const float2 dd = make_float2(dec, dec), xx = make_float2(x, x);
#pragma unroll
        for (int i = 0; i < NPH; ++i) {
          const float4 bc = cp[2 * i];
          const float2 pr = make_float2(S[2 * i], S[2 * i + 1]);
          const float2 sn = __ffma2_rn(pr, dd, __fmul2_rn(make_float2(bc.x, bc.y), xx));   // prior*decay + (B*dt)*x
          S[2 * i] = sn.x; S[2 * i + 1] = sn.y;
          ya = __ffma2_rn(pr, make_float2(bc.z, bc.w), ya);
          if (i < P8H) { m8a = fmaxf(m8a, fabsf(sn.x)); m8b = fmaxf(m8b, fabsf(sn.y)); }
          else         { m4a = fmaxf(m4a, fabsf(sn.x)); m4b = fmaxf(m4b, fabsf(sn.y)); }
        }
      }
      const float part = ya.x + ya.y;
      const float yacc = part + __shfl_xor_sync(0xffffffffu, part, 16);
      float m8 = fmaxf(m8a, m8b), m4 = fmaxf(m4a, m4b);
      m8 = fmaxf(m8, __shfl_xor_sync(0xffffffffu, m8, 16));
      m4 = fmaxf(m4, __shfl_xor_sync(0xffffffffu, m4, 16));
      float dots[7];
      {
        const float2 d01 = *reinterpret_cast<const float2*>(pv + F), d23 = *reinterpret_cast<const float2*>(pv + F + 2);
        const float2 pz = *reinterpret_cast<const float2*>(pv + NS);
        dots[0] = d01.x; dots[1] = d01.y; dots[2] = d23.x; dots[3] = d23.y; dots[4] = pv[F + 4];
        dots[5] = pz.x; dots[6] = pz.y;
      }
      TokenScales ts;
      const float out = token_tail_fold(yacc, m8, m4, x, dtv, dec, dv, dots, zz, ls2, nls2, ils2, ts);
      if (half == 0) yrow[(long long)(c0 + t) * P.y_st] = f2h(out);
      s8 = ts.s8; s4 = ts.s4;
      requant_row<2 * P8H, NPH>(S, ts);
    }
  }

  // ---- conv cache update (mode 1): raw columns of the newest positions ----
  if (MODE == 1) {
    uint16_t* cache = P.conv_cache + (long long)b * P.conv_cache_sb;
    const int nwrite = min(4, P.length);
    for (int i = 0; i < nwrite; ++i) {
      const int t = P.length - 1 - i;
      const int cs = (P.conv_pos + t) & 3;
      if (tid < dim) cache[cs * 10240 + h * dim + tid] = reinterpret_cast<const uint16_t*>(slot_of(t) + L::oX)[tid];
      if ((h % hpg) == 0) {
        cache[cs * 10240 + 8192 + g * 128 + tid] = P.B[(long long)b * P.b_sb + (long long)t * P.b_st + g * 128 + tid];
        cache[cs * 10240 + 9216 + g * 128 + tid] = P.C[(long long)b * P.c_sb + (long long)t * P.c_st + g * 128 + tid];
      }
    }
  }

  // ---- pack once (:163-181) and store coalesced ----
  __syncthreads();
  {
    const float i8 = s8 > 0.f ? __frcp_rn(s8) : 0.f;
    const float i4 = s4 > 0.f ? __frcp_rn(s4) : 0.f;
#pragma unroll
    for (int i = 0; i < P8H; ++i) {
      const int jp = 2 * i + half;
      const int qa = __float2int_rn(div_exact(S[2 * i], s8, i8));
      const int qb = __float2int_rn(div_exact(S[2 * i + 1], s8, i8));
      pLo[r * W8 + jp] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
      pHi[r * W8 + jp] = (unsigned char)(((qa >> 4) & 15) | (((qb >> 4) & 15) << 4));
    }
#pragma unroll
    for (int i = P8H; i < NPH; ++i) {
      const int qa = __float2int_rn(div_exact(S[2 * i], s4, i4));
      const int qb = __float2int_rn(div_exact(S[2 * i + 1], s4, i4));
      pQ4[r * W4 + 2 * (i - P8H) + half] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
    }
    if (half == 0) {
      pLat[r * 2 + 0] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.x, ls0, ils0), -448.f), 448.f));
      pLat[r * 2 + 1] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.y, ls1, ils1), -448.f), 448.f));
      pS8[r] = f2h(s8);
      pS4[r] = f2h(s4);
    }
  }
  __syncthreads();
  auto copy_out = [&](unsigned char* dst, const unsigned char* src, int bytes) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = tid; i < bytes / 16; i += 128) d[i] = s[i];
  };
  copy_out(P.lo + row0 * W8, pLo, rows * W8);
  copy_out(P.hi + row0 * W8, pHi, rows * W8);
  copy_out(P.q4 + row0 * W4, pQ4, rows * W4);
  copy_out(P.latent + row0 * 2, pLat, rows * 2);
  copy_out(reinterpret_cast<unsigned char*>(P.s8 + row0), reinterpret_cast<unsigned char*>(pS8), rows * 2);
  copy_out(reinterpret_cast<unsigned char*>(P.s4 + row0), reinterpret_cast<unsigned char*>(pS4), rows * 2);
}

template <int N8, int N4, int MODE>
int launch_half(const ScanParams& P, bool prepare_only, cudaStream_t stream) {
  using PL = PrepLayout<N8, N4>;
  constexpr int prep_smem = kPrepTokens * 256 * 4 + (PL::F * (PL::NZ + 1) * 4 + 15) / 16 * 16 +
                            (2 * PL::NZ * 4 + 15) / 16 * 16 + 128 * 4;
  constexpr int half_smem = HalfSmem<N8, N4>::kBytes;
  auto kp = scan_prep_kernel<N8, N4, MODE>;
  auto kc = ssu_half_kernel<N8, N4, MODE>;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kp, cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem) != cudaSuccess ||
        cudaFuncSetAttribute(kc, cudaFuncAttributeMaxDynamicSharedMemorySize, half_smem) != cudaSuccess ||
        cudaFuncSetAttribute(kc, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return kECuda;
    attr = true;
  }
  if (prepare_only) return kOk;
  dim3 gp((P.length + kPrepTokens - 1) / kPrepTokens, P.groups, P.batch);
  kp<<<gp, 256, prep_smem, stream>>>(P);
  dim3 gc(P.heads, P.batch);
  kc<<<gc, 128, half_smem, stream>>>(P);
  return launch_status();
}

// ============================================================================================
// Two-kernel path of the one-token decode step (mode 2: conv step numerics, conv ring).
//
// The single fused kernel redoes, in each of the eight CTAs of a B/C group, the staging of the
// group's predictor (F x NZ fp16), basis and conv taps and the F + 5 group dots; at batch 32-64
// that fixed cost dominates the step.  step_prep_kernel does it once per (batch, group):
//   bc   [B][G][256] fp16   conv'd B then conv'd C, tier order (conv step values are fp16)
//   pv   [B][G][FP]  fp32   cvec [0..NS) | pcz0 pcz1 | B.C (zero tier), b0.C, b1.C, b0.B, b1.B
//   ddt  [B][H]      float2 (dt after softplus, exp(A dt))
// and writes the new raw B/C columns into the ring; ssu_step_kernel then runs the rows of two
// heads (one thread per row) from those arrays, the conv'd x of its 128 channels, and writes
// the x columns into the ring.  Every value is computed by the same functions in the same
// order as the fused kernel's mode 2 (recur_row4 / token_tail_sums), so y, the state bytes and
// the ring are bit-identical to it, and to the persistent decode kernel.
// ============================================================================================

template <int N8, int N4>
__global__ void __launch_bounds__(256)
step_prep_kernel(const ScanParams P) {
  using PL = PrepLayout<N8, N4>;
  constexpr int NS = PL::NS, NZ = PL::NZ, F = PL::F, FP = PL::FP;
  constexpr int oPred = 256 * 4;                                     // sBC [256] fp32 first
  constexpr int oBasis = oPred + (F * (NZ + 1) * 4 + 15) / 16 * 16;
  constexpr int oPerm = oBasis + (2 * NZ * 4 + 15) / 16 * 16;
  extern __shared__ __align__(16) unsigned char smem[];
  float* sBC = reinterpret_cast<float*>(smem);                       // [256] conv'd B | C (tier order)
  float* sPred = reinterpret_cast<float*>(smem + oPred);             // [F][NZ+1]
  float* sBasis = reinterpret_cast<float*>(smem + oBasis);           // [2][NZ]
  int* sPerm = reinterpret_cast<int*>(smem + oPerm);                 // [128]
  uint16_t* rawPred = reinterpret_cast<uint16_t*>(smem + oPerm + 512);
  uint16_t* rawBasis = rawPred + (F * NZ * 2 + 15) / 16 * 8;
  uint8_t* rawPerm = reinterpret_cast<uint8_t*>(rawBasis + (NZ * 4 + 15) / 16 * 8);

  const int tid = threadIdx.x;
  const int g = blockIdx.x, b = blockIdx.y;
  stage16(rawPred, P.predictor + (long long)g * F * NZ, F * NZ * 2, tid, 256);
  stage16(rawBasis, P.basis + (long long)g * NZ * 2, NZ * 4, tid, 256);
  stage16(rawPerm, P.perm + g * 128, 128, tid, 256);
  cp_async_wait_all();
  __syncthreads();
  for (int i = tid; i < F * NZ; i += 256) {
    const int f = i / NZ, d = i - f * NZ;
    sPred[f * (NZ + 1) + d] = h2f(rawPred[i]);
  }
  for (int i = tid; i < NZ; i += 256) {
    sBasis[i] = h2f(rawBasis[2 * i + 0]);
    sBasis[NZ + i] = h2f(rawBasis[2 * i + 1]);
  }
  if (tid < 128) sPerm[tid] = rawPerm[tid];
  __syncthreads();

  // ---- conv step of B (tid < 128) or C (tid >= 128) at tier coordinate j ----
  {
    const int j = tid & 127;
    const bool isC = tid >= 128;
    const int n = sPerm[j];
    const int ch = (isC ? 9216 : 8192) + g * 128 + n;
    float w[5];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = h2f(P.conv_w[ch * 4 + i]);
    w[4] = h2f(P.conv_b[ch]);
    uint16_t* ring = P.conv_cache + (long long)b * P.conv_cache_sb;
    const float h1 = h2f(ring[((P.conv_pos - 3) & 3) * 10240 + ch]);
    const float h2 = h2f(ring[((P.conv_pos - 2) & 3) * 10240 + ch]);
    const float h3 = h2f(ring[((P.conv_pos - 1) & 3) * 10240 + ch]);
    const uint16_t rawb = (isC ? P.C + (long long)b * P.c_sb : P.B + (long long)b * P.b_sb)[g * 128 + n];
    const float v = conv_step_value(w, h1, h2, h3, h2f(rawb));
    sBC[tid] = v;
    P.prep_bc[((long long)b * P.groups + g) * 256 + tid] = f2h(v);   // v is an fp16 value: exact
    ring[(P.conv_pos & 3) * 10240 + ch] = rawb;                      // the newest raw column
  }
  // ---- dt / decay for the group's heads ----
  {
    const int hpg = P.heads / P.groups;
    for (int i = tid; i < hpg; i += 256) {
      const int h = g * hpg + i;
      const float bias = P.dt_bias_is_f32 ? reinterpret_cast<const float*>(P.dt_bias)[h]
                                          : h2f(reinterpret_cast<const uint16_t*>(P.dt_bias)[h]);
      const float dtv = softplus_ref(h2f(P.dt[(long long)b * P.dt_sb + h]) + bias);
      P.prep_ddt[(long long)b * P.heads + h] = make_float2(dtv, expf(P.A[h] * dtv));
    }
  }
  __syncthreads();
  // ---- group dots, the fused kernel's pairing and order ----
  float* pv = P.prep_pv + ((long long)b * P.groups + g) * FP;
  for (int f = tid; f < FP; f += 256) {
    float r = 0.f;
    if (f < F) {
      const float* pr = sPred + f * (NZ + 1);
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 4
      for (int d = 0; d < NZ; d += 2) {
        acc0 = fmaf(sBC[128 + NS + d], pr[d], acc0);
        acc1 = fmaf(sBC[128 + NS + d + 1], pr[d + 1], acc1);
      }
      r = acc0 + acc1;                                  // cvec (f < NS) or pcz (f = NS, NS + 1)
    } else if (f < F + 5) {
      const int k = f - F;   // 0: B.C (zero tier), 1: basis0.C, 2: basis1.C, 3: basis0.B, 4: basis1.B
      const float* us = (k == 0) ? nullptr : sBasis + ((k - 1) & 1) * NZ;
      const int voff = (k >= 3 || k == 0) ? 0 : 128;   // 0 -> B, 128 -> C
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 4
      for (int d = 0; d < NZ; d += 2) {
        const float u0 = (k == 0) ? sBC[NS + d] : us[d], u1 = (k == 0) ? sBC[NS + d + 1] : us[d + 1];
        const float v0 = (k == 0) ? sBC[128 + NS + d] : sBC[voff + NS + d];
        const float v1 = (k == 0) ? sBC[128 + NS + d + 1] : sBC[voff + NS + d + 1];
        acc0 = fmaf(u0, v0, acc0);
        acc1 = fmaf(u1, v1, acc1);
      }
      r = acc0 + acc1;
    }
    pv[f] = r;
  }
}

// Rows of the one-token step: one thread per state row, 128-thread CTAs of `hpc` heads.
template <int N8, int N4>
__global__ void __launch_bounds__(128, 4)
ssu_step_kernel(const ScanParams P) {
  using PL = PrepLayout<N8, N4>;
  constexpr int NS = N8 + N4, F = NS + 2, FP = PL::FP;
  constexpr int W8 = N8 / 2, W4 = N4 / 2, NP = NS / 2;
  constexpr int rows = 128;
  __shared__ __align__(16) unsigned char sPack[rows * 52];
  __shared__ __align__(16) float4 sP4[64];          // {b_j, b_j+1, c_j, c_j+1} per pair
  __shared__ __align__(16) float2 sV2[64];          // cvec pairs
  __shared__ float sDots[8];
  __shared__ float2 sDD[8];

  const int tid = threadIdx.x;
  const int dim = P.dim;
  const int hpc = 128 / dim;
  const int b = blockIdx.y;
  const int h0 = blockIdx.x * hpc;
  const int hl = tid / dim;
  const int p = tid - hl * dim;
  const int h = h0 + hl;
  const int hpg = P.heads / P.groups;
  const int g = h0 / hpg;
  const long long row0 = ((long long)b * P.heads + h0) * dim;

  unsigned char* pLo = sPack;
  unsigned char* pHi = pLo + rows * W8;
  unsigned char* pQ4 = pHi + rows * W8;
  unsigned char* pLat = pQ4 + rows * W4;
  uint16_t* pS8 = reinterpret_cast<uint16_t*>(pLat + rows * 2);
  uint16_t* pS4 = pS8 + rows;
  stage16(pLo, P.lo + row0 * W8, rows * W8, tid, 128);
  stage16(pHi, P.hi + row0 * W8, rows * W8, tid, 128);
  stage16(pQ4, P.q4 + row0 * W4, rows * W4, tid, 128);
  stage16(pLat, P.latent + row0 * 2, rows * 2, tid, 128);
  stage16(pS8, P.s8 + row0, rows * 2, tid, 128);
  stage16(pS4, P.s4 + row0, rows * 2, tid, 128);
  // the group's tables from the prep kernel
  {
    const uint16_t* bc = P.prep_bc + ((long long)b * P.groups + g) * 256;
    const float* pvg = P.prep_pv + ((long long)b * P.groups + g) * FP;
    if (tid < 64) {
      const __half2 bb = reinterpret_cast<const __half2*>(bc)[tid];
      const __half2 cc = reinterpret_cast<const __half2*>(bc + 128)[tid];
      const float2 bf = __half22float2(bb), cf = __half22float2(cc);
      sP4[tid] = make_float4(bf.x, bf.y, cf.x, cf.y);
      if (2 * tid < NS) sV2[tid] = make_float2(pvg[2 * tid], pvg[2 * tid + 1]);
    } else if (tid < 64 + 7) {
      const int k = tid - 64;                          // dots {B.C, b0.C, b1.C, b0.B, b1.B, pcz0, pcz1}
      sDots[k] = k < 5 ? pvg[F + k] : pvg[NS + k - 5];
    } else if (tid < 64 + 7 + hpc) {
      sDD[tid - 71] = P.prep_ddt[(long long)b * P.heads + h0 + tid - 71];
    }
  }
  // conv step of this thread's x channel (channel h0 * dim + tid); the newest raw column
  // goes into the ring
  float xv;
  {
    const int ch = h0 * dim + tid;
    float w[5];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = h2f(P.conv_w[ch * 4 + i]);
    w[4] = h2f(P.conv_b[ch]);
    uint16_t* ring = P.conv_cache + (long long)b * P.conv_cache_sb;
    const float h1 = h2f(ring[((P.conv_pos - 3) & 3) * 10240 + ch]);
    const float h2 = h2f(ring[((P.conv_pos - 2) & 3) * 10240 + ch]);
    const float h3 = h2f(ring[((P.conv_pos - 1) & 3) * 10240 + ch]);
    const uint16_t raw = P.x[(long long)b * P.x_sb + ch];
    xv = conv_step_value(w, h1, h2, h3, h2f(raw));
    ring[(P.conv_pos & 3) * 10240 + ch] = raw;
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- decode own row (:81-114) ----
  float S[NS];
  {
    const float s8 = h2f(pS8[tid]), s4 = h2f(pS4[tid]);
#pragma unroll
    for (int j = 0; j < N8; ++j) {
      int lo = (pLo[tid * W8 + j / 2] >> (4 * (j & 1))) & 15;
      int hi = (pHi[tid * W8 + j / 2] >> (4 * (j & 1))) & 15;
      int ub = (hi << 4) | lo;
      S[j] = (float)(ub - 256 * (ub > 127)) * s8;
    }
#pragma unroll
    for (int j = 0; j < N4; ++j) {
      int nib = (pQ4[tid * W4 + j / 2] >> (4 * (j & 1))) & 15;
      S[N8 + j] = (float)(nib - 16 * (nib > 7)) * s4;
    }
  }
  const float ls0 = h2f(P.latent_scale[g * 2 + 0]), ls1 = h2f(P.latent_scale[g * 2 + 1]);
  const float ils0 = __frcp_rn(ls0), ils1 = __frcp_rn(ls1);
  const float2 ls2 = make_float2(ls0, ls1), nls2 = make_float2(-ls0, -ls1), ils2 = make_float2(ils0, ils1);
  float2 zz = make_float2(e4m3_to_f32(pLat[tid * 2 + 0]) * ls0, e4m3_to_f32(pLat[tid * 2 + 1]) * ls1);
  const float dv = P.d_is_f32 ? reinterpret_cast<const float*>(P.D)[h] : h2f(reinterpret_cast<const uint16_t*>(P.D)[h]);

  // ---- one token: recurrence, four-stream readout, latent and INT requant (:115-162) ----
  float s8, s4;
  {
    const float dtv = sDD[hl].x, dec = sDD[hl].y;
    float dots[7];
#pragma unroll
    for (int i = 0; i < 7; ++i) dots[i] = sDots[i];
    float ysum, ycorr, m8, m4;
    recur_row4<N8, NP>(S, sP4, sV2, dec, dtv, xv, ysum, ycorr, m8, m4);
    TokenScales ts;
    const float out = token_tail_sums(ysum, ycorr, m8, m4, xv, dtv, dec, dv, dots, zz, ls2, nls2, ils2, ts);
    P.y[(long long)b * P.y_sb + (long long)h * dim + p] = f2h(out);
    s8 = ts.s8; s4 = ts.s4;
    requant_row<N8, NP>(S, ts);
  }

  // ---- pack (:163-181) and store coalesced ----
  __syncthreads();
  {
    const float i8 = s8 > 0.f ? __frcp_rn(s8) : 0.f;
    const float i4 = s4 > 0.f ? __frcp_rn(s4) : 0.f;
#pragma unroll
    for (int j = 0; j < N8; j += 2) {
      const int qa = __float2int_rn(div_exact(S[j], s8, i8));
      const int qb = __float2int_rn(div_exact(S[j + 1], s8, i8));
      pLo[tid * W8 + j / 2] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
      pHi[tid * W8 + j / 2] = (unsigned char)(((qa >> 4) & 15) | (((qb >> 4) & 15) << 4));
    }
#pragma unroll
    for (int j = 0; j < N4; j += 2) {
      const int qa = __float2int_rn(div_exact(S[N8 + j], s4, i4));
      const int qb = __float2int_rn(div_exact(S[N8 + j + 1], s4, i4));
      pQ4[tid * W4 + j / 2] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
    }
    pLat[tid * 2 + 0] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.x, ls0, ils0), -448.f), 448.f));
    pLat[tid * 2 + 1] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.y, ls1, ils1), -448.f), 448.f));
    pS8[tid] = f2h(s8);
    pS4[tid] = f2h(s4);
  }
  __syncthreads();
  auto copy_out = [&](unsigned char* dst, const unsigned char* src, int bytes) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = tid; i < bytes / 16; i += 128) d[i] = s[i];
  };
  copy_out(P.lo + row0 * W8, pLo, rows * W8);
  copy_out(P.hi + row0 * W8, pHi, rows * W8);
  copy_out(P.q4 + row0 * W4, pQ4, rows * W4);
  copy_out(P.latent + row0 * 2, pLat, rows * 2);
  copy_out(reinterpret_cast<unsigned char*>(P.s8 + row0), reinterpret_cast<unsigned char*>(pS8), rows * 2);
  copy_out(reinterpret_cast<unsigned char*>(P.s4 + row0), reinterpret_cast<unsigned char*>(pS4), rows * 2);
}

template <int N8, int N4>
int launch_step2(const ScanParams& P, bool prepare_only, cudaStream_t stream) {
  using PL = PrepLayout<N8, N4>;
  constexpr int smem = 256 * 4 + (PL::F * (PL::NZ + 1) * 4 + 15) / 16 * 16 + (2 * PL::NZ * 4 + 15) / 16 * 16 + 512 +
                       (PL::F * PL::NZ * 2 + 15) / 16 * 16 + (PL::NZ * 4 + 15) / 16 * 16 + 128;
  auto kp = step_prep_kernel<N8, N4>;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kp, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return kECuda;
    attr = true;
  }
  if (prepare_only) return kOk;
  kp<<<dim3(P.groups, P.batch), 256, smem, stream>>>(P);
  ssu_step_kernel<N8, N4><<<dim3(P.heads / (128 / P.dim), P.batch), 128, 0, stream>>>(P);
  return launch_status();
}

template <int N8, int N4, int KJ, int MODE, int TC = (MODE == 2 ? 1 : kTC)>
int launch_kj(const ScanParams& P, int hpc, cudaStream_t stream) {
  const size_t smem = ScanSmem<N8, N4, TC>::kBytes;
  auto kern = ssu_sq325_kernel<N8, N4, KJ, MODE, TC>;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return kECuda;
    attr = true;
  }
  if (hpc == 0) return kOk;                         // prepare-only call (attributes set, no launch)
  dim3 grid(P.heads / hpc, P.batch);
  kern<<<grid, hpc * P.dim, smem, stream>>>(P);
  return launch_status();
}

template <int N8, int N4>
int launch_t(const ScanParams& P, int hpc, cudaStream_t stream) {
  const int bd = hpc * P.dim;
  if (P.conv_mode != 2 && P.prep_bc && P.prep_pv && P.prep_ddt && P.dim == 64 && P.batch <= 2)
    return P.conv_mode == 1 ? launch_half<N8, N4, 1>(P, false, stream) : launch_half<N8, N4, 0>(P, false, stream);
  if (P.conv_mode != 2 && P.prep_bc && P.prep_pv && P.prep_ddt && bd == 128 && hpc <= 2)
    return P.conv_mode == 1 ? launch_chunked<N8, N4, 1>(P, false, stream) : launch_chunked<N8, N4, 0>(P, false, stream);
  if (P.conv_mode == 1) return bd == 128 ? launch_kj<N8, N4, 1, 1>(P, hpc, stream) : kEInval;
  if (P.conv_mode == 2 && P.prep_bc && P.prep_pv && P.prep_ddt && bd == 128 && hpc <= 2)
    return launch_step2<N8, N4>(P, false, stream);
  if (P.conv_mode == 2) return bd == 128 ? launch_kj<N8, N4, 1, 2>(P, hpc, stream) : kEInval;
  if (bd >= 128) return launch_kj<N8, N4, 1, 0>(P, hpc, stream);
  if (bd >= 64) return launch_kj<N8, N4, 2, 0>(P, hpc, stream);
  return launch_kj<N8, N4, 4, 0>(P, hpc, stream);
}

}  // namespace

template <int N8, int N4>
int prepare_t() {
  ScanParams P{};
  int st = kOk;
  st |= launch_kj<N8, N4, 1, 0>(P, 0, 0);
  st |= launch_kj<N8, N4, 2, 0>(P, 0, 0);
  st |= launch_kj<N8, N4, 4, 0>(P, 0, 0);
  st |= launch_kj<N8, N4, 1, 1>(P, 0, 0);
  st |= launch_kj<N8, N4, 1, 2>(P, 0, 0);
  st |= launch_chunked<N8, N4, 0>(P, true, 0);
  st |= launch_chunked<N8, N4, 1>(P, true, 0);
  st |= launch_step2<N8, N4>(P, true, 0);
  st |= launch_half<N8, N4, 0>(P, true, 0);
  st |= launch_half<N8, N4, 1>(P, true, 0);
  return st;
}

// Sets the shared-memory attributes of every scan instantiation up front (a graph capture
// must not be the first launch of a kernel that needs an attribute change).
int prepare_scan_kernels() {
  int st = prepare_t<32, 28>() | prepare_t<16, 60>() | prepare_t<8, 76>() | prepare_t<24, 44>() |
           prepare_t<36, 20>() | prepare_t<40, 12>() | prepare_t<44, 4>();
  return st ? kECuda : kOk;
}

namespace {
int prep_fp(int layout) {
  const int f = kLayouts[layout].n8 + kLayouts[layout].n4 + 2;
  return (f + 5 + 3) / 4 * 4;
}
long long round256(long long v) { return (v + 255) / 256 * 256; }
}  // namespace

long long scan_prep_bytes(int batch, int length, int heads, int groups, int layout) {
  if (layout < 0 || layout > 6 || batch <= 0 || length <= 0 || heads <= 0 || groups <= 0) return -1;
  const long long bt = (long long)batch * length;
  return round256(bt * groups * 512) + round256(bt * groups * prep_fp(layout) * 4) + round256(bt * heads * 8);
}

long long scan_prep_bytes_any_layout(int batch, int length, int heads, int groups) {
  long long m = 0;
  for (int l = 0; l < 7; ++l) m = std::max(m, scan_prep_bytes(batch, length, heads, groups, l));
  return m;
}

void scan_prep_bind(ScanParams& P, void* ws) {
  unsigned char* w = static_cast<unsigned char*>(ws);
  const long long bt = (long long)P.batch * P.length;
  P.prep_bc = reinterpret_cast<uint16_t*>(w);
  w += round256(bt * P.groups * 512);
  P.prep_pv = reinterpret_cast<float*>(w);
  w += round256(bt * P.groups * prep_fp(P.layout) * 4);
  P.prep_ddt = reinterpret_cast<float2*>(w);
}

int launch_scan(const ScanParams& P, cudaStream_t stream) {
  if (P.layout < 0 || P.layout > 6) return kEInval;
  if (P.batch <= 0 || P.length <= 0 || P.heads <= 0 || P.groups <= 0 || P.heads % P.groups) return kEInval;
  if (P.dim <= 0 || P.dim % 16 || P.dim > 128) return kEInval;
  if (P.conv_mode < 0 || P.conv_mode > 2) return kEInval;
  if (P.conv_mode != 0 && (!P.conv_w || !P.conv_b || !P.conv_cache || P.heads * P.dim + 2 * P.groups * 128 != 10240))
    return kEInval;
  if (P.conv_mode == 1 && P.conv_pos != 0) return kEInval;     // fused prefill only from a reset state
  if (P.conv_mode == 2 && (P.length != 1 || P.conv_pos <= 0)) return kEInval;
  if (P.conv_mode != 0 && ((((uintptr_t)P.conv_cache) & 15) || (P.conv_cache_sb & 7))) return kEInval;
  const int hpg = P.heads / P.groups;
  int hpc = 1;
  for (int c = 1; c <= hpg && c <= kMaxHpc; ++c)
    if (hpg % c == 0 && c * P.dim <= 128) hpc = c;
  if (hpc * P.dim < 32) return kEInval;
  switch (P.layout) {
    case 0: return launch_t<32, 28>(P, hpc, stream);
    case 1: return launch_t<16, 60>(P, hpc, stream);
    case 2: return launch_t<8, 76>(P, hpc, stream);
    case 3: return launch_t<24, 44>(P, hpc, stream);
    case 4: return launch_t<36, 20>(P, hpc, stream);
    case 5: return launch_t<40, 12>(P, hpc, stream);
    case 6: return launch_t<44, 4>(P, hpc, stream);
  }
  return kEInval;
}

}  // namespace sq
