// Per-row arithmetic of the SQ3.25 codec step, shared by the scan kernels (scan.cu) and
// the persistent decode kernel (decode.cu) so that every path computes the same bits.
// Semantics: scripts/fp4_zero_predictor_codec_v1.py:115-162 (recurrence, readout,
// latent and INT8/INT4 requant) and mamba2_recall/state_quant.py:283-317 (conv).
#pragma once
#include "common.cuh"

namespace sq {

// Exactly rounded fp32 quotient a/s given inv = RN(1/s): one FMA remainder and one FMA
// update (Markstein's correction) give RN(a/s) for normal operands.
__device__ __forceinline__ float div_exact(float a, float s, float inv) {
  float q0 = a * inv;
  float r = fmaf(-q0, s, a);
  return fmaf(r, inv, q0);
}
__device__ __forceinline__ float2 div_exact2(float2 a, float2 ns, float2 inv) {
  float2 q0 = __fmul2_rn(a, inv);
  float2 r = __ffma2_rn(q0, ns, a);           // a - q0*s, exact
  return __ffma2_rn(r, inv, q0);
}
__device__ __forceinline__ float softplus_ref(float v) {
  return v <= 20.0f ? logf(expf(v) + 1.0f) : v;   // :124
}
__device__ __forceinline__ float silu16(float v16) {
  return h2f(f2h(v16 / (1.0f + expf(-v16))));      // torch SiLU on fp16: fp32 math, fp16 out
}
// conv1d prefill numerics (state_quant.py:311-312): fp32 accumulate incl. bias -> fp16, SiLU -> fp16
__device__ __forceinline__ float conv_prefill_value(const float (&w)[5], float x0, float x1, float x2, float x3) {
  float acc = w[0] * x0 + w[1] * x1 + w[2] * x2 + w[3] * x3 + w[4];
  return silu16(h2f(f2h(acc)));
}
// conv step numerics (state_quant.py:291-297): fp16 products summed, fp16, + bias (fp16), SiLU
__device__ __forceinline__ float conv_step_value(const float (&w)[5], float x0, float x1, float x2, float x3) {
  float acc = h2f(f2h(x0 * w[0])) + h2f(f2h(x1 * w[1])) + h2f(f2h(x2 * w[2])) + h2f(f2h(x3 * w[3]));
  float s = h2f(f2h(acc));
  s = h2f(f2h(s + w[4]));
  return silu16(s);
}
// Stored-tier requant of a coordinate pair (:155-162): v = clip(round_half_away(S/s), +-lim) * s
// with S/s the correctly rounded quotient.  Computed on the magnitude: the clip moves in
// front of the rounding (lim is an integer), floor(a + 0.5) is taken exactly with two
// round-down adds (RD(a + 0.5) never crosses the integer below a + 0.5, and RD(t + 2^23)
// = floor(t) + 2^23 for 0 <= t < 2^23), the product (u - 2^23) * s is one FMA against the
// exact -2^23 * s, and the sign of S is put back last.  Bit-identical to the scalar chain.
constexpr float kMagic = 8388608.0f;   // 2^23
__device__ __forceinline__ void requant_pair(float& sa, float& sb, float2 ns, float2 inv, float lim, float2 s,
                                             float2 nms) {
  const float2 q = div_exact2(make_float2(sa, sb), ns, inv);
  float2 a = make_float2(fminf(fabsf(q.x), lim), fminf(fabsf(q.y), lim));
  a = __fadd2_rd(__fadd2_rd(a, make_float2(0.5f, 0.5f)), make_float2(kMagic, kMagic));
  const float2 v = __ffma2_rn(a, s, nms);
  sa = copysignf(v.x, sa);
  sb = copysignf(v.y, sb);
}

// Per-token scalar tail shared by both scan kernels, so their arithmetic is identical by
// construction: the readout (:139-147), the FP8 requant of both latent coefficients
// (:149-154) and the INT8/INT4 scales of the new state (:155-160), pairs in fp32x2.
// dots = {B.C, b0.C, b1.C, b0.B, b1.B, pcz0, pcz1}.
struct TokenScales { float s8, s4, i8, i4; };
__device__ __forceinline__ float token_tail_sums(float ysum, float ycorr, float m8, float m4, float x, float dtv,
                                                 float dec, float dv, const float (&dots)[7], float2& z, float2 ls,
                                                 float2 nls, float2 ils, TokenScales& ts) {
  const float xdt = x * dtv;
  const float zc = fmaf(z.x, dots[1], z.y * dots[2]);
  float out = ysum + fmaf(dec, zc, fmaf(xdt, dots[0], x * dv));
  out = fmaf(dec, fmaf(z.y, dots[6], fmaf(z.x, dots[5], ycorr)), out);
  // latent: z = z*dec + xdt*db, then RN-satfinite E4M3 of clip(z/ls) and back
  z = __ffma2_rn(z, make_float2(dec, dec), __fmul2_rn(make_float2(xdt, xdt), make_float2(dots[3], dots[4])));
  float2 q = div_exact2(z, nls, ils);
  q = make_float2(fminf(fmaxf(q.x, -448.f), 448.f), fminf(fmaxf(q.y, -448.f), 448.f));
  const __half2_raw hz = __nv_cvt_fp8x2_to_halfraw2(__nv_cvt_float2_to_fp8x2(q, __NV_SATFINITE, __NV_E4M3), __NV_E4M3);
  z = __fmul2_rn(__half22float2(*reinterpret_cast<const __half2*>(&hz)), ls);
  // scales: fp16(max(max|S| / {127, 7}, 1e-8))
  float2 sc = div_exact2(make_float2(m8, m4), make_float2(-127.f, -7.f), make_float2(1.0f / 127.0f, 1.0f / 7.0f));
  sc = __half22float2(__float22half2_rn(make_float2(fmaxf(sc.x, 1e-8f), fmaxf(sc.y, 1e-8f))));
  ts.s8 = sc.x; ts.s4 = sc.y;
  ts.i8 = sc.x > 0.f ? __frcp_rn(sc.x) : 0.f;
  ts.i4 = sc.y > 0.f ? __frcp_rn(sc.y) : 0.f;
  return out;
}

__device__ __forceinline__ float token_tail(float2 ya, float2 yb, float2 ca, float2 cb, float m8, float m4,
                                            float x, float dtv, float dec, float dv, const float (&dots)[7],
                                            float2& z, float2 ls, float2 nls, float2 ils, TokenScales& ts) {
  return token_tail_sums((ya.x + ya.y) + (yb.x + yb.y), (ca.x + ca.y) + (cb.x + cb.y), m8, m4, x, dtv, dec, dv, dots,
                         z, ls, nls, ils, ts);
}

// Token tail of the folded multi-token readout (recur_row_fold): the stored tiers' readout
// and the predictor correction arrive as one sum yacc = sum_j prior_j (C_j + cvec_j), and
// the stored tiers' current-token term x dt sum_j B_j C_j joins the zero tier's under
// dots[0] = B.C over all 128 coordinates:
//   out = dec (yacc + z0 c0 + z1 c1 + z0 pcz0 + z1 pcz1) + (x dt) B.C + x D
// (the same value as token_tail_sums with S_j = prior_j dec + (B_j dt) x substituted, summed
// in another order).  dots = {B.C (all), b0.C, b1.C, b0.B, b1.B, pcz0, pcz1}.  The latent
// update and the INT scales are token_tail_sums'.
__device__ __forceinline__ float token_tail_fold(float yacc, float m8, float m4, float x, float dtv, float dec,
                                                 float dv, const float (&dots)[7], float2& z, float2 ls, float2 nls,
                                                 float2 ils, TokenScales& ts) {
  const float xdt = x * dtv;
  const float zc = fmaf(z.x, dots[1], z.y * dots[2]);
  const float corr = fmaf(z.y, dots[6], fmaf(z.x, dots[5], yacc));
  const float out = fmaf(dec, corr + zc, fmaf(xdt, dots[0], x * dv));
  z = __ffma2_rn(z, make_float2(dec, dec), __fmul2_rn(make_float2(xdt, xdt), make_float2(dots[3], dots[4])));
  float2 q = div_exact2(z, nls, ils);
  q = make_float2(fminf(fmaxf(q.x, -448.f), 448.f), fminf(fmaxf(q.y, -448.f), 448.f));
  const __half2_raw hz = __nv_cvt_fp8x2_to_halfraw2(__nv_cvt_float2_to_fp8x2(q, __NV_SATFINITE, __NV_E4M3), __NV_E4M3);
  z = __fmul2_rn(__half22float2(*reinterpret_cast<const __half2*>(&hz)), ls);
  float2 sc = div_exact2(make_float2(m8, m4), make_float2(-127.f, -7.f), make_float2(1.0f / 127.0f, 1.0f / 7.0f));
  sc = __half22float2(__float22half2_rn(make_float2(fmaxf(sc.x, 1e-8f), fmaxf(sc.y, 1e-8f))));
  ts.s8 = sc.x; ts.s4 = sc.y;
  ts.i8 = sc.x > 0.f ? __frcp_rn(sc.x) : 0.f;
  ts.i4 = sc.y > 0.f ? __frcp_rn(sc.y) : 0.f;
  return out;
}

// Requant of every stored pair with the row's new scales.
template <int N8, int NP>
__device__ __forceinline__ void requant_row(float (&S)[2 * NP], const TokenScales& ts) {
  const float2 s82 = make_float2(ts.s8, ts.s8), ns82 = make_float2(-ts.s8, -ts.s8), i82 = make_float2(ts.i8, ts.i8);
  const float2 s42 = make_float2(ts.s4, ts.s4), ns42 = make_float2(-ts.s4, -ts.s4), i42 = make_float2(ts.i4, ts.i4);
  const float m8s = -kMagic * ts.s8, m4s = -kMagic * ts.s4;          // exact (power-of-two scaling)
  const float2 nm82 = make_float2(m8s, m8s), nm42 = make_float2(m4s, m4s);
#pragma unroll
  for (int jp = 0; jp < NP; ++jp) {
    const bool t8 = 2 * jp < N8;
    requant_pair(S[2 * jp], S[2 * jp + 1], t8 ? ns82 : ns42, t8 ? i82 : i42, t8 ? 127.f : 7.f,
                 t8 ? s82 : s42, t8 ? nm82 : nm42);
  }
}

// One token of the recurrence over the stored pairs of one row (:115-147): prior state S
// (already requantised), B/C pairs in tier order ({b_j, b_j+1, c_j, c_j+1}), the predictor
// readout pairs cvec, and per-row dt / decay / x.  S becomes the new unquantised state; the
// readout accumulators and the per-tier max |S| come back for the token tail.
template <int N8, int NP>
__device__ __forceinline__ void recur_row(float (&S)[2 * NP], const float4* __restrict__ cp,
                                          const float2* __restrict__ vp, float dec, float dtv, float x,
                                          float2& ya, float2& yb, float2& ca, float2& cb, float& m8, float& m4) {
  const float2 dd = make_float2(dec, dec), dt2 = make_float2(dtv, dtv), xx = make_float2(x, x);
  ya = yb = ca = cb = make_float2(0.f, 0.f);
  float m8a = 0.f, m8b = 0.f, m4a = 0.f, m4b = 0.f;
#pragma unroll
  for (int jp = 0; jp < NP; ++jp) {
    const float4 bc = cp[jp];
    const float2 cv = vp[jp];
    const float2 pr = make_float2(S[2 * jp], S[2 * jp + 1]);
    const float2 upd = __fmul2_rn(__fmul2_rn(make_float2(bc.x, bc.y), dt2), xx);   // (B*dt)*x
    const float2 sn = __ffma2_rn(pr, dd, upd);                                      // prior*decay + upd
    S[2 * jp] = sn.x; S[2 * jp + 1] = sn.y;
    if (jp & 1) { yb = __ffma2_rn(sn, make_float2(bc.z, bc.w), yb); cb = __ffma2_rn(pr, cv, cb); }
    else        { ya = __ffma2_rn(sn, make_float2(bc.z, bc.w), ya); ca = __ffma2_rn(pr, cv, ca); }
    if (2 * jp < N8) { m8a = fmaxf(m8a, fabsf(sn.x)); m8b = fmaxf(m8b, fabsf(sn.y)); }
    else             { m4a = fmaxf(m4a, fabsf(sn.x)); m4b = fmaxf(m4b, fabsf(sn.y)); }
  }
  m8 = fmaxf(m8a, m8b);
  m4 = fmaxf(m4a, m4b);
}

// Folded multi-token form of recur_row (pairs with token_tail_fold): one accumulation of
// prior_j (C_j + cvec_j) per pair instead of separate readout and correction sums.
// cp[jp].xy = {B_j, B_j+1} (times dt when PREMUL, rounded once, as B * dt here) and the
// pair {C_j + cvec_j, C_j+1 + cvec_j+1} is cp[jp].zw, or vp[jp] when SPLIT.  The new state is
// prior * dec + (B dt) x as in recur_row; the readout accumulates in two chains (even / odd
// pairs) added as (ya.x + ya.y) + (yb.x + yb.y).
template <int N8, int NP, bool PREMUL, bool SPLIT>
__device__ __forceinline__ float recur_row_fold(float (&S)[2 * NP], const float4* __restrict__ cp,
                                                const float2* __restrict__ vp, float dec, float dtv, float x,
                                                float& m8, float& m4) {
  const float2 dd = make_float2(dec, dec), dt2 = make_float2(dtv, dtv), xx = make_float2(x, x);
  float2 ya = make_float2(0.f, 0.f), yb = ya;
  float m8a = 0.f, m8b = 0.f, m4a = 0.f, m4b = 0.f;
#pragma unroll
  for (int jp = 0; jp < NP; ++jp) {
    const float4 bc = cp[jp];
    const float2 cc = SPLIT ? vp[jp] : make_float2(bc.z, bc.w);
    const float2 pr = make_float2(S[2 * jp], S[2 * jp + 1]);
    const float2 bdt = PREMUL ? make_float2(bc.x, bc.y) : __fmul2_rn(make_float2(bc.x, bc.y), dt2);
    const float2 sn = __ffma2_rn(pr, dd, __fmul2_rn(bdt, xx));                          // prior*decay + (B*dt)*x
    S[2 * jp] = sn.x; S[2 * jp + 1] = sn.y;
    if (jp & 1) yb = __ffma2_rn(pr, cc, yb);
    else        ya = __ffma2_rn(pr, cc, ya);
    if (2 * jp < N8) { m8a = fmaxf(m8a, fabsf(sn.x)); m8b = fmaxf(m8b, fabsf(sn.y)); }
    else             { m4a = fmaxf(m4a, fabsf(sn.x)); m4b = fmaxf(m4b, fabsf(sn.y)); }
  }
  m8 = fmaxf(m8a, m8b);
  m4 = fmaxf(m4a, m4b);
  return (ya.x + ya.y) + (yb.x + yb.y);
}

// The one-token step's form of recur_row: the readout and correction sums run as four
// streams (pair jp feeds stream jp % 4, in increasing jp) added as ((t0 + t1) + (t2 + t3)),
// t_k = y_k.x + y_k.y, so four threads of a row can each run one stream and combine them
// with the same result.  Same per-pair state update as recur_row.
template <int N8, int NP>
__device__ __forceinline__ void recur_row4(float (&S)[2 * NP], const float4* __restrict__ cp,
                                           const float2* __restrict__ vp, float dec, float dtv, float x, float& ysum,
                                           float& ycorr, float& m8, float& m4) {
  const float2 dd = make_float2(dec, dec), dt2 = make_float2(dtv, dtv), xx = make_float2(x, x);
  float2 y[4], c[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) y[k] = c[k] = make_float2(0.f, 0.f);
  float m8a = 0.f, m8b = 0.f, m4a = 0.f, m4b = 0.f;
#pragma unroll
  for (int jp = 0; jp < NP; ++jp) {
    const float4 bc = cp[jp];
    const float2 cv = vp[jp];
    const float2 pr = make_float2(S[2 * jp], S[2 * jp + 1]);
    const float2 upd = __fmul2_rn(__fmul2_rn(make_float2(bc.x, bc.y), dt2), xx);
    const float2 sn = __ffma2_rn(pr, dd, upd);
    S[2 * jp] = sn.x; S[2 * jp + 1] = sn.y;
    y[jp & 3] = __ffma2_rn(sn, make_float2(bc.z, bc.w), y[jp & 3]);
    c[jp & 3] = __ffma2_rn(pr, cv, c[jp & 3]);
    if (2 * jp < N8) { m8a = fmaxf(m8a, fabsf(sn.x)); m8b = fmaxf(m8b, fabsf(sn.y)); }
    else             { m4a = fmaxf(m4a, fabsf(sn.x)); m4b = fmaxf(m4b, fabsf(sn.y)); }
  }
  float ty[4], tc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) { ty[k] = y[k].x + y[k].y; tc[k] = c[k].x + c[k].y; }
  ysum = (ty[0] + ty[1]) + (ty[2] + ty[3]);
  ycorr = (tc[0] + tc[1]) + (tc[2] + tc[3]);
  m8 = fmaxf(m8a, m8b);
  m4 = fmaxf(m4a, m4b);
}

}  // namespace sq
