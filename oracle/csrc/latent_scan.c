/*
 * C restatement of the per-row work of the production SQ3.25 latent codec (CPU, test only).
 *
 * TEST INFRASTRUCTURE: loaded by oracle/cscan.py for tests/, never by the product.
 *
 * Restates scripts/fp4_zero_predictor_codec_v1.py:81-181 (decode, per-token recurrence,
 * readout, FP8 latent requant, INT8/INT4 requant via scripts/state_ppl_codec_v6.py:52-61,
 * pack) exactly as oracle/codec.py:latent_scan evaluates it with numpy, so that both give
 * the same bits:
 *   - every operation is one IEEE fp32 operation (build with -ffp-contract=off, no
 *     -ffast-math), in the order the numpy expressions evaluate;
 *   - reductions reproduce numpy's pairwise float32 sum over the kernel's padded tile width
 *     R (next power of two, zero padded): for R < 8 a left-to-right sum, for 8 <= R <= 128
 *     eight strided accumulators combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7));
 *   - the per-token scalars that need exp/log (dt after softplus, exp(A dt)) and the
 *     predictor correction einsum stay in numpy / torch on the caller side and come in as
 *     arrays, so no libm result can differ.
 * Rows (b, h, p) are independent given their group's B / C, so they run in parallel.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef uint16_t f16bits;

static float h2f(f16bits h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}
static f16bits f2h(float f) {
  _Float16 v = (_Float16)f;   /* IEEE round to nearest even */
  f16bits h;
  memcpy(&h, &v, 2);
  return h;
}

static float E4M3[256];
static void init_e4m3(void) {
  for (int b = 0; b < 256; ++b) {
    const int e = (b >> 3) & 15, m = b & 7;
    double v = e == 0 ? m * ldexp(1.0, -9) : (1.0 + m / 8.0) * ldexp(1.0, e - 7);
    if ((b & 0x7F) == 0x7F) v = NAN;
    E4M3[b] = (float)((b & 0x80) ? -v : v);
  }
}

/* fp32 -> E4M3FN byte, round to nearest even, saturating at 448 (inputs are pre-clamped);
 * the same grid arithmetic as oracle/codec.py:f32_to_e4m3, in double (exact). */
static uint8_t f32_to_e4m3(float value) {
  const int sign = signbit(value) ? 1 : 0;
  double a = fabs((double)value);
  if (a > 448.0) a = 448.0;
  int e;
  if (a > 0) {
    frexp(a, &e);
    e -= 1;                                   /* floor(log2(a)) */
  } else {
    e = 0;
  }
  if (e < -6) e = -6;
  if (e > 8) e = 8;
  const double ulp = ldexp(1.0, e - 3);
  double q = nearbyint(a / ulp) * ulp;        /* default rounding mode: ties to even */
  if (q > 448.0) q = 448.0;
  int byte;
  if (q == 0) {
    byte = 0;
  } else if (q < ldexp(1.0, -6)) {
    byte = (int)nearbyint(q / ldexp(1.0, -9));
  } else {
    int eq;
    frexp(q, &eq);
    eq -= 1;
    if (eq < -6) eq = -6;
    if (eq > 8) eq = 8;
    const int mant = (int)nearbyint((q / ldexp(1.0, eq) - 1.0) * 8.0);
    byte = ((eq + 7) << 3) | mant;
  }
  return (uint8_t)(byte | (sign << 7));
}

static int next_pow2(int n) {
  int r = 1;
  while (r < n) r <<= 1;
  return r;
}

/* numpy's float32 pairwise sum of a contiguous run of n <= 128 values */
static float np_sum(const float* a, int n) {
  if (n < 8) {
    float res = 0.f;
    for (int i = 0; i < n; ++i) res += a[i];
    return res;
  }
  float r[8];
  for (int j = 0; j < 8; ++j) r[j] = a[j];
  int i = 8;
  for (; i < n - (n % 8); i += 8)
    for (int j = 0; j < 8; ++j) r[j] += a[i + j];
  float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
  for (; i < n; ++i) res += a[i];
  return res;
}

static float round_half_away(float q) {
  const float a = fabsf(q);
  float r = floorf(a);
  if (a - r >= 0.5f) r = r + 1.0f;
  return q < 0 ? -r : r;
}

/* stored_quantize (state_ppl_codec_v6.py:52-61) of one value */
static int stored_quantize(float value, float scale, float limit) {
  const float safe = scale > 0 ? scale : 1.0f;
  const float quotient = value / safe;
  float r = round_half_away(quotient);
  r = fminf(fmaxf(r, -limit), limit);
  return scale > 0 ? (int)r : 0;
}

/* den = max(value / limit, 1e-8) -> fp16 -> fp32 */
static float tier_scale(float maxabs, float limit) {
  float den = maxabs / limit;
  if (!isnan(den) && den < 1e-8f) den = 1e-8f;   /* np.maximum: NaN propagates */
  return h2f(f2h(den));
}

#define RMAX 128

/*
 * Bt, L, H, P, G, n8, n4: geometry (H heads passed in; head_groups[h] = group of head h).
 * x, y: fp16 bits [Bt][L][H][P];  B, C: fp16 bits [Bt][L][G][128].
 * dtv, decay: fp32 [Bt][L][H] (softplus'd dt and exp(A dt), computed by numpy).
 * Dv: fp32 [H];  corr: fp32 [Bt][L][G][F], F = n8 + n4 + 2.
 * perm: u8 [G][128];  basis: fp16 bits [G][nz][2];  ls: fp32 [G][2] (fp16 values).
 * state: lo/hi [Bt][H][P][n8/2], q4 [Bt][H][P][n4/2], latent [Bt][H][P][2] (E4M3 bytes),
 * s8/s4 fp16 bits [Bt][H][P]; mutated in place.
 */
void latent_scan_rows(int Bt, int L, int H, int P, int G, int n8, int n4, const f16bits* x, const float* dtv,
                      const float* decay, const f16bits* B, const f16bits* C, const float* Dv, const float* corr,
                      const uint8_t* perm, const f16bits* basis, const float* ls, const int* head_groups,
                      uint8_t* lo, uint8_t* hi, uint8_t* q4, uint8_t* latent, f16bits* s8o, f16bits* s4o,
                      f16bits* y) {
  static int inited = 0;
  if (!inited) { init_e4m3(); inited = 1; }
  const int nz = 128 - n8 - n4, F = n8 + n4 + 2;
  const int R8 = next_pow2(n8), R4 = next_pow2(n4), RZ = next_pow2(nz);
  const int W8 = n8 / 2, W4 = n4 / 2;

  /* group-level values per (b, t, g): B / C in tier order and the five zero-tier dots */
  const long long nbtg = (long long)Bt * L * G;
  float* bc = (float*)malloc(sizeof(float) * nbtg * 256);       /* b[0..128) c[128..256) tier order */
  float* dots = (float*)malloc(sizeof(float) * nbtg * 5);       /* bc, c0, c1, b0, b1 */
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < nbtg; ++i) {
    const int g = (int)(i % G);
    const f16bits* bt = B + i * 128;
    const f16bits* ct = C + i * 128;
    float* o = bc + i * 256;
    for (int j = 0; j < 128; ++j) {
      o[j] = h2f(bt[perm[g * 128 + j]]);
      o[128 + j] = h2f(ct[perm[g * 128 + j]]);
    }
    float pbc[RMAX], pc0[RMAX], pc1[RMAX], pb0[RMAX], pb1[RMAX];
    for (int d = 0; d < RZ; ++d) {
      float bv = 0.f, cv = 0.f, u0 = 0.f, u1 = 0.f;
      if (d < nz) {
        bv = o[n8 + n4 + d];
        cv = o[128 + n8 + n4 + d];
        u0 = h2f(basis[(g * nz + d) * 2 + 0]);
        u1 = h2f(basis[(g * nz + d) * 2 + 1]);
      }
      pbc[d] = bv * cv;
      pc0[d] = u0 * cv;
      pc1[d] = u1 * cv;
      pb0[d] = u0 * bv;
      pb1[d] = u1 * bv;
    }
    dots[i * 5 + 0] = np_sum(pbc, RZ);
    dots[i * 5 + 1] = np_sum(pc0, RZ);
    dots[i * 5 + 2] = np_sum(pc1, RZ);
    dots[i * 5 + 3] = np_sum(pb0, RZ);
    dots[i * 5 + 4] = np_sum(pb1, RZ);
  }

  const long long rows = (long long)Bt * H * P;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < rows; ++r) {
    const int b = (int)(r / ((long long)H * P));
    const int h = (int)((r / P) % H);
    const int p = (int)(r % P);
    const int g = head_groups[h];
    float st8[RMAX], st4[RMAX], pr8[RMAX], pr4[RMAX], tmp[RMAX];
    int q8[RMAX], q4v[RMAX];
    /* decode (:81-114) */
    const float sc8 = h2f(s8o[r]), sc4 = h2f(s4o[r]);
    for (int j = 0; j < R8; ++j) {
      st8[j] = 0.f;
      if (j < n8) {
        const int l = (lo[r * W8 + j / 2] >> (4 * (j & 1))) & 15;
        const int hh = (hi[r * W8 + j / 2] >> (4 * (j & 1))) & 15;
        const int ub = (hh << 4) | l;
        st8[j] = (float)(ub - 256 * (ub > 127)) * sc8;
      }
    }
    for (int j = 0; j < R4; ++j) {
      st4[j] = 0.f;
      if (j < n4) {
        const int nib = (q4[r * W4 + j / 2] >> (4 * (j & 1))) & 15;
        st4[j] = (float)(nib - 16 * (nib > 7)) * sc4;
      }
    }
    const float ls0 = ls[g * 2 + 0], ls1 = ls[g * 2 + 1];
    float z0 = E4M3[latent[r * 2 + 0]] * ls0;
    float z1 = E4M3[latent[r * 2 + 1]] * ls1;
    const float dv = Dv[h];
    float s8 = sc8, s4 = sc4;
    for (int t = 0; t < L; ++t) {
      const long long bth = ((long long)b * L + t) * H + h;
      const long long btg = ((long long)b * L + t) * G + g;
      const float* cp = corr + btg * F;
      const float* o = bc + btg * 256;
      const float* dt5 = dots + btg * 5;
      const float xv = h2f(x[bth * P + p]);
      const float dtr = dtv[bth], dec = decay[bth];
      /* recurrence (:133-138): state = prior*decay + (B*dt)*x, padded lanes zero */
      for (int j = 0; j < R8; ++j) {
        pr8[j] = st8[j];
        const float bv = j < n8 ? o[j] : 0.f;
        st8[j] = j < n8 ? pr8[j] * dec + (bv * dtr) * xv : 0.f;
      }
      for (int j = 0; j < R4; ++j) {
        pr4[j] = st4[j];
        const float bv = j < n4 ? o[n8 + j] : 0.f;
        st4[j] = j < n4 ? pr4[j] * dec + (bv * dtr) * xv : 0.f;
      }
      /* readout (:139-147) */
      for (int j = 0; j < R8; ++j) tmp[j] = st8[j] * (j < n8 ? o[128 + j] : 0.f);
      const float ys8 = np_sum(tmp, R8);
      for (int j = 0; j < R4; ++j) tmp[j] = st4[j] * (j < n4 ? o[128 + n8 + j] : 0.f);
      const float ys4 = np_sum(tmp, R4);
      float out = ys8 + ys4;
      const float zc = z0 * dt5[1] + z1 * dt5[2];
      const float xdt = xv * dtr;
      out = out + ((dec * zc + xdt * dt5[0]) + xv * dv);
      for (int j = 0; j < R8; ++j) tmp[j] = pr8[j] * (j < n8 ? cp[j] : 0.f);
      const float c8 = np_sum(tmp, R8);
      for (int j = 0; j < R4; ++j) tmp[j] = pr4[j] * (j < n4 ? cp[n8 + j] : 0.f);
      const float c4 = np_sum(tmp, R4);
      out = out + dec * (((c8 + c4) + z0 * cp[n8 + n4]) + z1 * cp[n8 + n4 + 1]);
      y[bth * P + p] = f2h(out);
      /* latent update + FP8 requant (:149-154) */
      z0 = z0 * dec + xdt * dt5[3];
      z1 = z1 * dec + xdt * dt5[4];
      float v0 = z0 / ls0, v1 = z1 / ls1;
      v0 = fminf(fmaxf(v0, -448.f), 448.f);
      v1 = fminf(fmaxf(v1, -448.f), 448.f);
      z0 = E4M3[f32_to_e4m3(v0)] * ls0;
      z1 = E4M3[f32_to_e4m3(v1)] * ls1;
      /* INT8 / INT4 requant (:155-162) */
      float m8 = 0.f, m4 = 0.f;
      for (int j = 0; j < R8; ++j) m8 = fmaxf(m8, fabsf(st8[j]));
      for (int j = 0; j < R4; ++j) m4 = fmaxf(m4, fabsf(st4[j]));
      s8 = tier_scale(m8, 127.f);
      s4 = tier_scale(m4, 7.f);
      for (int j = 0; j < R8; ++j) {
        q8[j] = stored_quantize(st8[j], s8, 127.f);
        st8[j] = (float)q8[j] * s8;
      }
      for (int j = 0; j < R4; ++j) {
        q4v[j] = stored_quantize(st4[j], s4, 7.f);
        st4[j] = (float)q4v[j] * s4;
      }
    }
    /* pack + store once (:163-181) */
    for (int j = 0; j < n8; j += 2) {
      lo[r * W8 + j / 2] = (uint8_t)((q8[j] & 15) | ((q8[j + 1] & 15) << 4));
      hi[r * W8 + j / 2] = (uint8_t)(((q8[j] >> 4) & 15) | (((q8[j + 1] >> 4) & 15) << 4));
    }
    for (int j = 0; j < n4; j += 2) q4[r * W4 + j / 2] = (uint8_t)((q4v[j] & 15) | ((q4v[j + 1] & 15) << 4));
    float v0 = fminf(fmaxf(z0 / ls0, -448.f), 448.f);
    float v1 = fminf(fmaxf(z1 / ls1, -448.f), 448.f);
    latent[r * 2 + 0] = f32_to_e4m3(v0);
    latent[r * 2 + 1] = f32_to_e4m3(v1);
    s8o[r] = f2h(s8);
    s4o[r] = f2h(s4);
  }
  free(bc);
  free(dots);
}
