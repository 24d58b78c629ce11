// Standalone SQ3.25 row encode / decode (the scan kernel's prologue and epilogue
// as separate entry points).
//
// decode: packed rows -> fp32 tier values in tier (permuted) order and latent z
//         (scripts/fp4_zero_predictor_codec_v1.py:81-114).
// encode: fp32 tier values + latent z -> packed rows with the kernel's requant
//         rule (:149-181, scripts/state_ppl_codec_v6.py:52-61), or with the
//         diagnostic initializer of mamba2_recall/state_codec.py:299-331.
#include "common.cuh"
#include "scan.cuh"

namespace sq {
namespace {

__device__ __forceinline__ float div_exact2(float a, float s, float inv) {
  float q0 = a * inv;
  float r = fmaf(-q0, s, a);
  return fmaf(r, inv, q0);
}

__global__ void decode_rows_kernel(int n8, int n4, long long rows, int heads, int dim, int hpg,
                                   const uint8_t* lo, const uint8_t* hi, const uint8_t* q4,
                                   const uint8_t* latent, const uint16_t* s8p, const uint16_t* s4p,
                                   const uint16_t* latent_scale, float* tiers, float* z) {
  long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int w8 = n8 / 2, w4 = n4 / 2, nt = n8 + n4;
  const float s8 = h2f(s8p[r]), s4 = h2f(s4p[r]);
  for (int j = 0; j < n8; ++j) {
    int l = (lo[r * w8 + j / 2] >> (4 * (j & 1))) & 15;
    int hh = (hi[r * w8 + j / 2] >> (4 * (j & 1))) & 15;
    int ub = (hh << 4) | l;
    tiers[r * nt + j] = (float)(ub - 256 * (ub > 127)) * s8;
  }
  for (int j = 0; j < n4; ++j) {
    int nib = (q4[r * w4 + j / 2] >> (4 * (j & 1))) & 15;
    tiers[r * nt + n8 + j] = (float)(nib - 16 * (nib > 7)) * s4;
  }
  const int h = (int)((r / dim) % heads);
  const int g = h / hpg;
  z[r * 2 + 0] = e4m3_to_f32(latent[r * 2 + 0]) * h2f(latent_scale[g * 2 + 0]);
  z[r * 2 + 1] = e4m3_to_f32(latent[r * 2 + 1]) * h2f(latent_scale[g * 2 + 1]);
}

__global__ void encode_rows_kernel(int n8, int n4, long long rows, int heads, int dim, int hpg, int mode,
                                   const float* tiers, const float* z, const uint16_t* latent_scale,
                                   uint8_t* lo, uint8_t* hi, uint8_t* q4, uint8_t* latent,
                                   uint16_t* s8p, uint16_t* s4p) {
  long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int w8 = n8 / 2, w4 = n4 / 2, nt = n8 + n4;
  const float* v = tiers + r * nt;
  float m8 = 0.f, m4 = 0.f;
  for (int j = 0; j < n8; ++j) m8 = fmaxf(m8, fabsf(v[j]));
  for (int j = 0; j < n4; ++j) m4 = fmaxf(m4, fabsf(v[n8 + j]));
  float d8 = fmaxf(__fdiv_rn(m8, 127.f), 1e-8f), d4 = fmaxf(__fdiv_rn(m4, 7.f), 1e-8f);
  float s8, s4, div8, div4;
  if (mode == 0) {            // production requant: divide by the stored fp16 scale
    s8 = h2f(f2h(d8)); s4 = h2f(f2h(d4)); div8 = s8; div4 = s4;
  } else {                    // diagnostic encode_state_: fp32 denominators
    s8 = h2f(f2h(d8)); s4 = h2f(f2h(d4)); div8 = d8; div4 = d4;
  }
  auto quant = [&](float x, float s, float lim) -> int {
    if (mode == 0) {
      if (!(s > 0.f)) return 0;
      float q = round_half_away(div_exact2(x, s, __frcp_rn(s)));
      return (int)fminf(fmaxf(q, -lim), lim);
    }
    float zq = __fdiv_rn(x, s);
    float rq = copysignf(floorf(fabsf(zq) + 0.5f), zq);
    if (zq == 0.f) rq = 0.f;
    return (int)fminf(fmaxf(rq, -lim), lim);
  };
  for (int j = 0; j < n8; j += 2) {
    int a = quant(v[j], div8, 127.f), c = quant(v[j + 1], div8, 127.f);
    lo[r * w8 + j / 2] = (uint8_t)((a & 15) | ((c & 15) << 4));
    hi[r * w8 + j / 2] = (uint8_t)(((a >> 4) & 15) | (((c >> 4) & 15) << 4));
  }
  for (int j = 0; j < n4; j += 2) {
    int a = quant(v[n8 + j], div4, 7.f), c = quant(v[n8 + j + 1], div4, 7.f);
    q4[r * w4 + j / 2] = (uint8_t)((a & 15) | ((c & 15) << 4));
  }
  s8p[r] = f2h(s8); s4p[r] = f2h(s4);
  if (mode == 0) {
    const int h = (int)((r / dim) % heads);
    const int g = h / hpg;
    const float l0 = h2f(latent_scale[g * 2]), l1 = h2f(latent_scale[g * 2 + 1]);
    const float z0 = z[r * 2 + 0], z1 = z[r * 2 + 1];
    latent[r * 2 + 0] = f32_to_e4m3(fminf(fmaxf(__fdiv_rn(z0, l0), -448.f), 448.f));
    latent[r * 2 + 1] = f32_to_e4m3(fminf(fmaxf(__fdiv_rn(z1, l1), -448.f), 448.f));
  } else {
    latent[r * 2 + 0] = 0; latent[r * 2 + 1] = 0;
  }
}

}  // namespace

int launch_decode_rows(int layout, int batch, int heads, int dim, int groups,
                       const uint8_t* lo, const uint8_t* hi, const uint8_t* q4, const uint8_t* latent,
                       const uint16_t* s8, const uint16_t* s4, const uint16_t* latent_scale,
                       float* tiers, float* z, cudaStream_t st) {
  if (layout < 0 || layout > 6 || batch <= 0 || heads <= 0 || dim <= 0 || groups <= 0 || heads % groups)
    return kEInval;
  long long rows = (long long)batch * heads * dim;
  int th = 128;
  decode_rows_kernel<<<(unsigned)((rows + th - 1) / th), th, 0, st>>>(
      kLayouts[layout].n8, kLayouts[layout].n4, rows, heads, dim, heads / groups,
      lo, hi, q4, latent, s8, s4, latent_scale, tiers, z);
  return launch_status();
}

int launch_encode_rows(int layout, int batch, int heads, int dim, int groups, int mode,
                       const float* tiers, const float* z, const uint16_t* latent_scale,
                       uint8_t* lo, uint8_t* hi, uint8_t* q4, uint8_t* latent,
                       uint16_t* s8, uint16_t* s4, cudaStream_t st) {
  if (layout < 0 || layout > 6 || batch <= 0 || heads <= 0 || dim <= 0 || groups <= 0 || heads % groups ||
      (mode != 0 && mode != 1))
    return kEInval;
  long long rows = (long long)batch * heads * dim;
  int th = 128;
  encode_rows_kernel<<<(unsigned)((rows + th - 1) / th), th, 0, st>>>(
      kLayouts[layout].n8, kLayouts[layout].n4, rows, heads, dim, heads / groups, mode,
      tiers, z, latent_scale, lo, hi, q4, latent, s8, s4);
  return launch_status();
}

}  // namespace sq
