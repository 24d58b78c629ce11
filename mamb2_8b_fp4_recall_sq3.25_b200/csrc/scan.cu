// Fused SQ3.25 selective-state update (the production latent codec), sm_100a.
//
// Semantics: scripts/fp4_zero_predictor_codec_v1.py:76-181 (kernel) plus the
// host predictor correction of :221-225, which is folded in here (one group
// dot-product pass per token in shared memory instead of a separate einsum
// and an HBM round trip of the [B,L,G,F] correction tensor).
//
// Mapping: one thread owns one recurrent row (b,h,p) of 128 coordinates and
// keeps its n8+n4 stored coordinates in registers for the whole call (the
// zero tier carries no state).  A CTA holds `hpc` heads of the same B/C group.
// Per token the CTA stages the group's B/C values in tier order together with
// the predictor readout vector cvec (= the reference's `correction`) and the
// five zero-tier group dots, then every thread updates, reads out, and
// requantizes its row in registers.  Packed rows are read once at the start
// and written once at the end of the call, as in the reference.
#include "common.cuh"
#include "scan.cuh"

namespace sq {

namespace {

constexpr int kMaxF = 88;      // n8+n4+2 <= 86
constexpr int kMaxNz = 80;

struct __align__(16) Coord { float b, c, cvec, pad; };

// Exactly-rounded fp32 quotient a/s given inv = RN(1/s) (Markstein's
// correction step: one FMA remainder + one FMA update gives RN(a/s)).
__device__ __forceinline__ float div_exact(float a, float s, float inv) {
  float q0 = a * inv;
  float r = fmaf(-q0, s, a);
  return fmaf(r, inv, q0);
}

__device__ __forceinline__ float softplus_ref(float v) {
  // dt = dt <= 20 ? log(exp(dt) + 1) : dt   (:124)
  return v <= 20.0f ? logf(expf(v) + 1.0f) : v;
}

__device__ __forceinline__ float silu16(float v16) {
  // torch SiLU on an fp16 tensor: computed in fp32, rounded to fp16.
  float r = v16 / (1.0f + expf(-v16));
  return h2f(f2h(r));
}

// Causal conv step of StateQuant._convolution (mamba2_recall/state_quant.py:291-297):
// value = fp16(sum_k fp16(cache_k * w_k)) + bias (fp16), then SiLU -> fp16.
__device__ __forceinline__ float conv_step_value(const ScanParams& P, int b, int ch, uint16_t raw) {
  const uint16_t* ring = P.conv_cache + (long long)b * P.conv_cache_sb;
  float acc = 0.0f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint16_t v = (k == 3) ? raw : ring[((P.conv_pos - 3 + k) & 3) * 10240 + ch];
    float prod = h2f(f2h(h2f(v) * h2f(P.conv_w[ch * 4 + k])));
    acc += prod;
  }
  float s = h2f(f2h(acc));
  s = h2f(f2h(s + h2f(P.conv_b[ch])));
  return silu16(s);
}

template <int N8, int N4>
__global__ void __launch_bounds__(256)
ssu_sq325_kernel(const ScanParams P) {
  constexpr int NZ = 128 - N8 - N4;
  constexpr int F = N8 + N4 + 2;
  constexpr int W8 = N8 / 2, W4 = N4 / 2;
  static_assert(F <= kMaxF && NZ <= kMaxNz, "layout out of range");

  extern __shared__ __align__(16) unsigned char smem[];
  Coord* sCoord = reinterpret_cast<Coord*>(smem);                          // [128]
  float* sDots = reinterpret_cast<float*>(sCoord + 128);                   // [8]
  float* sPred = sDots + 8;                                                // [F][NZ+1]
  float* sBasis = sPred + F * (NZ + 1);                                    // [2][NZ]
  int* sPerm = reinterpret_cast<int*>(sBasis + 2 * NZ);                    // [128]
  unsigned char* sPack = reinterpret_cast<unsigned char*>(sPerm + 128);   // rows*52

  const int tid = threadIdx.x;
  const int bd = blockDim.x;
  const int dim = P.dim;
  const int hpc = bd / dim;
  const int b = blockIdx.y;
  const int h0 = blockIdx.x * hpc;
  const int hl = tid / dim;
  const int p = tid - hl * dim;
  const int h = h0 + hl;
  const int g = h0 / (P.heads / P.groups);
  const long long row0 = ((long long)b * P.heads + h0) * dim;   // first row of this CTA
  const int rows = bd;

  // ---- static tables for this group ----
  for (int i = tid; i < 128; i += bd) sPerm[i] = P.perm[g * 128 + i];
  for (int i = tid; i < F * NZ; i += bd) {
    int f = i / NZ, d = i - f * NZ;
    sPred[f * (NZ + 1) + d] = h2f(P.predictor[((long long)g * F + f) * NZ + d]);
  }
  for (int i = tid; i < NZ; i += bd) {
    sBasis[i] = h2f(P.basis[(g * NZ + i) * 2 + 0]);
    sBasis[NZ + i] = h2f(P.basis[(g * NZ + i) * 2 + 1]);
  }
  // ---- stage packed rows (coalesced 32-bit copies; regions are 4-byte multiples) ----
  unsigned char* pLo = sPack;
  unsigned char* pHi = pLo + rows * W8;
  unsigned char* pQ4 = pHi + rows * W8;
  unsigned char* pLat = pQ4 + rows * W4;
  uint16_t* pS8 = reinterpret_cast<uint16_t*>(pLat + rows * 2);
  uint16_t* pS4 = pS8 + rows;
  {
    auto copy_in = [&](unsigned char* dst, const unsigned char* src, int bytes) {
      const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
      uint32_t* d = reinterpret_cast<uint32_t*>(dst);
      for (int i = tid; i < bytes / 4; i += bd) d[i] = s[i];
    };
    copy_in(pLo, P.lo + row0 * W8, rows * W8);
    copy_in(pHi, P.hi + row0 * W8, rows * W8);
    copy_in(pQ4, P.q4 + row0 * W4, rows * W4);
    copy_in(pLat, P.latent + row0 * 2, rows * 2);
    copy_in(reinterpret_cast<unsigned char*>(pS8), reinterpret_cast<const unsigned char*>(P.s8 + row0), rows * 2);
    copy_in(reinterpret_cast<unsigned char*>(pS4), reinterpret_cast<const unsigned char*>(P.s4 + row0), rows * 2);
  }
  __syncthreads();

  // ---- decode own row (:81-114) ----
  float S8[N8 > 0 ? N8 : 1], S4[N4 > 0 ? N4 : 1];
  {
    float s8 = h2f(pS8[tid]), s4 = h2f(pS4[tid]);
#pragma unroll
    for (int j = 0; j < N8; ++j) {
      int lo = (pLo[tid * W8 + j / 2] >> (4 * (j & 1))) & 15;
      int hi = (pHi[tid * W8 + j / 2] >> (4 * (j & 1))) & 15;
      int ub = (hi << 4) | lo;
      int q = ub - 256 * (ub > 127);
      S8[j] = (float)q * s8;
    }
#pragma unroll
    for (int j = 0; j < N4; ++j) {
      int nib = (pQ4[tid * W4 + j / 2] >> (4 * (j & 1))) & 15;
      int q = nib - 16 * (nib > 7);
      S4[j] = (float)q * s4;
    }
  }
  const float ls0 = h2f(P.latent_scale[g * 2 + 0]);
  const float ls1 = h2f(P.latent_scale[g * 2 + 1]);
  float z0 = e4m3_to_f32(pLat[tid * 2 + 0]) * ls0;
  float z1 = e4m3_to_f32(pLat[tid * 2 + 1]) * ls1;
  const float av = P.A[h];
  const float dv = P.d_is_f32 ? reinterpret_cast<const float*>(P.D)[h] : h2f(reinterpret_cast<const uint16_t*>(P.D)[h]);
  const float bias = P.dt_bias_is_f32 ? reinterpret_cast<const float*>(P.dt_bias)[h]
                                      : h2f(reinterpret_cast<const uint16_t*>(P.dt_bias)[h]);
  const bool fuse_conv = P.conv_w != nullptr;

  // ---- token loop with one-token register prefetch ----
  constexpr int kMaxJ = 4;                  // 128 / min blockDim (32)
  uint16_t pre_b[kMaxJ], pre_c[kMaxJ], pre_x = 0, pre_dt = 0;
  auto prefetch = [&](int t) {
    const long long xo = (long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * dim + p;
    pre_x = P.x[xo];
    pre_dt = P.dt[(long long)b * P.dt_sb + (long long)t * P.dt_st + h];
    const uint16_t* Bt = P.B + (long long)b * P.b_sb + (long long)t * P.b_st + g * 128;
    const uint16_t* Ct = P.C + (long long)b * P.c_sb + (long long)t * P.c_st + g * 128;
#pragma unroll
    for (int i = 0; i < kMaxJ; ++i) {
      int j = tid + i * bd;
      if (j < 128) { int n = sPerm[j]; pre_b[i] = Bt[n]; pre_c[i] = Ct[n]; }
    }
  };
  prefetch(0);
  float S8n_max = 0.f, S4n_max = 0.f;   // last scales (kept for the final pack)
  float s8 = 0.f, s4 = 0.f;
  for (int t = 0; t < P.length; ++t) {
    __syncthreads();                                   // previous token done with sCoord
    float xv, dtraw;
#pragma unroll
    for (int i = 0; i < kMaxJ; ++i) {
      int j = tid + i * bd;
      if (j < 128) {
        float bv, cv;
        if (fuse_conv) {
          int n = sPerm[j];
          bv = conv_step_value(P, b, 8192 + g * 128 + n, pre_b[i]);
          cv = conv_step_value(P, b, 9216 + g * 128 + n, pre_c[i]);
        } else {
          bv = h2f(pre_b[i]); cv = h2f(pre_c[i]);
        }
        sCoord[j].b = bv; sCoord[j].c = cv;
      }
    }
    if (fuse_conv) xv = conv_step_value(P, b, h * dim + p, pre_x);
    else xv = h2f(pre_x);
    dtraw = h2f(pre_dt);
    if (fuse_conv) {
      // ring write of this token's raw values (slot pos%4 is not read this step)
      uint16_t* ring = P.conv_cache + (long long)b * P.conv_cache_sb + (P.conv_pos & 3) * 10240;
      ring[h * dim + p] = pre_x;
      if ((h0 % (P.heads / P.groups)) == 0) {
#pragma unroll
        for (int i = 0; i < kMaxJ; ++i) {
          int j = tid + i * bd;
          if (j < 128) { int n = sPerm[j]; ring[8192 + g * 128 + n] = pre_b[i]; ring[9216 + g * 128 + n] = pre_c[i]; }
        }
      }
    }
    if (t + 1 < P.length) prefetch(t + 1);
    __syncthreads();                                   // B/C of token t visible
    // group-level dots: cvec (the reference's host correction) and zero-tier dots
    for (int f = tid; f < F + 5; f += bd) {
      float acc = 0.f;
      if (f < F) {
        const float* pr = sPred + f * (NZ + 1);
#pragma unroll 8
        for (int d = 0; d < NZ; ++d) acc = fmaf(sCoord[N8 + N4 + d].c, pr[d], acc);
        if (f < N8 + N4) sCoord[f].cvec = acc; else sDots[5 + f - (N8 + N4)] = acc;
      } else {
        int k = f - F;
#pragma unroll 8
        for (int d = 0; d < NZ; ++d) {
          const Coord cz = sCoord[N8 + N4 + d];
          float u = (k == 0) ? cz.b : (k <= 2 ? sBasis[(k - 1) * NZ + d] : sBasis[(k - 3) * NZ + d]);
          float v = (k == 0) ? cz.c : (k <= 2 ? cz.c : cz.b);
          acc = fmaf(u, v, acc);
        }
        sDots[k] = acc;
      }
    }
    __syncthreads();                                   // cvec and dots visible

    // ---- per-row recurrence, readout and requant (:115-162) ----
    float dtv = softplus_ref(dtraw + bias);
    float dec = expf(av * dtv);
    float ysum = 0.f, ycorr = 0.f, m8 = 0.f, m4 = 0.f;
#pragma unroll
    for (int j = 0; j < N8; ++j) {
      const Coord c = sCoord[j];
      float pr = S8[j];
      float sn = fmaf(pr, dec, (c.b * dtv) * xv);
      S8[j] = sn;
      ysum = fmaf(sn, c.c, ysum);
      ycorr = fmaf(pr, c.cvec, ycorr);
      m8 = fmaxf(m8, fabsf(sn));
    }
#pragma unroll
    for (int j = 0; j < N4; ++j) {
      const Coord c = sCoord[N8 + j];
      float pr = S4[j];
      float sn = fmaf(pr, dec, (c.b * dtv) * xv);
      S4[j] = sn;
      ysum = fmaf(sn, c.c, ysum);
      ycorr = fmaf(pr, c.cvec, ycorr);
      m4 = fmaxf(m4, fabsf(sn));
    }
    const float dbc = sDots[0], dc0 = sDots[1], dc1 = sDots[2], db0 = sDots[3], db1 = sDots[4];
    const float pcz0 = sDots[5], pcz1 = sDots[6];
    const float xdt = xv * dtv;
    float out = ysum + (dec * (z0 * dc0 + z1 * dc1) + xdt * dbc + xv * dv);
    out = out + dec * (ycorr + z0 * pcz0 + z1 * pcz1);
    P.y[(long long)b * P.y_sb + (long long)t * P.y_st + (long long)h * dim + p] = f2h(out);
    // latent FP8 requant (:149-154)
    z0 = z0 * dec + xdt * db0;
    z1 = z1 * dec + xdt * db1;
    z0 = e4m3_to_f32(f32_to_e4m3(fminf(fmaxf(__fdiv_rn(z0, ls0), -448.f), 448.f))) * ls0;
    z1 = e4m3_to_f32(f32_to_e4m3(fminf(fmaxf(__fdiv_rn(z1, ls1), -448.f), 448.f))) * ls1;
    // INT8 / INT4 requant (:155-162, state_ppl_codec_v6.py:52-61)
    s8 = h2f(f2h(fmaxf(__fdiv_rn(m8, 127.f), 1e-8f)));
    s4 = h2f(f2h(fmaxf(__fdiv_rn(m4, 7.f), 1e-8f)));
    const float i8 = s8 > 0.f ? __frcp_rn(s8) : 0.f;
    const float i4 = s4 > 0.f ? __frcp_rn(s4) : 0.f;
#pragma unroll
    for (int j = 0; j < N8; ++j) {
      float q = round_half_away(div_exact(S8[j], s8, i8));
      q = fminf(fmaxf(q, -127.f), 127.f);
      S8[j] = q * s8;
    }
#pragma unroll
    for (int j = 0; j < N4; ++j) {
      float q = round_half_away(div_exact(S4[j], s4, i4));
      q = fminf(fmaxf(q, -7.f), 7.f);
      S4[j] = q * s4;
    }
  }
  (void)S8n_max; (void)S4n_max;

  // ---- pack once (:163-181) and store coalesced ----
  {
    const float i8 = s8 > 0.f ? __frcp_rn(s8) : 0.f;
    const float i4 = s4 > 0.f ? __frcp_rn(s4) : 0.f;
#pragma unroll
    for (int j = 0; j < N8; j += 2) {
      int qa = __float2int_rn(div_exact(S8[j], s8, i8));
      int qb = __float2int_rn(div_exact(S8[j + 1], s8, i8));
      pLo[tid * W8 + j / 2] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
      pHi[tid * W8 + j / 2] = (unsigned char)(((qa >> 4) & 15) | (((qb >> 4) & 15) << 4));
    }
#pragma unroll
    for (int j = 0; j < N4; j += 2) {
      int qa = __float2int_rn(div_exact(S4[j], s4, i4));
      int qb = __float2int_rn(div_exact(S4[j + 1], s4, i4));
      pQ4[tid * W4 + j / 2] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
    }
    pLat[tid * 2 + 0] = f32_to_e4m3(fminf(fmaxf(__fdiv_rn(z0, ls0), -448.f), 448.f));
    pLat[tid * 2 + 1] = f32_to_e4m3(fminf(fmaxf(__fdiv_rn(z1, ls1), -448.f), 448.f));
    pS8[tid] = f2h(s8);
    pS4[tid] = f2h(s4);
  }
  __syncthreads();
  {
    auto copy_out = [&](unsigned char* dst, const unsigned char* src, int bytes) {
      const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
      uint32_t* d = reinterpret_cast<uint32_t*>(dst);
      for (int i = tid; i < bytes / 4; i += bd) d[i] = s[i];
    };
    copy_out(P.lo + row0 * W8, pLo, rows * W8);
    copy_out(P.hi + row0 * W8, pHi, rows * W8);
    copy_out(P.q4 + row0 * W4, pQ4, rows * W4);
    copy_out(P.latent + row0 * 2, pLat, rows * 2);
    copy_out(reinterpret_cast<unsigned char*>(P.s8 + row0), reinterpret_cast<unsigned char*>(pS8), rows * 2);
    copy_out(reinterpret_cast<unsigned char*>(P.s4 + row0), reinterpret_cast<unsigned char*>(pS4), rows * 2);
  }
}

template <int N8, int N4>
int launch_t(const ScanParams& P, int hpc, cudaStream_t stream) {
  constexpr int NZ = 128 - N8 - N4;
  constexpr int F = N8 + N4 + 2;
  const int bd = hpc * P.dim;
  size_t smem = 128 * sizeof(Coord) + 8 * 4 + (size_t)F * (NZ + 1) * 4 + 2 * NZ * 4 + 128 * 4 + (size_t)bd * 52;
  auto kern = ssu_sq325_kernel<N8, N4>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return kECuda;
  }
  dim3 grid(P.heads / hpc, P.batch);
  kern<<<grid, bd, smem, stream>>>(P);
  return cudaGetLastError() == cudaSuccess ? kOk : kECuda;
}

}  // namespace

int launch_scan(const ScanParams& P, cudaStream_t stream) {
  if (P.layout < 0 || P.layout > 6) return kEInval;
  if (P.batch <= 0 || P.length <= 0 || P.heads <= 0 || P.groups <= 0 || P.heads % P.groups) return kEInval;
  if (P.dim <= 0 || P.dim % 16 || P.dim > 256) return kEInval;
  if (P.conv_w && P.length != 1) return kEInval;
  const int hpg = P.heads / P.groups;
  int hpc = 1;
  for (int c = 1; c <= hpg; ++c)
    if (hpg % c == 0 && c * P.dim <= 128) hpc = c;
  if (hpc * P.dim < 32 && hpg > hpc) return kEInval;
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
