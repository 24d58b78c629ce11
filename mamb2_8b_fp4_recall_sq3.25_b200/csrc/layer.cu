// Block / mixer elementwise kernels around the codec and the FP4 projections.
//
//  add_rmsnorm          mamba_ssm Block (unfused add, fp16 residual) + RMSNorm(eps)
//  conv_prefill         StateQuant._convolution prefill branch (mamba2_recall/state_quant.py:303-317)
//  resurface_gatednorm  resurface_native._Adapter.forward (:105-118) applied in the
//                       norm pre-hook (:201-222), then RMSNormGated(norm_before_gate=False,
//                       group_size=1024) as called at fp4_zero_predictor_codec_v1.py:356-359
//  ce_finalize / window_sum / argmax   the scoring and greedy heads
//                       (scripts/run_fp4_ridge_resurface_v3.py:105-109,
//                        scripts/infer_fp4_ridge_resurface_v1.py:103-105)
#include "common.cuh"
#include "device_util.cuh"
#include "layer.cuh"

namespace sq {
namespace {


// one CTA (256 threads) per row; D % 8 == 0, D <= 8192
__global__ void add_rmsnorm_kernel(const uint16_t* __restrict__ h, uint16_t* __restrict__ res, int has_res,
                                   const uint16_t* __restrict__ w, float eps, uint16_t* __restrict__ out, int D) {
  __shared__ float red[8];
  const long long row = blockIdx.x;
  const uint16_t* hr = h + row * D;
  uint16_t* rr = res + row * D;
  float vals[32];
  float ss = 0.f;
  int n = 0;
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8, ++n) {
    uint4 hv = *reinterpret_cast<const uint4*>(hr + c);
    const uint16_t* hp = reinterpret_cast<const uint16_t*>(&hv);
    uint4 ov;
    uint16_t* op = reinterpret_cast<uint16_t*>(&ov);
    if (has_res) {
      uint4 rv = *reinterpret_cast<const uint4*>(rr + c);
      const uint16_t* rp = reinterpret_cast<const uint16_t*>(&rv);
#pragma unroll
      for (int i = 0; i < 8; ++i) op[i] = f2h(h2f(hp[i]) + h2f(rp[i]));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) op[i] = hp[i];
    }
    *reinterpret_cast<uint4*>(rr + c) = ov;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float x = h2f(op[i]);
      vals[n * 8 + i] = x;
      ss += x * x;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float rstd = 1.0f / sqrtf(tot / (float)D + eps);
  n = 0;
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8, ++n) {
    uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const uint16_t* wp = reinterpret_cast<const uint16_t*>(&wv);
    uint4 ov;
    uint16_t* op = reinterpret_cast<uint16_t*>(&ov);
#pragma unroll
    for (int i = 0; i < 8; ++i) op[i] = f2h((vals[n * 8 + i] * rstd) * h2f(wp[i]));
    *reinterpret_cast<uint4*>(out + row * D + c) = ov;
  }
}

constexpr int kConvChunk = 64;

__device__ __forceinline__ float silu_f16(float v16) { return h2f(f2h(v16 / (1.0f + expf(-v16)))); }

// thread = (b, channel, chunk of kConvChunk positions)
__global__ void conv_prefill_kernel(const uint16_t* __restrict__ raw, long long raw_sb, long long raw_st,
                                    int B, int L, int C, const uint16_t* __restrict__ w,
                                    const uint16_t* __restrict__ bias, uint16_t* __restrict__ cache,
                                    long long cache_sb, int pos0, uint16_t* __restrict__ out,
                                    long long out_sb, long long out_st) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int chunk = blockIdx.y;
  const int b = blockIdx.z;
  if (c >= C) return;
  const int t0 = chunk * kConvChunk;
  if (t0 >= L) return;
  const int t1 = min(L, t0 + kConvChunk);
  const uint16_t* rb = raw + (long long)b * raw_sb + c;
  uint16_t* ring = cache + (long long)b * cache_sb + c;
  const float w0 = h2f(w[c * 4 + 0]), w1 = h2f(w[c * 4 + 1]), w2 = h2f(w[c * 4 + 2]), w3 = h2f(w[c * 4 + 3]);
  const float bb = h2f(bias[c]);
  // history: raw values at local positions t0-3 .. t0-1 (negative -> ring or zeros)
  float x0, x1, x2;
  auto hist = [&](int lt) -> float {
    if (lt >= 0) return h2f(rb[(long long)lt * raw_st]);
    const int ap = pos0 + lt;                  // absolute position
    if (ap < 0) return 0.f;
    return h2f(ring[(long long)(ap & 3) * C]);
  };
  x0 = hist(t0 - 3); x1 = hist(t0 - 2); x2 = hist(t0 - 1);
  for (int t = t0; t < t1; ++t) {
    const float x3 = h2f(rb[(long long)t * raw_st]);
    float acc = w0 * x0 + w1 * x1 + w2 * x2 + w3 * x3 + bb;
    float v = h2f(f2h(acc));
    out[(long long)b * out_sb + (long long)t * out_st + c] = f2h(silu_f16(v));
    x0 = x1; x1 = x2; x2 = x3;
  }
  if (chunk == 0) {
    // the only thread of this (b, c) that touches the ring: write the last raw columns
    for (int lt = max(0, L - 4); lt < L; ++lt) ring[(long long)((pos0 + lt) & 3) * C] = rb[(long long)lt * raw_st];
  }
}

// Adapter gate partial over channels [512 w, 512 w + 512): lane stride 8, warp sum.
__device__ __forceinline__ float gate_span(const uint16_t* Us, const uint16_t* Ws, int w, int lane) {
  float s = 0.f;
#pragma unroll
  for (int i = w * 512 + lane * 8; i < (w + 1) * 512; i += 256) {
    const uint4 uv = *reinterpret_cast<const uint4*>(Us + i);
    const uint4 wv = *reinterpret_cast<const uint4*>(Ws + i);
    const uint16_t* up = reinterpret_cast<const uint16_t*>(&uv);
    const uint16_t* wp = reinterpret_cast<const uint16_t*>(&wv);
#pragma unroll
    for (int k = 0; k < 8; ++k) s = fmaf(h2f(up[k]), h2f(wp[k]), s);
  }
  return warp_sum(s);
}

// A CTA of `gpb` warps (8 for long sequences, 1 for decode batches) covers gated-norm
// groups blockIdx.x*gpb .. +gpb-1 (warp w owns heads 16g..16g+15 of its group g) and
// processes tokens t = blockIdx.y, += gridDim.y.  The 128x128 head mix
// mix[i,p] = sum_j V[i,j] y[j,p] runs on the tensor cores (mma.sync m16n8k16, fp16 in,
// fp32 accumulate; V and the token's y staged in shared memory, B fragments through
// ldmatrix.trans), then each warp applies the gate correction and the gated RMSNorm of its
// group entirely in registers.
constexpr int kVPitch = 136;   // fp16 elements per staged V row (128 + 8 pad, 272 B)
constexpr int kYPitch = 72;    // fp16 elements per staged y row (64 + 8 pad, 144 B)

// [rows][64] fp16 tiles in shared memory with 16-byte chunk c of row h at chunk c ^ (h & 7),
// so that lanes reading the same column of eight consecutive rows hit different banks.
__device__ __forceinline__ int swz64(int h, int p) { return (h << 6) + ((((p >> 3) ^ h) & 7) << 3) + (p & 7); }
__device__ __forceinline__ void stage_swz64(uint16_t* dst, const uint16_t* src, int rows, int tid, int nth) {
  for (int i = tid; i < rows * 8; i += nth) cp_async16(dst + swz64(i >> 3, (i & 7) * 8), src + i * 8);
}

template <int GPB>
__global__ void __launch_bounds__(32 * GPB)
resurface_gatednorm_kernel(const uint16_t* __restrict__ y, const uint16_t* __restrict__ z, long long z_st,
                           const uint16_t* __restrict__ u, long long u_st, AdapterPtrs ad, int has_ad,
                           const uint16_t* __restrict__ nw, float eps, uint16_t* __restrict__ out, int T) {
  extern __shared__ __align__(16) unsigned char smraw[];
  uint16_t* Ys = reinterpret_cast<uint16_t*>(smraw);                  // [128][kYPitch]   this token's y
  uint16_t* Vs = Ys + 128 * kYPitch;                                  // [GPB*16][kVPitch] V rows
  uint16_t* Zs = Vs + GPB * 16 * kVPitch;                             // [GPB*16][64]     this token's z (swz64)
  uint16_t* Ns = Zs + GPB * 1024;                                     // [GPB*16][64]     norm weights (swz64)
  uint16_t* Us = Ns + GPB * 1024;                                     // [4096]           mixer input u
  uint16_t* Ws = Us + 4096;                                           // [4096]           gate weights
  __shared__ float spart[GPB];
  const int tid = threadIdx.x, nth = 32 * GPB;
  const int warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int grp0 = blockIdx.x * GPB;
  const int grp = grp0 + warp;                                        // norm group of this warp
  // per-CTA constants: V rows of the CTA's groups, gate weights, norm weights
  if (has_ad) {
    for (int i = tid; i < GPB * 16 * 16; i += nth) {
      const int r = i >> 4, c = (i & 15) * 8;
      cp_async16(Vs + r * kVPitch + c, ad.V + (grp0 * 16 + r) * 128 + c);
    }
    stage16(Ws, ad.w, 4096 * 2, tid, nth);
  }
  stage_swz64(Ns, nw + grp0 * 1024, GPB * 16, tid, nth);
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
    __syncthreads();                                   // previous token done with the staged rows
    const uint16_t* yr = y + (long long)t * 8192;
    for (int i = tid; i < 128 * 8; i += nth) {         // y[j][p] in 16-byte chunks
      const int r = i >> 3, c = (i & 7) * 8;
      cp_async16(Ys + r * kYPitch + c, yr + r * 64 + c);
    }
    stage_swz64(Zs, z + (long long)t * z_st + grp0 * 1024, GPB * 16, tid, nth);
    if (has_ad) stage16(Us, u + (long long)t * u_st, 4096 * 2, tid, nth);
    cp_async_wait_all();
    __syncthreads();
    float gate = 0.f;
    if (has_ad) {
      // gate logit = fp16(fp16(u . w) + b): eight 512-channel partials (lane stride 8, warp
      // sum each), added in order; with GPB = 8 each warp computes one, with GPB = 1 one warp
      // computes all eight
      float s = 0.f;
      if (GPB > 1) {
        const float p = gate_span(Us, Ws, warp, lane);
        if (lane == 0) spart[warp] = p;
        __syncthreads();
#pragma unroll
        for (int w = 0; w < GPB; ++w) s += spart[w];
      } else {
#pragma unroll 1
        for (int w = 0; w < 8; ++w) s += gate_span(Us, Ws, w, lane);
      }
      const float lg = h2f(f2h(h2f(f2h(s)) + h2f(ad.b[0])));
      gate = h2f(f2h(ad.hard ? (lg > 0.f ? 1.f : 0.f) : __frcp_rn(1.0f + expf(-lg))));
    }
    float acc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    if (has_ad) {
      const int i0 = warp * 16;                        // local V row of this warp's heads
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int k0 = 0; k0 < 128; k0 += 16) {
        uint32_t a[4];
        // matrices: (rows i0..+7, k0), (i0+8.., k0), (i0.., k0+8), (i0+8.., k0+8)
        ldsm_x4(a, Vs + (i0 + rr + (mi & 1) * 8) * kVPitch + k0 + (mi >> 1) * 8);
#pragma unroll
        for (int n2 = 0; n2 < 4; ++n2) {
          uint32_t bfr[4];
          // matrices: (j k0..+7, p n), (j k0+8.., p n), (j k0.., p n+8), (j k0+8.., p n+8)
          ldsm_x4_t(bfr, Ys + (k0 + rr + (mi & 1) * 8) * kYPitch + n2 * 16 + (mi >> 1) * 8);
          mma16816(acc[2 * n2], a, bfr[0], bfr[1]);
          mma16816(acc[2 * n2 + 1], a, bfr[2], bfr[3]);
        }
      }
    }
    // epilogue: correction, gated RMSNorm over this warp's group (1024 channels)
    uint16_t* zs = Zs + warp * 1024;                    // this warp's z rows, then its output rows
    const uint16_t* ns = Ns + warp * 1024;
    float xv[8][4];
    float ss = 0.f;
    const int ia = grp * 16 + gq, ib = ia + 8;          // heads (global)
    const int la = gq, lb = gq + 8;                      // heads within the group
    const float ga = has_ad ? h2f(f2h(gate * h2f(ad.g[ia]))) : 0.f;
    const float gb = has_ad ? h2f(f2h(gate * h2f(ad.g[ib]))) : 0.f;
    const __half2 ga2 = __float2half2_rn(ga), gb2 = __float2half2_rn(gb);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int p0 = n * 8 + 2 * tq;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int i = half ? ib : ia, li = half ? lb : la;
        const float2 x2 = resurface_pair(*reinterpret_cast<const uint32_t*>(Ys + i * kYPitch + p0),
                                         *reinterpret_cast<const uint32_t*>(zs + swz64(li, p0)), acc[n][2 * half],
                                         acc[n][2 * half + 1], half ? gb2 : ga2, has_ad);
        xv[n][2 * half] = x2.x;
        xv[n][2 * half + 1] = x2.y;
        ss += x2.x * x2.x;
        ss += x2.y * x2.y;
      }
    }
    ss = warp_sum(ss);
    const float rstd = 1.0f / sqrtf(ss / 1024.0f + eps);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int p0 = n * 8 + 2 * tq;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int li = half ? lb : la;
        const float2 w2 = __half22float2(*reinterpret_cast<const __half2*>(ns + swz64(li, p0)));
        const float o0 = (xv[n][2 * half] * rstd) * w2.x;
        const float o1 = (xv[n][2 * half + 1] * rstd) * w2.y;
        *reinterpret_cast<__half2*>(zs + swz64(li, p0)) = __floats2half2_rn(o0, o1);   // z already read
      }
    }
    __syncwarp();
    uint4* og = reinterpret_cast<uint4*>(out + (long long)t * 8192 + grp * 1024);
#pragma unroll
    for (int i = lane; i < 128; i += 32) og[i] = *reinterpret_cast<const uint4*>(zs + swz64(i >> 3, (i & 7) * 8));
  }
}

__global__ void ce_finalize_kernel(const float2* __restrict__ part, int nt, const float* __restrict__ tl,
                                   int rows, float* __restrict__ nll) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float2* p = part + (long long)row * nt;
  float mx = -INFINITY;
  for (int i = lane; i < nt; i += 32) mx = fmaxf(mx, p[i].x);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = 0.f;
  for (int i = lane; i < nt; i += 32) { float2 v = p[i]; if (v.y > 0.f) s += v.y * expf(v.x - mx); }
  s = warp_sum(s);
  if (lane == 0) nll[row] = (mx + logf(s)) - tl[row];
}

__global__ void window_sum_kernel(const float* __restrict__ nll, int per, const int* __restrict__ counts,
                                  double* __restrict__ out) {
  __shared__ double red[256];
  const int w = blockIdx.x;
  const int n = counts[w];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += (double)nll[(long long)w * per + i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o; o >>= 1) {
    if ((int)threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[w] = red[0];
}

// first-occurrence argmax in two stages: per (row, slice) partials, then per row
constexpr int kArgSlice = 4096;
__global__ void argmax_partial_kernel(const uint16_t* __restrict__ logits, int V, long long ld,
                                      float* __restrict__ pv, int* __restrict__ pi, int nslice) {
  __shared__ float sv[256];
  __shared__ int si[256];
  const int row = blockIdx.y, sl = blockIdx.x;
  const uint16_t* r = logits + (long long)row * ld;
  float best = -INFINITY; int idx = 0x7fffffff;
  const int end = min(V, (sl + 1) * kArgSlice);
  for (int i = sl * kArgSlice + threadIdx.x; i < end; i += blockDim.x) {
    const float v = h2f(r[i]);
    if (v > best) { best = v; idx = i; }
  }
  sv[threadIdx.x] = best; si[threadIdx.x] = idx;
  __syncthreads();
  for (int o = blockDim.x / 2; o; o >>= 1) {
    if ((int)threadIdx.x < o) argmax_merge(sv[threadIdx.x], si[threadIdx.x], sv[threadIdx.x + o], si[threadIdx.x + o]);
    __syncthreads();
  }
  if (threadIdx.x == 0) { pv[row * nslice + sl] = sv[0]; pi[row * nslice + sl] = si[0]; }
}
__global__ void argmax_final_kernel(const float* __restrict__ pv, const int* __restrict__ pi, int nslice,
                                    long long* __restrict__ out) {
  const int row = blockIdx.x, lane = threadIdx.x;
  float best = -INFINITY; int idx = 0x7fffffff;
  for (int i = lane; i < nslice; i += 32) argmax_merge(best, idx, pv[row * nslice + i], pi[row * nslice + i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    argmax_merge(best, idx, v2, i2);
  }
  if (lane == 0) out[row] = idx == 0x7fffffff ? 0 : idx;
}

int g_sms = 0;
int num_sms() {
  if (!g_sms) { int d = 0; cudaGetDevice(&d); cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, d); }
  return g_sms > 0 ? g_sms : 148;
}

}  // namespace

int launch_add_rmsnorm(const uint16_t* h, uint16_t* res, int has_res, const uint16_t* w, float eps,
                       uint16_t* out, int rows, int D, cudaStream_t st) {
  if (rows <= 0 || D % 8 || D > 8192) return kEInval;
  add_rmsnorm_kernel<<<rows, 256, 0, st>>>(h, res, has_res, w, eps, out, D);
  return launch_status();
}

int launch_conv_prefill(const uint16_t* raw, long long raw_sb, long long raw_st, int B, int L, int C,
                        const uint16_t* w, const uint16_t* bias, uint16_t* cache, long long cache_sb,
                        int pos0, uint16_t* out, long long out_sb, long long out_st, cudaStream_t st) {
  if (B <= 0 || L <= 0 || C <= 0 || pos0 < 0) return kEInval;
  dim3 grid((C + 255) / 256, (L + kConvChunk - 1) / kConvChunk, B);
  conv_prefill_kernel<<<grid, 256, 0, st>>>(raw, raw_sb, raw_st, B, L, C, w, bias, cache, cache_sb, pos0, out,
                                            out_sb, out_st);
  return launch_status();
}

template <int GPB>
int launch_rg(const uint16_t* y, const uint16_t* z, long long z_st, const uint16_t* u, long long u_st,
              const AdapterPtrs& a, int has_ad, const uint16_t* norm_w, float eps, uint16_t* out, int T, int ty,
              cudaStream_t st) {
  const size_t smem = (size_t)(128 * kYPitch + GPB * 16 * kVPitch + 2 * GPB * 1024 + 2 * 4096) * 2;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(resurface_gatednorm_kernel<GPB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return kECuda;
    attr = true;
  }
  if (!y) return kOk;                                // prepare-only call
  dim3 grid(8 / GPB, ty);
  resurface_gatednorm_kernel<GPB><<<grid, 32 * GPB, smem, st>>>(y, z, z_st, u, u_st, a, has_ad, norm_w, eps, out, T);
  return launch_status();
}

int prepare_layer_kernels() {
  AdapterPtrs a{};
  int st = launch_rg<1>(nullptr, nullptr, 0, nullptr, 0, a, 0, nullptr, 0.f, nullptr, 0, 0, 0) |
           launch_rg<8>(nullptr, nullptr, 0, nullptr, 0, a, 0, nullptr, 0.f, nullptr, 0, 0, 0);
  return st ? kECuda : kOk;
}

int launch_resurface_gatednorm(const uint16_t* y, const uint16_t* z, long long z_st, const uint16_t* u,
                               long long u_st, const AdapterPtrs* ad, const uint16_t* norm_w, float eps,
                               uint16_t* out, int T, cudaStream_t st) {
  if (T <= 0) return kEInval;
  if (((uintptr_t)y % 16) || ((uintptr_t)z % 16) || ((uintptr_t)u % 16) || ((uintptr_t)norm_w % 16) ||
      ((uintptr_t)out % 16) ||
      (z_st % 8) || (u_st % 8))
    return kEInval;
  const int has_ad = ad && ad->V;
  AdapterPtrs a{};
  if (has_ad) {
    a = *ad;
    if (((uintptr_t)a.V % 16) || ((uintptr_t)a.w % 16)) return kEInval;
  }
  // few tokens: one warp (one norm group) per CTA spreads a token over 8 SMs;
  // many tokens: 8 warps per CTA share one staged copy of each token's y
  if (T < 64) return launch_rg<1>(y, z, z_st, u, u_st, a, has_ad, norm_w, eps, out, T, T, st);
  const int ty = T < 2 * num_sms() ? T : 2 * num_sms();
  return launch_rg<8>(y, z, z_st, u, u_st, a, has_ad, norm_w, eps, out, T, ty, st);
}

int launch_ce_finalize(const float2* partials, int ntiles, const float* tlogit, int rows, float* nll,
                       cudaStream_t st) {
  if (rows <= 0 || ntiles <= 0) return kEInval;
  ce_finalize_kernel<<<(rows + 7) / 8, 256, 0, st>>>(partials, ntiles, tlogit, rows, nll);
  return launch_status();
}

int launch_window_sum(const float* nll, int windows, int per, const int* counts, double* out, cudaStream_t st) {
  if (windows <= 0 || per <= 0) return kEInval;
  window_sum_kernel<<<windows, 256, 0, st>>>(nll, per, counts, out);
  return launch_status();
}

int argmax_workspace_bytes(int rows, int V) {
  const int ns = (V + kArgSlice - 1) / kArgSlice;
  return rows * ns * 8;
}

int launch_argmax(const uint16_t* logits, int rows, int V, long long ld, long long* out, void* ws, cudaStream_t st) {
  if (rows <= 0 || V <= 0 || !ws) return kEInval;
  const int ns = (V + kArgSlice - 1) / kArgSlice;
  float* pv = reinterpret_cast<float*>(ws);
  int* pi = reinterpret_cast<int*>(pv + rows * ns);
  argmax_partial_kernel<<<dim3(ns, rows), 256, 0, st>>>(logits, V, ld, pv, pi, ns);
  argmax_final_kernel<<<rows, 32, 0, st>>>(pv, pi, ns, out);
  return launch_status();
}

}  // namespace sq
