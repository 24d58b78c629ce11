// Packed-resident FP4-E2M1 G16 weights: exact decode, skinny GEMM ("GEMV") on
// the tensor cores, and the embedding row gather.
//
// Decode semantics (mamba2_recall/fp4.py:100-103, 125-130, 151-154):
//   w = FP16( FP32( FP32(E2M1[code&7] * sign(code&8) * E4M3(block)) * global_f32 ) )
// with the low nibble of each byte holding the even input column and one E4M3
// block scale per 16 consecutive input columns.  E2M1 * E4M3 is exact in fp32;
// the product with the fp32 global scale rounds once to fp32 and then to fp16.
#include "common.cuh"
#include "fp4.cuh"

namespace sq {
namespace {

// Hardware conversions (sm_100a): four code bytes -> four f16x2 magnitudes*sign
// (element 2i in the low half), and one E4M3 byte -> {v, v} as f16x2.  Both are exact:
// every E2M1 and E4M3 value is representable in fp16.
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n.reg .b8 q0, q1, q2, q3;\nmov.b32 {q0, q1, q2, q3}, %4;\n"
      "cvt.rn.f16x2.e2m1x2 %0, q0;\ncvt.rn.f16x2.e2m1x2 %1, q1;\n"
      "cvt.rn.f16x2.e2m1x2 %2, q2;\ncvt.rn.f16x2.e2m1x2 %3, q3;\n}\n"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3]) : "r"(w));
}
__device__ __forceinline__ uint32_t e4m3_splat_f16x2(uint32_t byte) {
  uint32_t r;
  const uint16_t two = (uint16_t)(byte | (byte << 8));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;\n" : "=r"(r) : "h"(two));
  return r;
}

// Exact decode of one code pair: FP16(FP32(FP32(m*b)*g)).  m*b is exact in fp16 (<= 6
// significant bits, |m*b| <= 2688, >= 2^-10), so HMUL2 gives it exactly; the product with
// the fp32 global scale is then rounded once to fp32 and once to fp16, as the reference.
__device__ __forceinline__ uint32_t scale_pair(uint32_t m16x2, uint32_t b16x2, float2 g2) {
  __half2 p = __hmul2(*reinterpret_cast<__half2*>(&m16x2), *reinterpret_cast<__half2*>(&b16x2));
  const float2 f = __fmul2_rn(__half22float2(p), g2);
  __half2 r = __float22half2_rn(f);
  return *reinterpret_cast<uint32_t*>(&r);
}

__global__ void fp4_decode_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                  const float* __restrict__ gptr, long long rows, int cols,
                                  uint16_t* __restrict__ out, long long ldo) {
  // one thread = 8 consecutive elements (4 code bytes, one block scale)
  const long long per_row = cols / 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * per_row) return;
  const long long r = idx / per_row;
  const int c8 = (int)(idx - r * per_row);
  const float g = *gptr;
  const float2 g2 = make_float2(g, g);
  const uint32_t w = *reinterpret_cast<const uint32_t*>(codes + r * (cols / 2) + c8 * 4);
  const uint32_t bs = e4m3_splat_f16x2(scales[r * (cols / 16) + (c8 >> 1)]);
  uint32_t m[4];
  e2m1x8_to_f16x2(w, m);
  uint4 o;
  o.x = scale_pair(m[0], bs, g2);
  o.y = scale_pair(m[1], bs, g2);
  o.z = scale_pair(m[2], bs, g2);
  o.w = scale_pair(m[3], bs, g2);
  *reinterpret_cast<uint4*>(out + r * ldo + c8 * 8) = o;
}

__global__ void fp4_embed_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                 const float* __restrict__ gptr, int vocab, int cols,
                                 const long long* __restrict__ ids, int ntok, uint16_t* __restrict__ out,
                                 int* __restrict__ err) {
  const int t = blockIdx.x;
  if (t >= ntok) return;
  long long id = ids[t];
  if (id < 0 || id >= vocab) { if (threadIdx.x == 0) atomicOr(err, (int)kDevBadArgs); id = 0; }
  const float g = *gptr;
  const float2 g2 = make_float2(g, g);
  for (int c8 = threadIdx.x; c8 < cols / 8; c8 += blockDim.x) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(codes + id * (cols / 2) + c8 * 4);
    const uint32_t bs = e4m3_splat_f16x2(scales[id * (cols / 16) + (c8 >> 1)]);
    uint32_t m[4];
    e2m1x8_to_f16x2(w, m);
    uint4 o;
    o.x = scale_pair(m[0], bs, g2);
    o.y = scale_pair(m[1], bs, g2);
    o.z = scale_pair(m[2], bs, g2);
    o.w = scale_pair(m[3], bs, g2);
    *reinterpret_cast<uint4*>(out + (long long)t * cols + c8 * 8) = o;
  }
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Skinny GEMM Y[M,N] = X[M,K] . W[N,K]^T for M <= 8*MT.  A CTA owns 16 weight
// rows and KS warps split K; each warp streams 128-column chunks (64 code bytes
// per row), decodes them exactly into mma.sync A fragments, and multiplies
// against X.  K positions are permuted consistently between the A and B
// fragments so that every lane reads 16 contiguous code bytes per row.
template <int MT, int KS>
__global__ void __launch_bounds__(32 * KS)
fp4_gemv_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                const float* __restrict__ gptr, int N, int K,
                const uint16_t* __restrict__ X, long long ldx, int M,
                uint16_t* __restrict__ Y, long long ldy) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int n0 = blockIdx.x * 16;
  const float gsc = *gptr;
  const float2 g2 = make_float2(gsc, gsc);
  const int nchunks = K / 128;
  const int per = (nchunks + KS - 1) / KS;
  const int c_begin = warp * per, c_end = min(nchunks, c_begin + per);
  const int rA = min(n0 + gq, N - 1), rB = min(n0 + gq + 8, N - 1);
  const uint8_t* codeA = codes + (long long)rA * (K / 2) + tq * 16;
  const uint8_t* codeB = codes + (long long)rB * (K / 2) + tq * 16;
  const uint8_t* scA = scales + (long long)rA * (K / 16) + tq * 2;
  const uint8_t* scB = scales + (long long)rB * (K / 16) + tq * 2;
  float acc[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  uint4 ca, cb; uint16_t sa, sb;
  if (c_begin < c_end) {
    ca = __ldg(reinterpret_cast<const uint4*>(codeA + (long long)c_begin * 64));
    cb = __ldg(reinterpret_cast<const uint4*>(codeB + (long long)c_begin * 64));
    sa = __ldg(reinterpret_cast<const uint16_t*>(scA + (long long)c_begin * 8));
    sb = __ldg(reinterpret_cast<const uint16_t*>(scB + (long long)c_begin * 8));
  }
  for (int c = c_begin; c < c_end; ++c) {
    const uint4 cca = ca, ccb = cb; const uint16_t ssa = sa, ssb = sb;
    if (c + 1 < c_end) {
      ca = __ldg(reinterpret_cast<const uint4*>(codeA + (long long)(c + 1) * 64));
      cb = __ldg(reinterpret_cast<const uint4*>(codeB + (long long)(c + 1) * 64));
      sa = __ldg(reinterpret_cast<const uint16_t*>(scA + (long long)(c + 1) * 8));
      sb = __ldg(reinterpret_cast<const uint16_t*>(scB + (long long)(c + 1) * 8));
    }
    const uint32_t wa[4] = {cca.x, cca.y, cca.z, cca.w};
    const uint32_t wb[4] = {ccb.x, ccb.y, ccb.z, ccb.w};
    const uint32_t bsa0 = e4m3_splat_f16x2(ssa & 0xFF), bsa1 = e4m3_splat_f16x2(ssa >> 8);
    const uint32_t bsb0 = e4m3_splat_f16x2(ssb & 0xFF), bsb1 = e4m3_splat_f16x2(ssb >> 8);
    const int kbase = c * 128 + tq * 32;       // physical k of this lane's 32 elements
#pragma unroll
    for (int w4 = 0; w4 < 4; ++w4) {           // one 32-bit code word = 2 mma k-steps per row
      uint32_t ma[4], mb[4];
      e2m1x8_to_f16x2(wa[w4], ma);
      e2m1x8_to_f16x2(wb[w4], mb);
      const uint32_t bsA = (w4 < 2) ? bsa0 : bsa1, bsB = (w4 < 2) ? bsb0 : bsb1;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
      const int j = w4 * 2 + jj;
      uint32_t a[4];
      a[0] = scale_pair(ma[2 * jj], bsA, g2);
      a[1] = scale_pair(mb[2 * jj], bsB, g2);
      a[2] = scale_pair(ma[2 * jj + 1], bsA, g2);
      a[3] = scale_pair(mb[2 * jj + 1], bsB, g2);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int m = mt * 8 + gq;
        uint32_t b0 = 0, b1 = 0;
        if (m < M) {
          const uint2 xv = __ldg(reinterpret_cast<const uint2*>(X + (long long)m * ldx + kbase + 4 * j));
          b0 = xv.x; b1 = xv.y;
        }
        mma16816(acc[mt], a, b0, b1);
      }
      }
    }
  }
  // reduce the KS partial tiles through shared memory
  __shared__ float red[KS][MT][32][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][mt][lane][i] = acc[mt][i];
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      for (int w = 0; w < KS; ++w)
#pragma unroll
        for (int i = 0; i < 4; ++i) s[i] += red[w][mt][lane][i];
      const int m0 = mt * 8 + 2 * tq;
      const int na = n0 + gq, nb = n0 + gq + 8;
      if (m0 < M && na < N) Y[(long long)m0 * ldy + na] = f2h(s[0]);
      if (m0 + 1 < M && na < N) Y[(long long)(m0 + 1) * ldy + na] = f2h(s[1]);
      if (m0 < M && nb < N) Y[(long long)m0 * ldy + nb] = f2h(s[2]);
      if (m0 + 1 < M && nb < N) Y[(long long)(m0 + 1) * ldy + nb] = f2h(s[3]);
    }
  }
}

template <int MT>
int gemv_mt(const Fp4Weight& W, const uint16_t* X, long long ldx, int M, uint16_t* Y, long long ldy,
            cudaStream_t st) {
  const int grid = (W.rows + 15) / 16;
  const int chunks = W.cols / 128;
  if (chunks >= 64) {
    fp4_gemv_kernel<MT, 8><<<grid, 256, 0, st>>>(W.codes, W.scales, W.global_scale, W.rows, W.cols, X, ldx, M, Y, ldy);
  } else {
    fp4_gemv_kernel<MT, 4><<<grid, 128, 0, st>>>(W.codes, W.scales, W.global_scale, W.rows, W.cols, X, ldx, M, Y, ldy);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kECuda;
}

}  // namespace

int launch_fp4_decode(const Fp4Weight& W, uint16_t* out, long long ldo, cudaStream_t st) {
  if (W.rows <= 0 || W.cols <= 0 || W.cols % 16 || ldo < W.cols || ldo % 8) return kEInval;
  const long long n = (long long)W.rows * (W.cols / 8);
  const int th = 256;
  fp4_decode_kernel<<<(unsigned)((n + th - 1) / th), th, 0, st>>>(W.codes, W.scales, W.global_scale, W.rows,
                                                                   W.cols, out, ldo);
  return cudaGetLastError() == cudaSuccess ? kOk : kECuda;
}

int launch_fp4_embed(const Fp4Weight& E, const long long* ids, int ntok, uint16_t* out, int* err, cudaStream_t st) {
  if (E.cols % 16 || ntok <= 0) return kEInval;
  fp4_embed_kernel<<<ntok, 256, 0, st>>>(E.codes, E.scales, E.global_scale, E.rows, E.cols, ids, ntok, out, err);
  return cudaGetLastError() == cudaSuccess ? kOk : kECuda;
}

int launch_fp4_gemv(const Fp4Weight& W, const uint16_t* X, long long ldx, int M, uint16_t* Y, long long ldy,
                    cudaStream_t st) {
  if (M <= 0 || M > 64 || W.cols % 128 || ldx % 4) return kEInval;
  if (M <= 8) return gemv_mt<1>(W, X, ldx, M, Y, ldy, st);
  if (M <= 16) return gemv_mt<2>(W, X, ldx, M, Y, ldy, st);
  if (M <= 32) return gemv_mt<4>(W, X, ldx, M, Y, ldy, st);
  return gemv_mt<8>(W, X, ldx, M, Y, ldy, st);
}

}  // namespace sq
