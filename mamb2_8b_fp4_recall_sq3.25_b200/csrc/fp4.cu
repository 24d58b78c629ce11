// Packed-resident FP4-E2M1 G16 weights: exact decode, skinny GEMM ("GEMV") on
// the tensor cores, and the embedding row gather.
//
// Decode semantics (mamba2_recall/fp4.py:100-103, 125-130, 151-154):
//   w = FP16( FP32( FP32(E2M1[code&7] * sign(code&8) * E4M3(block)) * global_f32 ) )
// with the low nibble of each byte holding the even input column and one E4M3
// block scale per 16 consecutive input columns.  E2M1 * E4M3 is exact in fp32;
// the product with the fp32 global scale rounds once to fp32 and then to fp16.
#include "common.cuh"
#include "device_util.cuh"
#include "fp4.cuh"

namespace sq {
namespace {

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

// decode_packet's checks (mamba2_recall/fp4.py:235-249) over a packed matrix, one thread per
// 16-column group: bit 1 = a block scale that is negative or NaN ('Invalid stored scale'),
// bit 2 = a nonzero code (other than +-0) in a zero-scale group, bit 4 = a decoded weight
// that is not finite in fp16.
__global__ void fp4_validate_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                    const float* __restrict__ gptr, long long rows, int cols, int* __restrict__ flags) {
  const long long groups = rows * (cols / 16);
  const float g = *gptr;
  const float2 g2 = make_float2(g, g);
  int bad = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < groups;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / (cols / 16);
    const int gcol = (int)(i - r * (cols / 16));
    const uint8_t sb = scales[i];
    if ((sb & 0x7F) == 0x7F || ((sb & 0x80) && (sb & 0x7F))) bad |= 1;
    const uint4 w = *reinterpret_cast<const uint4*>(codes + r * (cols / 2) + gcol * 8);
    const uint32_t ws[2] = {w.x, w.y};
    if ((sb & 0x7F) == 0) {
      // every nibble must be 0 or 8 (+0 / -0)
      if (((ws[0] | ws[1]) & 0x77777777u) != 0) bad |= 2;
    } else {
      const uint32_t bs = e4m3_splat_f16x2(sb);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint32_t m[4];
        e2m1x8_to_f16x2(ws[q], m);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t v = scale_pair(m[k], bs, g2);
          // fp16 exponent all ones: inf or NaN
          if ((v & 0x7C00u) == 0x7C00u || (v & 0x7C000000u) == 0x7C000000u) bad |= 4;
        }
      }
    }
  }
  if (bad) atomicOr(flags, bad);
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

// ---------------------------------------------------------------------------------------
// Streaming skinny GEMM for M <= 8*MT, the decode-time projection kernel.
// Warp 0 (one lane) streams row tiles of 16 weight rows x KC columns (codes + block
// scales) into a STAGES-deep shared-memory ring with cp.async.bulk (non-multicast) and
// mbarrier transaction counts; warps 1..4 decode each stage exactly into mma.sync A
// fragments and multiply with X.  Every mbarrier wait is bounded (%globaltimer); on
// expiry the warp records an error bit and leaves.
constexpr int kGvRows = 16, kGvKC = 1024, kGvStages = 6, kGvConsumers = 4;
constexpr int kGvCodeBytes = kGvRows * kGvKC / 2;          // 8 KB
constexpr int kGvScaleBytes = kGvRows * kGvKC / 16;        // 1 KB
constexpr int kGvStageBytes = kGvCodeBytes + kGvScaleBytes;
constexpr unsigned long long kGvWaitNs = 2000000000ull;

__device__ __forceinline__ uint64_t gv_time() { uint64_t t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }
__device__ __forceinline__ bool gv_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok) : "r"(a), "r"(parity) : "memory");
  return ok != 0;
}
// Limit of the pipeline's waits (producer on a free stage, consumers on a loaded one),
// settable per device for failure-detection tests (set_gemv_wait_limit_ns).  The drain
// waits after an expiry keep the fixed kGvWaitNs, so copies already in flight always land
// before the CTA exits.
// A limit below kGvTimerNs (shorter than %globaltimer can resolve) makes the wait a single
// non-blocking test of the phase (mbarrier.try_wait itself may suspend the thread for a
// while before it reports an incomplete phase).
__device__ unsigned long long g_gv_wait_ns = kGvWaitNs;
constexpr unsigned long long kGvTimerNs = 2000;
__device__ __forceinline__ bool gv_test(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n.reg .pred p;\nmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok) : "r"(a), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool gv_wait_for(uint32_t a, uint32_t parity, unsigned long long limit) {
  if (limit < kGvTimerNs) return gv_test(a, parity);
  if (gv_try(a, parity)) return true;
  const uint64_t t0 = gv_time();
  for (;;) {
    for (int i = 0; i < 32; ++i) if (gv_try(a, parity)) return true;
    if (gv_time() - t0 > limit) return false;
  }
}
__device__ __forceinline__ bool gv_wait(uint32_t a, uint32_t parity) { return gv_wait_for(a, parity, g_gv_wait_ns); }
__device__ __forceinline__ bool gv_drain_wait(uint32_t a, uint32_t parity) { return gv_wait_for(a, parity, kGvWaitNs); }

__device__ __forceinline__ void gv_tma2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      :: "r"(dst), "l"(map), "r"(bar), "r"(x), "r"(y) : "memory");
}

// EXACT: every weight is decoded to FP16(FP32(m*b)*g) before the product (the reference's
// decoded-weight numerics).  Otherwise the exact fp16 products m*b enter the MMA and the
// fp32 global scale multiplies each fp32 accumulator once (factored scale): the weight seen
// by the product is then m*b*g unrounded instead of its fp16 rounding, one instruction per
// weight instead of about three.
template <int MT, bool EXACT>
__global__ void __launch_bounds__(32 * (1 + kGvConsumers))
fp4_gemv_stream_kernel(const __grid_constant__ CUtensorMap mcodes, const __grid_constant__ CUtensorMap mscales,
                       const float* __restrict__ gptr, int N, int K, int KC,
                       const uint16_t* __restrict__ X, long long ldx, int M,
                       uint16_t* __restrict__ Y, long long ldy, int* err) {
  extern __shared__ __align__(128) unsigned char gsm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(gsm + kGvStages * kGvStageBytes);
  uint64_t* empty = full + kGvStages;
  float* red = reinterpret_cast<float*>(empty + kGvStages);          // [consumers][MT][32][4]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(gsm);
  const uint32_t fbar = (uint32_t)__cvta_generic_to_shared(full);
  const uint32_t ebar = (uint32_t)__cvta_generic_to_shared(empty);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGvStages; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(fbar + 8 * i) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(ebar + 8 * i), "r"(kGvConsumers) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int tiles = (N + kGvRows - 1) / kGvRows;
  const int kchunks = K / KC;
  const int code_row = KC / 2, scale_row = KC / 16;
  if (warp == 0) {
    if (lane == 0) {
      int stage = 0; uint32_t phase = 0; int issued = 0; bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        for (int kc = 0; kc < kchunks; ++kc) {
          if (!gv_wait(ebar + 8 * stage, phase ^ 1)) { ok = false; break; }
          const uint32_t fb = fbar + 8 * stage;
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                       :: "r"(fb), "r"((uint32_t)(kGvRows * (code_row + scale_row))) : "memory");
          const uint32_t cdst = sbase + stage * kGvStageBytes, sdst = cdst + kGvCodeBytes;
          // one 16-row box each; x in u32 units (16-byte multiples), rows past N read zeros
          gv_tma2d(cdst, &mcodes, fb, kc * (code_row / 4), tile * kGvRows);
          gv_tma2d(sdst, &mscales, fb, kc * (scale_row / 4), tile * kGvRows);
          ++issued;
          if (++stage == kGvStages) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        atomicOr(err, (int)kDevTimeoutProducer);
        for (int i = 0; i < kGvStages && issued > 0; ++i, --issued) {   // drain own copies
          if (--stage < 0) { stage = kGvStages - 1; phase ^= 1; }
          gv_drain_wait(fbar + 8 * stage, phase);
        }
      }
    }
    return;
  }
  // ------------------------------------------------------------------ consumers
  const int cw = warp - 1;
  const int gq = lane >> 2, tq = lane & 3;
  const float gsc = *gptr;
  const float2 g2 = make_float2(gsc, gsc);
  const int subs = KC / 128;                      // 128-column sub-chunks per stage
  int stage = 0; uint32_t phase = 0; bool ok = true;
  for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    float acc[MT][4], acc2[MT][4];          // two accumulator chains (even / odd k-steps)
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][e] = acc2[i][e] = 0.f;
    for (int kc = 0; kc < kchunks; ++kc) {
      if (ok && !gv_wait(fbar + 8 * stage, phase)) ok = false;
      if (ok) {
        const unsigned char* cs = gsm + stage * kGvStageBytes;
        const unsigned char* ss = cs + kGvCodeBytes;
        for (int sub = cw; sub < subs; sub += kGvConsumers) {
          // all X (B-fragment) data of this sub-chunk first: 32 consecutive k per lane per m
          const int kb0 = kc * KC + sub * 128 + tq * 32;
          uint4 xr[MT][4];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int m = mt * 8 + gq;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              xr[mt][q] = (m < M) ? __ldg(reinterpret_cast<const uint4*>(X + (long long)m * ldx + kb0 + 8 * q))
                                  : make_uint4(0, 0, 0, 0);
          }
          const uint4 ca = *reinterpret_cast<const uint4*>(cs + gq * code_row + sub * 64 + tq * 16);
          const uint4 cb = *reinterpret_cast<const uint4*>(cs + (gq + 8) * code_row + sub * 64 + tq * 16);
          const uint16_t sa = *reinterpret_cast<const uint16_t*>(ss + gq * scale_row + sub * 8 + tq * 2);
          const uint16_t sb = *reinterpret_cast<const uint16_t*>(ss + (gq + 8) * scale_row + sub * 8 + tq * 2);
          const uint32_t wa[4] = {ca.x, ca.y, ca.z, ca.w};
          const uint32_t wb[4] = {cb.x, cb.y, cb.z, cb.w};
          const uint32_t bsa0 = e4m3_splat_f16x2(sa & 0xFF), bsa1 = e4m3_splat_f16x2(sa >> 8);
          const uint32_t bsb0 = e4m3_splat_f16x2(sb & 0xFF), bsb1 = e4m3_splat_f16x2(sb >> 8);
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            uint32_t ma[4], mb[4];
            e2m1x8_to_f16x2(wa[w4], ma);
            e2m1x8_to_f16x2(wb[w4], mb);
            const uint32_t bsA = (w4 < 2) ? bsa0 : bsa1, bsB = (w4 < 2) ? bsb0 : bsb1;
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const int j = w4 * 2 + jj;
              uint32_t a[4];
              if (EXACT) {
                a[0] = scale_pair(ma[2 * jj], bsA, g2);
                a[1] = scale_pair(mb[2 * jj], bsB, g2);
                a[2] = scale_pair(ma[2 * jj + 1], bsA, g2);
                a[3] = scale_pair(mb[2 * jj + 1], bsB, g2);
              } else {
                a[0] = hmul2_u32(ma[2 * jj], bsA);
                a[1] = hmul2_u32(mb[2 * jj], bsB);
                a[2] = hmul2_u32(ma[2 * jj + 1], bsA);
                a[3] = hmul2_u32(mb[2 * jj + 1], bsB);
              }
#pragma unroll
              for (int mt = 0; mt < MT; ++mt) {
                // x[m][kb0 + 4j .. +3] = 16-byte word j/2, half (j&1)
                const uint4 xq = xr[mt][j >> 1];
                const uint32_t b0 = (j & 1) ? xq.z : xq.x, b1 = (j & 1) ? xq.w : xq.y;
                mma16816((j & 1) ? acc2[mt] : acc[mt], a, b0, b1);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(ebar + 8 * stage) : "memory");
      }
      if (++stage == kGvStages) { stage = 0; phase ^= 1; }
    }
    // cross-warp reduction of the tile (consumers only: named barrier 1)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[((cw * MT + mt) * 32 + lane) * 4 + i] = acc[mt][i] + acc2[mt][i];
    asm volatile("bar.sync 1, %0;" :: "r"(32 * kGvConsumers) : "memory");
    if (cw == 0) {
      const int n0 = tile * kGvRows;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        float sacc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int w = 0; w < kGvConsumers; ++w)
#pragma unroll
          for (int i = 0; i < 4; ++i) sacc[i] += red[((w * MT + mt) * 32 + lane) * 4 + i];
        if (!EXACT)
#pragma unroll
          for (int i = 0; i < 4; ++i) sacc[i] *= gsc;
        const int m0 = mt * 8 + 2 * tq;
        const int na = n0 + gq, nb = n0 + gq + 8;
        if (m0 < M && na < N) Y[(long long)m0 * ldy + na] = f2h(sacc[0]);
        if (m0 + 1 < M && na < N) Y[(long long)(m0 + 1) * ldy + na] = f2h(sacc[1]);
        if (m0 < M && nb < N) Y[(long long)m0 * ldy + nb] = f2h(sacc[2]);
        if (m0 + 1 < M && nb < N) Y[(long long)(m0 + 1) * ldy + nb] = f2h(sacc[3]);
      }
    }
    asm volatile("bar.sync 1, %0;" :: "r"(32 * kGvConsumers) : "memory");
  }
  if (!ok && lane == 0) atomicOr(err, (int)kDevTimeoutEpilogue);
}

int g_gv_sms = 0;

int gemv_kc(int cols) {
  return (cols % kGvKC == 0) ? kGvKC : (cols % 512 == 0 ? 512 : (cols % 256 == 0 ? 256 : 0));
}

template <int MT, bool EXACT>
int gemv_stream(const Fp4Weight& W, const Fp4Maps* maps, const uint16_t* X, long long ldx, int M, uint16_t* Y,
                long long ldy, int* err, cudaStream_t st) {
  const int KC = gemv_kc(W.cols);
  if (!KC && W.codes) return kEInval;
  if (!g_gv_sms) {
    int d = 0; cudaGetDevice(&d);
    cudaDeviceGetAttribute(&g_gv_sms, cudaDevAttrMultiProcessorCount, d);
    if (g_gv_sms <= 0) g_gv_sms = 148;
  }
  const size_t smem = (size_t)kGvStages * kGvStageBytes + 2 * kGvStages * 8 + (size_t)kGvConsumers * MT * 32 * 16;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(fp4_gemv_stream_kernel<MT, EXACT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return kECuda;
    attr = true;
  }
  if (!W.codes) return kOk;                          // prepare-only call
  const int tiles = (W.rows + kGvRows - 1) / kGvRows;
  const int grid = tiles < 3 * g_gv_sms ? tiles : 3 * g_gv_sms;
  Fp4Maps local;
  if (!maps || !maps->valid || maps->kc != KC) {
    if (!make_fp4_maps(W, &local)) return kECuda;
    maps = &local;
  }
  fp4_gemv_stream_kernel<MT, EXACT><<<grid, 32 * (1 + kGvConsumers), smem, st>>>(
      maps->codes, maps->scales, W.global_scale, W.rows, W.cols, KC, X, ldx, M, Y, ldy, err);
  return launch_status();
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
  return launch_status();
}

}  // namespace

int launch_fp4_decode(const Fp4Weight& W, uint16_t* out, long long ldo, cudaStream_t st) {
  if (W.rows <= 0 || W.cols <= 0 || W.cols % 16 || ldo < W.cols || ldo % 8) return kEInval;
  const long long n = (long long)W.rows * (W.cols / 8);
  const int th = 256;
  fp4_decode_kernel<<<(unsigned)((n + th - 1) / th), th, 0, st>>>(W.codes, W.scales, W.global_scale, W.rows,
                                                                   W.cols, out, ldo);
  return launch_status();
}

int launch_fp4_validate(const Fp4Weight& W, int* flags, cudaStream_t st) {
  if (W.rows <= 0 || W.cols <= 0 || W.cols % 16 || ((uintptr_t)W.codes % 8) || !flags) return kEInval;
  const long long groups = (long long)W.rows * (W.cols / 16);
  const long long blocks = (groups + 255) / 256;
  fp4_validate_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, st>>>(
      W.codes, W.scales, W.global_scale, W.rows, W.cols, flags);
  return launch_status();
}

int launch_fp4_embed(const Fp4Weight& E, const long long* ids, int ntok, uint16_t* out, int* err, cudaStream_t st) {
  if (E.cols % 16 || ntok <= 0) return kEInval;
  fp4_embed_kernel<<<ntok, 256, 0, st>>>(E.codes, E.scales, E.global_scale, E.rows, E.cols, ids, ntok, out, err);
  return launch_status();
}

bool make_fp4_maps(const Fp4Weight& W, Fp4Maps* maps) {
  maps->valid = 0;
  const int KC = gemv_kc(W.cols);
  if (!KC || !W.codes || ((uintptr_t)W.codes % 16) || ((uintptr_t)W.scales % 16) || ((W.cols / 16) % 16))
    return false;
  maps->kc = KC;
  if (!encode_u32_map(&maps->codes, W.codes, W.rows, W.cols / 8, W.cols / 2, KC / 8, kGvRows)) return false;
  if (!encode_u32_map(&maps->scales, W.scales, W.rows, W.cols / 64, W.cols / 16, KC / 64, kGvRows)) return false;
  maps->valid = 1;
  return true;
}

int prepare_fp4_kernels() {
  Fp4Weight none{nullptr, nullptr, nullptr, 0, 1024};
  int st = gemv_stream<1, true>(none, nullptr, nullptr, 0, 1, nullptr, 0, nullptr, 0) |
           gemv_stream<2, true>(none, nullptr, nullptr, 0, 1, nullptr, 0, nullptr, 0) |
           gemv_stream<4, true>(none, nullptr, nullptr, 0, 1, nullptr, 0, nullptr, 0) |
           gemv_stream<8, true>(none, nullptr, nullptr, 0, 1, nullptr, 0, nullptr, 0) |
           gemv_stream<1, false>(none, nullptr, nullptr, 0, 1, nullptr, 0, nullptr, 0) |
           gemv_stream<2, false>(none, nullptr, nullptr, 0, 1, nullptr, 0, nullptr, 0) |
           gemv_stream<4, false>(none, nullptr, nullptr, 0, 1, nullptr, 0, nullptr, 0) |
           gemv_stream<8, false>(none, nullptr, nullptr, 0, 1, nullptr, 0, nullptr, 0);
  return st ? kECuda : kOk;
}

int set_gemv_wait_limit_ns(unsigned long long ns) {
  const unsigned long long v = ns ? ns : kGvWaitNs;
  return cudaMemcpyToSymbol(g_gv_wait_ns, &v, sizeof(v)) == cudaSuccess ? kOk : kECuda;
}

int launch_fp4_gemv_stream(const Fp4Weight& W, const Fp4Maps* maps, const uint16_t* X, long long ldx, int M,
                           uint16_t* Y, long long ldy, int* err, cudaStream_t st, bool exact) {
  if (M <= 0 || M > 64 || W.cols % 256 || ldx % 8 || !err) return kEInval;
  if (((uintptr_t)W.codes % 16) || ((uintptr_t)W.scales % 16) || ((uintptr_t)X % 16) || ((W.cols / 16) % 16))
    return kEInval;
  if (exact) {
    if (M <= 8) return gemv_stream<1, true>(W, maps, X, ldx, M, Y, ldy, err, st);
    if (M <= 16) return gemv_stream<2, true>(W, maps, X, ldx, M, Y, ldy, err, st);
    if (M <= 32) return gemv_stream<4, true>(W, maps, X, ldx, M, Y, ldy, err, st);
    return gemv_stream<8, true>(W, maps, X, ldx, M, Y, ldy, err, st);
  }
  if (M <= 8) return gemv_stream<1, false>(W, maps, X, ldx, M, Y, ldy, err, st);
  if (M <= 16) return gemv_stream<2, false>(W, maps, X, ldx, M, Y, ldy, err, st);
  if (M <= 32) return gemv_stream<4, false>(W, maps, X, ldx, M, Y, ldy, err, st);
  return gemv_stream<8, false>(W, maps, X, ldx, M, Y, ldy, err, st);
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
