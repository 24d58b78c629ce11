// The FP16-state control scan (the reference's s16 mode), sm_100a.
//
// Semantics: mamba2_recall/state_codec.py:65-102 (_s16_scan) and the statistics reduction
// of its host wrapper (:256-262).  Per token: dt = softplus(dt + bias) (threshold 20),
// decay = exp(A dt), state = state * decay + (B * dt) * x, y = sum_n state * C + x * D
// (fp32, stored fp16), then the carry is rounded to fp16.  With statistics, every row sums
// |fp16 carry| over the tokens; rows are summed per 4-row tile, tiles per 16-row block.
//
// Mapping: four lanes per state row; lane l holds the 32 coordinates n = 8 i + 2 l + e
// (i < 16, e < 2) in fp32 registers.  That split makes the readout sum the reference's
// (numpy's pairwise order over 128: eight strided accumulators r_j = sum_i p[8 i + j] in
// order, combined ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7))): lane l owns r_2l and
// r_2l+1 and two shuffles combine the pairs in the reference's tree.  Products and sums are
// single-rounded (__fmul_rn / __fadd_rn), never contracted.  A CTA is 32 rows of one head;
// B and C of the head's group stream through shared memory one token at a time.
#include "common.cuh"
#include "s16.cuh"

namespace sq {
namespace {

constexpr int kRowsPerCta = 32;

template <bool STATS>
__global__ void __launch_bounds__(128) s16_scan_kernel(const S16Params P) {
  __shared__ float sB[2][128], sC[2][128];
  const int tid = threadIdx.x, lane = tid & 31, l = tid & 3;
  const int row = blockIdx.x * kRowsPerCta + (tid >> 2);           // p
  const int h = blockIdx.y, b = blockIdx.z;
  const int g = h / (P.heads / P.groups);
  const bool valid = row < P.dim;
  const long long srow = ((long long)b * P.heads + h) * P.dim + (valid ? row : 0);
  uint16_t* sp = P.state + srow * 128;
  float st[32];
  float acc[STATS ? 32 : 1];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t pair = valid ? *reinterpret_cast<const uint32_t*>(sp + 8 * i + 2 * l) : 0u;
    st[2 * i] = h2f((uint16_t)(pair & 0xFFFF));
    st[2 * i + 1] = h2f((uint16_t)(pair >> 16));
    if (STATS) acc[2 * i] = acc[2 * i + 1] = 0.f;
  }
  const float av = P.A[h];
  const float dv = P.d_is_f32 ? reinterpret_cast<const float*>(P.D)[h] : h2f(reinterpret_cast<const uint16_t*>(P.D)[h]);
  const float bias = P.dt_bias_is_f32 ? reinterpret_cast<const float*>(P.dt_bias)[h]
                                      : h2f(reinterpret_cast<const uint16_t*>(P.dt_bias)[h]);
  auto stage = [&](int t, int buf) {
    const uint16_t* bsrc = P.B + (long long)b * P.b_sb + (long long)t * P.b_st + g * 128;
    const uint16_t* csrc = P.C + (long long)b * P.c_sb + (long long)t * P.c_st + g * 128;
    sB[buf][tid] = h2f(bsrc[tid]);
    sC[buf][tid] = h2f(csrc[tid]);
  };
  stage(0, 0);
  for (int t = 0; t < P.length; ++t) {
    const int buf = t & 1;
    __syncthreads();                                                  // token t staged; t-1 consumed
    if (t + 1 < P.length) stage(t + 1, buf ^ 1);
    const float xv = valid ? h2f(P.x[(long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * P.dim + row]) : 0.f;
    float dtv = h2f(P.dt[(long long)b * P.dt_sb + (long long)t * P.dt_st + h]) + bias;
    dtv = dtv <= 20.0f ? logf(expf(dtv) + 1.0f) : dtv;
    const float dec = expf(av * dtv);
    float r0 = 0.f, r1 = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = 8 * i + 2 * l + e;
        const float db = __fmul_rn(sB[buf][n], dtv);
        const float s = __fadd_rn(__fmul_rn(st[2 * i + e], dec), __fmul_rn(db, xv));
        st[2 * i + e] = s;
        const float prod = __fmul_rn(s, sC[buf][n]);
        if (e == 0) r0 = (i == 0) ? prod : __fadd_rn(r0, prod);
        else        r1 = (i == 0) ? prod : __fadd_rn(r1, prod);
      }
    }
    // ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)): lane l holds r_2l + r_2l+1
    const float pr = __fadd_rn(r0, r1);
    // (IEEE addition is commutative, so every lane of the row gets the same bits)
    const float q = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 1));          // lanes 0,1: p0+p1; 2,3: p2+p3
    const float tot = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, q, 2));
    if (valid && l == 0) {
      const float out = __fadd_rn(tot, __fmul_rn(xv, dv));
      P.y[(long long)b * P.y_sb + (long long)t * P.y_st + (long long)h * P.dim + row] = f2h(out);
    }
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      st[k] = h2f(f2h(st[k]));
      if (STATS) acc[k] = __fadd_rn(acc[k], valid ? fabsf(st[k]) : 0.f);
    }
  }
  if (valid) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t pair = (uint32_t)f2h(st[2 * i]) | ((uint32_t)f2h(st[2 * i + 1]) << 16);
      *reinterpret_cast<uint32_t*>(sp + 8 * i + 2 * l) = pair;
    }
  }
  if (STATS) {
    // rows 4k..4k+3 of a tile are lanes 16k'.. of the warp: sum them in row order, then the
    // four tiles of a 16-row block (one warp = 8 rows = 2 tiles; a CTA = 2 blocks of 16)
    __shared__ float sT[kRowsPerCta / 4][128];
    const int r_in_tile = (tid >> 2) & 3;
    const int tile = tid >> 4;                                       // 0..7 within the CTA
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      float v = __shfl_sync(0xffffffffu, acc[k], (lane & ~15) | l);   // row 0 of the tile
#pragma unroll
      for (int r = 1; r < 4; ++r) v = __fadd_rn(v, __shfl_sync(0xffffffffu, acc[k], (lane & ~15) | (4 * r) | l));
      if (r_in_tile == 0) sT[tile][8 * (k >> 1) + 2 * l + (k & 1)] = v;
    }
    __syncthreads();
    // 32 rows = 2 statistics blocks of 16 rows (4 tiles each)
    const int nblocks = (min(P.dim - (int)blockIdx.x * kRowsPerCta, kRowsPerCta) + 15) / 16;
    for (int i = tid; i < 2 * 128; i += 128) {
      const int blk = i >> 7, n = i & 127;
      if (blk < nblocks) {
        float v = sT[4 * blk][n];
        for (int k = 1; k < 4; ++k) v = __fadd_rn(v, sT[4 * blk + k][n]);
        const int gblk = blockIdx.x * (kRowsPerCta / 16) + blk;
        P.stats[(((long long)b * P.heads + h) * ((P.dim + 15) / 16) + gblk) * 128 + n] = v;
      }
    }
  }
}

}  // namespace

int launch_s16_scan(const S16Params& P, cudaStream_t st) {
  if (P.batch <= 0 || P.length <= 0 || P.heads <= 0 || P.dim <= 0 || P.groups <= 0 || P.heads % P.groups)
    return kEInval;
  if (((uintptr_t)P.state & 3)) return kEInval;
  dim3 grid((P.dim + kRowsPerCta - 1) / kRowsPerCta, P.heads, P.batch);
  if (P.stats) s16_scan_kernel<true><<<grid, 128, 0, st>>>(P);
  else s16_scan_kernel<false><<<grid, 128, 0, st>>>(P);
  return launch_status();
}

}  // namespace sq
