// The legacy sq3p25 scan and its straight-through (STE) training backward, sm_100a.
//
// sq3p25: the fixed tier split of mamba2_recall/state_codec.py (`_sq_scan` :105-176): per
// recurrent row 16 INT8 + 64 INT4 stored coordinates (permuted order of the group's
// permutation) and 48 pruned ones that only read out the current token's update; 52 bytes
// per row (lo / hi u8[8], q4 u8[32], s8 / s4 fp16).  Per token: dt = softplus(dt + bias),
// decay = exp(A dt), S = S decay + (B dt) x on the 80 live lanes, y = sum S C (live) +
// sum ((B dt) x) C (pruned) + x D, then den = max(max|S| / limit, 1e-8) (fp32), q =
// clip(round_half_away(S / den), +-limit), S = q * fp16(den).
//
// STE backward (mamba2_recall/state_training_scan.py :24-221), from a fresh zero carry:
//   ste_checkpoint_kernel  replays the carries and stores the one entering every chunk of K
//                          tokens (workspace cp [B][NC][H][P][80] fp32);
//   ste_history_kernel     replays one chunk from its checkpoint, storing the carry entering
//                          each token (workspace hist [B][K][H][P][80]);
//   ste_backward_kernel    walks that chunk's tokens in reverse: the derivative passes
//                          through the requantisation as identity on the 80 live lanes and as
//                          zero through the 48 pruned ones (the adjoint carry adj
//                          [B][H][P][80] crosses chunks), the current-token readout through
//                          all 128; stores dx and d(dt) (times the softplus slope) and the
//                          per-(head, 16-row tile) partial sums of dB / dC;
//   ste_bc_reduce_kernel   adds the dB / dC partials of the chunk in (head, tile) order and
//                          scatters them to the original coordinates.
// Mapping: one CTA per (head, batch); four threads per row of the head (dim <= 128).  Thread
// `sub` of a row owns, in every tier block of n lanes, the lanes q with q % 8 in {2 sub,
// 2 sub + 1}: 4 INT8 + 16 INT4 stored coordinates (and 16 of the 64-wide pruned block), kept
// in registers.  The group's B / C of a token are staged in shared memory in tier order.
// Arithmetic is unfused (__fmul_rn / __fadd_rn) like the reference's, quotients are
// correctly rounded, and every reduction runs in the order of the reference kernels' golden
// runs (Triton interpreter, i.e. numpy): a sum over a row's lanes in numpy's eight-running-
// sum pairwise order (the owner of lanes q % 8 = 2 sub, 2 sub + 1 holds running sums 2 sub
// and 2 sub + 1 whole; two shuffles combine them as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7))),
// a tile's 16 rows for d(dt) in the same pairwise order, a tile's rows for dB / dC
// sequentially, tiles and heads in program order.  Given the same softplus / exp values the
// results are bit-identical to the golden runs; no atomics, so gradients are deterministic.
#include "common.cuh"
#include "ste.cuh"

namespace sq {
namespace {

constexpr int kLive8 = 16, kLive = 80;   // stored lanes (16 INT8, then 64 INT4); lanes 80..127 are pruned
constexpr int kTPR = 4;                                // threads per state row
constexpr int kOwn8 = 4, kOwn4 = 16, kOwn = kOwn8 + kOwn4, kOwnD = 16;   // lanes per thread

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float ldf(const void* p, int is_f32, int i) {
  return is_f32 ? reinterpret_cast<const float*>(p)[i] : h2f(reinterpret_cast<const uint16_t*>(p)[i]);
}
// round half away from zero; a negative value that rounds to zero gives +0
__device__ __forceinline__ float round_away(float q) {
  const float a = fabsf(q);
  float r = floorf(a);
  r = (a - r >= 0.5f) ? r + 1.0f : r;
  return q < 0.f ? 0.0f - r : r;
}
// RN(a / d) for a normal divisor d given inv = RN(1 / d): the remainder a - q0 d is exact in
// one FMA and one corrected step gives the correctly rounded quotient (Markstein).  Quotients
// below 0.5 in magnitude, the only ones that can be subnormal here, round to code 0 either way.
__device__ __forceinline__ float div_rn_inv(float a, float d, float inv) {
  const float q0 = fmul(a, inv);
  const float r = fmaf(-q0, d, a);
  return fmaf(r, inv, q0);
}
__device__ __forceinline__ float softplus20(float v) { return v <= 20.0f ? logf(fadd(expf(v), 1.0f)) : v; }

// Lane ownership: the thread's k-th lane of a tier block (k = 2 i + e) is q = 8 i + 2 sub + e.
__device__ __forceinline__ int own_lane(int k, int sub) { return 8 * (k >> 1) + 2 * sub + (k & 1); }
// tier-order index j of the thread's m-th stored lane (m < 4: INT8 tier, else INT4 tier)
__device__ __forceinline__ int stored_j(int m, int sub) {
  return m < kOwn8 ? own_lane(m, sub) : kLive8 + own_lane(m - kOwn8, sub);
}
// running sum e = k & 1 of the thread's lanes in order; the first term is assigned
__device__ __forceinline__ void run_add(float (&acc)[2], int k, float v) {
  if (k < 2) acc[k & 1] = v;
  else acc[k & 1] = fadd(acc[k & 1], v);
}
// reductions over the row's four threads (adjacent lanes of one warp)
__device__ __forceinline__ float row_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float row_pairwise(const float (&acc)[2]) {
  float v = fadd(acc[0], acc[1]);
  v = fadd(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fadd(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

// Per-token staging shared by every kernel: B / C of the row's group in tier order and the
// head's dt / decay.  All threads of the CTA call it; returns after a CTA barrier.
struct TokenShared {
  float b[128], c[128];
  float dt, decay, raw;
};
__device__ void stage_token(const SteParams& P, int b, int t, int h, int g, const int* perm, TokenShared& s,
                            bool need_c) {
  __syncthreads();
  const uint16_t* Bp = P.B + (long long)b * P.b_sb + (long long)t * P.b_st + g * 128;
  const uint16_t* Cp = P.C + (long long)b * P.c_sb + (long long)t * P.c_st + g * 128;
  for (int j = threadIdx.x; j < 128; j += blockDim.x) {
    s.b[j] = h2f(Bp[perm[j]]);
    if (need_c) s.c[j] = h2f(Cp[perm[j]]);
  }
  if (threadIdx.x == 0) {
    const float raw = fadd(h2f(P.dt[(long long)b * P.dt_sb + (long long)t * P.dt_st + h]),
                           ldf(P.dt_bias, P.dt_bias_is_f32, h));
    const float d = softplus20(raw);
    s.raw = raw;
    s.dt = d;
    s.decay = expf(fmul(P.A[h], d));
  }
  __syncthreads();
}

// The forward scan and the backward's carry replays stage kTS tokens per pair of CTA
// barriers: B / C of the group in tier order, and dt / decay computed by kTS threads at once.
constexpr int kTS = 8;
struct ChunkShared {
  float b[kTS][128], c[kTS][128];
  float dt[kTS], decay[kTS];
};
// Stage tokens t0 .. t0 + n - 1 (n <= kTS); threads 0 .. n - 1 compute dt and decay.
__device__ void stage_tokens(const SteParams& P, int b, int t0, int n, int h, int g, const int* perm,
                             ChunkShared& s, bool need_c) {
  __syncthreads();
  for (int i = threadIdx.x; i < n * 128; i += blockDim.x) {
    const int tk = i >> 7, j = i & 127;
    s.b[tk][j] = h2f(P.B[(long long)b * P.b_sb + (long long)(t0 + tk) * P.b_st + g * 128 + perm[j]]);
    if (need_c) s.c[tk][j] = h2f(P.C[(long long)b * P.c_sb + (long long)(t0 + tk) * P.c_st + g * 128 + perm[j]]);
  }
  if (threadIdx.x < n) {
    const int t = t0 + threadIdx.x;
    const float raw = fadd(h2f(P.dt[(long long)b * P.dt_sb + (long long)t * P.dt_st + h]),
                           ldf(P.dt_bias, P.dt_bias_is_f32, h));
    const float d = softplus20(raw);
    s.dt[threadIdx.x] = d;
    s.decay[threadIdx.x] = expf(fmul(P.A[h], d));
  }
  __syncthreads();
}

// S = S decay + (B dt) x on the thread's stored lanes (bt: the token's staged B)
__device__ __forceinline__ void step_own(float (&S)[kOwn], const float* bt, float dt, float decay, float x, int sub) {
#pragma unroll
  for (int m = 0; m < kOwn; ++m) S[m] = fadd(fmul(S[m], decay), fmul(fmul(bt[stored_j(m, sub)], dt), x));
}
// requant of the thread's stored lanes with the row's scales; the codes through q when asked
__device__ __forceinline__ void requant(float (&S)[kOwn], float& sc8, float& sc4, float* q = nullptr) {
  float m8 = 0.f, m4 = 0.f;
#pragma unroll
  for (int m = 0; m < kOwn8; ++m) m8 = fmaxf(m8, fabsf(S[m]));
#pragma unroll
  for (int m = kOwn8; m < kOwn; ++m) m4 = fmaxf(m4, fabsf(S[m]));
  m8 = row_max(m8);
  m4 = row_max(m4);
  const float den8 = fmaxf(__fdiv_rn(m8, 127.0f), 1e-8f), den4 = fmaxf(__fdiv_rn(m4, 7.0f), 1e-8f);
  const float inv8 = __frcp_rn(den8), inv4 = __frcp_rn(den4);
  sc8 = h2f(f2h(den8));
  sc4 = h2f(f2h(den4));
#pragma unroll
  for (int m = 0; m < kOwn; ++m) {
    const bool t8 = m < kOwn8;
    const float lim = t8 ? 127.f : 7.f;
    const float qq = fminf(fmaxf(round_away(div_rn_inv(S[m], t8 ? den8 : den4, t8 ? inv8 : inv4)), -lim), lim);
    if (q) q[m] = qq;
    S[m] = fmul(qq, t8 ? sc8 : sc4);
  }
}

__device__ void load_perm(const SteParams& P, int g, int* perm) {
  for (int j = threadIdx.x; j < 128; j += blockDim.x) perm[j] = P.perm[g * 128 + j];
}

__device__ __forceinline__ float* carry_at(float* base, long long idx) { return base + idx * kLive; }

// ------------------------------------------------------------------------ forward scan
__global__ void __launch_bounds__(512) sq3p25_scan_kernel(const SteParams P) {
  __shared__ ChunkShared s;
  __shared__ int perm[128];
  const int h = blockIdx.x, b = blockIdx.y, r = threadIdx.x / kTPR, sub = threadIdx.x % kTPR;
  const int g = h / (P.heads / P.groups);
  const bool live = r < P.dim;
  const long long row = ((long long)b * P.heads + h) * P.dim + (live ? r : 0);
  load_perm(P, g, perm);
  float S[kOwn];
  {
    const float s8 = live ? h2f(P.s8[row]) : 0.f, s4 = live ? h2f(P.s4[row]) : 0.f;
#pragma unroll
    for (int m = 0; m < kOwn8; ++m) {
      const int q = own_lane(m, sub), sh = 4 * (q & 1);
      const int ub = (((P.hi[row * 8 + q / 2] >> sh) & 15) << 4) | ((P.lo[row * 8 + q / 2] >> sh) & 15);
      S[m] = fmul(live ? (float)(ub - 256 * (ub > 127)) : 0.f, s8);
    }
#pragma unroll
    for (int m = 0; m < kOwn4; ++m) {
      const int q = own_lane(m, sub);
      const int nib = (P.q4[row * 32 + q / 2] >> (4 * (q & 1))) & 15;
      S[kOwn8 + m] = fmul(live ? (float)(nib - 16 * (nib > 7)) : 0.f, s4);
    }
  }
  const float dv = ldf(P.D, P.d_is_f32, h);
  float sc8 = 0.f, sc4 = 0.f, qlast[kOwn];
  for (int t0 = 0; t0 < P.length; t0 += kTS) {
    const int n = min(kTS, P.length - t0);
    stage_tokens(P, b, t0, n, h, g, perm, s, true);
    for (int tk = 0; tk < n; ++tk) {
      const int t = t0 + tk;
      const float* bt = s.b[tk];
      const float* ct = s.c[tk];
      const float dtv = s.dt[tk];
      const float x = live ? h2f(P.x[(long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * P.dim + r]) : 0.f;
      step_own(S, bt, dtv, s.decay[tk], x, sub);
      float a8[2], a4[2], ad[2];
#pragma unroll
      for (int m = 0; m < kOwn8; ++m) run_add(a8, m, fmul(S[m], ct[own_lane(m, sub)]));
#pragma unroll
      for (int m = 0; m < kOwn4; ++m) run_add(a4, m, fmul(S[kOwn8 + m], ct[kLive8 + own_lane(m, sub)]));
      // pruned tier: the reference's 64-wide block, 48 coordinates then 16 masked zero lanes
#pragma unroll
      for (int k = 0; k < kOwnD; ++k) {
        const int q = own_lane(k, sub);
        const bool real = k < 12;                     // q < 48
        const float bj = real ? bt[kLive + q] : 0.0f, cj = real ? ct[kLive + q] : 0.0f;
        run_add(ad, k, fmul(fmul(fmul(bj, dtv), x), cj));
      }
      const float o8 = row_pairwise(a8), o4 = row_pairwise(a4), od = row_pairwise(ad);
      const float out = fadd(fadd(o8, o4), fadd(od, fmul(x, dv)));
      if (live && sub == 0) P.y[(long long)b * P.y_sb + (long long)t * P.y_st + (long long)h * P.dim + r] = f2h(out);
      if (t + 1 < P.length) requant(S, sc8, sc4);
      else requant(S, sc8, sc4, qlast);
    }
  }
  if (live) {
    // this thread's INT8 lanes are 2 sub, 2 sub + 1 (byte sub) and 2 sub + 8, 2 sub + 9 (byte
    // 4 + sub); its INT4 lanes 8 i + 2 sub + {0, 1} form byte 4 i + sub
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int c0 = (int)qlast[2 * p], c1 = (int)qlast[2 * p + 1];
      P.lo[row * 8 + 4 * p + sub] = (uint8_t)((c0 & 15) | ((c1 & 15) << 4));
      P.hi[row * 8 + 4 * p + sub] = (uint8_t)(((c0 >> 4) & 15) | (((c1 >> 4) & 15) << 4));
    }
#pragma unroll
    for (int i = 0; i < kOwn4 / 2; ++i) {
      const int c0 = (int)qlast[kOwn8 + 2 * i], c1 = (int)qlast[kOwn8 + 2 * i + 1];
      P.q4[row * 32 + 4 * i + sub] = (uint8_t)((c0 & 15) | ((c1 & 15) << 4));
    }
    if (sub == 0) {
      P.s8[row] = f2h(sc8);
      P.s4[row] = f2h(sc4);
    }
  }
}

// ------------------------------------------------------------------------ STE backward
__global__ void __launch_bounds__(512) ste_checkpoint_kernel(const SteParams P) {
  __shared__ ChunkShared s;
  __shared__ int perm[128];
  const int h = blockIdx.x, b = blockIdx.y, r = threadIdx.x / kTPR, sub = threadIdx.x % kTPR;
  const int g = h / (P.heads / P.groups);
  const bool live = r < P.dim;
  load_perm(P, g, perm);
  float S[kOwn];
#pragma unroll
  for (int m = 0; m < kOwn; ++m) S[m] = 0.f;
  float sc8, sc4;
  for (int c = 0; c < P.nchunk; ++c) {
    if (live) {
      float* dst = carry_at(P.cp, (((long long)b * P.nchunk + c) * P.heads + h) * P.dim + r);
#pragma unroll
      for (int m = 0; m < kOwn; ++m) dst[stored_j(m, sub)] = S[m];
    }
    const int cend = min(P.length, (c + 1) * P.chunk);
    for (int t0 = c * P.chunk; t0 < cend; t0 += kTS) {
      const int n = min(kTS, cend - t0);
      stage_tokens(P, b, t0, n, h, g, perm, s, false);
      for (int tk = 0; tk < n; ++tk) {
        const int t = t0 + tk;
        const float x = live ? h2f(P.x[(long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * P.dim + r]) : 0.f;
        step_own(S, s.b[tk], s.dt[tk], s.decay[tk], x, sub);
        requant(S, sc8, sc4);
      }
    }
  }
}

__global__ void __launch_bounds__(512) ste_history_kernel(const SteParams P, int c) {
  __shared__ ChunkShared s;
  __shared__ int perm[128];
  const int h = blockIdx.x, b = blockIdx.y, r = threadIdx.x / kTPR, sub = threadIdx.x % kTPR;
  const int g = h / (P.heads / P.groups);
  const bool live = r < P.dim;
  load_perm(P, g, perm);
  float S[kOwn];
  {
    const float* src = carry_at(P.cp, (((long long)b * P.nchunk + c) * P.heads + h) * P.dim + (live ? r : 0));
#pragma unroll
    for (int m = 0; m < kOwn; ++m) S[m] = live ? src[stored_j(m, sub)] : 0.f;
  }
  float sc8, sc4;
  const int cend = min(P.length, (c + 1) * P.chunk);
  for (int t0 = c * P.chunk; t0 < cend; t0 += kTS) {
    const int n = min(kTS, cend - t0);
    stage_tokens(P, b, t0, n, h, g, perm, s, false);
    for (int tk = 0; tk < n; ++tk) {
      const int t = t0 + tk, k = t - c * P.chunk;
      if (live) {
        float* dst = carry_at(P.hist, (((long long)b * P.chunk + k) * P.heads + h) * P.dim + r);
#pragma unroll
        for (int m = 0; m < kOwn; ++m) dst[stored_j(m, sub)] = S[m];
      }
      const float x = live ? h2f(P.x[(long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * P.dim + r]) : 0.f;
      step_own(S, s.b[tk], s.dt[tk], s.decay[tk], x, sub);
      requant(S, sc8, sc4);
    }
  }
}

constexpr int kStageLanes = 32;   // tier lanes of dB / dC terms staged per block

struct BackShared {
  TokenShared s;
  int perm[128];
  float stage[2][kStageLanes][129];   // [dB | dC][lane in block][row], padded
  float row_dl[128];
};

// Per-token quantities of one row in the reverse walk.
struct RowCtx {
  float x, gy, factor, ad;
  const float* prev;
  bool live;
  int r;
};

// A stored lane (adjoint index m, tier index j, position k in its tier's running sums).
__device__ __forceinline__ void back_live_lane(BackShared& sh, const RowCtx& rc, float (&adj)[kOwn], int m, int j,
                                               int k, float (&ax)[2], float (&al)[2]) {
  const TokenShared& s = sh.s;
  const float pj = rc.live ? rc.prev[j] : 0.f;
  const float bj = s.b[j], cj = s.c[j];
  const float bdt = fmul(bj, s.dt);
  const float v = fadd(fmul(rc.gy, cj), adj[m]);                 // STE: identity on live lanes
  const float hj = fadd(fmul(pj, s.decay), fmul(bdt, rc.x));
  const float e = fadd(fmul(pj, rc.ad), fmul(bj, rc.x));
  run_add(ax, k, fmul(v, bdt));
  run_add(al, k, fmul(v, e));
  sh.stage[0][j % kStageLanes][rc.r] = fmul(v, rc.factor);
  sh.stage[1][j % kStageLanes][rc.r] = fmul(hj, rc.gy);
  adj[m] = fmul(v, s.decay);
}
// A lane of the pruned block (position k of the thread's 16; k >= 12 are the masked zeros).
__device__ __forceinline__ void back_pruned_lane(BackShared& sh, const RowCtx& rc, int k, int sub, float (&ax)[2],
                                                 float (&al)[2]) {
  const TokenShared& s = sh.s;
  if (k < 12) {
    const int j = kLive + own_lane(k, sub);
    const float bj = s.b[j], cj = s.c[j];
    const float bdt = fmul(bj, s.dt);
    const float v = fmul(rc.gy, cj);
    run_add(ax, k, fmul(v, bdt));
    run_add(al, k, fmul(v, fmul(bj, rc.x)));
    sh.stage[0][j % kStageLanes][rc.r] = fmul(v, rc.factor);
    sh.stage[1][j % kStageLanes][rc.r] = fmul(fmul(bdt, rc.x), rc.gy);
  } else {
    const float v = fmul(rc.gy, 0.0f);
    run_add(ax, k, fmul(v, fmul(0.0f, s.dt)));
    run_add(al, k, fmul(v, fmul(0.0f, rc.x)));
  }
}
// Sum each row tile's 16 staged terms of lane block `blk` in row order into the partials.
__device__ __forceinline__ void flush_block(BackShared& sh, float* part, int blk, int ntile) {
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * kStageLanes * ntile; i += blockDim.x) {
    const int which = i / (kStageLanes * ntile), rem = i % (kStageLanes * ntile);
    const int tile = rem / kStageLanes, lane = rem % kStageLanes;
    const float* col = &sh.stage[which][lane][tile * 16];
    float acc = col[0];
#pragma unroll
    for (int q = 1; q < 16; ++q) acc = fadd(acc, col[q]);
    part[(tile * 2 + which) * 128 + blk * kStageLanes + lane] = acc;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(512) ste_backward_kernel(const SteParams P, int c) {
  __shared__ BackShared sh;
  const int h = blockIdx.x, b = blockIdx.y, r = threadIdx.x / kTPR, sub = threadIdx.x % kTPR;
  const int g = h / (P.heads / P.groups);
  const int ntile = (P.dim + 15) / 16;
  const bool live = r < P.dim;
  load_perm(P, g, sh.perm);
  const float av = P.A[h], dv = ldf(P.D, P.d_is_f32, h);
  float adj[kOwn];
  float* adj_row = carry_at(P.adj, ((long long)b * P.heads + h) * P.dim + (live ? r : 0));
#pragma unroll
  for (int m = 0; m < kOwn; ++m) adj[m] = live ? adj_row[stored_j(m, sub)] : 0.f;
  for (int rev = 0; rev < P.chunk; ++rev) {
    const int k = P.chunk - 1 - rev;
    const int t = c * P.chunk + k;
    if (t >= P.length) continue;
    stage_token(P, b, t, h, g, sh.perm, sh.s, true);
    const long long xo = (long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * P.dim + r;
    RowCtx rc;
    rc.live = live;
    rc.r = r;
    rc.x = live ? h2f(P.x[xo]) : 0.f;
    rc.gy = live ? h2f(P.dy[xo]) : 0.f;
    rc.factor = fmul(sh.s.dt, rc.x);                   // 0 on rows past dim (x = 0 there)
    rc.ad = fmul(av, sh.s.decay);
    rc.prev = carry_at(P.hist, (((long long)b * P.chunk + k) * P.heads + h) * P.dim + (live ? r : 0));
    // dB / dC partials of this (token, head): [tile][dB | dC][128 tier lanes]
    float* part = P.part + (((long long)b * P.chunk + k) * P.heads + h) * ntile * 256;
    float ax8[2], al8[2], ax4[2], al4[2], axd[2], ald[2];
    // lane block 0: INT8 lanes (tier 0..15) and INT4 lanes of tier 16..31
#pragma unroll
    for (int m = 0; m < kOwn8; ++m) back_live_lane(sh, rc, adj, m, own_lane(m, sub), m, ax8, al8);
#pragma unroll
    for (int m = 0; m < 4; ++m) back_live_lane(sh, rc, adj, kOwn8 + m, kLive8 + own_lane(m, sub), m, ax4, al4);
    flush_block(sh, part, 0, ntile);
    // block 1: INT4 lanes of tier 32..63
#pragma unroll
    for (int m = 4; m < 12; ++m) back_live_lane(sh, rc, adj, kOwn8 + m, kLive8 + own_lane(m, sub), m, ax4, al4);
    flush_block(sh, part, 1, ntile);
    // block 2: INT4 lanes of tier 64..79, pruned lanes of tier 80..95
#pragma unroll
    for (int m = 12; m < 16; ++m) back_live_lane(sh, rc, adj, kOwn8 + m, kLive8 + own_lane(m, sub), m, ax4, al4);
#pragma unroll
    for (int kd = 0; kd < 4; ++kd) back_pruned_lane(sh, rc, kd, sub, axd, ald);
    flush_block(sh, part, 2, ntile);
    // block 3: pruned lanes of tier 96..127, then the masked zero lanes of the 64-wide block
#pragma unroll
    for (int kd = 4; kd < kOwnD; ++kd) back_pruned_lane(sh, rc, kd, sub, axd, ald);
    flush_block(sh, part, 3, ntile);
    const float dx8 = row_pairwise(ax8), dx4 = row_pairwise(ax4), dxd = row_pairwise(axd);
    const float dl8 = row_pairwise(al8), dl4 = row_pairwise(al4), dld = row_pairwise(ald);
    if (live && sub == 0) P.dx[xo] = fadd(fadd(dx8, dx4), fadd(dxd, fmul(rc.gy, dv)));
    if (sub == 0) sh.row_dl[r] = live ? fadd(fadd(dl8, dl4), dld) : 0.f;
    __syncthreads();
    // d(dt raw): each tile's 16 rows in numpy's pairwise order, times softplus'(raw), added
    // over the tiles in order
    if (threadIdx.x == 0) {
      const float sig = sh.s.raw <= 20.0f ? __fdiv_rn(1.0f, fadd(1.0f, expf(-sh.s.raw))) : 1.0f;
      float acc = 0.0f;
      for (int i = 0; i < ntile; ++i) {
        const float* d = &sh.row_dl[i * 16];
        float q[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = fadd(d[j], d[j + 8]);
        const float tsum = fadd(fadd(fadd(q[0], q[1]), fadd(q[2], q[3])), fadd(fadd(q[4], q[5]), fadd(q[6], q[7])));
        acc = fadd(acc, fmul(tsum, sig));
      }
      P.ddt[((long long)b * P.length + t) * P.heads + h] = acc;
    }
  }
  if (live) {
#pragma unroll
    for (int m = 0; m < kOwn; ++m) adj_row[stored_j(m, sub)] = adj[m];
  }
}

// dB / dC of one chunk: for every (token, batch, group) and coordinate, the partials of the
// group's heads and row tiles added in (head, tile) order, scattered through the permutation.
__global__ void __launch_bounds__(256) ste_bc_reduce_kernel(const SteParams P, int c) {
  const int k = blockIdx.x, b = blockIdx.y, g = blockIdx.z;
  const int t = c * P.chunk + k;
  if (t >= P.length) return;
  const int which = threadIdx.x >> 7, lane = threadIdx.x & 127;
  const int per = P.heads / P.groups, ntile = (P.dim + 15) / 16;
  const float* part = P.part + ((long long)b * P.chunk + k) * P.heads * ntile * 256 + which * 128 + lane;
  float acc = 0.0f;
  for (int hh = g * per; hh < (g + 1) * per; ++hh)
    for (int tile = 0; tile < ntile; ++tile) acc = fadd(acc, part[((long long)hh * ntile + tile) * 256]);
  const long long o = (((long long)b * P.length + t) * P.groups + g) * 128 + P.perm[g * 128 + lane];
  (which ? P.dc : P.db)[o] = acc;
}

// four threads per row over whole 16-row tiles, so every tile's rows exist (rows past dim
// carry zeros, as the reference's masked rows)
int threads_for(int dim) { return kTPR * ((dim + 15) / 16 * 16); }

}  // namespace

int launch_sq3p25_scan(const SteParams& P, cudaStream_t st) {
  if (P.dim <= 0 || P.dim > 128 || P.heads <= 0 || P.groups <= 0 || P.heads % P.groups || P.batch <= 0 ||
      P.length <= 0)
    return kEInval;
  sq3p25_scan_kernel<<<dim3(P.heads, P.batch), threads_for(P.dim), 0, st>>>(P);
  return launch_status();
}

long long ste_workspace_bytes(int batch, int length, int heads, int dim, int chunk) {
  if (batch <= 0 || length <= 0 || heads <= 0 || dim <= 0 || chunk <= 0) return -1;
  const long long nc = (length + chunk - 1) / chunk, ntile = (dim + 15) / 16;
  return (long long)batch * (nc + chunk + 1) * heads * dim * kLive * 4 +   // carries
         (long long)batch * chunk * heads * ntile * 256 * 4;                // dB / dC partials
}

int launch_ste_backward(SteParams P, void* workspace, cudaStream_t st) {
  if (P.dim <= 0 || P.dim > 128 || P.heads <= 0 || P.groups <= 0 || P.heads % P.groups || P.batch <= 0 ||
      P.length <= 0 || P.chunk <= 0 || P.chunk > 256)
    return kEInval;
  P.nchunk = (P.length + P.chunk - 1) / P.chunk;
  float* w = static_cast<float*>(workspace);
  const long long rows = (long long)P.batch * P.heads * P.dim;
  P.cp = w;
  P.hist = P.cp + rows * P.nchunk * kLive;
  P.adj = P.hist + rows * P.chunk * kLive;
  P.part = P.adj + rows * kLive;
  // dx, d(dt), dB and dC are written in full by the kernels; only the adjoint carry starts at 0
  if (cudaMemsetAsync(P.adj, 0, rows * kLive * 4, st) != cudaSuccess) return kECuda;
  const dim3 grid(P.heads, P.batch);
  const int th = threads_for(P.dim);
  ste_checkpoint_kernel<<<grid, th, 0, st>>>(P);
  for (int c = P.nchunk - 1; c >= 0; --c) {
    ste_history_kernel<<<grid, th, 0, st>>>(P, c);
    ste_backward_kernel<<<grid, th, 0, st>>>(P, c);
    ste_bc_reduce_kernel<<<dim3(P.chunk, P.batch, P.groups), 256, 0, st>>>(P, c);
  }
  return launch_status();
}

}  // namespace sq
