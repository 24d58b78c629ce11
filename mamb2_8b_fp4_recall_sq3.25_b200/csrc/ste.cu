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
//                          all 128; dx is stored, d(dt) (times the softplus slope) and dB /
//                          dC are summed over the CTA's rows and added atomically.
//   ste_bc_reduce_kernel   adds the per-(head, row tile) dB / dC partials of the chunk in
//                          (head, tile) order and scatters them to the original coordinates.
// Mapping: one CTA per (head, batch), one thread per row of the head (dim <= 128); the
// group's B / C of a token are staged in shared memory in tier order.  Arithmetic is
// unfused (__fmul_rn / __fadd_rn) like the reference's, and every reduction runs in the order
// of the reference kernels' golden runs (Triton interpreter, i.e. numpy): sums over a row's
// lanes and over a tile's 16 rows for d(dt) in numpy's eight-accumulator pairwise order,
// sums over rows for dB / dC sequentially, tiles and heads in program order.  Given the same
// softplus / exp values the results are bit-identical to the golden runs, and no atomics are
// used, so gradients are deterministic run to run.
#include "common.cuh"
#include "ste.cuh"

namespace sq {
namespace {

constexpr int kLive8 = 16, kLive4 = 64, kLive = 80;   // stored lanes; lanes 80..127 are pruned

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
__device__ __forceinline__ float softplus20(float v) { return v <= 20.0f ? logf(fadd(expf(v), 1.0f)) : v; }

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

// S = S decay + (B dt) x on the live lanes, then the requant of both tiers; returns the codes
// of the last requant through q8 / q4 when asked.
__device__ __forceinline__ void step_live(float (&S)[kLive], const TokenShared& s, float x) {
#pragma unroll
  for (int j = 0; j < kLive; ++j) S[j] = fadd(fmul(S[j], s.decay), fmul(fmul(s.b[j], s.dt), x));
}
__device__ __forceinline__ void requant(float (&S)[kLive], float& sc8, float& sc4, float* q = nullptr) {
  float m8 = 0.f, m4 = 0.f;
#pragma unroll
  for (int j = 0; j < kLive8; ++j) m8 = fmaxf(m8, fabsf(S[j]));
#pragma unroll
  for (int j = kLive8; j < kLive; ++j) m4 = fmaxf(m4, fabsf(S[j]));
  const float den8 = fmaxf(__fdiv_rn(m8, 127.0f), 1e-8f), den4 = fmaxf(__fdiv_rn(m4, 7.0f), 1e-8f);
  sc8 = h2f(f2h(den8));
  sc4 = h2f(f2h(den4));
#pragma unroll
  for (int j = 0; j < kLive; ++j) {
    const bool t8 = j < kLive8;
    const float lim = t8 ? 127.f : 7.f;
    const float qq = fminf(fmaxf(round_away(__fdiv_rn(S[j], t8 ? den8 : den4)), -lim), lim);
    if (q) q[j] = qq;
    S[j] = fmul(qq, t8 ? sc8 : sc4);
  }
}

// numpy's float32 sum of n lanes (n % 8 == 0, 8 <= n <= 128): eight running sums over the
// lanes j, j + 8, j + 16, ..., combined as ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)).
// `q` is the lane's position within the sum (a compile-time constant in unrolled loops).
__device__ __forceinline__ void pw_add(float (&r)[8], int q, float v) {
  if (q < 8) r[q] = v;
  else r[q & 7] = fadd(r[q & 7], v);
}
__device__ __forceinline__ float pw_total(const float (&r)[8]) {
  return fadd(fadd(fadd(r[0], r[1]), fadd(r[2], r[3])), fadd(fadd(r[4], r[5]), fadd(r[6], r[7])));
}

__device__ void load_perm(const SteParams& P, int g, int* perm) {
  for (int j = threadIdx.x; j < 128; j += blockDim.x) perm[j] = P.perm[g * 128 + j];
}

// ------------------------------------------------------------------------ forward scan
__global__ void __launch_bounds__(128) sq3p25_scan_kernel(const SteParams P) {
  __shared__ TokenShared s;
  __shared__ int perm[128];
  const int h = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int g = h / (P.heads / P.groups);
  const bool live = r < P.dim;
  const long long row = ((long long)b * P.heads + h) * P.dim + r;
  load_perm(P, g, perm);
  float S[kLive];
  {
    float s8 = 0.f, s4 = 0.f;
    if (live) { s8 = h2f(P.s8[row]); s4 = h2f(P.s4[row]); }
#pragma unroll
    for (int j = 0; j < kLive8; ++j) {
      int v = 0;
      if (live) {
        const int lo = (P.lo[row * 8 + j / 2] >> (4 * (j & 1))) & 15;
        const int hi = (P.hi[row * 8 + j / 2] >> (4 * (j & 1))) & 15;
        const int ub = (hi << 4) | lo;
        v = ub - 256 * (ub > 127);
      }
      S[j] = fmul((float)v, s8);
    }
#pragma unroll
    for (int j = 0; j < kLive4; ++j) {
      int v = 0;
      if (live) {
        const int nib = (P.q4[row * 32 + j / 2] >> (4 * (j & 1))) & 15;
        v = nib - 16 * (nib > 7);
      }
      S[kLive8 + j] = fmul((float)v, s4);
    }
  }
  const float dv = ldf(P.D, P.d_is_f32, h);
  float sc8 = 0.f, sc4 = 0.f;
  uint32_t plo[2] = {0, 0}, phi[2] = {0, 0}, pq4[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int t = 0; t < P.length; ++t) {
    stage_token(P, b, t, h, g, perm, s, true);
    const float x = live ? h2f(P.x[(long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * P.dim + r]) : 0.f;
    step_live(S, s, x);
    float acc[8], o8, o4, od;
#pragma unroll
    for (int j = 0; j < kLive8; ++j) pw_add(acc, j, fmul(S[j], s.c[j]));
    o8 = pw_total(acc);
#pragma unroll
    for (int j = kLive8; j < kLive; ++j) pw_add(acc, j - kLive8, fmul(S[j], s.c[j]));
    o4 = pw_total(acc);
    // pruned tier: the reference's 64-wide block, 48 coordinates and 16 masked zero lanes
#pragma unroll
    for (int q = 0; q < 64; ++q) {
      const float bj = q < 48 ? s.b[kLive + q] : 0.0f, cj = q < 48 ? s.c[kLive + q] : 0.0f;
      pw_add(acc, q, fmul(fmul(fmul(bj, s.dt), x), cj));
    }
    od = pw_total(acc);
    const float out = fadd(fadd(o8, o4), fadd(od, fmul(x, dv)));
    if (live) P.y[(long long)b * P.y_sb + (long long)t * P.y_st + (long long)h * P.dim + r] = f2h(out);
    if (t + 1 < P.length) {
      requant(S, sc8, sc4);
    } else {
      float q[kLive];
      requant(S, sc8, sc4, q);
#pragma unroll
      for (int j = 0; j < kLive8; ++j) {
        const int c = (int)q[j];
        plo[j / 8] |= (uint32_t)(c & 15) << (4 * (j % 8));
        phi[j / 8] |= (uint32_t)((c >> 4) & 15) << (4 * (j % 8));
      }
#pragma unroll
      for (int j = 0; j < kLive4; ++j) pq4[j / 8] |= (uint32_t)((int)q[kLive8 + j] & 15) << (4 * (j % 8));
    }
  }
  if (live) {
    uint32_t* lo = reinterpret_cast<uint32_t*>(P.lo + row * 8);
    uint32_t* hi = reinterpret_cast<uint32_t*>(P.hi + row * 8);
    uint32_t* q4 = reinterpret_cast<uint32_t*>(P.q4 + row * 32);
    lo[0] = plo[0]; lo[1] = plo[1]; hi[0] = phi[0]; hi[1] = phi[1];
#pragma unroll
    for (int i = 0; i < 8; ++i) q4[i] = pq4[i];
    P.s8[row] = f2h(sc8);
    P.s4[row] = f2h(sc4);
  }
}

// ------------------------------------------------------------------------ STE backward
__device__ __forceinline__ float* carry_at(float* base, long long idx) { return base + idx * kLive; }

__global__ void __launch_bounds__(128) ste_checkpoint_kernel(const SteParams P) {
  __shared__ TokenShared s;
  __shared__ int perm[128];
  const int h = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int g = h / (P.heads / P.groups);
  const bool live = r < P.dim;
  load_perm(P, g, perm);
  float S[kLive];
#pragma unroll
  for (int j = 0; j < kLive; ++j) S[j] = 0.f;
  float sc8, sc4;
  for (int c = 0; c < P.nchunk; ++c) {
    if (live) {
      float* dst = carry_at(P.cp, (((long long)b * P.nchunk + c) * P.heads + h) * P.dim + r);
#pragma unroll
      for (int j = 0; j < kLive; ++j) dst[j] = S[j];
    }
    for (int k = 0; k < P.chunk; ++k) {
      const int t = c * P.chunk + k;
      if (t >= P.length) break;
      stage_token(P, b, t, h, g, perm, s, false);
      const float x = live ? h2f(P.x[(long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * P.dim + r]) : 0.f;
      step_live(S, s, x);
      requant(S, sc8, sc4);
    }
  }
}

__global__ void __launch_bounds__(128) ste_history_kernel(const SteParams P, int c) {
  __shared__ TokenShared s;
  __shared__ int perm[128];
  const int h = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int g = h / (P.heads / P.groups);
  const bool live = r < P.dim;
  load_perm(P, g, perm);
  float S[kLive];
  {
    const float* src = carry_at(P.cp, (((long long)b * P.nchunk + c) * P.heads + h) * P.dim + (live ? r : 0));
#pragma unroll
    for (int j = 0; j < kLive; ++j) S[j] = live ? src[j] : 0.f;
  }
  float sc8, sc4;
  for (int k = 0; k < P.chunk; ++k) {
    const int t = c * P.chunk + k;
    if (t >= P.length) break;
    if (live) {
      float* dst = carry_at(P.hist, (((long long)b * P.chunk + k) * P.heads + h) * P.dim + r);
#pragma unroll
      for (int j = 0; j < kLive; ++j) dst[j] = S[j];
    }
    stage_token(P, b, t, h, g, perm, s, false);
    const float x = live ? h2f(P.x[(long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * P.dim + r]) : 0.f;
    step_live(S, s, x);
    requant(S, sc8, sc4);
  }
}

// Sum over a 16-row tile (lanes of one half-warp) in numpy's pairwise order: rows j and
// j + 8, then neighbours, pairs and halves; every lane of the tile receives the sum.
__device__ __forceinline__ float tile_pairwise16(float v) {
  v = fadd(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fadd(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = fadd(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = fadd(v, __shfl_xor_sync(0xffffffffu, v, 4));
  return v;
}

constexpr int kStageLanes = 32;   // lanes of dB / dC terms staged per block

__global__ void __launch_bounds__(128) ste_backward_kernel(const SteParams P, int c) {
  __shared__ TokenShared s;
  __shared__ int perm[128];
  __shared__ float stage[2][kStageLanes][129];       // [dB | dC][lane][row], padded
  __shared__ float tile_dl[8];
  const int h = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int g = h / (P.heads / P.groups);
  const int ntile = (P.dim + 15) / 16;
  const bool live = r < P.dim;
  load_perm(P, g, perm);
  const float av = P.A[h], dv = ldf(P.D, P.d_is_f32, h);
  float adj[kLive];
  float* adj_row = carry_at(P.adj, ((long long)b * P.heads + h) * P.dim + (live ? r : 0));
#pragma unroll
  for (int j = 0; j < kLive; ++j) adj[j] = live ? adj_row[j] : 0.f;
  for (int rev = 0; rev < P.chunk; ++rev) {
    const int k = P.chunk - 1 - rev;
    const int t = c * P.chunk + k;
    if (t >= P.length) continue;
    stage_token(P, b, t, h, g, perm, s, true);
    const long long xo = (long long)b * P.x_sb + (long long)t * P.x_st + (long long)h * P.dim + r;
    const float x = live ? h2f(P.x[xo]) : 0.f;
    const float gy = live ? h2f(P.dy[xo]) : 0.f;
    const float factor = fmul(s.dt, x);                 // 0 on rows past dim (x = 0 there)
    const float ad = fmul(av, s.decay);
    const float* prev = carry_at(P.hist, (((long long)b * P.chunk + k) * P.heads + h) * P.dim + (live ? r : 0));
    // dB / dC partials of this (token, head): [tile][dB | dC][128 tier lanes]
    float* part = P.part + (((long long)b * P.chunk + k) * P.heads + h) * ntile * 256;
    float ax[8], al[8];
    float dx8 = 0.f, dl8 = 0.f, dx4 = 0.f, dl4 = 0.f;
#pragma unroll
    for (int j = 0; j < 128; ++j) {
      float pb, pc;                                     // this row's dB and dC terms of lane j
      if (j < kLive) {                                  // STE: identity through the live lanes
        const float pj = live ? prev[j] : 0.f;
        const float bj = s.b[j], cj = s.c[j];
        const float bdt = fmul(bj, s.dt);
        const float v = fadd(fmul(gy, cj), adj[j]);
        const float hj = fadd(fmul(pj, s.decay), fmul(bdt, x));
        const float e = fadd(fmul(pj, ad), fmul(bj, x));
        const int q = j < kLive8 ? j : j - kLive8;
        pw_add(ax, q, fmul(v, bdt));
        pw_add(al, q, fmul(v, e));
        pb = fmul(v, factor);
        pc = fmul(hj, gy);
        adj[j] = fmul(v, s.decay);
        if (j == kLive8 - 1) { dx8 = pw_total(ax); dl8 = pw_total(al); }
        if (j == kLive - 1) { dx4 = pw_total(ax); dl4 = pw_total(al); }
      } else {                                          // pruned lanes: readout only
        const float bj = s.b[j], cj = s.c[j];
        const float bdt = fmul(bj, s.dt);
        const float v = fmul(gy, cj);
        pw_add(ax, j - kLive, fmul(v, bdt));
        pw_add(al, j - kLive, fmul(v, fmul(bj, x)));
        pb = fmul(v, factor);
        pc = fmul(fmul(bdt, x), gy);
      }
      stage[0][j % kStageLanes][r] = pb;
      stage[1][j % kStageLanes][r] = pc;
      if (j % kStageLanes == kStageLanes - 1) {
        __syncthreads();
        // each tile's 16 rows summed in row order (numpy's order for a sum over rows)
        for (int i = threadIdx.x; i < 2 * kStageLanes * ntile; i += blockDim.x) {
          const int which = i / (kStageLanes * ntile), rem = i % (kStageLanes * ntile);
          const int tile = rem / kStageLanes, lane = rem % kStageLanes;
          const float* col = &stage[which][lane][tile * 16];
          float acc = col[0];
#pragma unroll
          for (int q = 1; q < 16; ++q) acc = fadd(acc, col[q]);
          part[(tile * 2 + which) * 128 + (j + 1 - kStageLanes) + lane] = acc;
        }
        __syncthreads();
      }
    }
    // the pruned block is 64 wide in the reference: 16 masked zero lanes close the sums
#pragma unroll
    for (int q = 48; q < 64; ++q) {
      const float v = fmul(gy, 0.0f);
      pw_add(ax, q, fmul(v, fmul(0.0f, s.dt)));
      pw_add(al, q, fmul(v, fmul(0.0f, x)));
    }
    const float dxd = pw_total(ax), dld = pw_total(al);
    if (live) P.dx[xo] = fadd(fadd(dx8, dx4), fadd(dxd, fmul(gy, dv)));
    const float dl = tile_pairwise16(live ? fadd(fadd(dl8, dl4), dld) : 0.f);
    if ((r & 15) == 0 && (r >> 4) < ntile) tile_dl[r >> 4] = dl;
    __syncthreads();
    // d(dt raw) = sum over tiles, in tile order, of (tile sum) * softplus'(raw)
    if (threadIdx.x == 0) {
      const float sig = s.raw <= 20.0f ? __fdiv_rn(1.0f, fadd(1.0f, expf(-s.raw))) : 1.0f;
      float acc = 0.0f;
      for (int i = 0; i < ntile; ++i) acc = fadd(acc, fmul(tile_dl[i], sig));
      P.ddt[((long long)b * P.length + t) * P.heads + h] = acc;
    }
  }
  if (live) {
#pragma unroll
    for (int j = 0; j < kLive; ++j) adj_row[j] = adj[j];
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

int threads_for(int dim) { return (dim + 31) / 32 * 32; }

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
