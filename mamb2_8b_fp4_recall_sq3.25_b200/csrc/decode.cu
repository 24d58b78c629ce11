// Persistent batch-1 greedy decode (one cooperative launch runs all requested tokens).
//
// Same arithmetic, operation for operation, as the multi-kernel decode step it replaces
// (fp4_embed, add_rmsnorm, the factored-scale streaming GEMV, the one-token scan step with
// the conv ring, resurface_gatednorm, argmax), so tokens, logits and state bytes are
// identical; what changes is the schedule:
//   * grid = one CTA per SM, 10 warps: warps 0-7 compute, warp 8 lane 0 is the weight
//     producer, warp 9 lane 0 the stager.  Each CTA owns fixed 16-row tiles of in_proj,
//     out_proj and lm_head and streams them (1024-column chunks of codes + block scales,
//     2-D TMA, no multicast) through a 12-stage mbarrier ring in the order the consumers
//     use them, running ahead across phases and layers.  The stager brings each layer's
//     token-independent inputs (norm / adapter weights, the scan head's tables, packed state
//     rows and conv history) one layer ahead.
//   * per layer: norm (every CTA, redundant) -> in_proj -> grid barrier (gate dot and the
//     head's state unpack inside it) -> scan step (one head per CTA) -> grid barrier (state
//     requant / write-back inside it) -> resurface + gated norm (every CTA, redundant: the
//     128x128 head mix needs all heads) -> out_proj -> grid barrier.
//   * data another CTA wrote during this launch is read through L2 only (ld.global.cg,
//     cp.async.cg); every wait (ring slot, staging copy, grid barrier) is bounded by
//     %globaltimer and observes a shared abort flag, after which the launch finishes without
//     waiting and reports through the error word.
#include <cstring>

#include "common.cuh"
#include "decode.cuh"
#include "device_util.cuh"
#include "scan.cuh"
#include "scan_math.cuh"

namespace sq {
namespace {

constexpr int kWarps = 10, kThreads = 32 * kWarps, kCompute = 256;   // 8 compute, producer, stager
constexpr int kNst = 12;                               // ring stages
constexpr int kRows = 16, kKc = 1024;                  // tile rows, columns per chunk
constexpr int kCodeBytes = kRows * kKc / 2, kScaleBytes = kRows * kKc / 16, kStageBytes = kCodeBytes + kScaleBytes;
constexpr int kDModel = 4096, kDInner = 8192, kZx = 18560, kHeads = 128, kGroups = 8;
constexpr unsigned long long kWaitNs = 500000000ull;   // 0.5 s per wait

// shared-memory plan (bytes).  Per-layer tensors are staged well before use (the stager
// brings adapter V and weights, gated-norm weights and scan tables one layer ahead; the next
// layer's norm weight is copied one layer ahead; z right after the in_proj barrier).
// V and the gated-norm weights arrive as SWIZZLE_128B TMA tiles and z / the gated-norm
// output use the same layout (see swz), so the Resurface epilogue and the head mix read
// shared memory without bank conflicts; both tiles start on 1024-byte boundaries.
constexpr int kScanBytes = 20608;
constexpr int oRing = 0;                               // kNst x 9216 (1024-byte multiples)
constexpr int oV = oRing + kNst * kStageBytes;         // adapter V, 2 x [128][64] swizzled
constexpr int oGnw = oV + 128 * 128 * 2;               // gated RMSNorm weights [128][64] swizzled
constexpr int oYn = oGnw + kDInner * 2;                // z staging, then the gated-norm output [128][64] swizzled
constexpr int oHn = oYn + kDInner * 2;                 // normed layer input [4096] fp16
constexpr int oScan = oHn + kDModel * 2;               // scan item staging / y staging
constexpr int oAdw = oScan + kScanBytes;               // adapter gate weights [4096] fp16
constexpr int oNw = oAdw + kDModel * 2;                // Block norm weights [4096] fp16 (the next layer's copied in after each norm)
constexpr int oAdg = oNw + kDModel * 2;                // adapter g [128] fp16
constexpr int oRed = oAdg + 256;                       // GEMV cross-warp sums [2][4][32][4] f32
constexpr int oBar = oRed + 2 * 4 * 32 * 4 * 4;        // full[kNst], empty[kNst]
constexpr int oSBar = oBar + 2 * kNst * 8;             // staging mbarriers: layer inputs, norm weight, (unused), inputs free
constexpr int oMisc = oSBar + 32;                      // small scratch (reductions, flags)
constexpr int kSmem = oMisc + 512;
// scan region
constexpr int sPred = 0, sBasis = 8448, sPerm = 8768, sRows = 8896, sWx = 12224, sBx = 12736, sWbc = 12864,
              sBbc = 14912, sHist = 15424, sP4o = 17344, sV2o = 18368, sXo = 18880, sDotso = 19136, sDDo = 19168,
              sLs = 19200, sDv = 19232, sDtb = 19488, sAv = 19744;   // latent scales, D, dt_bias, A
constexpr int kYPitch = 72;                            // y staging rows (64 + 8 pad) for ldmatrix
static_assert(oV % 1024 == 0 && oGnw % 1024 == 0, "swizzled tiles need 1024-byte alignment");
// Element (h, p) of an [rows][64] fp16 tile in the SWIZZLE_128B layout: row h is 128 bytes,
// its 16-byte chunk c sits at chunk c ^ (h & 7).
__device__ __forceinline__ int swz(int h, int p) { return (h << 6) + ((((p >> 3) ^ h) & 7) << 3) + (p & 7); }

__device__ __forceinline__ void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ uint64_t now_ns() { uint64_t t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }
__device__ __forceinline__ int ld_abort(const DecodeSync* s) { return *reinterpret_cast<const volatile int*>(&s->abort); }
__device__ __forceinline__ void set_abort(const DecodeParams& P, int bit) {
  atomicOr(P.err, bit);
  atomicExch(&P.sync->abort, 1);
}
__device__ __forceinline__ uint4 ldcg4(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint16_t ldcg16(const uint16_t* p) {
  return __ldcg(reinterpret_cast<const unsigned short*>(p));
}

__device__ __forceinline__ bool mb_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok) : "r"(a), "r"(parity) : "memory");
  return ok != 0;
}
// bounded wait on an mbarrier phase; gives up on expiry or when another CTA aborted
__device__ __forceinline__ bool mb_wait(uint32_t a, uint32_t parity, const DecodeSync* s) {
  if (mb_try(a, parity)) return true;
  const uint64_t t0 = now_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i) if (mb_try(a, parity)) return true;
    if (ld_abort(s) || now_ns() - t0 > kWaitNs) return false;
  }
}
// Weight tiles are read once per token: they are loaded with an L2 evict-first policy so the
// stream does not push the kernel's code, activations and staged tensors out of L2.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Time-bounded wait that ignores the abort flag: before a CTA exits, every copy it issued
// must have landed in its shared memory.
__device__ __forceinline__ bool mb_drain(uint32_t a, uint32_t parity) {
  const uint64_t t0 = now_ns();
  while (!mb_try(a, parity))
    if (now_ns() - t0 > kWaitNs) return false;
  return true;
}
__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                      uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;"
      :: "r"(dst), "l"(map), "r"(bar), "r"(x), "r"(y), "l"(policy) : "memory");
}
__device__ __forceinline__ void tma2d_plain(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      :: "r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(map), "r"(bar), "r"(x), "r"(y) : "memory");
}

// Phase timestamps of two CTAs for the first layers, compiled only with SQ_DECODE_TRACE
// (a profiling build); the product build records nothing.
#ifdef SQ_DECODE_TRACE
__device__ unsigned long long g_decode_trace[2][64][16];
#define DTRACE(layer, slot)                                                                         \
  do {                                                                                              \
    if (threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1) && (layer) < 64)       \
      g_decode_trace[blockIdx.x == 0 ? 0 : 1][(layer)][(slot)] = now_ns();                          \
  } while (0)
__device__ unsigned long long g_decode_arrive[4][256];
__device__ unsigned long long g_decode_warp[4][16];
#define DWARP(layer, which)                                                                         \
  do {                                                                                              \
    if ((threadIdx.x & 31) == 0 && blockIdx.x == 0 && (layer) == 10)                                \
      g_decode_warp[(which)][threadIdx.x >> 5] = now_ns();                                          \
  } while (0)
#define DARRIVE(layer, which)                                                                       \
  do {                                                                                              \
    if (threadIdx.x == 0 && (layer) == 10) g_decode_arrive[(which)][blockIdx.x] = now_ns();         \
  } while (0)
#else
#define DTRACE(layer, slot) do { } while (0)
#define DARRIVE(layer, which) do { } while (0)
#define DWARP(layer, which) do { } while (0)
#endif

// Grid barrier for the compute warps of every CTA (the producer and stager warps never
// join).  One release add on a 64-bit arrival counter (zeroed before the launch); every CTA
// passes the same sequence of barriers, so barrier k of the launch completes when the counter
// reaches (k + 1) * gridDim.x and the add needs no reply.
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
// Split-phase form: grid_arrive adds this CTA's arrival (after a CTA barrier, so the release
// covers every thread's earlier writes) and returns the count to wait for; work that does not
// depend on the other CTAs can run before grid_wait.  The arrival never waits on a load (an
// abort is seen by the wait's polling loop instead).  `nbar` counts the barriers of the launch
// (the same in every thread).
__device__ unsigned long long grid_arrive(const DecodeParams& P, unsigned& nbar) {
  bar_sync(1, kCompute);
  const unsigned long long target = (unsigned long long)(++nbar) * gridDim.x;
  if (threadIdx.x == 0) red_release_add(&P.sync->count, 1ull);
  return target;
}
__device__ bool grid_wait(const DecodeParams& P, unsigned long long target, int* flag) {
  if (threadIdx.x == 0) {
    const DecodeSync* s = P.sync;
    int ok = target != 0;
    if (ok) {
      const uint64_t t0 = now_ns();
      int spins = 0;
      while (ld_acquire_u64(&s->count) < target) {   // one load in flight per poll
        if ((++spins & 15) == 0) {
          if (ld_abort(s)) { ok = 0; break; }
          if (now_ns() - t0 > kWaitNs) { set_abort(P, (int)kDevTimeoutEpilogue); ok = 0; break; }
        }
        if (spins > 64) __nanosleep(20);
      }
    }
    *flag = ok;
  }
  bar_sync(1, kCompute);
  return *flag != 0;
}
__device__ bool grid_sync(const DecodeParams& P, unsigned& nbar, int* flag) {
  return grid_wait(P, grid_arrive(P, nbar), flag);
}

// Block residual + RMSNorm over 4096 channels with 256 threads, the add_rmsnorm_kernel
// arithmetic: res = fp16(h + res) (or h), out = fp16((res * rstd) * w).  The layer-0 input
// is the embedding row of `tok` decoded exactly in place (fp4_embed_kernel arithmetic).
__device__ void block_norm(const DecodeParams& P, const uint16_t* hsrc, const uint16_t* res_in, uint16_t* res_out,
                           const uint16_t* w, long long emb_id, uint16_t* out, float* red8) {
  const int tid = threadIdx.x;
  float vals[16];
  float ss = 0.f;
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    const int c = tid * 8 + n * 2048;
    uint4 ov;
    uint16_t* op = reinterpret_cast<uint16_t*>(&ov);
    if (emb_id >= 0) {
      const int c8 = c / 8;
      const uint32_t cw = *reinterpret_cast<const uint32_t*>(P.emb_codes + emb_id * (kDModel / 2) + c8 * 4);
      const uint32_t bs = e4m3_splat_f16x2(P.emb_scales[emb_id * (kDModel / 16) + (c8 >> 1)]);
      const float g = *P.emb_g;
      const float2 g2 = make_float2(g, g);
      uint32_t m[4];
      e2m1x8_to_f16x2(cw, m);
      ov.x = scale_pair(m[0], bs, g2);
      ov.y = scale_pair(m[1], bs, g2);
      ov.z = scale_pair(m[2], bs, g2);
      ov.w = scale_pair(m[3], bs, g2);
    } else {
      const uint4 hv = ldcg4(hsrc + c);
      const uint16_t* hp = reinterpret_cast<const uint16_t*>(&hv);
      if (res_in) {
        const uint4 rv = ldcg4(res_in + c);
        const uint16_t* rp = reinterpret_cast<const uint16_t*>(&rv);
#pragma unroll
        for (int i = 0; i < 8; ++i) op[i] = f2h(h2f(hp[i]) + h2f(rp[i]));
      } else {
        ov = hv;
      }
    }
    if (res_out) *reinterpret_cast<uint4*>(res_out + c) = ov;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = h2f(op[i]);
      vals[n * 8 + i] = x;
      ss += x * x;
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red8[tid >> 5] = ss;
  bar_sync(1, kCompute);
  float tot = 0.f;
  for (int i = 0; i < 8; ++i) tot += red8[i];
  const float rstd = 1.0f / sqrtf(tot / (float)kDModel + P.eps);
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    const int c = tid * 8 + n * 2048;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const uint16_t* wp = reinterpret_cast<const uint16_t*>(&wv);
    uint4 ov;
    uint16_t* op = reinterpret_cast<uint16_t*>(&ov);
#pragma unroll
    for (int i = 0; i < 8; ++i) op[i] = f2h((vals[n * 8 + i] * rstd) * h2f(wp[i]));
    *reinterpret_cast<uint4*>(out + c) = ov;
  }
  bar_sync(1, kCompute);
}

// Ring of kNst stages.  tag[stage] holds the chunk counter the producer last armed the
// stage with (written before the arming arrive, read after the consumer's acquire), because
// a parity wait alone cannot tell a stage's current lap from the one two laps back, and
// consumers may wait on chunks several laps ahead.
struct Ring {
  uint32_t base, full, empty;
  volatile int* tag;
};

__device__ __forceinline__ bool wait_chunk(const Ring& R, int c, const DecodeSync* s) {
  const int stage = c % kNst;
  const uint32_t a = R.full + 8 * stage, parity = (uint32_t)(c / kNst) & 1u;
  const uint64_t t0 = now_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mb_try(a, parity) && R.tag[stage] == c) return true;
    if (ld_abort(s) || now_ns() - t0 > kWaitNs) return false;
  }
}

// One chunk (16 rows x 1024 columns in ring stage `cs`) of a tile: warp cw of the group takes
// 128-column sub-chunks cw and cw + 4, decodes them into mma.sync A fragments and accumulates
// even / odd k-steps in acc / acc2.  EXACT: every weight FP16(FP32(m b) g), the reference's
// decoded weight (g2 = the global scale twice); otherwise the exact fp16 products m b, the
// global scale applied per output by the caller.  xoff[s2][qq]: offset of the 8 input values
// k = sub * 128 + tq * 32 + 8 qq of the chunk (x_offsets).
template <bool EXACT>
__device__ __forceinline__ void chunk_mma(const unsigned char* cs, const uint16_t* Xs, int kc, int cw, int lane,
                                          const int (&xoff)[2][4], float2 g2, float (&acc)[4], float (&acc2)[4]) {
  const int gq = lane >> 2, tq = lane & 3;
  constexpr int code_row = kKc / 2, scale_row = kKc / 16;
  const unsigned char* ss = cs + kCodeBytes;
#pragma unroll
  for (int s2 = 0; s2 < 2; ++s2) {
    const int sub = cw + 4 * s2;
    uint4 xr[4];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq)
      xr[qq] = (gq == 0) ? *reinterpret_cast<const uint4*>(Xs + kc * kKc + xoff[s2][qq]) : make_uint4(0, 0, 0, 0);
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
        const uint4 xq = xr[j >> 1];
        const uint32_t b0 = (j & 1) ? xq.z : xq.x, b1 = (j & 1) ? xq.w : xq.y;
        mma16816((j & 1) ? acc2 : acc, a, b0, b1);
      }
    }
  }
}

// Offsets (within a 1024-column chunk) of the input values a lane reads: linear, or for an
// input stored as swizzled rows of 64 (swz) the same elements there.  Column k = sub * 128 +
// tq * 32 + 8 qq lies in row 2 sub + (tq >> 1) + 16 kc, chunk (tq & 1) * 4 + qq; the row's low
// three bits do not depend on kc, so the offsets are constant over a phase.
template <bool XSWZ>
__device__ __forceinline__ void x_offsets(int cw, int tq, int (&xoff)[2][4]) {
#pragma unroll
  for (int s2 = 0; s2 < 2; ++s2)
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      const int sub = cw + 4 * s2, h = 2 * sub + (tq >> 1), c = (tq & 1) * 4 + qq;
      xoff[s2][qq] = XSWZ ? h * 64 + (((c ^ h) & 7) << 3) : sub * 128 + tq * 32 + 8 * qq;
    }
}

// One projection phase: this CTA's tiles [t0, t1) of a 16-row-tiled matrix, chunks of 1024
// columns from ring counter ctr on (cpt per tile, cpt even); tiles alternate between the two
// 4-warp consumer groups, and the producer issues each pair of tiles chunk-interleaved (tile
// 2m chunk kc at ctr + 2m cpt + 2 kc, tile 2m + 1 one after it) so that both groups see the
// whole ring ahead of them; per tile the fp4_gemv_stream_kernel arithmetic (EXACT: weights
// decoded exactly; else the factored global scale), chunks taken two per wait, the four
// warps' sums added in order.
template <bool XSWZ, bool EXACT>
__device__ void gemv_phase(const DecodeParams& P, const Ring& R, const unsigned char* sm, int ctr, int t0, int t1,
                           int cpt, const uint16_t* Xs, const float* gptr, uint16_t* Y, float* red, bool argmax,
                           float& best, int& bidx, bool& ok) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp >> 2, cw = warp & 3;
  const int gq = lane >> 2, tq = lane & 3;
  const float gsc = *gptr;
  const float2 g2 = make_float2(gsc, gsc);
  int xoff[2][4];
  x_offsets<XSWZ>(cw, tq, xoff);
  for (int i = q; i < t1 - t0; i += 2) {
    const int tile = t0 + i;
    // ring position of chunk kc: tiles 2m and 2m + 1 (one per group) are issued interleaved
    const int base = ctr + (i >> 1) * 2 * cpt, paired = (i | 1) < t1 - t0;
    const int step = paired ? 2 : 1, off = paired ? (i & 1) : 0;
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
    for (int kc = 0; kc < cpt; kc += 2) {
      const int c = base + kc * step + off, c1 = c + step;
      const int st0 = c % kNst, st1 = c1 % kNst;
      if (ok && !(wait_chunk(R, c, P.sync) && wait_chunk(R, c1, P.sync))) {
        ok = false;
        set_abort(P, (int)kDevTimeoutMma);
      }
      if (ok) {
        chunk_mma<EXACT>(sm + oRing + st0 * kStageBytes, Xs, kc, cw, lane, xoff, g2, acc, acc2);
        chunk_mma<EXACT>(sm + oRing + st1 * kStageBytes, Xs, kc + 1, cw, lane, xoff, g2, acc, acc2);
      }
      __syncwarp();
      if (lane == 0) {
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(R.empty + 8 * st0) : "memory");
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(R.empty + 8 * st1) : "memory");
      }
    }
    float* rq = red + q * (4 * 32 * 4);
#pragma unroll
    for (int e = 0; e < 4; ++e) rq[(cw * 32 + lane) * 4 + e] = acc[e] + acc2[e];
    bar_sync(2 + q, 128);
    if (cw == 0) {
      float sacc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int w = 0; w < 4; ++w)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[e] += rq[(w * 32 + lane) * 4 + e];
      if (!EXACT)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[e] *= gsc;
      if (tq == 0) {
        const int na = tile * kRows + gq, nb = na + 8;
        const uint16_t ya = f2h(sacc[0]), yb = f2h(sacc[2]);
        Y[na] = ya;
        Y[nb] = yb;
        if (argmax) {
          argmax_merge(best, bidx, h2f(ya), na);
          argmax_merge(best, bidx, h2f(yb), nb);
        }
      }
    }
    bar_sync(2 + q, 128);
  }
}

// Producer: the CTA's chunks in consumption order (per layer: in_proj tiles x 4 chunks,
// out_proj tiles x 8 chunks; then lm_head tiles x 4 chunks).  No separate L2 prefetch: bulk
// L2 prefetches of the next rows measured slower (they occupy the same copy engine).
struct TileRange { int t0, t1; };
__device__ __forceinline__ TileRange tile_range(int ntiles, int cta, int ncta) {
  return TileRange{(int)((long long)ntiles * cta / ncta), (int)((long long)ntiles * (cta + 1) / ncta)};
}

__device__ void producer(const DecodeParams& P, const Ring& R) {
  const int cta = blockIdx.x, ncta = gridDim.x;
  const TileRange rin = tile_range(kZx / kRows, cta, ncta), rout = tile_range(kDModel / kRows, cta, ncta);
  const TileRange rhead = tile_range(P.vocab / kRows, cta, ncta);
  int ctr = 0;
  bool ok = true;
  const uint64_t policy = evict_first_policy();
  auto issue = [&](const CUtensorMap* mc, const CUtensorMap* ms, int tile, int kc) {
    const int stage = ctr % kNst;
    const uint32_t par = (uint32_t)(ctr / kNst) & 1u;
    if (ok && !mb_wait(R.empty + 8 * stage, par ^ 1u, P.sync)) {
      ok = false;
      set_abort(P, (int)kDevTimeoutProducer);
    }
    if (ok) {
      const uint32_t fb = R.full + 8 * stage;
      R.tag[stage] = ctr;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(fb), "r"((uint32_t)kStageBytes)
                   : "memory");
      const uint32_t dst = R.base + stage * kStageBytes;
      tma2d(dst, mc, fb, kc * (kKc / 8), tile * kRows, policy);
      tma2d(dst + kCodeBytes, ms, fb, kc * (kKc / 64), tile * kRows, policy);
    }
    ++ctr;
  };
  // tiles [r.t0, r.t1) in the consumers' order: pairs of tiles chunk-interleaved
  auto issue_tiles = [&](const CUtensorMap* m, TileRange r, int cpt) {
    for (int t = r.t0; t < r.t1; t += 2)
      for (int kc = 0; kc < cpt; ++kc)
        for (int u = t; u < t + 2 && u < r.t1; ++u) issue(m, m + 1, u, kc);
  };
  for (int step = 0; step < P.steps && ok; ++step) {
  for (int l = 0; l < P.n_layer && ok; ++l) {
    const CUtensorMap* mi = P.maps + (2 * l) * 2;
    issue_tiles(mi, rin, kDModel / kKc);
    const CUtensorMap* mo = P.maps + (2 * l + 1) * 2;
    issue_tiles(mo, rout, kDInner / kKc);
  }
  const CUtensorMap* mh = P.maps + (2 * P.n_layer) * 2;
  for (int t = rhead.t0; t < rhead.t1 && ok; t += 2) {
    issue_tiles(mh, TileRange{t, min(rhead.t1, t + 2)}, kDModel / kKc);
  }
  }
  // every issued copy has landed before the CTA may exit
  const int issued = ctr;
  for (int i = 0; i < kNst && i < issued; ++i) {
    const int c = issued - 1 - i;
    if (!mb_drain(R.full + 8 * (c % kNst), (uint32_t)(c / kNst) & 1u)) break;
  }
}

// ---------------------------------------------------------------- scan step of one head
// The one-token codec step of ssu_sq325_kernel (MODE 2, TC 1) for the 64 rows of head
// `hh`, in three parts: scan_unpack decodes the stored pairs (before the token's inputs
// exist), scan_step runs the conv step on the raw in_proj columns with the ring history, the
// group dots, recurrence, readout and the token tail (scales), and publishes y; scan_finish
// requantises and packs the state (after y is out).  256 threads: B/C conv one channel each,
// dots one task each, rows on four lanes each.  One code path for all seven layouts: the
// row's stored pairs live in shared memory (pair-major, [np][64] float2) and runtime loops
// run the same per-pair operations, in the same order, as recur_row / requant_row, so the
// step is compact enough to stay in the instruction caches.
struct Geo { int n8, n4, ns, nz, f, np, w8, w4; };
__device__ __forceinline__ Geo geo_of(int layout) {
  Geo g;
  switch (layout) {                                   // the seven tier layouts (index order of the C ABI)
    case 0: g.n8 = 32; g.n4 = 28; break;
    case 1: g.n8 = 16; g.n4 = 60; break;
    case 2: g.n8 = 8; g.n4 = 76; break;
    case 3: g.n8 = 24; g.n4 = 44; break;
    case 4: g.n8 = 36; g.n4 = 20; break;
    case 5: g.n8 = 40; g.n4 = 12; break;
    default: g.n8 = 44; g.n4 = 4; break;
  }
  g.ns = g.n8 + g.n4;
  g.nz = 128 - g.ns;
  g.f = g.ns + 2;
  g.np = g.ns / 2;
  g.w8 = g.n8 / 2;
  g.w4 = g.n4 / 2;
  return g;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ void mb_expect(uint32_t bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}

// The step's static inputs in kScanPieces pieces (each a multiple of 16 bytes, both ends
// 16-byte aligned): predictor table, basis, permutation, the head's packed rows, conv taps /
// biases, the conv ring history and the per-head scalars.
constexpr int kScanPieces = 28;
__device__ __forceinline__ unsigned scan_stage_bytes(const Geo& G) {
  return G.f * G.nz * 2 + G.nz * 4 + 128 + 64 * (2 * G.w8 + G.w4) + 3 * 128 + 512 + 128 + 2048 + 512 + 3 * 640 + 32 +
         256 + 256 + 512;
}
struct Piece { void* d; const void* s; int bytes; };
__device__ __forceinline__ Piece scan_stage_piece(const DecLayer& L, int hh, unsigned char* sc, int k, int pos) {
  const Geo G = geo_of(L.layout);
  const int g = hh / (kHeads / kGroups);
  const long long row0 = (long long)hh * 64;
  unsigned char* rows = sc + sRows;
  void* d = nullptr;
  const void* src = nullptr;
  int bytes = 0;
  switch (k) {
    case 0: d = sc + sPred; src = L.predictor + (long long)g * G.f * G.nz; bytes = G.f * G.nz * 2; break;
    case 1: d = sc + sBasis; src = L.basis + (long long)g * G.nz * 2; bytes = G.nz * 4; break;
    case 2: d = sc + sPerm; src = L.perm + g * 128; bytes = 128; break;
    case 3: d = rows; src = L.lo + row0 * G.w8; bytes = 64 * G.w8; break;
    case 4: d = rows + 64 * G.w8; src = L.hi + row0 * G.w8; bytes = 64 * G.w8; break;
    case 5: d = rows + 128 * G.w8; src = L.q4 + row0 * G.w4; bytes = 64 * G.w4; break;
    case 6: d = rows + 128 * G.w8 + 64 * G.w4; src = L.latent + row0 * 2; bytes = 128; break;
    case 7: d = rows + 128 * G.w8 + 64 * G.w4 + 128; src = L.s8 + row0; bytes = 128; break;
    case 8: d = rows + 128 * G.w8 + 64 * G.w4 + 256; src = L.s4 + row0; bytes = 128; break;
    case 9: d = sc + sWx; src = L.conv_w + (long long)hh * 64 * 4; bytes = 512; break;
    case 10: d = sc + sBx; src = L.conv_b + hh * 64; bytes = 128; break;
    case 11: d = sc + sWbc; src = L.conv_w + (long long)(8192 + g * 128) * 4; bytes = 1024; break;
    case 12: d = sc + sWbc + 1024; src = L.conv_w + (long long)(9216 + g * 128) * 4; bytes = 1024; break;
    case 13: d = sc + sBbc; src = L.conv_b + 8192 + g * 128; bytes = 256; break;
    case 14: d = sc + sBbc + 256; src = L.conv_b + 9216 + g * 128; bytes = 256; break;
    case 24: d = sc + sLs; src = L.latent_scale; bytes = kGroups * 2 * 2; break;
    case 25: d = sc + sDv; src = L.D; bytes = kHeads * 2; break;
    case 26: d = sc + sDtb; src = L.dt_bias; bytes = kHeads * 2; break;
    case 27: d = sc + sAv; src = L.A; bytes = kHeads * 4; break;
    default: {                                        // 15..23: conv ring history, 3 slots x 3 pieces
      const int hk = (k - 15) / 3, part = (k - 15) % 3;
      const uint16_t* rs = L.ring + ((pos - 3 + hk) & 3) * 10240;
      unsigned char* hd = sc + sHist + hk * 640;
      if (part == 0) { d = hd; src = rs + hh * 64; bytes = 128; }
      else if (part == 1) { d = hd + 128; src = rs + 8192 + g * 128; bytes = 256; }
      else { d = hd + 384; src = rs + 9216 + g * 128; bytes = 256; }
    }
  }
  return Piece{d, src, bytes};
}

// A lane's stored pairs of its row: pair jp = k + 4 i in v[i] (k = lane of the row, at most
// 11 pairs a lane for 42 pairs a row), in registers from the unpack to the requant.
constexpr int kRowPairs = 11;
struct RowState { float2 v[kRowPairs]; };

__device__ void scan_step(const DecodeParams& P, const DecLayer& L, int hh, unsigned char* sc, RowState& rs,
                          int layer, int pos, TokenScales& ts, float2& zlat) {
  const Geo G = geo_of(L.layout);
  const int NS = G.ns, NZ = G.nz, F = G.f, W8 = G.w8, W4 = G.w4, NP = G.np, N8 = G.n8;
  const int tid = threadIdx.x, g = hh / (kHeads / kGroups);
  const bool group_leader = (hh % (kHeads / kGroups)) == 0;
  const uint16_t* rawPred = reinterpret_cast<const uint16_t*>(sc + sPred);
  const uint16_t* rawBasis = reinterpret_cast<const uint16_t*>(sc + sBasis);
  const uint8_t* perm = sc + sPerm;
  const uint16_t* hist = reinterpret_cast<const uint16_t*>(sc + sHist);   // [3][x 64 | B 128 | C 128]
  float* sPf = reinterpret_cast<float*>(sc + sP4o);
  float* sV = reinterpret_cast<float*>(sc + sV2o);
  float* sX = reinterpret_cast<float*>(sc + sXo);
  float* sDots = reinterpret_cast<float*>(sc + sDotso);
  float* sDD = reinterpret_cast<float*>(sc + sDDo);
  const int slot = pos & 3;
  uint16_t* ring_new = L.ring + slot * 10240;
  // -- conv step (state_quant.py:291-297) of B/C in tier order, x of own channels, dt --
  {
    const int j = tid & 127;
    const int isC = tid >> 7;
    const int n = perm[j];
    const uint16_t rawbits = ldcg16(P.zx + 2 * kDInner + isC * 1024 + g * 128 + n);     // raw B | C
    const uint16_t* wbc = reinterpret_cast<const uint16_t*>(sc + sWbc) + (isC * 128 + n) * 4;
    const uint16_t* bbc = reinterpret_cast<const uint16_t*>(sc + sBbc) + isC * 128 + n;
    float w[5];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = h2f(wbc[i]);
    w[4] = h2f(*bbc);
    const int hoff = 64 + isC * 128 + n;
    const float v = conv_step_value(w, h2f(hist[0 * 320 + hoff]), h2f(hist[1 * 320 + hoff]),
                                    h2f(hist[2 * 320 + hoff]), h2f(rawbits));
    sPf[(j >> 1) * 4 + (j & 1) + 2 * isC] = v;
    if (group_leader) {                                // newest raw B/C columns, channel order
      const int ch = tid & 127;
      ring_new[8192 + isC * 1024 + g * 128 + ch] = ldcg16(P.zx + 2 * kDInner + isC * 1024 + g * 128 + ch);
    }
  }
  if (tid < 64) {
    const uint16_t rawbits = ldcg16(P.zx + kDInner + hh * 64 + tid);                    // raw x
    const uint16_t* wx = reinterpret_cast<const uint16_t*>(sc + sWx) + tid * 4;
    float w[5];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = h2f(wx[i]);
    w[4] = h2f(reinterpret_cast<const uint16_t*>(sc + sBx)[tid]);
    sX[tid] = conv_step_value(w, h2f(hist[0 * 320 + tid]), h2f(hist[1 * 320 + tid]), h2f(hist[2 * 320 + tid]),
                              h2f(rawbits));
    ring_new[hh * 64 + tid] = rawbits;
  } else if (tid == 64) {
    const float dtv = softplus_ref(h2f(ldcg16(P.zx + 2 * kDInner + 2 * 1024 + hh)) +
                                   h2f(reinterpret_cast<const uint16_t*>(sc + sDtb)[hh]));
    sDD[0] = dtv;
    sDD[1] = expf(reinterpret_cast<const float*>(sc + sAv)[hh] * dtv);
  }
  bar_sync(1, kCompute);
  DTRACE(layer, 10);
  // -- group dots (fp4_zero_predictor_codec_v1.py:221-225 and the zero-tier dots) --
  for (int f = tid; f < F + 5; f += kCompute) {
    float acc0 = 0.f, acc1 = 0.f;
    if (f < F) {
      const uint16_t* pr = rawPred + f * NZ;
#pragma unroll 4
      for (int d = 0; d < NZ; d += 2) {
        const int j0 = NS + d;
        acc0 = fmaf(sPf[(j0 >> 1) * 4 + 2], h2f(pr[d]), acc0);
        acc1 = fmaf(sPf[(j0 >> 1) * 4 + 3], h2f(pr[d + 1]), acc1);
      }
      const float acc = acc0 + acc1;
      if (f < NS) sV[f] = acc;
      else sDots[5 + f - NS] = acc;
    } else {
      const int k = f - F;   // 0: B.C, 1: basis0.C, 2: basis1.C, 3: basis0.B, 4: basis1.B
      const int voff = (k >= 3 || k == 0) ? 0 : 2;
#pragma unroll 4
      for (int d = 0; d < NZ; d += 2) {
        const int j0 = NS + d;
        const float* q = sPf + (j0 >> 1) * 4;
        const float u0 = (k == 0) ? q[0] : h2f(rawBasis[2 * d + ((k - 1) & 1)]);
        const float u1 = (k == 0) ? q[1] : h2f(rawBasis[2 * (d + 1) + ((k - 1) & 1)]);
        const float v0 = (k == 0) ? q[2] : q[voff], v1 = (k == 0) ? q[3] : q[voff + 1];
        acc0 = fmaf(u0, v0, acc0);
        acc1 = fmaf(u1, v1, acc1);
      }
      sDots[k] = acc0 + acc1;
    }
  }
  bar_sync(1, kCompute);
  DTRACE(layer, 11);
  // -- per-row recurrence and readout: row p = tid / 4 on four adjacent lanes, lane k = tid % 4
  //    takes the pairs jp = k, k + 4, ... (readout stream k of recur_row4); the stored pairs
  //    were decoded into rs by scan_unpack --
  const unsigned char* pLat = sc + sRows + 64 * (2 * W8 + W4);
  {
    const int p = tid >> 2, k = tid & 3;
    const uint16_t* lsv = reinterpret_cast<const uint16_t*>(sc + sLs);
    const float ls0 = h2f(lsv[g * 2 + 0]), ls1 = h2f(lsv[g * 2 + 1]);
    const float ils0 = __frcp_rn(ls0), ils1 = __frcp_rn(ls1);
    const float2 ls2 = make_float2(ls0, ls1), nls2 = make_float2(-ls0, -ls1), ils2 = make_float2(ils0, ils1);
    float2 zz = make_float2(e4m3_to_f32(pLat[p * 2 + 0]) * ls0, e4m3_to_f32(pLat[p * 2 + 1]) * ls1);
    const float dv = h2f(reinterpret_cast<const uint16_t*>(sc + sDv)[hh]);
    const float dtv = sDD[0], dec = sDD[1], x = sX[p];
    // recur_row4, stream k on this lane
    const float2 dd = make_float2(dec, dec), dt2 = make_float2(dtv, dtv), xx = make_float2(x, x);
    float2 ys = make_float2(0.f, 0.f), cs = ys;
    float m8a = 0.f, m8b = 0.f, m4a = 0.f, m4b = 0.f;
    const float4* cpp = reinterpret_cast<const float4*>(sPf);
    const float2* vpp = reinterpret_cast<const float2*>(sV);
#pragma unroll
    for (int i = 0; i < kRowPairs; ++i) {
      const int jp = k + 4 * i;
      if (jp < NP) {
        const float4 bc = cpp[jp];
        const float2 cv = vpp[jp];
        const float2 pr = rs.v[i];
        const float2 upd = __fmul2_rn(__fmul2_rn(make_float2(bc.x, bc.y), dt2), xx);   // (B*dt)*x
        const float2 sn = __ffma2_rn(pr, dd, upd);                                      // prior*decay + upd
        rs.v[i] = sn;
        ys = __ffma2_rn(sn, make_float2(bc.z, bc.w), ys);
        cs = __ffma2_rn(pr, cv, cs);
        if (2 * jp < N8) { m8a = fmaxf(m8a, fabsf(sn.x)); m8b = fmaxf(m8b, fabsf(sn.y)); }
        else             { m4a = fmaxf(m4a, fabsf(sn.x)); m4b = fmaxf(m4b, fabsf(sn.y)); }
      }
    }
    // combine the four lanes of the row: ((t0 + t1) + (t2 + t3)); max over the lanes
    const float ty = ys.x + ys.y, tc = cs.x + cs.y;
    const unsigned mask = 0xffffffffu;
    const int base = (threadIdx.x & 31) & ~3;
    float ty4[4], tc4[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      ty4[q] = __shfl_sync(mask, ty, base + q);
      tc4[q] = __shfl_sync(mask, tc, base + q);
    }
    const float ysum = (ty4[0] + ty4[1]) + (ty4[2] + ty4[3]);
    const float ycorr = (tc4[0] + tc4[1]) + (tc4[2] + tc4[3]);
    float m8 = fmaxf(m8a, m8b), m4 = fmaxf(m4a, m4b);
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      m8 = fmaxf(m8, __shfl_xor_sync(mask, m8, o));
      m4 = fmaxf(m4, __shfl_xor_sync(mask, m4, o));
    }
    float dots[7];
#pragma unroll
    for (int i = 0; i < 7; ++i) dots[i] = sDots[i];
    const float out = token_tail_sums(ysum, ycorr, m8, m4, x, dtv, dec, dv, dots, zz, ls2, nls2, ils2, ts);  // same in the four lanes
    zlat = zz;
    if (k == 0) P.y[hh * 64 + p] = f2h(out);
  }
}

// The stored pairs of the head's 64 rows (packed rows staged in shared memory) as fp32 pairs
// in the lanes' registers: the INT8 / INT4 codes times the row scales.  Depends only on the
// previous step's state, so it runs before the token's inputs exist.
__device__ void scan_unpack(const DecLayer& L, const unsigned char* sc, RowState& rs) {
  const Geo G = geo_of(L.layout);
  const int W8 = G.w8, W4 = G.w4, NP = G.np, N8 = G.n8;
  const unsigned char* pLo = sc + sRows;
  const unsigned char* pHi = pLo + 64 * W8;
  const unsigned char* pQ4 = pHi + 64 * W8;
  const uint16_t* pS8 = reinterpret_cast<const uint16_t*>(pQ4 + 64 * W4 + 128);
  const uint16_t* pS4 = pS8 + 64;
  const int p = threadIdx.x >> 2, k = threadIdx.x & 3;
  const float s8 = h2f(pS8[p]), s4 = h2f(pS4[p]);
#pragma unroll
  for (int i = 0; i < kRowPairs; ++i) {
    const int jp = k + 4 * i;
    if (jp < NP) {
      float v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = 2 * jp + e;
        if (j < N8) {
          const int lo = (pLo[p * W8 + j / 2] >> (4 * (j & 1))) & 15;
          const int hi = (pHi[p * W8 + j / 2] >> (4 * (j & 1))) & 15;
          const int ub = (hi << 4) | lo;
          v[e] = (float)(ub - 256 * (ub > 127)) * s8;
        } else {
          const int j4 = j - N8;
          const int nib = (pQ4[p * W4 + j4 / 2] >> (4 * (j4 & 1))) & 15;
          v[e] = (float)(nib - 16 * (nib > 7)) * s4;
        }
      }
      rs.v[i] = make_float2(v[0], v[1]);
    }
  }
}

// The rest of the step, which only this CTA's next step reads: requant of the new pairs with
// the row scales ts, the codes packed into the staged rows, the latent bytes and scales, and
// the rows copied back to the layer state.  Runs after the readout y has been published.
__device__ void scan_finish(const DecLayer& L, int hh, unsigned char* sc, const RowState& rs, const TokenScales& ts,
                            float2 zz) {
  const Geo G = geo_of(L.layout);
  const int W8 = G.w8, W4 = G.w4, NP = G.np, N8 = G.n8;
  const int tid = threadIdx.x, g = hh / (kHeads / kGroups);
  unsigned char* pLo = sc + sRows;
  unsigned char* pHi = pLo + 64 * W8;
  unsigned char* pQ4 = pHi + 64 * W8;
  unsigned char* pLat = pQ4 + 64 * W4;
  uint16_t* pS8 = reinterpret_cast<uint16_t*>(pLat + 128);
  uint16_t* pS4 = pS8 + 64;
  {
    const int p = tid >> 2, k = tid & 3;
    // requant + pack of this lane's pairs: v = requant(S), then the codes of v
    const float s8 = ts.s8, s4 = ts.s4;
    const float2 s82 = make_float2(s8, s8), ns82 = make_float2(-s8, -s8), i82 = make_float2(ts.i8, ts.i8);
    const float2 s42 = make_float2(s4, s4), ns42 = make_float2(-s4, -s4), i42 = make_float2(ts.i4, ts.i4);
    const float m8s = -kMagic * s8, m4s = -kMagic * s4;
    const float2 nm82 = make_float2(m8s, m8s), nm42 = make_float2(m4s, m4s);
    const float i8 = s8 > 0.f ? __frcp_rn(s8) : 0.f;
    const float i4 = s4 > 0.f ? __frcp_rn(s4) : 0.f;
#pragma unroll
    for (int i = 0; i < kRowPairs; ++i) {
      const int jp = k + 4 * i;
      if (jp >= NP) break;
      const bool t8 = 2 * jp < N8;
      float2 v = rs.v[i];
      requant_pair(v.x, v.y, t8 ? ns82 : ns42, t8 ? i82 : i42, t8 ? 127.f : 7.f, t8 ? s82 : s42, t8 ? nm82 : nm42);
      if (t8) {
        const int qa = __float2int_rn(div_exact(v.x, s8, i8));
        const int qb = __float2int_rn(div_exact(v.y, s8, i8));
        pLo[p * W8 + jp] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
        pHi[p * W8 + jp] = (unsigned char)(((qa >> 4) & 15) | (((qb >> 4) & 15) << 4));
      } else {
        const int qa = __float2int_rn(div_exact(v.x, s4, i4));
        const int qb = __float2int_rn(div_exact(v.y, s4, i4));
        pQ4[p * W4 + (jp - N8 / 2)] = (unsigned char)((qa & 15) | ((qb & 15) << 4));
      }
    }
    if (k == 0) {
      const uint16_t* lsv = reinterpret_cast<const uint16_t*>(sc + sLs);
      const float ls0 = h2f(lsv[g * 2 + 0]), ls1 = h2f(lsv[g * 2 + 1]);
      const float ils0 = __frcp_rn(ls0), ils1 = __frcp_rn(ls1);
      pLat[p * 2 + 0] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.x, ls0, ils0), -448.f), 448.f));
      pLat[p * 2 + 1] = f32_to_e4m3(fminf(fmaxf(div_exact(zz.y, ls1, ils1), -448.f), 448.f));
      pS8[p] = f2h(s8);
      pS4[p] = f2h(s4);
    }
  }
  bar_sync(1, kCompute);
  const long long row0 = (long long)hh * 64;
  auto copy_out = [&](unsigned char* dst, const unsigned char* src, int bytes) {
    for (int i = tid; i < bytes / 16; i += kCompute)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  };
  copy_out(L.lo + row0 * W8, pLo, 64 * W8);
  copy_out(L.hi + row0 * W8, pHi, 64 * W8);
  copy_out(L.q4 + row0 * W4, pQ4, 64 * W4);
  copy_out(L.latent + row0 * 2, pLat, 128);
  copy_out(reinterpret_cast<unsigned char*>(L.s8 + row0), reinterpret_cast<unsigned char*>(pS8), 128);
  copy_out(reinterpret_cast<unsigned char*>(L.s4 + row0), reinterpret_cast<unsigned char*>(pS4), 128);
}

// Adapter gate partial of warp w: the dot u . w over channels [512 w, 512 w + 512), lane
// stride 8, then the warp sum.  The gate logit is the sum of the eight partials in warp
// order (the summation of the multi-kernel resurface_gatednorm_kernel).
__device__ __forceinline__ float gate_partial(const uint16_t* Us, const uint16_t* Ws, int w, int lane) {
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

// Resurface adapter + gated RMSNorm for one token, warp w = norm group w: the
// resurface_gatednorm_kernel arithmetic with one group per CTA (head mix on the tensor
// cores, correction, x = y * silu(z), RMSNorm over 1024 channels).  The gate partials were
// computed earlier (gpart[8]); V (staged one layer ahead) and y sit in shared memory.
__device__ void resurface_norm(const DecodeParams& P, const DecLayer& L, const float* gpart, const uint16_t* Ys,
                               const uint16_t* Vs, const uint16_t* Gs, const uint16_t* Ns, uint16_t* zout, int layer) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int grp = warp;
  const bool has_ad = L.ad_V != nullptr;
  float gate = 0.f;
  if (has_ad) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += gpart[w];
    const float lg = h2f(f2h(h2f(f2h(s)) + h2f(L.ad_b[0])));
    gate = h2f(f2h(L.hard ? (lg > 0.f ? 1.f : 0.f) : __frcp_rn(1.0f + expf(-lg))));
  }
  DTRACE(layer, 13);
  float acc[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  if (has_ad) {
    const int mi = lane >> 3, rr = lane & 7;
    const int i0 = grp * 16;                          // V rows of this group's heads
#pragma unroll
    for (int k0 = 0; k0 < 128; k0 += 16) {
      uint32_t a[4];
      const int vr = i0 + rr + (mi & 1) * 8, vc = k0 + (mi >> 1) * 8;   // V row, first column of the 8
      ldsm_x4(a, Vs + (vc >> 6) * 128 * 64 + swz(vr, vc & 63));
#pragma unroll
      for (int n2 = 0; n2 < 4; ++n2) {
        uint32_t bfr[4];
        ldsm_x4_t(bfr, Ys + (k0 + rr + (mi & 1) * 8) * kYPitch + n2 * 16 + (mi >> 1) * 8);
        mma16816(acc[2 * n2], a, bfr[0], bfr[1]);
        mma16816(acc[2 * n2 + 1], a, bfr[2], bfr[3]);
      }
    }
  }
  DTRACE(layer, 14);
  // The mix results and the x values go through this warp's 16 V rows (4 KB, no longer read).
  float* scr0 = reinterpret_cast<float*>(const_cast<uint16_t*>(Vs) + grp * 16 * 64);      // 512 floats
  float* scr1 = reinterpret_cast<float*>(const_cast<uint16_t*>(Vs) + 128 * 64 + grp * 16 * 64);
  auto scr_at = [&](int n, int e) { return (n < 4 ? scr0 + (n * 4 + e) * 32 : scr1 + ((n - 4) * 4 + e) * 32) + lane; };
  __syncwarp();
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) *scr_at(n, e) = acc[n][e];
  const uint16_t* zs = zout + grp * 1024;               // z of this group, staged where yn goes
  const uint16_t* ns = Ns + grp * 1024;
  float ss = 0.f;
  const int ia = grp * 16 + gq, ib = ia + 8;
  const int la = gq, lb = gq + 8;
  const float ga = has_ad ? h2f(f2h(gate * h2f(Gs[ia]))) : 0.f;
  const float gb = has_ad ? h2f(f2h(gate * h2f(Gs[ib]))) : 0.f;
  const __half2 ga2 = __float2half2_rn(ga), gb2 = __float2half2_rn(gb);
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int p0 = n * 8 + 2 * tq;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int i = half ? ib : ia, li = half ? lb : la;
      float* sp = scr_at(n, 2 * half);
      const float2 x2 = resurface_pair(*reinterpret_cast<const uint32_t*>(Ys + i * kYPitch + p0),
                                       *reinterpret_cast<const uint32_t*>(zs + swz(li, p0)), sp[0], sp[32],
                                       half ? gb2 : ga2, has_ad);
      sp[0] = x2.x;
      sp[32] = x2.y;
      ss += x2.x * x2.x;
      ss += x2.y * x2.y;
    }
  }
  ss = warp_sum(ss);
  const float rstd = 1.0f / sqrtf(ss / 1024.0f + P.eps);
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int p0 = n * 8 + 2 * tq;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int li = half ? lb : la;
      const float* sp = scr_at(n, 2 * half);
      const float2 w2 = __half22float2(*reinterpret_cast<const __half2*>(ns + swz(li, p0)));
      const float o0 = (sp[0] * rstd) * w2.x;
      const float o1 = (sp[32] * rstd) * w2.y;
      __half2 hv = __floats2half2_rn(o0, o1);
      *reinterpret_cast<__half2*>(zout + grp * 1024 + swz(li, p0)) = hv;   // each lane's own z slots
    }
  }
}


// Stager (one lane of its own warp): the per-layer inputs that do not depend on the token
// (gated-norm weights, adapter V / gate weights / g; for CTAs with a scan head the scan
// statics, the head's packed rows and the conv ring history) as bulk / TMA copies on `full`,
// one layer ahead: layer g
// (counted over all steps) is issued once the compute warps have released the buffers of
// layer g - 1 (`free`, arrived after that layer's Resurface).  Issuing ~30 copies takes
// microseconds while the weight stream occupies the copy engine, so it runs off the compute
// warps' path.  The state rows and conv ring it reads were written by the previous step and
// made visible by the grid barriers since; the proxy fence orders them before the copies.
__device__ void stager(const DecodeParams& P, unsigned char* sm, uint32_t full, uint32_t free_bar, int item) {
  unsigned char* sc = sm + oScan;
  uint16_t* Ws = reinterpret_cast<uint16_t*>(sm + oAdw);
  uint16_t* Gn = reinterpret_cast<uint16_t*>(sm + oGnw);
  uint16_t* Ag = reinterpret_cast<uint16_t*>(sm + oAdg);
  uint16_t* Vs = reinterpret_cast<uint16_t*>(sm + oV);
  int armed = 0;
  for (int step = 0; step < P.steps; ++step)
    for (int l = 0; l < P.n_layer; ++l) {
      const int g = step * P.n_layer + l;
      if (g > 0 && !mb_wait(free_bar, (uint32_t)(g - 1) & 1u, P.sync)) {
        set_abort(P, (int)kDevTimeoutProducer);
        goto drain;
      }
      {
        const DecLayer& L = P.layers[l];
        asm volatile("fence.proxy.async;" ::: "memory");
        unsigned bytes = kDInner * 2;
        if (L.ad_V) bytes += kDModel * 2 + kHeads * 2 + 128 * 128 * 2;
        if (item >= 0) bytes += scan_stage_bytes(geo_of(L.layout));
        mb_expect(full, bytes);
        ++armed;
        tma2d_plain(Gn, P.aux_maps + 2 * l + 1, full, 0, 0);          // [128][64] swizzled
        if (L.ad_V) {
          bulk_g2s(Ws, L.ad_w, kDModel * 2, full);
          bulk_g2s(Ag, L.ad_g, kHeads * 2, full);
          tma2d_plain(Vs, P.aux_maps + 2 * l, full, 0, 0);             // 2 x [128][64] swizzled
          tma2d_plain(Vs + 128 * 64, P.aux_maps + 2 * l, full, 64, 0);
        }
        if (item >= 0)
          for (int k = 0; k < kScanPieces; ++k) {
            const Piece pc = scan_stage_piece(L, item, sc, k, P.pos + step);
            bulk_g2s(pc.d, pc.s, (unsigned)pc.bytes, full);
          }
      }
    }
drain:
  // every issued copy has landed before the CTA may exit
  if (armed) mb_drain(full, (uint32_t)(armed - 1) & 1u);
}

template <bool EXACT>
__global__ void __launch_bounds__(kThreads, 1)
decode_step_kernel(const __grid_constant__ DecodeParams P) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const int tid = threadIdx.x, warp = tid >> 5;
  if ((__cvta_generic_to_shared(sm) & 1023u) != 0) {    // the swizzled tiles assume a 1024-byte aligned base
    if (tid == 0) atomicOr(P.err, (int)kDevBadArgs);
    return;
  }
  Ring R;
  R.base = (uint32_t)__cvta_generic_to_shared(sm + oRing);
  R.full = (uint32_t)__cvta_generic_to_shared(sm + oBar);
  R.empty = R.full + 8 * kNst;
  R.tag = reinterpret_cast<volatile int*>(sm + oMisc + 320);
  if (tid == 0) {
    for (int i = 0; i < kNst; ++i) R.tag[i] = -1;
    for (int i = 0; i < 4; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;"
                   :: "r"((uint32_t)__cvta_generic_to_shared(sm + oSBar) + 8 * i) : "memory");
    for (int i = 0; i < kNst; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(R.full + 8 * i) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" :: "r"(R.empty + 8 * i) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const uint32_t sbIn = (uint32_t)__cvta_generic_to_shared(sm + oSBar), sbNw = sbIn + 8, sbFree = sbIn + 24;
  if (warp == kWarps - 2) {
    if ((tid & 31) == 0) producer(P, R);
    return;
  }
  if (warp == kWarps - 1) {
    if ((tid & 31) == 0) stager(P, sm, sbIn, sbFree, blockIdx.x < kHeads ? (int)blockIdx.x : -1);
    return;
  }
  // ------------------------------------------------------------ compute warps
  uint16_t* hn = reinterpret_cast<uint16_t*>(sm + oHn);
  uint16_t* yn = reinterpret_cast<uint16_t*>(sm + oYn);
  unsigned char* sc = sm + oScan;
  float* red = reinterpret_cast<float*>(sm + oRed);
  float* misc = reinterpret_cast<float*>(sm + oMisc);
  int* flag = reinterpret_cast<int*>(sm + oMisc + 256);
  const int cta = blockIdx.x, ncta = gridDim.x;
  const TileRange rin = tile_range(kZx / kRows, cta, ncta), rout = tile_range(kDModel / kRows, cta, ncta);
  const TileRange rhead = tile_range(P.vocab / kRows, cta, ncta);
  const int item = cta < kHeads ? cta : -1;           // scan head of this CTA (batch 1)
  bool ok = true;
  int ctr = 0;
  uint16_t* Vs = reinterpret_cast<uint16_t*>(sm + oV);
  uint16_t* Ws = reinterpret_cast<uint16_t*>(sm + oAdw);
  uint16_t* Gn = reinterpret_cast<uint16_t*>(sm + oGnw);
  uint16_t* Ag = reinterpret_cast<uint16_t*>(sm + oAdg);
  uint16_t* Nw = reinterpret_cast<uint16_t*>(sm + oNw);
  auto stage_wait = [&](uint32_t bar, uint32_t parity) {
    if (ok && !mb_wait(bar, parity, P.sync)) {
      ok = false;
      set_abort(P, (int)kDevTimeoutProducer);
    }
  };
  int nw_phase = 0, in_phase = 0;
  unsigned nbar = 0;                                   // grid barriers passed
  unsigned arms_nw = 1;                                // bulk-copy phases armed by thread 0
  if (tid == 0) {
    mb_expect(sbNw, kDModel * 2);
    bulk_g2s(Nw, P.layers[0].norm_w, kDModel * 2, sbNw);
  }
  for (int step = 0; step < P.steps; ++step) {
  // the token of this step: the caller's for the first, then the previous step's pick
  long long id = __ldcg(P.tok);
  if (id < 0 || id >= P.vocab) {
    if (tid == 0 && cta == 0) atomicOr(P.err, (int)kDevBadArgs);
    id = 0;
  }
  const int pos = P.pos + step;
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int l = 0; l < P.n_layer; ++l) {
    const DecLayer& L = P.layers[l];
    DTRACE(l, 0);
    DARRIVE(l, 3);
    // this layer's norm weight was staged one layer ahead (layer 0: at the start)
    stage_wait(sbNw, (uint32_t)nw_phase);
    nw_phase ^= 1;
    uint16_t* res_out = cta == 0 ? P.res + ((l + 1) & 1) * kDModel : nullptr;
    block_norm(P, P.h, l > 0 ? P.res + (l & 1) * kDModel : nullptr, res_out, Nw,
               l == 0 ? id : -1, hn, misc);
    // next layer's norm weight (norm_f after the last layer): block_norm's last CTA barrier
    // has passed every read of this one
    if (tid == 0) {
      asm volatile("fence.proxy.async;" ::: "memory");
      mb_expect(sbNw, kDModel * 2);
      ++arms_nw;
      bulk_g2s(Nw, l + 1 < P.n_layer ? P.layers[l + 1].norm_w : P.norm_f, kDModel * 2, sbNw);
    }
    DTRACE(l, 1);
    DWARP(l, 0);
    gemv_phase<false, EXACT>(P, R, sm, ctr, rin.t0, rin.t1, kDModel / kKc, hn, L.in_g, P.zx, red, false, best, bidx,
                             ok);
    DWARP(l, 1);
    ctr += (rin.t1 - rin.t0) * (kDModel / kKc);
    DTRACE(l, 2);
    DARRIVE(l, 0);
    RowState rs;                                         // the head's row pairs (CTAs with a scan head)
    {
      const unsigned long long tk = grid_arrive(P, nbar);
      stage_wait(sbIn, (uint32_t)in_phase);              // this layer's staged inputs
      in_phase ^= 1;
      if (L.ad_V) {                                      // adapter gate partials of this layer's input
        const float gp = gate_partial(hn, Ws, warp, tid & 31);
        if ((tid & 31) == 0) misc[24 + warp] = gp;
      }
      if (item >= 0) scan_unpack(L, sc, rs);             // the previous step's state of the head
      if (!grid_wait(P, tk, flag)) ok = false;
    }
    DTRACE(l, 3);
    // z columns for the gated norm (swizzled rows of 64), staged where yn will be written
    for (int i = tid; i < kDInner / 8; i += kCompute) cp_async16(yn + swz(i >> 3, (i & 7) * 8), P.zx + i * 8);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    {
      TokenScales ts;
      float2 zlat;
      if (item >= 0) {
        DTRACE(l, 9);
        scan_step(P, L, item, sc, rs, l, pos, ts, zlat);
      }
      DTRACE(l, 4);
      DARRIVE(l, 1);
      const unsigned long long tk = grid_arrive(P, nbar);      // y is published
      if (item >= 0) scan_finish(L, item, sc, rs, ts, zlat);
      if (!grid_wait(P, tk, flag)) ok = false;
    }
    DTRACE(l, 5);
    {
      uint16_t* Ys = reinterpret_cast<uint16_t*>(sc);
      for (int i = tid; i < 128 * 8; i += kCompute) {
        const int r = i >> 3, c = (i & 7) * 8;
        cp_async16(Ys + r * kYPitch + c, P.y + r * 64 + c);
      }
      cp_async_wait_all();
      bar_sync(1, kCompute);
      DTRACE(l, 12);
      resurface_norm(P, L, misc + 24, Ys, Vs, Ag, Gn, yn, l);
      bar_sync(1, kCompute);
      // the staged layer inputs are no longer read: the stager may bring the next layer's
      if (tid == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(sbFree) : "memory");
    }
    DTRACE(l, 6);
    DWARP(l, 2);
    gemv_phase<true, EXACT>(P, R, sm, ctr, rout.t0, rout.t1, kDInner / kKc, yn, L.out_g, P.h, red, false, best, bidx,
                            ok);
    DWARP(l, 3);
    ctr += (rout.t1 - rout.t0) * (kDInner / kKc);
    DTRACE(l, 7);
    DARRIVE(l, 2);
    if (!grid_sync(P, nbar, flag)) ok = false;
    DTRACE(l, 8);
  }
  DTRACE(63, 0);
  stage_wait(sbNw, (uint32_t)nw_phase);                          // norm_f
  nw_phase ^= 1;
  // final norm (norm_f) and the greedy head
  block_norm(P, P.h, P.res + (P.n_layer & 1) * kDModel, nullptr, Nw, -1, hn, misc);
  if (step + 1 < P.steps && tid == 0) {                          // next token's layer-0 norm weight
    asm volatile("fence.proxy.async;" ::: "memory");
    mb_expect(sbNw, kDModel * 2);
    ++arms_nw;
    bulk_g2s(Nw, P.layers[0].norm_w, kDModel * 2, sbNw);
  }
  gemv_phase<false, EXACT>(P, R, sm, ctr, rhead.t0, rhead.t1, kDModel / kKc, hn, P.head_g, P.logits, red, true, best,
                           bidx, ok);
  ctr += (rhead.t1 - rhead.t0) * (kDModel / kKc);
  // CTA candidate: warps 0 and 4 hold the per-lane picks of their group
  if ((warp & 3) == 0) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bidx, o);
      argmax_merge(best, bidx, v2, i2);
    }
    if ((tid & 31) == 0) {
      misc[16 + (warp >> 2)] = best;
      reinterpret_cast<int*>(misc)[18 + (warp >> 2)] = bidx;
    }
  }
  bar_sync(1, kCompute);
  if (tid == 0) {
    float bv = misc[16];
    int bi = reinterpret_cast<int*>(misc)[18];
    argmax_merge(bv, bi, misc[17], reinterpret_cast<int*>(misc)[19]);
    P.part_v[cta] = bv;
    P.part_i[cta] = bi;
  }
  DTRACE(63, 1);
  grid_sync(P, nbar, flag);
  DTRACE(63, 2);
  if (cta == 0 && warp == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < ncta; i += 32) argmax_merge(bv, bi, __ldcg(P.part_v + i), __ldcg(P.part_i + i));
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_merge(bv, bi, v2, i2);
    }
    if (tid == 0) {
      const long long pick = bi == 0x7fffffff ? 0 : bi;
      *P.tok = pick;
      if (P.out_tokens) P.out_tokens[step] = pick;
    }
  }
  if (step + 1 < P.steps) grid_sync(P, nbar, flag);                    // every CTA reads the pick next
  }
  // after an abort some staged copies were never waited for: let them land before exiting
  cp_async_wait_all();
  if (tid == 0) {
    if (arms_nw) mb_drain(sbNw, (arms_nw - 1) & 1u);
  }
  (void)ok;
}

}  // namespace

int decode_smem_bytes() { return kSmem; }

#ifdef SQ_DECODE_TRACE
extern "C" int sq_decode_trace_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, g_decode_trace, sizeof(g_decode_trace)) == cudaSuccess ? 0 : 4;
}
extern "C" int sq_decode_warp_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, g_decode_warp, sizeof(g_decode_warp)) == cudaSuccess ? 0 : 4;
}
extern "C" int sq_decode_arrive_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, g_decode_arrive, sizeof(g_decode_arrive)) == cudaSuccess ? 0 : 4;
}
#endif

int prepare_decode_kernel() {
  static bool done = false;
  if (done) return kOk;
  if (cudaFuncSetAttribute(decode_step_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
          cudaSuccess ||
      cudaFuncSetAttribute(decode_step_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return kECuda;
  done = true;
  return kOk;
}

int decode_grid() {
  int dev = 0, sms = 0, coop = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  if (!coop || sms <= 0) return -1;
  if (prepare_decode_kernel() != kOk) return -1;
  int per_sm_exact = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel<false>, kThreads, kSmem) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_exact, decode_step_kernel<true>, kThreads, kSmem) !=
          cudaSuccess ||
      per_sm < 1 || per_sm_exact < 1)
    return -1;
  return sms;
}

int launch_decode_step(const DecodeParams& p, int grid, cudaStream_t st) {
  if (grid < kHeads) return kEInval;                 // one scan head per CTA needs >= 128 CTAs
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = p.exact ? cudaLaunchKernelEx(&cfg, decode_step_kernel<true>, p)
                                : cudaLaunchKernelEx(&cfg, decode_step_kernel<false>, p);
  if (e != cudaSuccess) { cudaGetLastError(); last_launch_error() = e; return kECuda; }
  return kOk;
}

}  // namespace sq
