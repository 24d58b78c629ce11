// FP4-G16 linear on the 5th-generation tensor cores with the weight decode fused in, for
// activation batches of 1..256 rows (decode steps at batch > 1, short prompts, the BASELINE
// config-2 shapes).  Y[m, n] = X[m, k] . W[n, k]^T with W decoded exactly as the reference
// (mamba2_recall/fp4.py:151-154: FP16(FP32(FP32(code * block) * global))), fp32 accumulation,
// fp16 output: the nn.Linear the reference runs over its decoded FP16 weights.  Optionally
// (exact = false) the fp32 global scale is applied once per output instead of per weight:
// the MMA then sees the exact fp16 products code * block.
//
// Weights are the MMA's A operand ("swap AB"): a CTA owns 128 weight rows and one slice of K,
// so every packed weight byte is read from HBM once.  The K walk advances in stages of 128
// columns (two 64-column SWIZZLE_128B atoms): per stage the MMA thread waits twice, issues
// eight tcgen05.mma (M = 128 weight rows, N = the batch rounded up to 16, K = 16) and commits
// twice, so the per-stage handshake cost is spread over 16K weights.  At small N an MMA's
// pipeline latency, not its work, sets the rate when every MMA accumulates into the same
// TMEM tile, so the eight MMAs of a stage rotate over four accumulators (K-step kk adds into
// accumulator kk % 4) and the epilogue sums them, ((a0 + a1) + a2) + a3.  Roles, by warp:
//   0        TMA lane: packed codes (SWIZZLE_128B) and E4M3 block scales, 256-column chunks,
//            4-deep ring;
//   1        TMEM owner and the elected MMA issuer;
//   2        TMA lane: activation stages (2 boxes of 64 columns x batch, SWIZZLE_128B) into
//            their own ring, as deep as the shared memory left allows;
//   3..18    converters (four per SM sub-partition): decode each 128-column stage into the
//            K-major SWIZZLE_128B fp16 tile.  A thread owns one 8-column group and four rows
//            32 apart, so its four items share every address term but the row and run
//            unrolled side by side;
//   4..7     also the epilogue: read the accumulator back (tcgen05.ld, one weight row per
//            lane; warp w may only touch TMEM lanes 32 (w % 4) .. +31).
// When the matrix has few 128-row tiles (out_proj: 32) K is split over a cluster of 2 or 4
// CTAs (grid y).  Each CTA then parks its fp32 partial [batch x 128] in its own (by then idle)
// ring memory, and after a cluster barrier rank t sums the partials of all ranks, in rank
// order, for its share of the rows through distributed shared memory and stores Y.
// Batches above 128 rows run as two launches over the row halves (each streams the weights
// once more; the accumulator and the activation ring are sized for 128 rows).
//
// Every wait is bounded (tc::mbar_wait, 2 s): on expiry a role records an error bit, drains
// the copies / MMAs it has in flight, and the CTA frees its TMEM before leaving.  The cluster
// barriers are reached by every thread on every path.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "device_util.cuh"
#include "fp4.cuh"
#include "tc_util.cuh"

namespace sq {
namespace {
using namespace tc;

constexpr int kRowsW = 128;                 // weight rows per CTA (MMA M)
constexpr int kChunk = 256;                 // K columns per packed chunk
constexpr int kStage = 128;                 // K columns per decoded / activation stage
constexpr int kAtom = 64;                   // K columns per SWIZZLE_128B atom (128 B of fp16)
constexpr int kNP = 4;                      // packed-chunk ring depth
constexpr int kNAMax = 3, kNXMax = 8;       // decoded-stage / activation-stage ring depths (max)
constexpr int kMaxBatch = 128;              // rows per launch (larger batches: two launches)
constexpr int kNAcc = 4;                    // independent TMEM accumulators (4 x 128 columns max)
constexpr int kCodeBytes = kRowsW * kChunk / 2;          // 16 KB, SWIZZLE_128B rows of 128 B
constexpr int kScaleBytes = kRowsW * kChunk / 16;        // 2 KB, rows of 16 B
constexpr int kPBytes = kCodeBytes + kScaleBytes;        // 18 KB (a 1024-multiple)
constexpr int kAtomBytes = kRowsW * kAtom * 2;           // 16 KB
constexpr int kABytes = 2 * kAtomBytes;                  // 32 KB per decoded stage
constexpr int kConv = 16;                                // converter warps
constexpr int kConvThreads = 32 * kConv;
constexpr int kItems = kRowsW * kStage / 8;              // 8-column outputs per stage (2048)
constexpr int kItemsPerThread = kItems / kConvThreads;   // 4: rows r0, r0 + 32, r0 + 64, r0 + 96
static_assert(kItemsPerThread * kConvThreads == kItems && kConvThreads / 16 == 32, "item map");
constexpr int kWarps = 3 + kConv;
constexpr int kThreads = 32 * kWarps;
// shared memory (offsets from a 1024-byte aligned base)
constexpr int oP = 0;
constexpr int oA = oP + kNP * kPBytes;                   // 72 KB
constexpr int oEnd = 224 * 1024;                         // A ring + X ring end here
constexpr int oBar = oEnd;
// barriers: pfull[kNP], pempty[kNP], afull[kNAMax], aempty[kNAMax], xfull[kNXMax], xempty[kNXMax],
// dfull, drain
constexpr int kBars = 2 * kNP + 2 * kNAMax + 2 * kNXMax + 2;
constexpr int kSmem = oBar + kBars * 8 + 16 + 1024;     // + TMEM slot, + alignment slack
static_assert(kSmem <= 227 * 1024, "fits one CTA per SM");
// split-K partial [batch][128] fp32 in the packed / decoded rings (idle once D is complete)
static_assert(kRowsW * kMaxBatch * 4 <= oA + 2 * kABytes, "split-K partial fits the idle rings");

struct LinArgs {
  int N, K, M, mbox, ksplit, exact;
  uint16_t* Y; long long ldy;
  const float* g;
  int* err;
};

// Instruction descriptor of tcgen05.mma.kind::f16: fp32 D, fp16 A and B, both K-major,
// M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kRowsW >> 4) << 24);
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
// fp16 pair m * b, optionally times the fp32 global scale rounded once to fp32 then fp16.
__device__ __forceinline__ uint32_t decode_pair(uint32_t m16x2, uint32_t b16x2, float2 g2, bool exact) {
  return exact ? scale_pair(m16x2, b16x2, g2) : hmul2_u32(m16x2, b16x2);
}

template <bool EXACT>
__global__ void __launch_bounds__(kThreads, 1)
fp4_mma_linear_kernel(const __grid_constant__ CUtensorMap mcodes, const __grid_constant__ CUtensorMap mscales,
                      const __grid_constant__ CUtensorMap mx, const LinArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned base derived by pointer arithmetic on the shared array, so that the
  // compiler keeps every converter access a shared-memory (not generic) load / store
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + oBar;
  auto PFULL = [&](int s) { return bar0 + 8u * s; };
  auto PEMPTY = [&](int s) { return bar0 + 8u * (kNP + s); };
  auto AFULL = [&](int s) { return bar0 + 8u * (2 * kNP + s); };
  auto AEMPTY = [&](int s) { return bar0 + 8u * (2 * kNP + kNAMax + s); };
  auto XFULL = [&](int s) { return bar0 + 8u * (2 * kNP + 2 * kNAMax + s); };
  auto XEMPTY = [&](int s) { return bar0 + 8u * (2 * kNP + 2 * kNAMax + kNXMax + s); };
  const uint32_t DFULL = bar0 + 8u * (kBars - 2), DRAIN = bar0 + 8u * (kBars - 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + oBar + kBars * 8);

  const int n0 = blockIdx.x * kRowsW;
  const int kspan = args.K / args.ksplit;              // this CTA's K columns (multiple of 256)
  const int k0 = blockIdx.y * kspan;
  const int nstage = kspan / kStage;
  const int nchunk = kspan / kChunk;
  const uint32_t xatom = (uint32_t)args.mbox * kAtom * 2;          // one activation atom
  const uint32_t xbytes = 2 * xatom;                                 // one activation stage
  // ring carve-up: 3 decoded stages up to batch 64, else 2; the activation ring takes the rest
  const int nA = args.mbox <= 64 ? kNAMax : 2;
  const uint32_t oX = (uint32_t)(oA + nA * kABytes);
  const int nX = min(kNXMax, (int)((oEnd - oX) / xbytes));
  // TMEM: kNAcc accumulators of mbox fp32 columns each, accumulator a at column a * mbox
  const uint32_t tcols = args.mbox <= 16 ? 64 : (args.mbox <= 32 ? 128 : (args.mbox <= 64 ? 256 : 512));

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNP; ++s) { mbar_init(PFULL(s), 1); mbar_init(PEMPTY(s), kConv); }
    for (int s = 0; s < nA; ++s) { mbar_init(AFULL(s), kConv); mbar_init(AEMPTY(s), 1); }
    for (int s = 0; s < nX; ++s) { mbar_init(XFULL(s), 1); mbar_init(XEMPTY(s), 1); }
    mbar_init(DFULL, 1);
    mbar_init(DRAIN, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(tcols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- packed-weight producer
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int c = 0; c < nchunk; ++c) {
        const int ps = c % kNP;
        if (!mbar_wait(PEMPTY(ps), ((c / kNP) & 1) ^ 1)) { ok = false; break; }
        const uint32_t pdst = sbase + oP + ps * kPBytes;
        mbar_expect_tx(PFULL(ps), kPBytes);
        tma_load_2d(pdst, &mcodes, PFULL(ps), (k0 + c * kChunk) / 2, n0);
        tma_load_2d(pdst + kCodeBytes, &mscales, PFULL(ps), (k0 + c * kChunk) / 16, n0);
        ++issued;
      }
      if (!ok) {
        atomicOr(args.err, (int)kDevTimeoutProducer);
        for (int i = 1; i <= kNP && i <= issued; ++i) {   // issued copies land before the CTA leaves
          const int c = issued - i;
          mbar_wait(PFULL(c % kNP), (c / kNP) & 1);
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- activation producer
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      int xs = 0, xph = 0;
      for (int t = 0; t < nstage; ++t) {
        if (!mbar_wait(XEMPTY(xs), xph ^ 1)) { ok = false; break; }
        const uint32_t dst = sbase + oX + xs * xbytes;
        mbar_expect_tx(XFULL(xs), xbytes);
        tma_load_2d(dst, &mx, XFULL(xs), k0 + t * kStage, 0);
        tma_load_2d(dst + xatom, &mx, XFULL(xs), k0 + t * kStage + kAtom, 0);
        ++issued;
        if (++xs == nX) { xs = 0; xph ^= 1; }
      }
      if (!ok) {
        atomicOr(args.err, (int)kDevTimeoutProducer);
        for (int i = 1; i <= nX && i <= issued; ++i) {
          const int t = issued - i;
          mbar_wait(XFULL(t % nX), (t / nX) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = true;
      const uint32_t idesc = idesc_f16(args.mbox);
      int as = 0, aph = 0, xs = 0, xph = 0;
      for (int t = 0; t < nstage; ++t) {
        if (!mbar_wait(AFULL(as), aph) || !mbar_wait(XFULL(xs), xph)) { ok = false; break; }
        tc_fence_after();
        const uint64_t da = sw128_desc(sbase + oA + as * kABytes);
        const uint64_t dx = sw128_desc(sbase + oX + xs * xbytes);
        const uint64_t da1 = da + (kAtomBytes >> 4), dx1 = dx + (xatom >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)            // descriptor address field: 16-byte units
          umma_f16(tmem + (uint32_t)(kk * args.mbox), da + 2 * kk, dx + 2 * kk, idesc, t != 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem + (uint32_t)(kk * args.mbox), da1 + 2 * kk, dx1 + 2 * kk, idesc, 1);
        umma_commit(AEMPTY(as));
        umma_commit(XEMPTY(xs));
        if (++as == nA) { as = 0; aph ^= 1; }
        if (++xs == nX) { xs = 0; xph ^= 1; }
      }
      if (ok) umma_commit(DFULL);
      else atomicOr(args.err, (int)kDevTimeoutMma);
      umma_commit(DRAIN);                       // every issued MMA retires before TMEM is freed
      mbar_wait(DRAIN, 0);
    }
  } else {
    // ---------------------------------------------------------------- converters
    // Thread ct owns the 8-column group q = ct % 16 of rows r0 + 32 i (i < 4), r0 = ct / 16.
    // Rows 32 apart share r % 8, hence every swizzle term: item i only adds i * 32 rows.
    const int ct = (warp - 3) * 32 + lane;
    const int q = ct & 15, r0 = ct >> 4, kc = q & 7, sw = r0 & 7;
    const float gsc = *args.g;
    const float2 g2 = make_float2(gsc, gsc);
    const int out_off = (q >> 3) * kAtomBytes + r0 * 128 + ((kc ^ sw) << 4);
    int code_off[2], scale_off[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      // codes: bytes s*64 + q*4 .. +3 of the row = 16-byte chunk 4s + q/4 at offset (q % 4) * 4,
      // stored at chunk position (4s + q/4) ^ (r % 8) (SWIZZLE_128B); block scale s*8 + q/2
      code_off[s] = r0 * 128 + (((s * 4 + (q >> 2)) ^ sw) << 4) + (q & 3) * 4;
      scale_off[s] = kCodeBytes + r0 * 16 + s * 8 + (q >> 1);
    }
    bool ok = true;
    int as = 0, aph = 0;
    for (int c = 0; c < nchunk && ok; ++c) {
      const int ps = c % kNP;
      if (!mbar_wait(PFULL(ps), (c / kNP) & 1)) { ok = false; break; }
      const unsigned char* pc = smem + oP + ps * kPBytes;
      for (int s = 0; s < kChunk / kStage && ok; ++s) {
        if (!mbar_wait(AEMPTY(as), aph ^ 1)) { ok = false; break; }
        unsigned char* pa = smem + oA + as * kABytes + out_off;
        const unsigned char* pcs = pc + code_off[s];
        const unsigned char* pss = pc + scale_off[s];
        uint32_t w[kItemsPerThread], bs[kItemsPerThread];
#pragma unroll
        for (int i = 0; i < kItemsPerThread; ++i) {
          w[i] = *reinterpret_cast<const uint32_t*>(pcs + i * 32 * 128);
          bs[i] = pss[i * 32 * 16];
        }
#pragma unroll
        for (int i = 0; i < kItemsPerThread; ++i) {
          const uint32_t b2 = e4m3_splat_f16x2(bs[i]);
          uint32_t m[4];
          e2m1x8_to_f16x2(w[i], m);
          uint4 o;
          o.x = decode_pair(m[0], b2, g2, EXACT);
          o.y = decode_pair(m[1], b2, g2, EXACT);
          o.z = decode_pair(m[2], b2, g2, EXACT);
          o.w = decode_pair(m[3], b2, g2, EXACT);
          *reinterpret_cast<uint4*>(pa + i * 32 * 128) = o;
        }
        // generic-proxy writes become visible to the tensor core's async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(AFULL(as));
        if (++as == nA) { as = 0; aph ^= 1; }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(PEMPTY(ps));
    }
    if (!ok && lane == 0) atomicOr(args.err, (int)kDevTimeoutEpilogue);
  }
  // ------------------------------------------------------------------ epilogue (warps 4..7)
  if (warp >= 4 && warp < 8) {
    const int qd = warp & 3;                    // TMEM lane quadrant of this warp (warp % 4)
    if (mbar_wait(DFULL, 0)) {
      tc_fence_after();
      const int r = qd * 32 + lane;             // weight row within the tile
      const int n = n0 + r;
      const float gsc = EXACT ? 1.0f : *args.g;
      float* part = reinterpret_cast<float*>(smem + oP);   // [mbox][128], split-K only
      const uint32_t trow = tmem + ((uint32_t)(qd * 32) << 16);
      // 32 batch columns at a time: s[i] = ((a0 + a1) + a2) + a3 of column c0 + i
      for (int c0 = 0; c0 < args.mbox; c0 += 32) {
        float sacc[32];
        uint32_t u[32];
        if (args.mbox == 16) {                  // the four 16-column accumulators in two loads
          tmem_ld32(trow, u);
#pragma unroll
          for (int i = 0; i < 16; ++i) sacc[i] = __uint_as_float(u[i]) + __uint_as_float(u[16 + i]);
          tmem_ld32(trow + 32, u);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            sacc[i] = (sacc[i] + __uint_as_float(u[i])) + __uint_as_float(u[16 + i]);
            sacc[16 + i] = 0.f;
          }
        } else {
          tmem_ld32(trow + (uint32_t)c0, u);
#pragma unroll
          for (int i = 0; i < 32; ++i) sacc[i] = __uint_as_float(u[i]);
#pragma unroll
          for (int a = 1; a < kNAcc; ++a) {
            tmem_ld32(trow + (uint32_t)(a * args.mbox + c0), u);
#pragma unroll
            for (int i = 0; i < 32; ++i) sacc[i] += __uint_as_float(u[i]);
          }
        }
        const int ncol = min(32, args.mbox - c0);
        if (args.ksplit > 1) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < ncol) part[(c0 + i) * kRowsW + r] = sacc[i];
        } else if (n < args.N) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < ncol && c0 + i < args.M)
              args.Y[(long long)(c0 + i) * args.ldy + n] = f2h(EXACT ? sacc[i] : sacc[i] * gsc);
        }
      }
    } else if (lane == 0) {
      atomicOr(args.err, (int)kDevTimeoutEpilogue);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (args.ksplit > 1) {
    // ---------------------------------------------------------------- split-K reduction
    cluster_sync_all();                         // every rank's partial is in its shared memory
    const uint32_t rank = cluster_rank();
    const int rows = kRowsW / args.ksplit;      // rows reduced by this rank
    const uint32_t part0 = sbase + oP;
    const float gsc = EXACT ? 1.0f : *args.g;
    for (int idx = threadIdx.x; idx < rows * args.M; idx += kThreads) {
      const int c = idx / rows, r = (int)rank * rows + idx % rows;
      const uint32_t off = part0 + (uint32_t)(c * kRowsW + r) * 4u;
      float acc = 0.f;
      for (int s = 0; s < args.ksplit; ++s) acc += ld_cluster_f32(map_rank(off, (uint32_t)s));
      if (n0 + r < args.N) args.Y[(long long)c * args.ldy + n0 + r] = f2h(EXACT ? acc : acc * gsc);
    }
    cluster_sync_all();                         // no rank leaves while its partial is read
  }
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(tcols));
}

bool g_attr = false;

// K split over a cluster: the smallest of 1, 2, 4 that gives >= 120 CTAs (about 0.8 of the
// 148 SMs) while every slice stays a multiple of the 256-column chunk.
int choose_ksplit(int ntiles, int K) {
  int s = 1;
  while (s < 4 && ntiles * s < 120 && (K / (2 * s)) % kChunk == 0 && K % (2 * s) == 0) s *= 2;
  return s;
}

int launch_rows(const Fp4Weight& W, const uint16_t* X, long long ldx, int M, uint16_t* Y, long long ldy, int* err,
                bool exact, cudaStream_t st) {
  const int mbox = (M + 15) / 16 * 16;
  CUtensorMap mc, ms, mx;
  // codes: u8 [rows][cols/2], boxes of 128 B x 128 rows, SWIZZLE_128B
  if (!encode_2d_map(&mc, CU_TENSOR_MAP_DATA_TYPE_UINT8, W.codes, W.rows, W.cols / 2, W.cols / 2, kChunk / 2, kRowsW,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      // block scales: u8 [rows][cols/16], boxes of 16 B x 128 rows
      !encode_2d_map(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT8, W.scales, W.rows, W.cols / 16, W.cols / 16, kChunk / 16,
                     kRowsW, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      // activations: fp16 [M][cols], boxes of 64 columns (128 B) x mbox rows, SWIZZLE_128B
      !encode_2d_map(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X, M, W.cols, ldx * 2, kAtom, mbox,
                     CU_TENSOR_MAP_SWIZZLE_128B))
    return kECuda;
  const int ntiles = (W.rows + kRowsW - 1) / kRowsW;
  LinArgs a;
  a.N = W.rows; a.K = W.cols; a.M = M; a.mbox = mbox; a.ksplit = choose_ksplit(ntiles, W.cols);
  a.exact = exact ? 1 : 0;
  a.Y = Y; a.ldy = ldy; a.g = W.global_scale; a.err = err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ntiles, a.ksplit, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = a.ksplit;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.ksplit > 1 ? 1 : 0;
  const cudaError_t e = exact ? cudaLaunchKernelEx(&cfg, fp4_mma_linear_kernel<true>, mc, ms, mx, a)
                              : cudaLaunchKernelEx(&cfg, fp4_mma_linear_kernel<false>, mc, ms, mx, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    last_launch_error() = e;
    return kECuda;
  }
  return launch_status();
}

}  // namespace

int prepare_fp4_mma_kernel() {
  if (g_attr) return kOk;
  if (cudaFuncSetAttribute(fp4_mma_linear_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
          cudaSuccess ||
      cudaFuncSetAttribute(fp4_mma_linear_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
          cudaSuccess)
    return kECuda;
  g_attr = true;
  return kOk;
}

int launch_fp4_mma_linear(const Fp4Weight& W, const uint16_t* X, long long ldx, int M, uint16_t* Y, long long ldy,
                          int* err, cudaStream_t st, bool exact) {
  if (M <= 0 || M > 2 * kMaxBatch || W.rows <= 0 || W.cols % kChunk || ldx < W.cols || ldy < W.rows || !err)
    return kEInval;
  if (((uintptr_t)W.codes % 16) || ((uintptr_t)W.scales % 16) || ((uintptr_t)X % 16) || (ldx % 8)) return kEInval;
  if (prepare_fp4_mma_kernel() != kOk) return kECuda;
  if (M <= kMaxBatch) return launch_rows(W, X, ldx, M, Y, ldy, err, exact, st);
  const int m1 = ((M + 1) / 2 + 15) & ~15;   // first half: a multiple of 16 rows
  if (int s = launch_rows(W, X, ldx, m1, Y, ldy, err, exact, st)) return s;
  return launch_rows(W, X + (long long)m1 * ldx, ldx, M - m1, Y + (long long)m1 * ldy, ldy, err, exact, st);
}

}  // namespace sq
