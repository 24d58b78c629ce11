// FP4-G16 linear on the 5th-generation tensor cores with the weight decode fused in, for
// activation batches of 1..256 rows (decode steps at batch > 1, short prompts, the BASELINE
// config-2 shapes).  Y[m, n] = X[m, k] . W[n, k]^T with W decoded exactly as the reference
// (mamba2_recall/fp4.py:151-154: FP16(FP32(FP32(code * block) * global))), fp32 accumulation,
// fp16 output: the nn.Linear the reference runs over its decoded FP16 weights.
//
// Weights are the MMA's A operand ("swap AB"): one CTA owns 128 weight rows and walks all
// of K, so every packed weight byte is read from HBM once.  Per 256-column chunk a TMA lane
// brings the packed codes (SWIZZLE_128B) and E4M3 block scales into a ring; eight converter
// warps decode each 64-column slab into a K-major SWIZZLE_128B fp16 tile; one elected
// thread issues tcgen05.mma.kind::f16 (M = 128 weight rows, N = the batch rounded up to
// 16, K = 16) against the activation slab, which TMA streams with the same swizzle; the
// accumulator D^T [128 weight rows x batch] lives in TMEM.  Four of the converter warps read
// it back (tcgen05.ld, one weight row per lane) and store Y with the batch row outermost,
// 32 consecutive outputs per warp store.
//
// Every wait is bounded (tc::mbar_wait, 2 s): on expiry a role records an error bit, drains
// the copies / MMAs it has in flight, and the CTA frees its TMEM before leaving.
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
constexpr int kSlab = 64;                   // K columns per MMA slab (128 B of fp16)
constexpr int kNP = 2, kNA = 4, kNX = 3;    // ring depths: packed chunks, decoded slabs, X slabs
constexpr int kMaxBatch = 256;
constexpr int kCodeBytes = kRowsW * kChunk / 2;          // 16 KB, SWIZZLE_128B rows of 128 B
constexpr int kScaleBytes = kRowsW * kChunk / 16;        // 2 KB, rows of 16 B
constexpr int kPBytes = kCodeBytes + kScaleBytes;
constexpr int kABytes = kRowsW * kSlab * 2;              // 16 KB
constexpr int kXMaxBytes = kMaxBatch * kSlab * 2;        // 32 KB
constexpr int kConv = 8;                                 // converter warps
constexpr int kThreads = 32 * (2 + kConv);
// shared memory (offsets from a 1024-byte aligned base)
constexpr int oP = 0;
constexpr int oA = oP + kNP * kPBytes;                   // 36 KB (a 1024-multiple)
constexpr int oX = oA + kNA * kABytes;
constexpr int oBar = oX + kNX * kXMaxBytes;
// barriers: pfull[kNP], pempty[kNP], afull[kNA], aempty[kNA], xfull[kNX], xempty[kNX], dfull, drain
constexpr int kBars = 2 * kNP + 2 * kNA + 2 * kNX + 2;
constexpr int kSmem = oBar + kBars * 8 + 16 + 1024;     // + TMEM slot, + alignment slack

struct LinArgs {
  int N, K, M, mbox;
  uint16_t* Y; long long ldy;
  const float* g;
  int* err;
};

// Instruction descriptor of tcgen05.mma.kind::f16: fp32 D, fp16 A and B, both K-major,
// M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kRowsW >> 4) << 24);
}

__global__ void __launch_bounds__(kThreads, 1)
fp4_mma_linear_kernel(const __grid_constant__ CUtensorMap mcodes, const __grid_constant__ CUtensorMap mscales,
                      const __grid_constant__ CUtensorMap mx, const LinArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + oBar;
  auto PFULL = [&](int s) { return bar0 + 8u * s; };
  auto PEMPTY = [&](int s) { return bar0 + 8u * (kNP + s); };
  auto AFULL = [&](int s) { return bar0 + 8u * (2 * kNP + s); };
  auto AEMPTY = [&](int s) { return bar0 + 8u * (2 * kNP + kNA + s); };
  auto XFULL = [&](int s) { return bar0 + 8u * (2 * kNP + 2 * kNA + s); };
  auto XEMPTY = [&](int s) { return bar0 + 8u * (2 * kNP + 2 * kNA + kNX + s); };
  const uint32_t DFULL = bar0 + 8u * (kBars - 2), DRAIN = bar0 + 8u * (kBars - 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + oBar + kBars * 8);

  const int n0 = blockIdx.x * kRowsW;
  const int nslab = args.K / kSlab;
  const int nchunk = args.K / kChunk;
  const uint32_t xbytes = (uint32_t)args.mbox * kSlab * 2;
  const uint32_t tcols = args.mbox <= 32 ? 32 : (args.mbox <= 64 ? 64 : (args.mbox <= 128 ? 128 : 256));

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNP; ++s) { mbar_init(PFULL(s), 1); mbar_init(PEMPTY(s), kConv); }
    for (int s = 0; s < kNA; ++s) { mbar_init(AFULL(s), kConv); mbar_init(AEMPTY(s), 1); }
    for (int s = 0; s < kNX; ++s) { mbar_init(XFULL(s), 1); mbar_init(XEMPTY(s), 1); }
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
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      bool ok = true;
      int issued_p = 0, issued_x = 0;
      for (int c = 0; c < nchunk && ok; ++c) {
        const int ps = c % kNP;
        if (!mbar_wait(PEMPTY(ps), ((c / kNP) & 1) ^ 1)) { ok = false; break; }
        const uint32_t pdst = sbase + oP + ps * kPBytes;
        mbar_expect_tx(PFULL(ps), kPBytes);
        tma_load_2d(pdst, &mcodes, PFULL(ps), c * (kChunk / 2), n0);
        tma_load_2d(pdst + kCodeBytes, &mscales, PFULL(ps), c * (kChunk / 16), n0);
        ++issued_p;
        for (int s = 0; s < kChunk / kSlab; ++s) {
          const int j = c * (kChunk / kSlab) + s, xs = j % kNX;
          if (!mbar_wait(XEMPTY(xs), ((j / kNX) & 1) ^ 1)) { ok = false; break; }
          mbar_expect_tx(XFULL(xs), xbytes);
          tma_load_2d(sbase + oX + xs * kXMaxBytes, &mx, XFULL(xs), j * kSlab, 0);
          ++issued_x;
        }
      }
      if (!ok) {
        atomicOr(args.err, (int)kDevTimeoutProducer);
        // drain: the copies already issued into each ring land before the CTA leaves
        for (int i = 1; i <= kNP && i <= issued_p; ++i) {
          const int c = issued_p - i;
          mbar_wait(PFULL(c % kNP), (c / kNP) & 1);
        }
        for (int i = 1; i <= kNX && i <= issued_x; ++i) {
          const int j = issued_x - i;
          mbar_wait(XFULL(j % kNX), (j / kNX) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = true;
      const uint32_t idesc = idesc_f16(args.mbox);
      for (int j = 0; j < nslab; ++j) {
        const int as = j % kNA, xs = j % kNX;
        if (!mbar_wait(AFULL(as), (j / kNA) & 1) || !mbar_wait(XFULL(xs), (j / kNX) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = sbase + oA + as * kABytes, sx = sbase + oX + xs * kXMaxBytes;
#pragma unroll
        for (int kk = 0; kk < kSlab / 16; ++kk)
          umma_f16(tmem, sw128_desc(sa + kk * 32), sw128_desc(sx + kk * 32), idesc, (j | kk) != 0);
        umma_commit(AEMPTY(as));
        umma_commit(XEMPTY(xs));
      }
      if (ok) umma_commit(DFULL);
      else atomicOr(args.err, (int)kDevTimeoutMma);
      umma_commit(DRAIN);                       // every issued MMA retires before TMEM is freed
      mbar_wait(DRAIN, 0);
    }
  } else {
    // ---------------------------------------------------------------- converters
    const int ct = threadIdx.x - 64;            // 0..255
    const float gsc = *args.g;
    const float2 g2 = make_float2(gsc, gsc);
    bool ok = true;
    for (int c = 0; c < nchunk && ok; ++c) {
      const int ps = c % kNP;
      if (!mbar_wait(PFULL(ps), (c / kNP) & 1)) { ok = false; break; }
      const unsigned char* pc = smem + oP + ps * kPBytes;
      const unsigned char* psc = pc + kCodeBytes;
      for (int s = 0; s < kChunk / kSlab && ok; ++s) {
        const int j = c * (kChunk / kSlab) + s, as = j % kNA;
        if (!mbar_wait(AEMPTY(as), ((j / kNA) & 1) ^ 1)) { ok = false; break; }
        unsigned char* pa = smem + oA + as * kABytes;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // output chunk (row r, 8-column chunk kc) of the 128 x 64 fp16 slab
          const int idx = ct + 256 * i, r = idx >> 3, kc = idx & 7;
          // its 8 codes: bytes s*32 + kc*4 .. +3 of row r, i.e. 16-byte chunk 2s + kc/4, offset
          // (kc % 4) * 4, the chunk stored at position chunk ^ (r % 8) (SWIZZLE_128B)
          const int lc = s * 2 + (kc >> 2);
          const uint32_t w = *reinterpret_cast<const uint32_t*>(pc + r * 128 + ((lc ^ (r & 7)) << 4) + (kc & 3) * 4);
          const uint32_t bs = e4m3_splat_f16x2(psc[r * 16 + s * 4 + (kc >> 1)]);
          uint32_t m[4];
          e2m1x8_to_f16x2(w, m);
          uint4 o;
          o.x = scale_pair(m[0], bs, g2);
          o.y = scale_pair(m[1], bs, g2);
          o.z = scale_pair(m[2], bs, g2);
          o.w = scale_pair(m[3], bs, g2);
          *reinterpret_cast<uint4*>(pa + r * 128 + ((kc ^ (r & 7)) << 4)) = o;
        }
        // generic-proxy writes become visible to the tensor core's async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(AFULL(as));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(PEMPTY(ps));
    }
    if (!ok && lane == 0) atomicOr(args.err, (int)kDevTimeoutEpilogue);
    // ---------------------------------------------------------------- epilogue (4 warps)
    if (ok && warp < 6) {
      const int q = warp & 3;                   // TMEM lane quadrant of this warp
      if (mbar_wait(DFULL, 0)) {
        tc_fence_after();
        const int n = n0 + q * 32 + lane;
        for (int c0 = 0; c0 < args.mbox; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
          if (n < args.N) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c0 + i < args.M) args.Y[(long long)(c0 + i) * args.ldy + n] = f2h(__uint_as_float(v[i]));
          }
        }
      } else if (lane == 0) {
        atomicOr(args.err, (int)kDevTimeoutEpilogue);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(tcols));
}

bool g_attr = false;

}  // namespace

int prepare_fp4_mma_kernel() {
  if (g_attr) return kOk;
  if (cudaFuncSetAttribute(fp4_mma_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return kECuda;
  g_attr = true;
  return kOk;
}

int launch_fp4_mma_linear(const Fp4Weight& W, const uint16_t* X, long long ldx, int M, uint16_t* Y, long long ldy,
                          int* err, cudaStream_t st) {
  if (M <= 0 || M > kMaxBatch || W.rows <= 0 || W.cols % kChunk || ldx < W.cols || ldy < W.rows || !err)
    return kEInval;
  if (((uintptr_t)W.codes % 16) || ((uintptr_t)W.scales % 16) || ((uintptr_t)X % 16) || (ldx % 8)) return kEInval;
  const int mbox = (M + 15) / 16 * 16;
  CUtensorMap mc, ms, mx;
  // codes: u8 [rows][cols/2], boxes of 128 B x 128 rows, SWIZZLE_128B
  if (!encode_2d_map(&mc, CU_TENSOR_MAP_DATA_TYPE_UINT8, W.codes, W.rows, W.cols / 2, W.cols / 2, kChunk / 2, kRowsW,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      // block scales: u8 [rows][cols/16], boxes of 16 B x 128 rows
      !encode_2d_map(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT8, W.scales, W.rows, W.cols / 16, W.cols / 16, kChunk / 16,
                     kRowsW, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      // activations: fp16 [M][cols], boxes of 64 columns (128 B) x mbox rows, SWIZZLE_128B
      !encode_2d_map(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X, M, W.cols, ldx * 2, kSlab, mbox,
                     CU_TENSOR_MAP_SWIZZLE_128B))
    return kECuda;
  if (prepare_fp4_mma_kernel() != kOk) return kECuda;
  LinArgs a;
  a.N = W.rows; a.K = W.cols; a.M = M; a.mbox = mbox; a.Y = Y; a.ldy = ldy; a.g = W.global_scale; a.err = err;
  const int grid = (W.rows + kRowsW - 1) / kRowsW;
  fp4_mma_linear_kernel<<<grid, kThreads, kSmem, st>>>(mc, ms, mx, a);
  return launch_status();
}

}  // namespace sq
