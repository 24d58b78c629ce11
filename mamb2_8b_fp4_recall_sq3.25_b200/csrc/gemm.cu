// Persistent, warp-specialised tcgen05 GEMM for sm_100a:
//   C[M,N] = A[M,K] . B[N,K]^T   (fp16 operands, both K-major; fp32 accumulate in TMEM)
//
// Roles (192 threads):
//   warp 0      TMA producer: 128x64 A tile + 256x64 B tile per stage (SWIZZLE_128B),
//               4-stage ring, mbarrier complete_tx.  No multicast.
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and one
//               elected lane issues tcgen05.mma.cta_group::1.kind::f16 (M=128,N=256,K=16),
//               committing each stage back to the producer and each finished tile
//               to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld 32x32b.x32 per lane quadrant, then either fp16
//               stores or the fused cross-entropy partials of the scoring head.
// Every mbarrier wait is bounded by wall time (globaltimer); on expiry the role sets a
// device error bit, drains what it has in flight, and leaves; TMEM is always freed.
#include <cuda.h>
#include <cudaTypedefs.h>
#include "common.cuh"
#include "fp4.cuh"
#include "tc_util.cuh"

namespace sq {
namespace {
using namespace tc;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;           // 16 KB
constexpr int B_BYTES = BN * BK * 2;           // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int GROUP_M = 32;                    // raster: 32 M-tiles (32 MB of A) share each pass over N
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

struct TileSched {
  int mt, nt, total;
  __device__ void coords(int t, int& mb, int& nb) const {
    const int per_group = GROUP_M * nt;
    const int grp = t / per_group;
    const int first_m = grp * GROUP_M;
    const int gm = min(GROUP_M, mt - first_m);
    const int r = t - grp * per_group;
    mb = first_m + r % gm;
    nb = r / gm;
  }
};

struct GemmArgs {
  int M, N, K;
  uint16_t* C; long long ldc;
  int mode;
  const long long* targets; float2* partials; float* tlogit;
  int n_offset, ntiles_total;
  int vec;                      // C rows are 16-byte aligned: vector stores allowed
  int* err;
};

__global__ void __launch_bounds__(192, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
               const GemmArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2], drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = smem_u32(bars);
  auto FULL = [&](int s) { return bar0 + 8u * s; };
  auto EMPTY = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto TFULL = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto TEMPTY = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t DRAIN = bar0 + 8u * (2 * STAGES + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(FULL(s), 1); mbar_init(EMPTY(s), 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(TFULL(a), 1); mbar_init(TEMPTY(a), 128); }
    mbar_init(DRAIN, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" :: "r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  TileSched ts;
  ts.mt = (args.M + BM - 1) / BM;
  ts.nt = (args.N + BN - 1) / BN;
  ts.total = ts.mt * ts.nt;
  const int kblocks = args.K / BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0; uint32_t phase = 0; bool ok = true;
      long long issued = 0;
      for (int t = blockIdx.x; t < ts.total && ok; t += gridDim.x) {
        int mb, nb; ts.coords(t, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(EMPTY(stage), phase ^ 1)) { ok = false; break; }
          const uint32_t sa = sbase + stage * STAGE_BYTES;
          mbar_expect_tx(FULL(stage), STAGE_BYTES);
          tma_load_2d(sa, &mapA, FULL(stage), kb * BK, mb * BM);
          tma_load_2d(sa + A_BYTES, &mapB, FULL(stage), kb * BK, nb * BN);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        atomicOr(args.err, (int)kDevTimeoutProducer);
        // drain: wait (bounded) for the loads already issued into each stage
        for (int i = 0; i < STAGES && issued > 0; ++i, --issued) {
          if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
          mbar_wait(FULL(stage), phase);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0; uint32_t phase = 0; bool ok = true;
      int acc = 0; uint32_t aphase = 0;
      for (int t = blockIdx.x; t < ts.total && ok; t += gridDim.x) {
        if (!mbar_wait(TEMPTY(acc), aphase ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dt = tmem + (uint32_t)(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(FULL(stage), phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = sbase + stage * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16(dt, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), kIdesc, (kb | kk) != 0);
          umma_commit(EMPTY(stage));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(TFULL(acc));
        if (++acc == 2) { acc = 0; aphase ^= 1; }
      }
      if (!ok) atomicOr(args.err, (int)kDevTimeoutMma);
      // make sure every issued MMA has retired before TMEM is released
      umma_commit(DRAIN);
      mbar_wait(DRAIN, 0);
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrant (warp % 4)
    const int q = warp & 3;
    int acc = 0; uint32_t aphase = 0; bool ok = true;
    for (int t = blockIdx.x; t < ts.total; t += gridDim.x) {
      int mb, nb; ts.coords(t, mb, nb);
      if (!mbar_wait(TFULL(acc), aphase)) { ok = false; break; }
      tc_fence_after();
      const int row = mb * BM + q * 32 + lane;
      const int n0 = nb * BN;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      if (args.mode == 0) {
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c0, r);
          if (row < args.M) {
            uint16_t* dst = args.C + (long long)row * args.ldc + n0 + c0;
            if (args.vec && n0 + c0 + 32 <= args.N) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint4 o;
                __half2 h0 = __floats2half2_rn(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
                __half2 h1 = __floats2half2_rn(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
                __half2 h2 = __floats2half2_rn(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
                __half2 h3 = __floats2half2_rn(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
                o.x = *reinterpret_cast<uint32_t*>(&h0); o.y = *reinterpret_cast<uint32_t*>(&h1);
                o.z = *reinterpret_cast<uint32_t*>(&h2); o.w = *reinterpret_cast<uint32_t*>(&h3);
                *reinterpret_cast<uint4*>(dst + 8 * v) = o;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (n0 + c0 + i < args.N) dst[i] = f2h(__uint_as_float(r[i]));
            }
          }
        }
      } else {
        // fused cross-entropy partials over fp16-rounded logits
        float mx = -INFINITY, sm = 0.f, tv = 0.f;
        bool have_t = false;
        long long tgt = (row < args.M) ? args.targets[row] : -1;
        const long long tl = tgt - (long long)(args.n_offset + n0);
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c0, r);
          float v[32];
          float cm = -INFINITY;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = __half2float(__float2half_rn(__uint_as_float(r[i])));
            if (n0 + c0 + i >= args.N) v[i] = -INFINITY;
            cm = fmaxf(cm, v[i]);
            if (tl == c0 + i) { tv = v[i]; have_t = true; }
          }
          const float nm = fmaxf(mx, cm);
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) s += expf(v[i] - nm);       // CUDA's accurate expf
          sm = (mx == -INFINITY ? 0.f : sm * expf(mx - nm)) + s;
          mx = nm;
        }
        if (row < args.M) {
          args.partials[(long long)row * args.ntiles_total + args.n_offset / BN + nb] = make_float2(mx, sm);
          if (have_t) args.tlogit[row] = tv;
        }
      }
      tc_fence_before();
      mbar_arrive(TEMPTY(acc));
      if (++acc == 2) { acc = 0; aphase ^= 1; }
    }
    if (!ok && lane == 0) atomicOr(args.err, (int)kDevTimeoutEpilogue);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" :: "r"(tmem));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld, int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int g_num_sms = 0;

}  // namespace

// 2-D tiled tensor map over a row-major matrix: dims {cols, rows} elements of `dtype`, row
// stride `row_bytes`, box {box_cols, box_rows}, the given swizzle, zero fill out of bounds.
bool encode_2d_map(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, long long rows, long long cols,
                   long long row_bytes, int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D tiled tensor map over a row-major matrix of 4-byte elements (used by the FP4 GEMV
// to stream code / block-scale tiles): dims {cols, rows}, box {box_cols, box_rows}.
bool encode_u32_map(CUtensorMap* m, const void* base, long long rows, long long cols_u32, long long row_bytes,
                    int box_cols, int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols_u32, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D tiled tensor map over a row-major fp16 matrix [rows][cols] whose box rows are 64
// elements (128 bytes) wide, loaded with SWIZZLE_128B: 16-byte chunk c of box row r lands at
// chunk c ^ (r & 7) of that row in shared memory (destination 1024-byte aligned).
bool encode_f16_sw128_map(CUtensorMap* m, const void* base, long long rows, long long cols, int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int gemm_num_ntiles(int N) { return (N + BN - 1) / BN; }

static bool g_gemm_attr = false;
int prepare_gemm_kernel() {
  if (g_gemm_attr) return kOk;
  const size_t smem = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
  if (cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return kECuda;
  g_gemm_attr = true;
  return kOk;
}

int launch_gemm_f16(const uint16_t* A, long long lda, const uint16_t* B, long long ldb,
                    uint16_t* C, long long ldc, int M, int N, int K, int mode, const GemmCE* ce,
                    int* dev_err, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0 || K % BK) return kEInval;
  if ((lda * 2) % 16 || (ldb * 2) % 16 || ((uintptr_t)A % 16) || ((uintptr_t)B % 16)) return kEInval;
  if (mode == 0 && (!C || ldc < N)) return kEInval;
  if (mode == 1 && (!ce || !ce->targets || !ce->partials || !ce->target_logit)) return kEInval;
  if (!dev_err) return kEInval;
  CUtensorMap ma, mb;
  if (!make_map(&ma, A, M, K, lda, BM) || !make_map(&mb, B, N, K, ldb, BN)) return kECuda;
  if (!g_num_sms) {
    int dev = 0; cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  const size_t smem = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
  if (prepare_gemm_kernel() != kOk) return kECuda;
  GemmArgs a;
  a.M = M; a.N = N; a.K = K; a.C = C; a.ldc = ldc; a.mode = mode;
  a.targets = ce ? ce->targets : nullptr; a.partials = ce ? ce->partials : nullptr;
  a.tlogit = ce ? ce->target_logit : nullptr; a.err = dev_err;
  a.n_offset = ce ? ce->n_offset : 0; a.ntiles_total = ce ? ce->ntiles_total : 0;
  a.vec = (mode == 0 && ldc % 8 == 0 && ((uintptr_t)C % 16) == 0) ? 1 : 0;
  if (mode == 1 && (a.n_offset % BN || a.ntiles_total < a.n_offset / BN + (N + BN - 1) / BN)) return kEInval;
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = tiles < g_num_sms ? tiles : g_num_sms;
  tc_gemm_kernel<<<grid, 192, smem, st>>>(ma, mb, a);
  return launch_status();
}

}  // namespace sq
