// sq_fp4_linear_static: the FP4-G16 linear (same math and kernels as sq_fp4_linear) for
// callers that cannot allocate device memory.  Such callers are foreign-language bindings
// (cgo / JNI / ctypes) that own no device allocator and are handed only the operand
// buffers, and serving processes whose device memory is carved up once at start-up, where a
// cudaMalloc would synchronise the device and can fail mid-run.  Instead of the
// caller-provided workspace of sq_fp4_linear, the decoded weight rows are staged in the
// file-scope device array below and the matrix is processed in row chunks that fit it.
//
// Nothing here allocates: no cudaMalloc / cudaFree, no allocating library routine.  The
// array lives in this library's device image; its address is taken once per device with
// cudaGetSymbolAddress.  The entry point has no counterpart in the reference.
#include <mutex>
#include <string>

#include "../../include/sq325.h"
#include "common.cuh"
#include "fp4.cuh"

namespace sq {
int set_last_error(int code, const char* msg);  // abi.cu
}

using namespace sq;

namespace {

constexpr size_t kHeaderBytes = 256;  // error word (must start each call at zero), padded
constexpr size_t kStageBytes = SQ_FP4_LINEAR_STATIC_STAGE_BYTES;
constexpr int kTileRows = 256;        // tcgen05 GEMM N tile: chunks are whole tiles
constexpr int kMaxDevices = 64;

// [0, 256): int error word written by bounded device waits; [256, 256 + stage): fp16 rows.
static __device__ __align__(256) unsigned char g_linear_scratch[kHeaderBytes + kStageBytes];

std::mutex g_setup_mutex;
unsigned char* g_scratch_addr[kMaxDevices] = {};

// Per-device set-up on the first call with that device current: resolves the array's
// address (with lazy module loading this is also when the driver loads the module image)
// and sets the kernels' shared-memory attributes.
int scratch_for_current_device(unsigned char** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_last_error(SQ_ECUDA, "fp4_linear_static: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return set_last_error(SQ_EINVAL, "fp4_linear_static: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_linear_scratch);
    if (e != cudaSuccess || !p) {
      std::string msg = std::string("fp4_linear_static: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e);
      return set_last_error(SQ_ECUDA, msg.c_str());
    }
    if (prepare_fp4_kernels() != kOk || prepare_gemm_kernel() != kOk)
      return set_last_error(SQ_ECUDA, "fp4_linear_static: kernel attribute set-up failed");
    g_scratch_addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch_addr[dev];
  return SQ_OK;
}

int launch_error(int st, const char* what) {
  if (st == kOk) return SQ_OK;
  if (st == kECuda) {
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = last_launch_error();   // the launcher consumed it and recorded it
    last_launch_error() = cudaSuccess;
    std::string msg = std::string(what) + ": " + cudaGetErrorString(e);
    return set_last_error(SQ_ECUDA, msg.c_str());
  }
  return set_last_error(st, (std::string(what) + ": invalid arguments").c_str());
}

}  // namespace

extern "C" {

int64_t sq_fp4_linear_static_max_k(void) { return (int64_t)(kStageBytes / (2 * kTileRows)); }

int sq_fp4_linear_static(const uint8_t* codes, const uint8_t* block_scales, const float* global_scale, int n,
                         int k, const uint16_t* x, int64_t ldx, int m, uint16_t* y, int64_t ldy, void* stream) {
  if (!codes || !block_scales || !global_scale || !x || !y)
    return set_last_error(SQ_EINVAL, "fp4_linear_static: null pointer");
  if (m <= 0 || n <= 0 || k <= 0 || k % 128)
    return set_last_error(SQ_EINVAL, "fp4_linear_static: k must be a positive multiple of 128");
  if (((uintptr_t)codes % 16) || ((uintptr_t)x % 16))
    return set_last_error(SQ_EINVAL, "fp4_linear_static: misaligned buffers");
  // Row strides are checked here, before any chunk runs: the chunked GEMM below sees only
  // `rows` output columns per launch, so it cannot catch ldy < n itself.
  if (ldx < k || ldy < n)
    return set_last_error(SQ_EINVAL, "fp4_linear_static: row strides must satisfy ldx >= k and ldy >= n");
  if (m > 64 && k > sq_fp4_linear_static_max_k())
    return set_last_error(SQ_EINVAL,
                          "fp4_linear_static: k exceeds the static scratch (256 decoded rows of k fp16 must fit "
                          "SQ_FP4_LINEAR_STATIC_STAGE_BYTES = 16 MiB, so k <= 32768 when m > 64)");
  unsigned char* scratch = nullptr;
  if (int s = scratch_for_current_device(&scratch)) return s;
  int* d_err = reinterpret_cast<int*>(scratch);
  uint16_t* stage = reinterpret_cast<uint16_t*>(scratch + kHeaderBytes);
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(d_err, 0, sizeof(int), st) != cudaSuccess)
    return set_last_error(SQ_ECUDA, "fp4_linear_static: clearing the error word failed");

  Fp4Weight w{codes, block_scales, global_scale, n, k};
  if (m <= 64) {
    int s;
    if (k % 256 == 0 && ((uintptr_t)block_scales % 16) == 0 && ldx % 8 == 0)
      s = launch_error(launch_fp4_gemv_stream(w, nullptr, x, ldx, m, y, ldy, d_err, st), "fp4 gemv");
    else
      s = launch_error(launch_fp4_gemv(w, x, ldx, m, y, ldy, st), "fp4 gemv");
    if (s) return s;
  } else {
    // Rows per chunk: as many whole GEMM tiles of decoded rows as the stage holds.
    const int chunk = (int)((kStageBytes / (2 * (size_t)k)) / kTileRows) * kTileRows;
    for (int r0 = 0; r0 < n; r0 += chunk) {
      const int rows = n - r0 < chunk ? n - r0 : chunk;
      Fp4Weight part{codes + (size_t)r0 * (k / 2), block_scales + (size_t)r0 * (k / 16), global_scale, rows, k};
      if (int s = launch_error(launch_fp4_decode(part, stage, k, st), "fp4 decode")) return s;
      if (int s = launch_error(launch_gemm_f16(x, ldx, stage, k, y + r0, ldy, m, rows, k, 0, nullptr, d_err, st),
                               "tcgen05 gemm"))
        return s;
    }
  }
  // Synchronous completion: the stage is reused by the next call and the error word is read.
  int h = 0;
  if (cudaMemcpyAsync(&h, d_err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    std::string msg = std::string("fp4_linear_static: ") + cudaGetErrorString(cudaGetLastError());
    return set_last_error(SQ_ECUDA, msg.c_str());
  }
  if (h) return set_last_error(SQ_ETIMEOUT, "fp4_linear_static: a bounded device wait expired");
  return SQ_OK;
}

}  // extern "C"
