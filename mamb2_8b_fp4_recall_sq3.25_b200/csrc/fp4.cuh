// Packed FP4-E2M1 G16 weight descriptor and kernel launchers.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sq {

// One packed matrix exactly as the reference checkpoint stores it
// (mamba2_recall/fp4_checkpoint.py:100-114): codes u8[rows, cols/2] (low nibble =
// even column), block_scale_bytes u8[rows, cols/16] (E4M3FN), global_scale f32.
struct Fp4Weight {
  const uint8_t* codes;
  const uint8_t* scales;
  const float* global_scale;   // device pointer to one fp32
  int rows, cols;
};

int launch_fp4_decode(const Fp4Weight& W, uint16_t* out, long long ldo, cudaStream_t st);
// decode_packet's checks; ORs 1 (invalid scale), 2 (nonzero code in a zero-scale group),
// 4 (nonfinite decoded weight) into *flags (device int, caller-cleared).
int launch_fp4_validate(const Fp4Weight& W, int* flags, cudaStream_t st);
int launch_fp4_embed(const Fp4Weight& E, const long long* ids, int ntok, uint16_t* out, int* err, cudaStream_t st);
int launch_fp4_gemv(const Fp4Weight& W, const uint16_t* X, long long ldx, int M, uint16_t* Y, long long ldy,
                    cudaStream_t st);
// TMA descriptors of one packed matrix for the streaming GEMV (codes and block scales as
// u32 matrices, 16-row boxes).  Built once per matrix.
struct Fp4Maps {
  CUtensorMap codes;
  CUtensorMap scales;
  int kc;          // columns per pipeline stage
  int valid;
};
bool make_fp4_maps(const Fp4Weight& W, Fp4Maps* maps);
bool encode_u32_map(CUtensorMap* m, const void* base, long long rows, long long cols_u32, long long row_bytes,
                    int box_cols, int box_rows);
bool encode_f16_sw128_map(CUtensorMap* m, const void* base, long long rows, long long cols, int box_rows);
// Same product through the TMA-pipelined kernel (cols % 256 == 0, 16-byte aligned rows);
// `maps` may be null (built on the fly); `err` receives an error bit if a bounded wait expires.
// exact = false applies the fp32 global scale once per output instead of per weight.
int launch_fp4_gemv_stream(const Fp4Weight& W, const Fp4Maps* maps, const uint16_t* X, long long ldx, int M,
                           uint16_t* Y, long long ldy, int* err, cudaStream_t st, bool exact = true);

// tcgen05 GEMM: C[M,N] = A[M,K] . B[N,K]^T, fp16 in, fp32 accumulate in TMEM.
// mode 0: store fp16 C.  mode 1: cross-entropy partials of fp16-rounded logits
// (per row and 256-column tile: running max and sum of exp), plus the target
// logit, never writing C.
struct GemmCE {
  const long long* targets;    // [M] target column per row (row < M), in the full vocabulary
  float2* partials;            // [M, ntiles_total]
  float* target_logit;         // [M]
  int n_offset;                // first vocabulary column of this launch (multiple of 256)
  int ntiles_total;            // row stride of `partials` (tiles over the full vocabulary)
};
int launch_gemm_f16(const uint16_t* A, long long lda, const uint16_t* B, long long ldb,
                    uint16_t* C, long long ldc, int M, int N, int K, int mode, const GemmCE* ce,
                    int* dev_err, cudaStream_t st);
// Limit (ns) of the skinny GEMM's pipeline waits on the current device; 0 restores the
// default 2 s.  A short limit makes the waits expire: the kernel sets its error bit,
// drains its copies and returns (failure-detection tests).
int set_gemv_wait_limit_ns(unsigned long long ns);
bool encode_2d_map(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, long long rows, long long cols,
                   long long row_bytes, int box_cols, int box_rows, CUtensorMapSwizzle swizzle);
// Y[M, N] = X[M, K] . W[N, K]^T on the tensor cores with the FP4 decode fused in
// (fp4mma.cu), 1 <= M <= 256, K % 256 == 0, 16-byte aligned rows.  One CTA per 128 weight
// rows and K slice; `err` receives an error bit if a bounded wait expires.  exact = false
// applies the fp32 global scale once per output instead of per weight.
int launch_fp4_mma_linear(const Fp4Weight& W, const uint16_t* X, long long ldx, int M, uint16_t* Y, long long ldy,
                          int* err, cudaStream_t st, bool exact = true);
int prepare_fp4_mma_kernel();
int gemm_num_ntiles(int N);
int prepare_fp4_kernels();
int prepare_gemm_kernel();
int prepare_layer_kernels();

}  // namespace sq
