// Per-layer elementwise / normalisation / head kernels of the Mamba-2 block.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sq {

// Block residual + RMSNorm (mamba_ssm Block with fused_add_norm=False,
// residual_in_fp32=False): res = fp16(h + res) (res = h when has_res == 0),
// out = fp16((res * rstd) * w), rstd = 1/sqrt(mean(res^2) + eps).
int launch_add_rmsnorm(const uint16_t* h, uint16_t* res, int has_res, const uint16_t* w, float eps,
                       uint16_t* out, int rows, int D, cudaStream_t st);

// Causal depthwise conv (width 4) + bias + SiLU over `L` new positions starting at
// absolute position pos0, for the 10240 xBC channels read from `raw` (row stride
// raw_st per token, batch stride raw_sb).  The previous 3 raw columns come from
// the ring `cache` ([B,4,C], slot = position % 4) when pos0 > 0, zeros otherwise;
// the ring is updated with the last min(L,4) raw columns.
int launch_conv_prefill(const uint16_t* raw, long long raw_sb, long long raw_st, int B, int L, int C,
                        const uint16_t* w, const uint16_t* bias, uint16_t* cache, long long cache_sb,
                        int pos0, uint16_t* out, long long out_sb, long long out_st, cudaStream_t st);

// Resurface post-D adapter (optional) + gated RMSNorm (norm_before_gate=False,
// group 1024) for `T` tokens.  y [T,8192] fp16 (scan output), z rows at z + t*z_st,
// u rows at u + t*u_st (mixer input).  Adapter: V [128,128], g [128], w [4096], b [1]
// fp16; hard != 0 selects the threshold gate.
struct AdapterPtrs { const uint16_t* V; const uint16_t* g; const uint16_t* w; const uint16_t* b; int hard; };
int launch_resurface_gatednorm(const uint16_t* y, const uint16_t* z, long long z_st, const uint16_t* u,
                               long long u_st, const AdapterPtrs* ad, const uint16_t* norm_w, float eps,
                               uint16_t* out, int T, cudaStream_t st);

// Cross-entropy finalisation: per row lse from the GEMM partials, nll = lse - target logit.
int launch_ce_finalize(const float2* partials, int ntiles, const float* tlogit, int rows, float* nll,
                       cudaStream_t st);
// Per-window fp64 sums of nll over `per` consecutive rows.
int launch_window_sum(const float* nll, int windows, int per, const int* counts, double* out, cudaStream_t st);
// First-occurrence argmax over fp16 rows (two stages; `ws` >= argmax_workspace_bytes).
int argmax_workspace_bytes(int rows, int V);
int launch_argmax(const uint16_t* logits, int rows, int V, long long ld, long long* out, void* ws, cudaStream_t st);

}  // namespace sq
