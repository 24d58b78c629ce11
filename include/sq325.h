/*
 * sq325.h — C ABI of the B200-native (sm_100a) Mamba-2 8B hot path with FP4-E2M1 G16
 * packed-resident weights and the 52-byte "SQ3.25" latent recurrent state.
 *
 * Plain C: device pointers are passed as typed pointers, sizes as ints, the CUDA stream
 * as an opaque `void*` (a cudaStream_t; NULL = legacy default stream).  Every entry point
 * returns an sq_status; the message of the last failure on the calling thread is
 * available from sq_last_error().  All buffers are owned by the caller except the
 * workspaces that an sq_model allocates in sq_model_reserve().
 *
 * Each declaration names the reference interface it replaces, as path:line in
 * EndlessChasing/mamb2_8B_FP4_Recall_SQ3.25.
 */
#ifndef SQ325_H_
#define SQ325_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SQ325_ABI_VERSION 1

typedef enum sq_status {
  SQ_OK = 0,
  SQ_EINVAL = 1,     /* geometry / dtype / layout / pointer contract violated (reference: ValueError) */
  SQ_ESTATE = 2,     /* ordering or controller state error (reference: RuntimeError) */
  SQ_ENONFINITE = 3, /* non-finite values detected (reference: FloatingPointError) */
  SQ_ECUDA = 4,      /* CUDA runtime error */
  SQ_ETIMEOUT = 5,   /* a bounded device-side wait expired; the context stays usable */
  SQ_ENOMEM = 6      /* workspace allocation failed */
} sq_status;

int sq_abi_version(void);
const char* sq_last_error(void);

/* ---------------------------------------------------------------- layouts
 * The seven tier layouts of scripts/w4_state_repair_codec_v2.py:22-28 after the latent
 * shift of scripts/fp4_zero_predictor_codec_v1.py:28-36 (n4 -= 4, nzero += 4).
 * Index order: 32_32_64, 16_64_48, 8_80_40, 24_48_56, 36_24_68, 40_16_72, 44_8_76. */
int sq_layout_index(const char* name);                                  /* -1 if unknown */
int sq_layout_counts(int layout, int* n8, int* n4, int* nzero);         /* layout_descriptor :28 */
int64_t sq_state_bytes(int batch, int heads, int dim);                  /* 52 B/row (:71-72) */

/* ---------------------------------------------------------------- codec scan
 * Replaces scan(x, dt, A, B, C, D, dt_bias, state, permutation, basis, latent_scale,
 * predictor, *, layout) -> (y, None)   scripts/fp4_zero_predictor_codec_v1.py:184-236,
 * including the host predictor correction (:221-225) and _latent_scan (:76-181).
 * All arrays are device pointers.  fp16 arrays are uint16_t bit patterns.
 * Activation element (b,t,h,p) of x / y lives at ptr + b*batch_stride + t*token_stride
 * + h*dim + p; dt (b,t,h) at dt + b*sb + t*st + h; B/C (b,t,g,n) at ptr + b*sb + t*st +
 * g*128 + n.  The state is mutated in place and y is written for every token.
 * workspace (optional, >= sq_scan_workspace(...) bytes, 256-byte aligned) enables the
 * two-kernel multi-token path (group-level dots computed once per group instead of once
 * per CTA); with NULL the single fused kernel runs.  Results are identical. */
typedef struct sq_scan_args {
  int32_t batch, length, heads, dim, groups, layout;
  const uint16_t* x;  int64_t x_batch_stride, x_token_stride;
  const uint16_t* dt; int64_t dt_batch_stride, dt_token_stride;
  const float* A;                                     /* [H] fp32, = -exp(A_log) */
  const uint16_t* B;  int64_t b_batch_stride, b_token_stride;
  const uint16_t* C;  int64_t c_batch_stride, c_token_stride;
  const void* D;       int32_t d_is_f32;              /* [H] fp16 or fp32 */
  const void* dt_bias; int32_t dt_bias_is_f32;        /* [H] fp16 or fp32 */
  const uint8_t* permutation;                         /* [G,128] u8 */
  const uint16_t* basis;                              /* [G,nzero,2] fp16 */
  const uint16_t* latent_scale;                       /* [G,2] fp16, > 0 */
  const uint16_t* predictor;                          /* [G,n8+n4+2,nzero] fp16 */
  uint8_t* lo; uint8_t* hi; uint8_t* q4; uint8_t* latent; uint16_t* s8; uint16_t* s4; /* PackedState */
  uint16_t* y; int64_t y_batch_stride, y_token_stride;
  void* workspace; int64_t workspace_bytes;           /* optional, may be NULL / 0 */
} sq_scan_args;
int64_t sq_scan_workspace(int batch, int length, int heads, int groups, int layout);
int sq_scan(const sq_scan_args* args, void* stream);
/* The causal depthwise conv of StateQuant._convolution (mamba2_recall/state_quant.py:283-317)
 * fused in front of the scan, as PredictorState._forward runs them
 * (fp4_zero_predictor_codec_v1.py:341-352).  x / B / C of `args` point at the RAW in_proj
 * xBC columns (channel h*dim+p, 8192+g*128+n, 9216+g*128+n; heads*dim = 8192 and
 * groups*128 = 1024), and the conv output feeds the scan without a round trip.
 * position == 0: prefill of `length` tokens from a reset (zero) ring, conv1d numerics
 * (fp32 accumulate + bias, one fp16 rounding, SiLU); the ring receives the last four raw
 * columns.  position > 0 requires length == 1: the one-token step numerics (fp16
 * products summed, fp16, + bias, SiLU) over the three previous raw columns in the ring
 * plus this token's, which replaces slot position % 4.  A continuing multi-token prefill
 * is not fused (SQ_EINVAL).  args->workspace selects the two-kernel path as in sq_scan
 * (prefill only). */
typedef struct sq_conv_args {
  const uint16_t* weight;     /* [10240,4] fp16 = conv1d.weight[:,0,:] */
  const uint16_t* bias;       /* [10240] fp16 */
  uint16_t* ring;             /* [batch][4][10240] fp16, slot = absolute position % 4 */
  int64_t ring_batch_stride;  /* elements, >= 4*10240 */
  int32_t position;           /* tokens this request consumed before the call */
} sq_conv_args;
int sq_scan_conv(const sq_scan_args* args, const sq_conv_args* conv, void* stream);

/* ---------------------------------------------------------------- S16 control scan
 * Replaces scan(..., state) for the FP16-state mode 's16' of mamba2_recall/state_codec.py
 * (_s16_scan :65-102, host wrapper :203-262), the reference's control / teacher arm: the
 * carry fp16 [batch,heads,dim,128] is updated in place (fp32 arithmetic, rounded to fp16
 * after every token) and y fp16 is written for every token.  Strides as in sq_scan_args.
 * stats (optional, NULL = off): fp32 [batch,heads,ceil(dim/16),128], per 16-row block the
 * sum over tokens and rows of |fp16 carry| (collect_stats=True). */
typedef struct sq_s16_args {
  int32_t batch, length, heads, dim, groups;
  const uint16_t* x;  int64_t x_batch_stride, x_token_stride;
  const uint16_t* dt; int64_t dt_batch_stride, dt_token_stride;
  const float* A;
  const uint16_t* B;  int64_t b_batch_stride, b_token_stride;
  const uint16_t* C;  int64_t c_batch_stride, c_token_stride;
  const void* D;       int32_t d_is_f32;
  const void* dt_bias; int32_t dt_bias_is_f32;
  uint16_t* state;
  uint16_t* y; int64_t y_batch_stride, y_token_stride;
  float* stats;
} sq_s16_args;
int sq_s16_scan(const sq_s16_args* args, void* stream);

/* ---------------------------------------------------------------- legacy sq3p25 scan + STE
 * sq_sq3p25_scan replaces scan(..., state) for the mode 'sq3p25' of
 * mamba2_recall/state_codec.py (`_sq_scan` :105-176, host wrapper :204-262): a fixed split
 * of each row into 16 INT8 + 64 INT4 stored coordinates and 48 pruned ones (the group's
 * permutation orders them), 52 bytes per row: lo / hi u8 [batch,heads,dim,8], q4 u8
 * [...,32], s8 / s4 fp16 [batch,heads,dim], updated in place; y fp16 for every token.
 * sq_ste_backward is the straight-through backward of scan_training
 * (mamba2_recall/state_training_scan.py :24-221) for a scan from a fresh zero state:
 * inputs contiguous as in the forward call, dy fp16 [B,L,H,P]; writes dx fp32 [B,L,H,P],
 * d(dt) fp32 [B,L,H], dB / dC fp32 [B,L,G,128] (every element written; sums in the
 * reference's order, no atomics, so the results are deterministic).  chunk = tokens between
 * carry checkpoints (1..256); the workspace holds the checkpoints, one chunk of carries, the
 * adjoint carry and one chunk of per-(head, row tile) dB / dC partials:
 * sq_ste_workspace(batch, length, heads, dim, chunk) bytes. */
typedef struct sq_sq3p25_args {
  int32_t batch, length, heads, dim, groups;
  const uint16_t* x;  int64_t x_batch_stride, x_token_stride;
  const uint16_t* dt; int64_t dt_batch_stride, dt_token_stride;
  const float* A;
  const uint16_t* B;  int64_t b_batch_stride, b_token_stride;
  const uint16_t* C;  int64_t c_batch_stride, c_token_stride;
  const void* D;       int32_t d_is_f32;
  const void* dt_bias; int32_t dt_bias_is_f32;
  const uint8_t* permutation;
  uint8_t* lo; uint8_t* hi; uint8_t* q4; uint16_t* s8; uint16_t* s4;
  uint16_t* y; int64_t y_batch_stride, y_token_stride;
} sq_sq3p25_args;
int sq_sq3p25_scan(const sq_sq3p25_args* args, void* stream);
int64_t sq_ste_workspace(int batch, int length, int heads, int dim, int chunk);
int sq_ste_backward(const sq_sq3p25_args* args, int chunk, const uint16_t* dy, float* dx, float* ddt, float* db,
                    float* dc, void* workspace, int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- standalone codec
 * decode: rows (b,h,p) of the six PackedState buffers (mamba2_recall/state_codec.py:29-48,
 * fp4_zero_predictor_codec_v1.py:39-49) -> tiers fp32 [rows, n8+n4] in tier order and
 * latent z fp32 [rows, 2] (= e4m3 * latent_scale[g]) — the kernel prologue :81-114.
 * encode: the inverse with the kernel's requant rule (:149-181 with
 * scripts/state_ppl_codec_v6.py:52-61) when mode == 0, or the diagnostic initializer
 * encode_state_ (mamba2_recall/state_codec.py:299-331) when mode == 1 (latent bytes 0). */
int sq_state_decode(int layout, int batch, int heads, int dim, int groups,
                    const uint8_t* lo, const uint8_t* hi, const uint8_t* q4, const uint8_t* latent,
                    const uint16_t* s8, const uint16_t* s4, const uint16_t* latent_scale,
                    float* tiers, float* z, void* stream);
int sq_state_encode(int layout, int batch, int heads, int dim, int groups, int mode,
                    const float* tiers, const float* z, const uint16_t* latent_scale,
                    uint8_t* lo, uint8_t* hi, uint8_t* q4, uint8_t* latent, uint16_t* s8, uint16_t* s4,
                    void* stream);

/* ---------------------------------------------------------------- FP4-E2M1 G16 weights
 * Packed matrix as stored by mamba2_recall/fp4_checkpoint.py:100-114: codes u8[rows,cols/2]
 * (low nibble = even column), block scales u8[rows,cols/16] (E4M3FN bytes), one fp32 global
 * scale (device pointer).
 * sq_fp4_decode replaces fp4.decode_packet (mamba2_recall/fp4.py:225-250), bit-exact. */
int sq_fp4_decode(const uint8_t* codes, const uint8_t* block_scales, const float* global_scale,
                  int rows, int cols, uint16_t* out, int64_t ldo, void* stream);
/* The content checks of fp4.decode_packet (mamba2_recall/fp4.py:235-249) on the device;
 * synchronous.  SQ_EINVAL (the reference's ValueError) with its message: "Invalid stored
 * scale" (a negative or NaN E4M3 block scale), "Nonzero code in a zero-scale group", or
 * "Nonfinite decoded FP16 weights".  Calls on one device share a flag word: serialise them. */
int sq_fp4_validate(const uint8_t* codes, const uint8_t* block_scales, const float* global_scale,
                    int rows, int cols, void* stream);
/* Y[m,n] = X[m,k] . W[n,k]^T with W decoded exactly on the fly; replaces the FP16
 * nn.Linear calls mx.in_proj / mx.out_proj / model.lm_head
 * (fp4_zero_predictor_codec_v1.py:338,357,360; run_fp4_ridge_resurface_v3.py:107).
 * m <= 64 runs the packed skinny-GEMM kernel (no workspace); larger m decodes into
 * `workspace` (>= sq_fp4_linear_workspace(m,n,k) bytes) and runs the tcgen05 GEMM. */
int64_t sq_fp4_linear_workspace(int m, int n, int k);
/* Asynchronous on `stream`.  A bounded device wait that expires (the context stays usable)
 * sets this device's sticky error word, which sq_device_check() reports and clears. */
int sq_fp4_linear(const uint8_t* codes, const uint8_t* block_scales, const float* global_scale,
                  int n, int k, const uint16_t* x, int64_t ldx, int m, uint16_t* y, int64_t ldy,
                  void* workspace, int64_t workspace_bytes, void* stream);
/* sq_fp4_linear without any device allocation (no counterpart in the reference): for
 * callers that cannot allocate, i.e. FFI bindings that own no device allocator, and
 * serving processes whose device memory is fixed at start-up (a cudaMalloc synchronises
 * the device and can fail mid-run).  Same result as sq_fp4_linear; for m > 64 the decoded
 * weight rows are staged, in chunks of whole 256-row tiles, in a static device array of
 * SQ_FP4_LINEAR_STATIC_STAGE_BYTES inside this library, so k <= 32768 there
 * (sq_fp4_linear_static_max_k()); larger k returns SQ_EINVAL, and so do row strides
 * ldx < k or ldy < n (checked before any work, leaving y untouched).
 * The first call on each device does set-up (resolves the array's address, which may load
 * the module, and sets kernel attributes): make it before any stream capture.  The call is
 * synchronous on `stream`.  The array is shared by all callers in the process: calls that
 * overlap in time (two host threads, or two streams) race on it and must be serialised. */
#define SQ_FP4_LINEAR_STATIC_STAGE_BYTES (16u << 20)
int64_t sq_fp4_linear_static_max_k(void);
int sq_fp4_linear_static(const uint8_t* codes, const uint8_t* block_scales, const float* global_scale,
                         int n, int k, const uint16_t* x, int64_t ldx, int m, uint16_t* y, int64_t ldy,
                         void* stream);
/* tcgen05 fp16 GEMM C[m,n] = A[m,k] . B[n,k]^T (fp32 accumulate), k % 64 == 0.
 * Asynchronous; expired waits are reported by sq_device_check(). */
int sq_gemm_f16(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb,
                uint16_t* c, int64_t ldc, int m, int n, int k, void* stream);
/* Synchronises `stream`, then reads and clears the current device's error word of the
 * standalone entry points above (sq_fp4_linear, sq_gemm_f16): SQ_ETIMEOUT if a bounded
 * device-side wait of one of their kernels expired since the last check.  The model
 * runtime has its own word (sq_model_check).  The reference reports no such condition
 * (its GEMMs are cuBLAS calls); this replaces nothing. */
int sq_device_check(void* stream);
/* Failure detection: the limit, in nanoseconds, of the skinny-GEMM kernel's pipeline waits
 * (sq_fp4_linear with m <= 64, the model's decode-step projections and greedy head) on
 * the current device; 0 restores the default of 2 s, and a limit under 2 us (finer than the
 * device timer resolves) makes each wait a single non-blocking test.  When a wait
 * reaches the limit the
 * kernel records an error bit, waits (with the default limit) for its own copies in
 * flight and returns, leaving the context usable; the call's check (sq_device_check or
 * sq_model_check) then returns SQ_ETIMEOUT.  Tests set a tiny limit to drive that path;
 * no reference counterpart (its GEMMs are cuBLAS calls). */
int sq_set_wait_limit_ns(uint64_t ns);

/* ---------------------------------------------------------------- model runtime
 * A native replacement for PredictorState (fp4_zero_predictor_codec_v1.py:239-367) driving
 * all layers of the Mamba-2 LM (MambaLMHeadModel geometry, mamba2_recall/runtime.py:25-33)
 * without monkey-patching: embedding -> per layer [Block add+RMSNorm, in_proj, causal conv,
 * SQ3.25 scan, Resurface, gated RMSNorm, out_proj] -> norm_f, plus the scoring and greedy
 * heads.  Weights and states are caller-owned device buffers bound by pointer. */
typedef struct sq_model sq_model;

typedef struct sq_model_config {
  int32_t n_layer;     /* 56 */
  int32_t vocab;       /* 256000 (any multiple of 16 >= 16 for tests) */
  float eps;           /* RMSNorm epsilon, 1e-5 */
} sq_model_config;

typedef struct sq_fp4_matrix {
  const uint8_t* codes; const uint8_t* block_scales; const float* global_scale; int32_t rows, cols;
} sq_fp4_matrix;

typedef struct sq_layer_desc {
  sq_fp4_matrix in_proj;            /* [18560, 4096] */
  sq_fp4_matrix out_proj;           /* [4096, 8192] */
  const uint16_t* norm_weight;      /* Block RMSNorm [4096] */
  const uint16_t* conv_weight;      /* [10240,4] */
  const uint16_t* conv_bias;        /* [10240] */
  const float* A;                   /* [128] = -exp(A_log) */
  const uint16_t* D;                /* [128] */
  const uint16_t* dt_bias;          /* [128] */
  const uint16_t* gated_norm_weight;/* [8192] */
  int32_t layout;                   /* 0..6 */
  const uint8_t* permutation;       /* [8,128] */
  const uint16_t* basis;            /* [8,nzero,2] */
  const uint16_t* latent_scale;     /* [8,2] */
  const uint16_t* predictor;        /* [8,n8+n4+2,nzero] */
} sq_layer_desc;

int sq_model_create(const sq_model_config* cfg, sq_model** out);
int sq_model_destroy(sq_model* model);
int sq_model_set_layer(sq_model* model, int layer, const sq_layer_desc* desc);
int sq_model_set_globals(sq_model* model, const sq_fp4_matrix* embedding, const sq_fp4_matrix* lm_head,
                         const uint16_t* norm_f_weight);
/* Resurface adapter of one layer (resurface_native.py:105-118, install_fp16 :363-375);
 * V == NULL removes it.  V [128,128], g [128], w [4096], b [1] fp16; hard != 0: threshold gate. */
int sq_model_set_adapter(sq_model* model, int layer, const uint16_t* V, const uint16_t* g,
                         const uint16_t* w, const uint16_t* b, int hard);
/* Per-layer state of a request batch: the six PackedState buffers [batch,128,64,w] and the
 * conv ring [batch,4,10240] fp16 (slot = position % 4). */
int sq_model_bind_state(sq_model* model, int layer, int batch, uint8_t* lo, uint8_t* hi, uint8_t* q4,
                        uint8_t* latent, uint16_t* s8, uint16_t* s4, uint16_t* conv_ring);
/* Allocate workspaces for up to max_tokens = batch*tokens rows per forward. */
int sq_model_reserve(sq_model* model, int max_tokens);
/* StateQuant.backbone (mamba2_recall/state_quant.py:196-219): ids int64 [batch,tokens];
 * pos0 = tokens already consumed by this request (0 after reset).  hidden_out fp16
 * [batch*tokens, 4096] after norm_f. */
int sq_model_forward(sq_model* model, const int64_t* ids, int batch, int tokens, int pos0,
                     uint16_t* hidden_out, void* stream);
/* One mixer layer, PredictorState._forward (fp4_zero_predictor_codec_v1.py:314-367): u is
 * the Block's normed input fp16 [batch*tokens, 4096] (what mamba_ssm's Block hands the
 * mixer), out receives the mixer output fp16 [batch*tokens, 4096].  in_proj -> causal conv
 * -> SQ3.25 scan (the layer's bound state, advanced in place) -> Resurface -> gated
 * RMSNorm -> out_proj, with the same kernels and numerics as sq_model_forward.  pos0 is
 * the number of tokens this layer's state has consumed. */
int sq_model_mixer_forward(sq_model* model, int layer, const uint16_t* u, int batch, int tokens, int pos0,
                           uint16_t* out, void* stream);
/* Scoring head (run_fp4_ridge_resurface_v3.py:105-109): per-row next-token NLL of the
 * fp16 logits lm_head(hidden).float(), computed without materialising the logits. */
int sq_model_score(sq_model* model, const uint16_t* hidden, int rows, const int64_t* targets,
                   float* nll, void* stream);
/* Greedy head (infer_fp4_ridge_resurface_v1.py:103-105): fp16 logits [rows,vocab] (optional,
 * may be NULL) and first-occurrence argmax tokens [rows]. */
int sq_model_greedy(sq_model* model, const uint16_t* hidden, int rows, uint16_t* logits_out,
                    int64_t* tokens_out, void* stream);
/* Synchronises the stream and reports a device-side failure (bad token id, expired wait). */
int sq_model_check(sq_model* model, void* stream);
/* Greedy decode at batch 1 with one persistent cooperative launch for all `steps` tokens
 * (the loop of infer_fp4_ridge_resurface_v1.py:100-110 after the prompt): step s feeds tokens[0] at
 * position pos + s, runs all layers, the final norm, lm_head and argmax, overwrites
 * tokens[0] with the pick and stores it in out_tokens[s] (device, may be NULL).  Requires
 * batch-1 states (pos > 0: prompt already consumed) and reserve(); the projections and the
 * head follow sq_model_set_exact_skinny (factored global scale by default, the exactly
 * decoded fp16 weights when set); the logits of the last step are left in the model's greedy
 * workspace.  Same tokens and states as sq_model_forward + sq_model_greedy per step, in
 * either mode. */
int sq_model_decode(sq_model* model, int64_t* tokens, int pos, int steps, int64_t* out_tokens, void* stream);
/* Inspection (the role of the reference's per-layer forward hooks, e.g. the Resurface
 * capture hooks of mamba2_recall/resurface_native.py:168-169): when `out` is non-NULL every
 * later sq_model_forward with batch*tokens <= rows also copies each layer's mixer output
 * (the out_proj result the Block adds to the residual) to out + layer*rows*4096, fp16
 * [rows, 4096] per layer.  NULL turns it off.  The persistent decode kernel does not
 * capture. */
int sq_model_set_capture(sq_model* model, uint16_t* out, int64_t rows);
/* Numerics of the one-token decode-step projections and of the greedy head (at most 64
 * rows).  exact = 0 (default): the exact fp16 products E2M1*E4M3 enter the tensor-core
 * product and the fp32 global scale multiplies each fp32 output once (factored scale), the
 * bandwidth-bound form.  exact = 1: every weight is first rounded to fp16 as the reference's
 * decoded FP16 weights (fp4.py:100-103), about three ALU instructions per weight.  Prompts,
 * scoring windows and the scoring head always use the exactly decoded weights. */
int sq_model_set_exact_skinny(sq_model* model, int exact);
/* Measurement: with enable = 1, every later large-M in_proj GEMM launch of sq_model_forward
 * (the tcgen05 GEMM of prompts and scoring windows, more than 256 rows) is bracketed by a pair
 * of CUDA events on its stream (not while the stream is being captured); enable = 0 stops.
 * Either call discards earlier records.  sq_model_gemm_time waits for the recorded launches
 * and returns their summed device time and count, then discards them. */
int sq_model_time_gemm(sq_model* model, int enable);
int sq_model_gemm_time(sq_model* model, double* seconds, int64_t* launches);

#ifdef __cplusplus
}
#endif
#endif /* SQ325_H_ */
