// C-ABI entry points (include/sq325.h) and the native model runtime that sequences the
// per-layer kernels.  Host code only; all device work is in scan.cu / codec.cu / fp4.cu /
// gemm.cu / layer.cu.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/sq325.h"
#include "common.cuh"
#include "decode.cuh"
#include "fp4.cuh"
#include "layer.cuh"
#include "s16.cuh"
#include "ste.cuh"
#include "scan.cuh"

namespace sq {
cudaError_t& last_launch_error() {
  static thread_local cudaError_t e = cudaSuccess;
  return e;
}
int launch_decode_rows(int layout, int batch, int heads, int dim, int groups, const uint8_t* lo,
                       const uint8_t* hi, const uint8_t* q4, const uint8_t* latent, const uint16_t* s8,
                       const uint16_t* s4, const uint16_t* latent_scale, float* tiers, float* z, cudaStream_t st);
int launch_encode_rows(int layout, int batch, int heads, int dim, int groups, int mode, const float* tiers,
                       const float* z, const uint16_t* latent_scale, uint8_t* lo, uint8_t* hi, uint8_t* q4,
                       uint8_t* latent, uint16_t* s8, uint16_t* s4, cudaStream_t st);
}  // namespace sq

using namespace sq;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
int cuda_fail(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = last_launch_error();     // a launcher already consumed it
  last_launch_error() = cudaSuccess;
  return fail(SQ_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
int check(int st, const char* what) {
  if (st == kOk) return SQ_OK;
  if (st == kECuda) return cuda_fail(what);
  return fail(st, std::string(what) + ": invalid arguments");
}
#define SQ_TRY(expr, what)                 \
  do {                                     \
    int _s = check((expr), (what));        \
    if (_s != SQ_OK) return _s;            \
  } while (0)

bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

constexpr int kDModel = 4096, kDInner = 8192, kXbc = 10240, kZx = 18560, kHeads = 128, kHeadDim = 64,
              kGroups = 8;
constexpr int kLmChunk = 32768;    // lm_head rows decoded per staging pass

// Device error word of the standalone entry points (sq_fp4_linear, sq_gemm_f16), one per
// device, allocated on the first call made with that device current.  Kernels whose
// bounded waits expire OR a bit into it; it stays set until sq_device_check() reads and
// clears it.
constexpr int kMaxDevices = 64;
std::mutex g_err_mutex;
int* g_dev_err[kMaxDevices] = {};

int device_error_word(int** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return cuda_fail("cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(SQ_EINVAL, "device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_err_mutex);
  if (!g_dev_err[dev]) {
    int* p = nullptr;
    // [0]: the sticky error word; [1]: per-call flags of sq_fp4_validate
    if (cudaMalloc(&p, 2 * sizeof(int)) != cudaSuccess) return cuda_fail("cudaMalloc (error word)");
    if (cudaMemset(p, 0, 2 * sizeof(int)) != cudaSuccess) { cudaFree(p); return cuda_fail("cudaMemset (error word)"); }
    g_dev_err[dev] = p;
  }
  *out = g_dev_err[dev];
  return SQ_OK;
}

}  // namespace

struct sq_model {
  sq_model_config cfg;
  std::vector<sq_layer_desc> layers;
  std::vector<AdapterPtrs> adapters;
  std::vector<Fp4Maps> in_maps, out_maps;     // streaming-GEMV TMA descriptors per layer
  Fp4Maps head_maps{};
  struct St { int batch = 0; uint8_t *lo = 0, *hi = 0, *q4 = 0, *latent = 0; uint16_t *s8 = 0, *s4 = 0, *ring = 0; };
  std::vector<St> states;
  sq_fp4_matrix embed{}, head{};
  const uint16_t* norm_f = nullptr;
  int max_tokens = 0;
  // workspaces
  uint16_t *h = 0, *res = 0, *hn = 0, *zx = 0, *xbc = 0, *y = 0, *yn = 0, *stage = 0, *logits = 0;
  float2* partials = 0;
  float* tlogit = 0;
  void* prep = 0;                             // two-kernel scan workspace (any layout)
  bool exact_skinny = false;                  // decode steps / greedy head: per-weight fp16 decode
  // persistent batch-1 decode: device copies of the layer table and TMA maps, step buffers
  DecLayer* d_dlayers = 0;
  CUtensorMap* d_dmaps = 0;
  unsigned char* d_dbuf = 0;                  // h | res[2] | zx | y | argmax partials | sync
  bool dec_dirty = true;
  int dec_grid = 0;
  int* d_err = 0;
  size_t stage_elems = 0;
  uint16_t* capture = nullptr;                // per-layer mixer outputs [n_layer][capture_rows][4096]
  long long capture_rows = 0;
  // opt-in timing of the large-M in_proj tcgen05 GEMM launches (sq_model_time_gemm): an
  // event pair per launch on the launching stream, read by sq_model_gemm_time
  bool gemm_timing = false;
  std::vector<cudaEvent_t> gemm_events;
  size_t gemm_events_used = 0;
  std::atomic<int> busy{0};
};

namespace {

Fp4Weight fw(const sq_fp4_matrix& m) { return Fp4Weight{m.codes, m.block_scales, m.global_scale, m.rows, m.cols}; }

void free_ws(sq_model* m) {
  void* ptrs[] = {m->h, m->res, m->hn, m->zx, m->xbc, m->y, m->yn, m->stage, m->logits, m->partials, m->tlogit,
                  m->prep};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  m->h = m->res = m->hn = m->zx = m->xbc = m->y = m->yn = m->stage = m->logits = nullptr;
  m->partials = nullptr; m->tlogit = nullptr; m->prep = nullptr;
  m->max_tokens = 0;
}

// Routing by batch rows M: one row -> the packed skinny GEMM; 2..256 rows -> the tensor-core
// linear with the decode fused in; more -> exact decode into the staging matrix + the tcgen05
// GEMM.  exact = per-weight fp16 decode (the reference's); false (one-token decode steps
// unless set_exact_skinny) applies the fp32 global scale once per output.
constexpr int kSkinnyMax = 1, kFusedMax = 256;
// Event pair around one timed GEMM launch; nullptr when timing is off or the stream is being
// captured into a graph.
cudaEvent_t* gemm_event_pair(sq_model* m, cudaStream_t st) {
  if (!m->gemm_timing) return nullptr;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return nullptr;
  while (m->gemm_events.size() < m->gemm_events_used + 2) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    m->gemm_events.push_back(e);
  }
  cudaEvent_t* pair = &m->gemm_events[m->gemm_events_used];
  m->gemm_events_used += 2;
  return pair;
}

int linear(sq_model* m, const sq_fp4_matrix& W, const Fp4Maps* maps, const uint16_t* X, long long ldx, int M,
           uint16_t* Y, long long ldy, bool exact, cudaStream_t st, bool timed = false) {
  const Fp4Weight w = fw(W);
  if (M <= kSkinnyMax) return check(launch_fp4_gemv_stream(w, maps, X, ldx, M, Y, ldy, m->d_err, st, exact), "fp4 gemv");
  if (M <= kFusedMax)
    return check(launch_fp4_mma_linear(w, X, ldx, M, Y, ldy, m->d_err, st, exact), "fp4 tensor-core linear");
  if ((size_t)W.rows * W.cols > m->stage_elems) return fail(SQ_EINVAL, "staging buffer too small");
  SQ_TRY(launch_fp4_decode(w, m->stage, W.cols, st), "fp4 decode");
  cudaEvent_t* ev = timed ? gemm_event_pair(m, st) : nullptr;
  if (ev) cudaEventRecord(ev[0], st);
  const int s = check(launch_gemm_f16(X, ldx, m->stage, W.cols, Y, ldy, M, W.rows, W.cols, 0, nullptr, m->d_err, st),
                      "tcgen05 gemm");
  if (ev) cudaEventRecord(ev[1], st);
  return s;
}

}  // namespace

namespace sq {
// Records `msg` as the calling thread's last error (used by entry points in other files).
int set_last_error(int code, const char* msg) { return fail(code, msg); }
}  // namespace sq

extern "C" {

int sq_abi_version(void) { return SQ325_ABI_VERSION; }
const char* sq_last_error(void) { return g_err.c_str(); }

int sq_layout_index(const char* name) {
  if (!name) return -1;
  for (int i = 0; i < 7; ++i)
    if (std::strcmp(name, kLayouts[i].name) == 0) return i;
  return -1;
}

int sq_layout_counts(int layout, int* n8, int* n4, int* nzero) {
  if (layout < 0 || layout > 6) return fail(SQ_EINVAL, "unknown layout index");
  if (n8) *n8 = kLayouts[layout].n8;
  if (n4) *n4 = kLayouts[layout].n4;
  if (nzero) *nzero = kLayouts[layout].nz;
  return SQ_OK;
}

int64_t sq_state_bytes(int batch, int heads, int dim) { return (int64_t)batch * heads * dim * 52; }

int64_t sq_scan_workspace(int batch, int length, int heads, int groups, int layout) {
  return scan_prep_bytes(batch, length, heads, groups, layout);
}

namespace {
// Checks the pointer contract of sq_scan_args and fills the kernel parameter block.
int scan_params(const sq_scan_args* a, ScanParams& P) {
  if (!a) return fail(SQ_EINVAL, "null scan args");
  const void* req[] = {a->x, a->dt, a->A, a->B, a->C, a->D, a->dt_bias, a->permutation, a->basis,
                       a->latent_scale, a->predictor, a->lo, a->hi, a->q4, a->latent, a->s8, a->s4, a->y};
  for (const void* p : req)
    if (!p) return fail(SQ_EINVAL, "scan: null pointer argument");
  const void* st16[] = {a->lo, a->hi, a->q4, a->latent, a->s8, a->s4, a->permutation, a->basis, a->predictor};
  for (const void* p : st16)
    if (!aligned(p, 16)) return fail(SQ_EINVAL, "scan: state buffers and static tables must be 16-byte aligned");
  P = ScanParams{};
  P.batch = a->batch; P.length = a->length; P.heads = a->heads; P.dim = a->dim; P.groups = a->groups;
  P.layout = a->layout;
  P.x = a->x; P.x_sb = a->x_batch_stride; P.x_st = a->x_token_stride;
  P.dt = a->dt; P.dt_sb = a->dt_batch_stride; P.dt_st = a->dt_token_stride;
  P.A = a->A;
  P.B = a->B; P.b_sb = a->b_batch_stride; P.b_st = a->b_token_stride;
  P.C = a->C; P.c_sb = a->c_batch_stride; P.c_st = a->c_token_stride;
  P.D = a->D; P.d_is_f32 = a->d_is_f32; P.dt_bias = a->dt_bias; P.dt_bias_is_f32 = a->dt_bias_is_f32;
  P.perm = a->permutation; P.basis = a->basis; P.latent_scale = a->latent_scale; P.predictor = a->predictor;
  P.lo = a->lo; P.hi = a->hi; P.q4 = a->q4; P.latent = a->latent; P.s8 = a->s8; P.s4 = a->s4;
  P.y = a->y; P.y_sb = a->y_batch_stride; P.y_st = a->y_token_stride;
  if (a->workspace) {
    const long long need = scan_prep_bytes(a->batch, a->length, a->heads, a->groups, a->layout);
    if (need < 0 || a->workspace_bytes < need || !aligned(a->workspace, 256))
      return fail(SQ_EINVAL, "scan: workspace smaller than sq_scan_workspace() or not 256-byte aligned");
    scan_prep_bind(P, a->workspace);
  }
  return SQ_OK;
}
}  // namespace

int sq_scan(const sq_scan_args* a, void* stream) {
  ScanParams P;
  if (int s = scan_params(a, P)) return s;
  return check(launch_scan(P, (cudaStream_t)stream), "sq_scan");
}

int sq_scan_conv(const sq_scan_args* a, const sq_conv_args* c, void* stream) {
  if (!c || !c->weight || !c->bias || !c->ring) return fail(SQ_EINVAL, "scan_conv: null conv argument");
  ScanParams P;
  if (int s = scan_params(a, P)) return s;
  if (P.heads * P.dim + 2 * P.groups * 128 != kXbc)
    return fail(SQ_EINVAL, "scan_conv: heads*dim + 2*groups*128 must equal the 10240 conv channels");
  if (!aligned(c->ring, 16) || c->ring_batch_stride % 8 || c->ring_batch_stride < 4LL * kXbc)
    return fail(SQ_EINVAL, "scan_conv: ring must be 16-byte aligned with a batch stride >= 4*10240 (multiple of 8)");
  if (c->position < 0 || (c->position > 0 && P.length != 1))
    return fail(SQ_EINVAL, "scan_conv: position 0 (prefill from a reset ring) or a one-token step (position > 0)");
  P.conv_mode = c->position == 0 ? 1 : 2;   // with a workspace, both run the two-kernel path
  P.conv_w = c->weight; P.conv_b = c->bias; P.conv_cache = c->ring; P.conv_pos = c->position;
  P.conv_cache_sb = c->ring_batch_stride;
  return check(launch_scan(P, (cudaStream_t)stream), "sq_scan_conv");
}

int sq_s16_scan(const sq_s16_args* a, void* stream) {
  if (!a || !a->x || !a->dt || !a->A || !a->B || !a->C || !a->D || !a->dt_bias || !a->state || !a->y)
    return fail(SQ_EINVAL, "s16_scan: null pointer argument");
  if (a->batch <= 0 || a->length <= 0 || a->heads <= 0 || a->dim <= 0 || a->groups <= 0 || a->heads % a->groups)
    return fail(SQ_EINVAL, "heads must be divisible by B/C groups");
  if (!aligned(a->state, 4)) return fail(SQ_EINVAL, "s16_scan: state must be 4-byte aligned");
  S16Params P{};
  P.batch = a->batch; P.length = a->length; P.heads = a->heads; P.dim = a->dim; P.groups = a->groups;
  P.x = a->x; P.x_sb = a->x_batch_stride; P.x_st = a->x_token_stride;
  P.dt = a->dt; P.dt_sb = a->dt_batch_stride; P.dt_st = a->dt_token_stride;
  P.A = a->A;
  P.B = a->B; P.b_sb = a->b_batch_stride; P.b_st = a->b_token_stride;
  P.C = a->C; P.c_sb = a->c_batch_stride; P.c_st = a->c_token_stride;
  P.D = a->D; P.d_is_f32 = a->d_is_f32; P.dt_bias = a->dt_bias; P.dt_bias_is_f32 = a->dt_bias_is_f32;
  P.state = a->state; P.y = a->y; P.y_sb = a->y_batch_stride; P.y_st = a->y_token_stride;
  P.stats = a->stats;
  return check(launch_s16_scan(P, (cudaStream_t)stream), "sq_s16_scan");
}

namespace {
int ste_params(const sq_sq3p25_args* a, SteParams& P, bool forward) {
  if (!a || !a->x || !a->dt || !a->A || !a->B || !a->C || !a->D || !a->dt_bias || !a->permutation)
    return fail(SQ_EINVAL, "sq3p25: null pointer argument");
  if (forward && (!a->lo || !a->hi || !a->q4 || !a->s8 || !a->s4 || !a->y))
    return fail(SQ_EINVAL, "sq3p25: null state or output");
  if (a->batch <= 0 || a->length <= 0 || a->heads <= 0 || a->dim <= 0 || a->groups <= 0 || a->heads % a->groups)
    return fail(SQ_EINVAL, "heads must be divisible by B/C groups");
  if (a->dim > 128) return fail(SQ_EINVAL, "sq3p25: dim must be at most 128");
  if (forward && (!aligned(a->lo, 8) || !aligned(a->hi, 8) || !aligned(a->q4, 16)))
    return fail(SQ_EINVAL, "sq3p25: state buffers must be 16-byte aligned");
  P = SteParams{};
  P.batch = a->batch; P.length = a->length; P.heads = a->heads; P.dim = a->dim; P.groups = a->groups;
  P.x = a->x; P.x_sb = a->x_batch_stride; P.x_st = a->x_token_stride;
  P.dt = a->dt; P.dt_sb = a->dt_batch_stride; P.dt_st = a->dt_token_stride;
  P.A = a->A;
  P.B = a->B; P.b_sb = a->b_batch_stride; P.b_st = a->b_token_stride;
  P.C = a->C; P.c_sb = a->c_batch_stride; P.c_st = a->c_token_stride;
  P.D = a->D; P.d_is_f32 = a->d_is_f32; P.dt_bias = a->dt_bias; P.dt_bias_is_f32 = a->dt_bias_is_f32;
  P.perm = a->permutation;
  P.lo = a->lo; P.hi = a->hi; P.q4 = a->q4; P.s8 = a->s8; P.s4 = a->s4;
  P.y = a->y; P.y_sb = a->y_batch_stride; P.y_st = a->y_token_stride;
  return SQ_OK;
}
}  // namespace

int sq_sq3p25_scan(const sq_sq3p25_args* a, void* stream) {
  SteParams P;
  if (int s = ste_params(a, P, true)) return s;
  return check(launch_sq3p25_scan(P, (cudaStream_t)stream), "sq_sq3p25_scan");
}

int64_t sq_ste_workspace(int batch, int length, int heads, int dim, int chunk) {
  return ste_workspace_bytes(batch, length, heads, dim, chunk);
}

int sq_ste_backward(const sq_sq3p25_args* a, int chunk, const uint16_t* dy, float* dx, float* ddt, float* db,
                    float* dc, void* workspace, int64_t workspace_bytes, void* stream) {
  SteParams P;
  if (int s = ste_params(a, P, false)) return s;
  if (!dy || !dx || !ddt || !db || !dc || !workspace) return fail(SQ_EINVAL, "ste_backward: null pointer argument");
  if (chunk < 1 || chunk > 256) return fail(SQ_EINVAL, "chunk_size must be an integer in [1,256]");
  const long long L = a->length, H = a->heads, Pd = a->dim, G = a->groups;
  if (a->x_token_stride != H * Pd || a->x_batch_stride != L * H * Pd || a->dt_token_stride != H ||
      a->dt_batch_stride != L * H || a->b_token_stride != G * 128 || a->b_batch_stride != L * G * 128 ||
      a->c_token_stride != G * 128 || a->c_batch_stride != L * G * 128)
    return fail(SQ_EINVAL, "ste_backward: inputs must be contiguous");
  const long long need = ste_workspace_bytes(a->batch, a->length, a->heads, a->dim, chunk);
  if (need < 0 || workspace_bytes < need || !aligned(workspace, 16))
    return fail(SQ_EINVAL, "ste_backward: workspace smaller than sq_ste_workspace() or not 16-byte aligned");
  P.dy = dy; P.dx = dx; P.ddt = ddt; P.db = db; P.dc = dc; P.chunk = chunk;
  return check(launch_ste_backward(P, workspace, (cudaStream_t)stream), "sq_ste_backward");
}

int sq_state_decode(int layout, int batch, int heads, int dim, int groups, const uint8_t* lo, const uint8_t* hi,
                    const uint8_t* q4, const uint8_t* latent, const uint16_t* s8, const uint16_t* s4,
                    const uint16_t* latent_scale, float* tiers, float* z, void* stream) {
  if (!lo || !hi || !q4 || !latent || !s8 || !s4 || !latent_scale || !tiers || !z)
    return fail(SQ_EINVAL, "state_decode: null pointer");
  return check(launch_decode_rows(layout, batch, heads, dim, groups, lo, hi, q4, latent, s8, s4, latent_scale,
                                  tiers, z, (cudaStream_t)stream), "sq_state_decode");
}

int sq_state_encode(int layout, int batch, int heads, int dim, int groups, int mode, const float* tiers,
                    const float* z, const uint16_t* latent_scale, uint8_t* lo, uint8_t* hi, uint8_t* q4,
                    uint8_t* latent, uint16_t* s8, uint16_t* s4, void* stream) {
  if (!lo || !hi || !q4 || !latent || !s8 || !s4 || !tiers || (mode == 0 && (!z || !latent_scale)))
    return fail(SQ_EINVAL, "state_encode: null pointer");
  return check(launch_encode_rows(layout, batch, heads, dim, groups, mode, tiers, z, latent_scale, lo, hi, q4,
                                  latent, s8, s4, (cudaStream_t)stream), "sq_state_encode");
}

int sq_fp4_decode(const uint8_t* codes, const uint8_t* block_scales, const float* global_scale, int rows, int cols,
                  uint16_t* out, int64_t ldo, void* stream) {
  if (!codes || !block_scales || !global_scale || !out) return fail(SQ_EINVAL, "fp4_decode: null pointer");
  if (!aligned(codes, 4) || !aligned(out, 16)) return fail(SQ_EINVAL, "fp4_decode: misaligned buffers");
  Fp4Weight w{codes, block_scales, global_scale, rows, cols};
  return check(launch_fp4_decode(w, out, ldo, (cudaStream_t)stream), "sq_fp4_decode");
}

int sq_fp4_validate(const uint8_t* codes, const uint8_t* block_scales, const float* global_scale, int rows, int cols,
                    void* stream) {
  if (!codes || !block_scales || !global_scale) return fail(SQ_EINVAL, "fp4_validate: null pointer");
  if (rows <= 0 || cols <= 0 || cols % 16) return fail(SQ_EINVAL, "fp4_validate: Invalid packet shape");
  if (!aligned(codes, 8)) return fail(SQ_EINVAL, "fp4_validate: codes must be 8-byte aligned");
  int* d_err = nullptr;
  if (int s = device_error_word(&d_err)) return s;
  int* flags = d_err + 1;                            // per-call flags, cleared on the stream
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(flags, 0, sizeof(int), st) != cudaSuccess) return cuda_fail("fp4_validate: clear flags");
  Fp4Weight w{codes, block_scales, global_scale, rows, cols};
  SQ_TRY(launch_fp4_validate(w, flags, st), "fp4_validate");
  int h = 0;
  if (cudaMemcpyAsync(&h, flags, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return cuda_fail("fp4_validate: read flags");
  if (h & 1) return fail(SQ_EINVAL, "Invalid stored scale");
  if (h & 2) return fail(SQ_EINVAL, "Nonzero code in a zero-scale group");
  if (h & 4) return fail(SQ_EINVAL, "Nonfinite decoded FP16 weights");   // ValueError, as the reference
  return SQ_OK;
}

int64_t sq_fp4_linear_workspace(int m, int n, int k) {
  // rows up to 256 run a kernel that needs no staging (k % 256 == 0 there)
  return (m <= 64 || (m <= kFusedMax && k % 256 == 0)) ? 0 : (int64_t)n * k * 2;
}

int sq_fp4_linear(const uint8_t* codes, const uint8_t* block_scales, const float* global_scale, int n, int k,
                  const uint16_t* x, int64_t ldx, int m, uint16_t* y, int64_t ldy, void* workspace,
                  int64_t workspace_bytes, void* stream) {
  if (!codes || !block_scales || !global_scale || !x || !y) return fail(SQ_EINVAL, "fp4_linear: null pointer");
  if (m <= 0 || n <= 0 || k <= 0 || k % 128) return fail(SQ_EINVAL, "fp4_linear: k must be a positive multiple of 128");
  if (!aligned(codes, 16) || !aligned(x, 16)) return fail(SQ_EINVAL, "fp4_linear: misaligned buffers");
  if (ldx < k || ldy < n) return fail(SQ_EINVAL, "fp4_linear: row strides must satisfy ldx >= k and ldy >= n");
  Fp4Weight w{codes, block_scales, global_scale, n, k};
  cudaStream_t st = (cudaStream_t)stream;
  int* d_err = nullptr;
  if (int s = device_error_word(&d_err)) return s;
  const bool tma_ok = k % 256 == 0 && aligned(block_scales, 16) && aligned(x, 16) && ldx % 8 == 0;
  if (m <= kSkinnyMax || (m <= 64 && !tma_ok)) {
    if (tma_ok) return check(launch_fp4_gemv_stream(w, nullptr, x, ldx, m, y, ldy, d_err, st), "fp4 gemv");
    return check(launch_fp4_gemv(w, x, ldx, m, y, ldy, st), "fp4 gemv");
  }
  if (m <= kFusedMax && tma_ok)
    return check(launch_fp4_mma_linear(w, x, ldx, m, y, ldy, d_err, st), "fp4 tensor-core linear");
  if (!workspace || workspace_bytes < sq_fp4_linear_workspace(m, n, k) || !aligned(workspace, 16))
    return fail(SQ_EINVAL, "fp4_linear: workspace too small");
  uint16_t* stg = (uint16_t*)workspace;
  SQ_TRY(launch_fp4_decode(w, stg, k, st), "fp4 decode");
  return check(launch_gemm_f16(x, ldx, stg, k, y, ldy, m, n, k, 0, nullptr, d_err, st), "tcgen05 gemm");
}

int sq_gemm_f16(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, uint16_t* c, int64_t ldc, int m,
                int n, int k, void* stream) {
  if (!a || !b || !c) return fail(SQ_EINVAL, "gemm: null pointer");
  int* d_err = nullptr;
  if (int s = device_error_word(&d_err)) return s;
  return check(launch_gemm_f16(a, lda, b, ldb, c, ldc, m, n, k, 0, nullptr, d_err, (cudaStream_t)stream),
               "tcgen05 gemm");
}

int sq_set_wait_limit_ns(uint64_t ns) {
  return check(set_gemv_wait_limit_ns((unsigned long long)ns), "set_wait_limit");
}

int sq_device_check(void* stream) {
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return cuda_fail("stream synchronize");
  int* d_err = nullptr;
  if (int s = device_error_word(&d_err)) return s;
  int h = 0;
  if (cudaMemcpy(&h, d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return cuda_fail("read error word");
  if (h) {
    if (cudaMemset(d_err, 0, sizeof(int)) != cudaSuccess) return cuda_fail("clear error word");
    return fail(SQ_ETIMEOUT, "device: a bounded wait of sq_fp4_linear / sq_gemm_f16 expired (code " +
                                 std::to_string(h) + ")");
  }
  return SQ_OK;
}

// ---------------------------------------------------------------- model runtime

int sq_model_create(const sq_model_config* cfg, sq_model** out) {
  if (!cfg || !out) return fail(SQ_EINVAL, "model_create: null pointer");
  if (cfg->n_layer <= 0 || cfg->vocab < 16 || cfg->vocab % 16 || !(cfg->eps > 0.f))
    return fail(SQ_EINVAL, "model_create: invalid config");
  sq_model* m = new sq_model();
  m->cfg = *cfg;
  m->layers.resize(cfg->n_layer);
  std::memset(m->layers.data(), 0, sizeof(sq_layer_desc) * cfg->n_layer);
  m->adapters.assign(cfg->n_layer, AdapterPtrs{});
  m->in_maps.assign(cfg->n_layer, Fp4Maps{});
  m->out_maps.assign(cfg->n_layer, Fp4Maps{});
  m->states.resize(cfg->n_layer);
  if (cudaMalloc(&m->d_err, sizeof(int)) != cudaSuccess) { delete m; return cuda_fail("cudaMalloc"); }
  cudaMemset(m->d_err, 0, sizeof(int));
  // kernel attributes are set here, so later launches (and graph captures) never change them
  if (prepare_scan_kernels() != kOk || prepare_fp4_kernels() != kOk || prepare_gemm_kernel() != kOk ||
      prepare_layer_kernels() != kOk || prepare_fp4_mma_kernel() != kOk) {
    cudaFree(m->d_err);
    delete m;
    return cuda_fail("kernel attribute setup");
  }
  *out = m;
  return SQ_OK;
}

int sq_model_destroy(sq_model* m) {
  if (!m) return SQ_OK;
  free_ws(m);
  void* dec[] = {m->d_dlayers, m->d_dmaps, m->d_dbuf};
  for (void* p : dec)
    if (p) cudaFree(p);
  if (m->d_err) cudaFree(m->d_err);
  for (cudaEvent_t e : m->gemm_events) cudaEventDestroy(e);
  delete m;
  return SQ_OK;
}

static bool fp4_ok(const sq_fp4_matrix& w, int rows, int cols) {
  return w.codes && w.block_scales && w.global_scale && w.rows == rows && w.cols == cols && aligned(w.codes, 16);
}

int sq_model_set_layer(sq_model* m, int layer, const sq_layer_desc* d) {
  if (!m || !d || layer < 0 || layer >= m->cfg.n_layer) return fail(SQ_EINVAL, "set_layer: bad layer");
  if (!fp4_ok(d->in_proj, kZx, kDModel) || !fp4_ok(d->out_proj, kDModel, kDInner))
    return fail(SQ_EINVAL, "set_layer: projection geometry differs ([18560,4096] / [4096,8192])");
  if (d->layout < 0 || d->layout > 6) return fail(SQ_EINVAL, "set_layer: unknown layout");
  const void* req[] = {d->norm_weight, d->conv_weight, d->conv_bias, d->A, d->D, d->dt_bias, d->gated_norm_weight,
                       d->permutation, d->basis, d->latent_scale, d->predictor};
  for (const void* p : req)
    if (!p) return fail(SQ_EINVAL, "set_layer: null pointer");
  if (!aligned(d->permutation, 16) || !aligned(d->basis, 16) || !aligned(d->predictor, 16))
    return fail(SQ_EINVAL, "set_layer: permutation / basis / predictor must be 16-byte aligned");
  m->layers[layer] = *d;
  m->dec_dirty = true;
  if (!make_fp4_maps(fw(d->in_proj), &m->in_maps[layer]) || !make_fp4_maps(fw(d->out_proj), &m->out_maps[layer]))
    return fail(SQ_EINVAL, "set_layer: projection rows must be 16-byte aligned for the TMA streams");
  return SQ_OK;
}

int sq_model_set_globals(sq_model* m, const sq_fp4_matrix* e, const sq_fp4_matrix* h, const uint16_t* nf) {
  if (!m || !e || !h || !nf) return fail(SQ_EINVAL, "set_globals: null pointer");
  if (!fp4_ok(*e, m->cfg.vocab, kDModel) || !fp4_ok(*h, m->cfg.vocab, kDModel))
    return fail(SQ_EINVAL, "set_globals: embedding / lm_head must be [vocab,4096]");
  m->embed = *e; m->head = *h; m->norm_f = nf;
  m->dec_dirty = true;
  if (!make_fp4_maps(fw(*h), &m->head_maps)) return fail(SQ_EINVAL, "set_globals: lm_head rows must be 16-byte aligned");
  return SQ_OK;
}

int sq_model_set_adapter(sq_model* m, int layer, const uint16_t* V, const uint16_t* g, const uint16_t* w,
                         const uint16_t* b, int hard) {
  if (!m || layer < 0 || layer >= m->cfg.n_layer) return fail(SQ_EINVAL, "set_adapter: bad layer");
  if (V && (!g || !w || !b)) return fail(SQ_EINVAL, "set_adapter: null pointer");
  m->adapters[layer] = AdapterPtrs{V, g, w, b, hard};
  m->dec_dirty = true;
  return SQ_OK;
}

int sq_model_bind_state(sq_model* m, int layer, int batch, uint8_t* lo, uint8_t* hi, uint8_t* q4, uint8_t* latent,
                        uint16_t* s8, uint16_t* s4, uint16_t* ring) {
  if (!m || layer < 0 || layer >= m->cfg.n_layer || batch <= 0) return fail(SQ_EINVAL, "bind_state: bad layer/batch");
  const void* p[] = {lo, hi, q4, latent, s8, s4, ring};
  for (const void* q : p)
    if (!q || !aligned(q, 16)) return fail(SQ_EINVAL, "bind_state: null or misaligned (16 B) buffer");
  sq_model::St& s = m->states[layer];
  s.batch = batch; s.lo = lo; s.hi = hi; s.q4 = q4; s.latent = latent; s.s8 = s8; s.s4 = s4; s.ring = ring;
  m->dec_dirty = true;
  return SQ_OK;
}

int sq_model_reserve(sq_model* m, int max_tokens) {
  if (!m || max_tokens <= 0) return fail(SQ_EINVAL, "reserve: bad size");
  if (max_tokens <= m->max_tokens) return SQ_OK;
  free_ws(m);
  const size_t T = (size_t)max_tokens;
  const int nt = gemm_num_ntiles(m->cfg.vocab);
  size_t stage = (size_t)kZx * kDModel;
  stage = std::max(stage, (size_t)kDModel * kDInner);
  stage = std::max(stage, (size_t)std::min(m->cfg.vocab, kLmChunk) * kDModel);
  struct A { void** p; size_t bytes; } allocs[] = {
      {(void**)&m->h, T * kDModel * 2}, {(void**)&m->res, T * kDModel * 2}, {(void**)&m->hn, T * kDModel * 2},
      {(void**)&m->zx, T * kZx * 2}, {(void**)&m->xbc, T * kXbc * 2}, {(void**)&m->y, T * kDInner * 2},
      {(void**)&m->yn, T * kDInner * 2}, {(void**)&m->stage, stage * 2},
      {(void**)&m->logits, (size_t)64 * m->cfg.vocab * 2},
      {(void**)&m->partials, std::max(T * nt * sizeof(float2), (size_t)argmax_workspace_bytes(64, m->cfg.vocab))},
      {(void**)&m->tlogit, T * sizeof(float)},
      {(void**)&m->prep, (size_t)scan_prep_bytes_any_layout(1, max_tokens, kHeads, kGroups)}};
  for (auto& a : allocs) {
    if (cudaMalloc(a.p, a.bytes) != cudaSuccess) {
      cudaGetLastError();
      free_ws(m);
      return fail(SQ_ENOMEM, "reserve: cudaMalloc failed");
    }
  }
  m->stage_elems = stage;
  m->max_tokens = max_tokens;
  return SQ_OK;
}

namespace {
struct Busy {
  sq_model* m; bool ok;
  explicit Busy(sq_model* mm) : m(mm) { int z = 0; ok = m->busy.compare_exchange_strong(z, 1); }
  ~Busy() { if (ok) m->busy.store(0); }
};
}  // namespace

namespace {
// One mixer layer, PredictorState._forward (fp4_zero_predictor_codec_v1.py:314-367): u is the
// Block's normed input [batch*tokens, 4096]; the result goes to `out` [batch*tokens, 4096].
// in_proj -> causal conv -> SQ3.25 scan -> Resurface (router on u) -> gated RMSNorm -> out_proj.
// Workspaces zx / xbc / y / yn / prep / stage are the model's.
int mixer_forward(sq_model* m, int l, const uint16_t* u, int batch, int tokens, int pos0, uint16_t* out,
                  cudaStream_t st) {
  const sq_layer_desc& L = m->layers[l];
  const sq_model::St& S = m->states[l];
  const int M = batch * tokens;
  const bool step = pos0 > 0 && tokens == 1;
  int s = linear(m, L.in_proj, &m->in_maps[l], u, kDModel, M, m->zx, kZx, !step || m->exact_skinny, st, true);
  if (s != SQ_OK) return s;
  ScanParams P{};
  P.batch = batch; P.length = tokens; P.heads = kHeads; P.dim = kHeadDim; P.groups = kGroups; P.layout = L.layout;
  P.dt = m->zx + 2 * kDInner + 2 * 1024; P.dt_sb = (long long)tokens * kZx; P.dt_st = kZx;
  P.A = L.A; P.D = L.D; P.d_is_f32 = 0; P.dt_bias = L.dt_bias; P.dt_bias_is_f32 = 0;
  P.perm = L.permutation; P.basis = L.basis; P.latent_scale = L.latent_scale; P.predictor = L.predictor;
  P.lo = S.lo; P.hi = S.hi; P.q4 = S.q4; P.latent = S.latent; P.s8 = S.s8; P.s4 = S.s4;
  P.y = m->y; P.y_sb = (long long)tokens * kDInner; P.y_st = kDInner;
  if (step || pos0 == 0) {
    // conv fused into the scan: step numerics for a one-token step, conv1d numerics
    // for a prefill from a reset state
    const uint16_t* raw = m->zx + kDInner;
    P.x = raw; P.B = raw + kDInner; P.C = raw + kDInner + 1024;
    P.x_sb = P.b_sb = P.c_sb = (long long)tokens * kZx; P.x_st = P.b_st = P.c_st = kZx;
    P.conv_mode = step ? 2 : 1;
    P.conv_w = L.conv_weight; P.conv_b = L.conv_bias; P.conv_cache = S.ring; P.conv_pos = pos0;
    P.conv_cache_sb = 4LL * kXbc;
  } else {
    SQ_TRY(launch_conv_prefill(m->zx + kDInner, (long long)tokens * kZx, kZx, batch, tokens, kXbc, L.conv_weight,
                               L.conv_bias, S.ring, 4LL * kXbc, pos0, m->xbc, (long long)tokens * kXbc, kXbc, st),
           "conv prefill");
    P.x = m->xbc; P.B = m->xbc + kDInner; P.C = m->xbc + kDInner + 1024;
    P.x_sb = P.b_sb = P.c_sb = (long long)tokens * kXbc; P.x_st = P.b_st = P.c_st = kXbc;
  }
  scan_prep_bind(P, m->prep);
  SQ_TRY(launch_scan(P, st), "ssu scan");
  const AdapterPtrs& ad = m->adapters[l];
  SQ_TRY(launch_resurface_gatednorm(m->y, m->zx, kZx, u, kDModel, ad.V ? &ad : nullptr, L.gated_norm_weight,
                                    m->cfg.eps, m->yn, M, st), "resurface + gated norm");
  return linear(m, L.out_proj, &m->out_maps[l], m->yn, kDInner, M, out, kDModel, !step || m->exact_skinny, st);
}
}  // namespace

int sq_model_mixer_forward(sq_model* m, int layer, const uint16_t* u, int batch, int tokens, int pos0, uint16_t* out,
                           void* stream) {
  if (!m || !u || !out || batch <= 0 || tokens <= 0 || pos0 < 0 || layer < 0 || layer >= (m ? m->cfg.n_layer : 0))
    return fail(SQ_EINVAL, "mixer_forward: bad args");
  Busy busy(m);
  if (!busy.ok) return fail(SQ_ESTATE, "mixer_forward: concurrent/reentrant use of one model context");
  if (batch * tokens > m->max_tokens) return fail(SQ_EINVAL, "mixer_forward: batch*tokens exceeds reserved workspace");
  if (!m->layers[layer].in_proj.codes) return fail(SQ_ESTATE, "mixer_forward: layer weights not set");
  if (m->states[layer].batch != batch) return fail(SQ_ESTATE, "mixer_forward: state batch differs from the call");
  if (!aligned(u, 16) || !aligned(out, 16)) return fail(SQ_EINVAL, "mixer_forward: u / out must be 16-byte aligned");
  return mixer_forward(m, layer, u, batch, tokens, pos0, out, (cudaStream_t)stream);
}

int sq_model_forward(sq_model* m, const int64_t* ids, int batch, int tokens, int pos0, uint16_t* hidden_out,
                     void* stream) {
  if (!m || !ids || !hidden_out || batch <= 0 || tokens <= 0 || pos0 < 0) return fail(SQ_EINVAL, "forward: bad args");
  Busy busy(m);
  if (!busy.ok) return fail(SQ_ESTATE, "forward: concurrent/reentrant use of one model context");
  const int M = batch * tokens;
  if (M > m->max_tokens) return fail(SQ_EINVAL, "forward: batch*tokens exceeds reserved workspace");
  if (!m->embed.codes || !m->norm_f) return fail(SQ_ESTATE, "forward: globals not set");
  cudaStream_t st = (cudaStream_t)stream;
  SQ_TRY(launch_fp4_embed(fw(m->embed), (const long long*)ids, M, m->h, m->d_err, st), "embedding");
  for (int l = 0; l < m->cfg.n_layer; ++l) {
    const sq_layer_desc& L = m->layers[l];
    if (!L.in_proj.codes) return fail(SQ_ESTATE, "forward: layer weights not set");
    if (m->states[l].batch != batch) return fail(SQ_ESTATE, "forward: state batch differs from the call (reset required)");
    SQ_TRY(launch_add_rmsnorm(m->h, m->res, l > 0, L.norm_weight, m->cfg.eps, m->hn, M, kDModel, st), "add_rmsnorm");
    if (int s = mixer_forward(m, l, m->hn, batch, tokens, pos0, m->h, st)) return s;
    if (m->capture && M <= m->capture_rows &&
        cudaMemcpyAsync(m->capture + (size_t)l * m->capture_rows * kDModel, m->h, (size_t)M * kDModel * 2,
                        cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return cuda_fail("forward: layer capture copy");
  }
  SQ_TRY(launch_add_rmsnorm(m->h, m->res, 1, m->norm_f, m->cfg.eps, hidden_out, M, kDModel, st), "norm_f");
  return SQ_OK;
}

int sq_model_score(sq_model* m, const uint16_t* hidden, int rows, const int64_t* targets, float* nll, void* stream) {
  if (!m || !hidden || !targets || !nll || rows <= 0) return fail(SQ_EINVAL, "score: bad args");
  Busy busy(m);
  if (!busy.ok) return fail(SQ_ESTATE, "score: concurrent/reentrant use of one model context");
  if (rows > m->max_tokens) return fail(SQ_EINVAL, "score: rows exceed reserved workspace");
  cudaStream_t st = (cudaStream_t)stream;
  const int V = m->cfg.vocab;
  const int nt = gemm_num_ntiles(V);
  for (int n0 = 0; n0 < V; n0 += kLmChunk) {
    const int nc = std::min(kLmChunk, V - n0);
    Fp4Weight w = fw(m->head);
    w.codes += (size_t)n0 * (kDModel / 2);
    w.scales += (size_t)n0 * (kDModel / 16);
    w.rows = nc;
    SQ_TRY(launch_fp4_decode(w, m->stage, kDModel, st), "lm_head decode");
    GemmCE ce{(const long long*)targets, m->partials, m->tlogit, n0, nt};
    SQ_TRY(launch_gemm_f16(hidden, kDModel, m->stage, kDModel, nullptr, 0, rows, nc, kDModel, 1, &ce, m->d_err, st),
           "lm_head gemm + ce");
  }
  return check(launch_ce_finalize(m->partials, nt, m->tlogit, rows, nll, st), "ce finalize");
}

int sq_model_greedy(sq_model* m, const uint16_t* hidden, int rows, uint16_t* logits_out, int64_t* tokens_out,
                    void* stream) {
  if (!m || !hidden || !tokens_out || rows <= 0 || rows > 64) return fail(SQ_EINVAL, "greedy: rows must be 1..64");
  Busy busy(m);
  if (!busy.ok) return fail(SQ_ESTATE, "greedy: concurrent/reentrant use of one model context");
  if (!m->logits) return fail(SQ_ESTATE, "greedy: reserve() first");
  cudaStream_t st = (cudaStream_t)stream;
  uint16_t* lg = logits_out ? logits_out : m->logits;
  if (rows <= kSkinnyMax)
    SQ_TRY(launch_fp4_gemv_stream(fw(m->head), &m->head_maps, hidden, kDModel, rows, lg, m->cfg.vocab, m->d_err, st,
                                  m->exact_skinny),
           "lm_head gemv");
  else
    SQ_TRY(launch_fp4_mma_linear(fw(m->head), hidden, kDModel, rows, lg, m->cfg.vocab, m->d_err, st,
                                 m->exact_skinny),
           "lm_head tensor-core linear");
  return check(launch_argmax(lg, rows, m->cfg.vocab, m->cfg.vocab, (long long*)tokens_out, m->partials, st),
               "argmax");
}

namespace {
constexpr size_t kDecH = 0, kDecRes = kDecH + 4096 * 2, kDecZx = kDecRes + 2 * 4096 * 2, kDecY = kDecZx + kZx * 2,
                 kDecPv = kDecY + kDInner * 2, kDecPi = kDecPv + 1024 * 4, kDecSync = kDecPi + 1024 * 4,
                 kDecBytes = kDecSync + 256;

// Device copies of everything the persistent decode kernel reads through pointers.
int decode_setup(sq_model* m) {
  const int L = m->cfg.n_layer;
  if (!m->d_dlayers) {
    if (cudaMalloc(&m->d_dlayers, sizeof(DecLayer) * L) != cudaSuccess ||
        cudaMalloc(&m->d_dmaps, sizeof(CUtensorMap) * ((2 * L + 1) * 2 + 2 * L)) != cudaSuccess ||
        cudaMalloc(&m->d_dbuf, kDecBytes) != cudaSuccess)
      return fail(SQ_ENOMEM, "decode: cudaMalloc failed");
    if (cudaMemset(m->d_dbuf, 0, kDecBytes) != cudaSuccess) return cuda_fail("decode: cudaMemset");
  }
  std::vector<DecLayer> dl(L);
  std::vector<CUtensorMap> maps((2 * L + 1) * 2 + 2 * L);
  CUtensorMap* aux = maps.data() + (2 * L + 1) * 2;
  for (int l = 0; l < L; ++l) {
    const sq_layer_desc& d = m->layers[l];
    const sq_model::St& st = m->states[l];
    const AdapterPtrs& ad = m->adapters[l];
    if (!d.in_proj.codes) return fail(SQ_ESTATE, "decode: layer weights not set");
    if (st.batch != 1) return fail(SQ_ESTATE, "decode: the persistent kernel decodes batch 1 (bind batch-1 states)");
    // every tensor the kernel bulk-copies must start on a 16-byte boundary
    const void* a16[] = {d.conv_weight, d.conv_bias, d.norm_weight, d.gated_norm_weight, d.latent_scale, d.D,
                         d.dt_bias, d.A, ad.w, ad.V, ad.g};
    for (const void* q : a16)
      if (q && !aligned(q, 16)) return fail(SQ_EINVAL, "decode: layer tensors must be 16-byte aligned");
    if (!m->in_maps[l].valid || !m->out_maps[l].valid || m->in_maps[l].kc != 1024 || m->out_maps[l].kc != 1024)
      return fail(SQ_ESTATE, "decode: projection stream maps missing");
    DecLayer& x = dl[l];
    std::memset(&x, 0, sizeof(x));
    x.norm_w = d.norm_weight; x.conv_w = d.conv_weight; x.conv_b = d.conv_bias; x.A = d.A; x.D = d.D;
    x.dt_bias = d.dt_bias; x.gnorm_w = d.gated_norm_weight;
    x.in_g = d.in_proj.global_scale; x.out_g = d.out_proj.global_scale;
    x.perm = d.permutation; x.basis = d.basis; x.latent_scale = d.latent_scale; x.predictor = d.predictor;
    x.ad_V = ad.V; x.ad_g = ad.g; x.ad_w = ad.w; x.ad_b = ad.b; x.hard = ad.hard;
    x.lo = st.lo; x.hi = st.hi; x.q4 = st.q4; x.latent = st.latent; x.s8 = st.s8; x.s4 = st.s4; x.ring = st.ring;
    x.layout = d.layout;
    maps[(2 * l) * 2 + 0] = m->in_maps[l].codes; maps[(2 * l) * 2 + 1] = m->in_maps[l].scales;
    maps[(2 * l + 1) * 2 + 0] = m->out_maps[l].codes; maps[(2 * l + 1) * 2 + 1] = m->out_maps[l].scales;
    std::memset(aux + 2 * l, 0, 2 * sizeof(CUtensorMap));
    if ((ad.V && !encode_f16_sw128_map(aux + 2 * l, ad.V, 128, 128, 128)) ||
        !encode_f16_sw128_map(aux + 2 * l + 1, d.gated_norm_weight, 128, 64, 128))
      return fail(SQ_ECUDA, "decode: tensor map encoding failed");
  }
  if (!m->head.codes || !m->head_maps.valid || m->head_maps.kc != 1024) return fail(SQ_ESTATE, "decode: lm_head not set");
  if (!aligned(m->norm_f, 16) || !aligned(m->embed.codes, 4)) return fail(SQ_EINVAL, "decode: norm_f must be 16-byte aligned");
  maps[(2 * L) * 2 + 0] = m->head_maps.codes; maps[(2 * L) * 2 + 1] = m->head_maps.scales;
  if (cudaMemcpy(m->d_dlayers, dl.data(), sizeof(DecLayer) * L, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(m->d_dmaps, maps.data(), sizeof(CUtensorMap) * maps.size(), cudaMemcpyHostToDevice) != cudaSuccess)
    return cuda_fail("decode: table upload");
  if (!m->dec_grid) m->dec_grid = decode_grid();
  if (m->dec_grid < 128) return fail(SQ_ECUDA, "decode: cooperative launch of one CTA per SM (>= 128 SMs) unavailable");
  m->dec_dirty = false;
  return SQ_OK;
}
}  // namespace

int sq_model_decode(sq_model* m, int64_t* tokens, int pos, int steps, int64_t* out_tokens, void* stream) {
  if (!m || !tokens || steps <= 0 || pos <= 0) return fail(SQ_EINVAL, "decode: bad arguments (pos > 0: prefill first)");
  Busy busy(m);
  if (!busy.ok) return fail(SQ_ESTATE, "decode: concurrent/reentrant use of one model context");
  if (!m->logits || !m->norm_f) return fail(SQ_ESTATE, "decode: reserve() and set_globals() first");
  if (m->dec_dirty) {
    const int s = decode_setup(m);
    if (s != SQ_OK) return s;
  }
  DecodeParams P{};
  P.layers = m->d_dlayers; P.maps = m->d_dmaps;
  P.aux_maps = m->d_dmaps + (2 * m->cfg.n_layer + 1) * 2;
  P.head_codes = m->head.codes; P.head_scales = m->head.block_scales;
  P.emb_codes = m->embed.codes; P.emb_scales = m->embed.block_scales; P.emb_g = m->embed.global_scale;
  P.head_g = m->head.global_scale; P.norm_f = m->norm_f;
  P.h = reinterpret_cast<uint16_t*>(m->d_dbuf + kDecH); P.res = reinterpret_cast<uint16_t*>(m->d_dbuf + kDecRes);
  P.zx = reinterpret_cast<uint16_t*>(m->d_dbuf + kDecZx); P.y = reinterpret_cast<uint16_t*>(m->d_dbuf + kDecY);
  P.logits = m->logits;
  P.part_v = reinterpret_cast<float*>(m->d_dbuf + kDecPv); P.part_i = reinterpret_cast<int*>(m->d_dbuf + kDecPi);
  P.sync = reinterpret_cast<DecodeSync*>(m->d_dbuf + kDecSync);
  P.err = m->d_err; P.tok = (long long*)tokens; P.out_tokens = (long long*)out_tokens;
  P.n_layer = m->cfg.n_layer; P.vocab = m->cfg.vocab; P.eps = m->cfg.eps;
  P.exact = m->exact_skinny ? 1 : 0;
  // fresh barrier words (an aborted launch leaves its count and abort flag behind)
  if (cudaMemsetAsync(P.sync, 0, sizeof(DecodeSync), (cudaStream_t)stream) != cudaSuccess)
    return cuda_fail("decode: barrier reset");
  P.pos = pos;
  P.steps = steps;
  SQ_TRY(launch_decode_step(P, m->dec_grid, (cudaStream_t)stream), "persistent decode");
  return SQ_OK;
}

int sq_model_set_capture(sq_model* m, uint16_t* out, int64_t rows) {
  if (!m || (out && rows <= 0)) return fail(SQ_EINVAL, "set_capture: bad arguments");
  if (out && !aligned(out, 16)) return fail(SQ_EINVAL, "set_capture: buffer must be 16-byte aligned");
  m->capture = out;
  m->capture_rows = out ? rows : 0;
  return SQ_OK;
}

int sq_model_time_gemm(sq_model* m, int enable) {
  if (!m) return fail(SQ_EINVAL, "time_gemm: null model");
  m->gemm_timing = enable != 0;
  m->gemm_events_used = 0;
  return SQ_OK;
}

int sq_model_gemm_time(sq_model* m, double* seconds, int64_t* launches) {
  if (!m || !seconds || !launches) return fail(SQ_EINVAL, "gemm_time: null argument");
  double total = 0.0;
  for (size_t i = 0; i + 1 < m->gemm_events_used; i += 2) {
    if (cudaEventSynchronize(m->gemm_events[i + 1]) != cudaSuccess) return cuda_fail("gemm_time: event synchronize");
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, m->gemm_events[i], m->gemm_events[i + 1]) != cudaSuccess)
      return cuda_fail("gemm_time: elapsed time");
    total += ms * 1e-3;
  }
  *seconds = total;
  *launches = (int64_t)(m->gemm_events_used / 2);
  m->gemm_events_used = 0;
  return SQ_OK;
}

int sq_model_set_exact_skinny(sq_model* m, int exact) {
  if (!m) return fail(SQ_EINVAL, "set_exact_skinny: null model");
  m->exact_skinny = exact != 0;
  return SQ_OK;
}

int sq_model_check(sq_model* m, void* stream) {
  if (!m) return fail(SQ_EINVAL, "check: null model");
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return cuda_fail("stream synchronize");
  int h = 0;
  if (cudaMemcpy(&h, m->d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return cuda_fail("read error word");
  if (h) {
    cudaMemset(m->d_err, 0, sizeof(int));
    if (h & (int)kDevBadArgs) return fail(SQ_EINVAL, "device: token id outside the vocabulary");
    return fail(SQ_ETIMEOUT, "device: a bounded wait expired (code " + std::to_string(h) + ")");
  }
  return SQ_OK;
}

}  // extern "C"
