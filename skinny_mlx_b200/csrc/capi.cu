// C-ABI entry points: host-side validation, then stream-ordered kernel launches.
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/skinny_b200.h"
#include "qmm_layout.cuh"

namespace skinny {
int device_sm_count(int dev);
cudaError_t qmm_tc_launch(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M, int N,
                          int K, void* ws, int C, cudaStream_t stream, bool pdl);
cudaError_t qmm_tc_launch_grouped(int n, const void* const* x, const int* ldx, const void* const* w_tc,
                                  void* const* out, const int* ldo, const int* N, const int* K, int M,
                                  void* ws, cudaStream_t stream, bool pdl);
cudaError_t qmm_repack_launch(const uint32_t* w, const uint16_t* s, const uint16_t* b, void* w_tc,
                              int N, int K, cudaStream_t stream);
cudaError_t qmm_simt_launch(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M,
                            int N, int K, cudaStream_t stream);
bool qmm_noalloc_fits(int N, int K);
size_t spec_accept_ws_bytes();
cudaError_t gdn_recurrent_launch(const void* q, const void* k, const void* v, const float* g,
                                 const float* beta, float* state, void* y, float* ckpt, int T, int Hv,
                                 int Hk, cudaStream_t stream);
struct GdnRollbackParams;
cudaError_t gdn_rollback_call(int n_layers, float* const* state, const float* const* ckpt,
                             void* const* conv, const void* const* conv_full, long long state_elems,
                             int keep, int fed, int W, int C, cudaStream_t stream);
bool spec_accept_fits(int rows, int V);
cudaError_t spec_accept_launch(const void* logits, int ld, int rows, int V, const int32_t* draft,
                               int32_t* result, int32_t* pred, void* ws, cudaStream_t stream);
cudaError_t qmm_tc_launch_noalloc(const void* x, int ldx, const void* w_tc, void* out, int ldo,
                                  int M, int N, int K, cudaStream_t stream);
}  // namespace skinny

namespace {
thread_local int g_last_cuda = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return SKINNY_OK;
  g_last_cuda = static_cast<int>(e);
  return SKINNY_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return dev;
}

int ctas_for(int N, int K) {
  const skinny::QmmShape sh = skinny::qmm_shape(N, K);
  long long C = skinny::device_sm_count(current_device());
  if (C > sh.U) C = sh.U;
  return static_cast<int>(C);
}

int check_qmm_shape(int N, int K) {
  if (N < 1 || K < skinny::kGroup) return SKINNY_ERR_SHAPE;
  if (N > skinny::kMaxTiles * skinny::kTileRows) return SKINNY_ERR_SHAPE;
  if (K % skinny::kGroup != 0) return SKINNY_ERR_SHAPE;
  return SKINNY_OK;
}
}  // namespace

extern "C" {

int skinny_version(void) { return 100; }

const char* skinny_strerror(int status) {
  switch (status) {
    case SKINNY_OK: return "ok";
    case SKINNY_ERR_INVALID_ARG: return "invalid argument (null pointer or negative size)";
    case SKINNY_ERR_SHAPE:
      return "unsupported shape (K must be a positive multiple of 64 up to 131072, N >= 1; grouped: "
             "at most 16384 row tiles and 2048 input groups in total)";
    case SKINNY_ERR_TOKENS: return "token count outside [1, 16]";
    case SKINNY_ERR_ALIGNMENT: return "pointer or leading dimension not 16-byte aligned";
    case SKINNY_ERR_WORKSPACE: return "workspace missing or smaller than required";
    case SKINNY_ERR_CUDA: return "CUDA runtime call failed";
    case SKINNY_ERR_DEVICE: return "kernel recorded an error in the workspace";
    case SKINNY_ERR_UNSUPPORTED: return "unsupported device or option";
    case SKINNY_ERR_SCRATCH_LIMIT:
      return "shape exceeds the static scratch of skinny_qmm_w4g64_noalloc (N <= 262144 rows, "
             "K <= 32768 columns)";
    default: return "unknown status";
  }
}

int skinny_last_cuda_error(void) { return g_last_cuda; }

size_t skinny_repack_bytes(int N, int K) {
  if (check_qmm_shape(N, K) != SKINNY_OK) return 0;
  const skinny::QmmShape sh = skinny::qmm_shape(N, K);
  return static_cast<size_t>(sh.U) * skinny::kUnitWBytes;
}

int skinny_repack_w4g64(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                        void* w_tc, int N, int K, void* stream) {
  if (!w || !scales || !biases || !w_tc) return SKINNY_ERR_INVALID_ARG;
  const int st = check_qmm_shape(N, K);
  if (st != SKINNY_OK) return st;
  if (!aligned16(w_tc)) return SKINNY_ERR_ALIGNMENT;
  return cuda_status(skinny::qmm_repack_launch(w, scales, biases, w_tc, N, K,
                                               static_cast<cudaStream_t>(stream)));
}

size_t skinny_qmm_workspace_bytes(int N, int K) {
  if (check_qmm_shape(N, K) != SKINNY_OK) return 0;
  return skinny::ws_layout(skinny::device_sm_count(current_device())).total;
}

int skinny_qmm_w4g64(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M, int N,
                     int K, void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !w_tc || !out) return SKINNY_ERR_INVALID_ARG;
  int st = check_qmm_shape(N, K);
  if (st != SKINNY_OK) return st;
  if (M < 1 || M > skinny::kMaxTokens) return SKINNY_ERR_TOKENS;
  if (ldx < K || ldo < N) return SKINNY_ERR_INVALID_ARG;
  if (!aligned16(x) || (ldx % 8) != 0 || !aligned16(w_tc)) return SKINNY_ERR_ALIGNMENT;
  if (K / skinny::kGroup > skinny::kMaxXGroups) return SKINNY_ERR_SHAPE;
  const int C = ctas_for(N, K);
  const skinny::WsLayout wl = skinny::ws_layout(skinny::device_sm_count(current_device()));
  if (!workspace || workspace_bytes < wl.total || !aligned16(workspace)) return SKINNY_ERR_WORKSPACE;
  return cuda_status(skinny::qmm_tc_launch(x, ldx, w_tc, out, ldo, M, N, K, workspace, C,
                                           static_cast<cudaStream_t>(stream), true));
}

int skinny_qmm_w4g64_grouped(int n, const void* const* x, const int* ldx, const void* const* w_tc,
                             void* const* out, const int* ldo, const int* N, const int* K, int M,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (n < 1 || n > SKINNY_QMM_MAX_GROUP || !x || !ldx || !w_tc || !out || !ldo || !N || !K)
    return SKINNY_ERR_INVALID_ARG;
  if (M < 1 || M > skinny::kMaxTokens) return SKINNY_ERR_TOKENS;
  long long tiles = 0;
  int distinct = 0;
  long long xgroups = 0;
  for (int i = 0; i < n; ++i) {
    if (!x[i] || !w_tc[i] || !out[i]) return SKINNY_ERR_INVALID_ARG;
    const int st = check_qmm_shape(N[i], K[i]);
    if (st != SKINNY_OK) return st;
    if (ldx[i] < K[i] || ldo[i] < N[i]) return SKINNY_ERR_INVALID_ARG;
    if (!aligned16(x[i]) || (ldx[i] % 8) != 0 || !aligned16(w_tc[i])) return SKINNY_ERR_ALIGNMENT;
    tiles += skinny::qmm_shape(N[i], K[i]).T;
    bool seen = false;
    for (int q = 0; q < i; ++q)
      if (x[q] == x[i] && K[q] == K[i] && ldx[q] == ldx[i]) seen = true;
    if (!seen) {
      ++distinct;
      xgroups += K[i] / skinny::kGroup;
    }
  }
  if (tiles > skinny::kMaxTiles || distinct > SKINNY_QMM_MAX_GROUP_INPUTS ||
      xgroups > skinny::kMaxXGroups)
    return SKINNY_ERR_SHAPE;
  const skinny::WsLayout wl = skinny::ws_layout(skinny::device_sm_count(current_device()));
  if (!workspace || workspace_bytes < wl.total || !aligned16(workspace)) return SKINNY_ERR_WORKSPACE;
  return cuda_status(skinny::qmm_tc_launch_grouped(n, x, ldx, w_tc, out, ldo, N, K, M, workspace,
                                                   static_cast<cudaStream_t>(stream), true));
}

int skinny_qmm_w4g64_simt(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M,
                          int N, int K, void* stream) {
  if (!x || !w_tc || !out) return SKINNY_ERR_INVALID_ARG;
  int st = check_qmm_shape(N, K);
  if (st != SKINNY_OK) return st;
  if (M < 1 || M > skinny::kMaxTokens) return SKINNY_ERR_TOKENS;
  if (ldx < K || ldo < N) return SKINNY_ERR_INVALID_ARG;
  return cuda_status(skinny::qmm_simt_launch(x, ldx, w_tc, out, ldo, M, N, K,
                                             static_cast<cudaStream_t>(stream)));
}

int skinny_qmm_w4g64_noalloc(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M,
                             int N, int K, void* stream) {
  if (!x || !w_tc || !out) return SKINNY_ERR_INVALID_ARG;
  int st = check_qmm_shape(N, K);
  if (st != SKINNY_OK) return st;
  if (!skinny::qmm_noalloc_fits(N, K)) return SKINNY_ERR_SCRATCH_LIMIT;
  if (M < 1 || M > skinny::kMaxTokens) return SKINNY_ERR_TOKENS;
  if (ldx < K || ldo < N) return SKINNY_ERR_INVALID_ARG;
  if (!aligned16(x) || (ldx % 8) != 0 || !aligned16(w_tc)) return SKINNY_ERR_ALIGNMENT;
  return cuda_status(skinny::qmm_tc_launch_noalloc(x, ldx, w_tc, out, ldo, M, N, K,
                                                   static_cast<cudaStream_t>(stream)));
}

size_t skinny_spec_accept_workspace_bytes(void) { return skinny::spec_accept_ws_bytes(); }

int skinny_spec_accept(const void* logits, int ld, int rows, int V, const int32_t* draft,
                       int32_t* result, int32_t* pred, void* workspace, size_t workspace_bytes,
                       void* stream) {
  if (!logits || !result || (rows > 1 && !draft)) return SKINNY_ERR_INVALID_ARG;
  if (!skinny::spec_accept_fits(rows, V) || ld < V) return SKINNY_ERR_SHAPE;
  if (!aligned16(logits) || (ld % 8) != 0) return SKINNY_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < skinny::spec_accept_ws_bytes() || !aligned16(workspace))
    return SKINNY_ERR_WORKSPACE;
  return cuda_status(skinny::spec_accept_launch(logits, ld, rows, V, draft, result, pred, workspace,
                                                static_cast<cudaStream_t>(stream)));
}

int skinny_gdn_recurrent(const void* q, const void* k, const void* v, const float* g,
                         const float* beta, float* state, void* y, float* ckpt, int T, int Hv, int Hk,
                         int Dk, int Dv, void* stream) {
  if (!q || !k || !v || !g || !beta || !state || !y) return SKINNY_ERR_INVALID_ARG;
  if (T < 1 || Hv < 1 || Hk < 1 || Hv % Hk != 0 || Dk != 128 || Dv != 128) return SKINNY_ERR_SHAPE;
  if (!aligned16(state) || (ckpt && !aligned16(ckpt))) return SKINNY_ERR_ALIGNMENT;
  return cuda_status(skinny::gdn_recurrent_launch(q, k, v, g, beta, state, y, ckpt, T, Hv, Hk,
                                                  static_cast<cudaStream_t>(stream)));
}

int skinny_gdn_rollback(int n_layers, float* const* state, const float* const* ckpt,
                        void* const* conv, const void* const* conv_full, long long state_elems,
                        int keep, int fed, int W, int C, void* stream) {
  if (n_layers < 1 || n_layers > SKINNY_GDN_MAX_LAYERS || !state || !ckpt) return SKINNY_ERR_INVALID_ARG;
  if (keep < 1 || keep > fed || state_elems < 4 || state_elems % 4 != 0) return SKINNY_ERR_SHAPE;
  if (conv && (!conv_full || W < 0 || C < 1)) return SKINNY_ERR_INVALID_ARG;
  for (int l = 0; l < n_layers; ++l) {
    if (!state[l] || (keep < fed && !ckpt[l])) return SKINNY_ERR_INVALID_ARG;
    if (!aligned16(state[l]) || (ckpt[l] && !aligned16(ckpt[l]))) return SKINNY_ERR_ALIGNMENT;
    if (conv && (!conv[l] || !conv_full[l])) return SKINNY_ERR_INVALID_ARG;
  }
  return cuda_status(skinny::gdn_rollback_call(n_layers, state, ckpt, conv, conv_full, state_elems,
                                               keep, fed, W, C, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
