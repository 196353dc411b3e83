// C-ABI entry points: host-side validation, then stream-ordered kernel launches.
#include <cstdint>
#include <cstring>
#include <utility>
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
cudaError_t qmm_launch_config(int M, int N, int K, int* token_cols, int* split, int* ctas);
cudaError_t qmm_noalloc_error_copy(void* dst, cudaStream_t stream);
cudaError_t qmm_dequant_launch(const void* w_tc, int N, int K, void* out, int ldo, cudaStream_t stream);
bool qmm_noalloc_fits(int N, int K);
size_t spec_accept_ws_bytes();
cudaError_t qmm_tc_launch_prepared(const void* xq, const void* w_tc, void* out, int ldo, int M, int N, int K,
                                   void* ws, const void* const* xq_ranks, int xq_gpr, const skinny_peer_sync* sync,
                                   cudaStream_t stream, void* swiglu_xq = nullptr);
cudaError_t prep_launch(int mode, const void* x, int ldx, const void* d, int ldd, int dseg_cols,
                        const void* const* dseg, void* h_out, int ldh, const float* w, float eps, int K, int M,
                        void* xq, void* a_out, const skinny_peer_sync* sync, cudaStream_t stream);
int prep_max_k();
cudaError_t embed_launch(const int64_t* ids, int M, const void* w, const void* sc, const void* bi, int V, int K,
                         void* out, int ldo, cudaStream_t stream);
struct GdnFusedParamsHost {
  const void* proj;
  int ldp;
  void* conv;
  void* conv_full;
  const float* conv_w;
  const float* A_log;
  const float* dt_bias;
  const float* norm_w;
  float eps;
  float* state;
  float* ckpt;
  void* xq;
  void* o_out;
  uint32_t* err;
  const int32_t* parent;
  int T, Hv, Hk, W;
};
cudaError_t gdn_fused_call(const GdnFusedParamsHost& prm, cudaStream_t stream);
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
size_t attn_ws_bytes(int T, int nh, int nkv, int max_len);
bool attn_fits(int T, int nh, int nkv);
cudaError_t attn_fused_launch(const void* proj, int ldp, const float* qn_w, const float* kn_w,
                              const float* inv_freq, int rot, int gated, float eps, void* kc, void* vc, int L0,
                              const int* len_dev, int max_len, int T, int nh, int nkv, void* ws, void* xq,
                              void* o_out, const skinny_peer_sync* sync, const int32_t* parent, cudaStream_t stream);
cudaError_t spec_accept_tree_launch(const void* logits, int ld, int rows, int V, const int32_t* tokens,
                                    const int32_t* parent, int32_t* result, int32_t* pred, void* ws,
                                    cudaStream_t stream);
bool kv_compact_fits(int n_layers, int n, int row_bytes);
cudaError_t kv_compact_launch(int n_layers, void* const* k, void* const* v, const int* L0, const int* path, int n,
                              int row_bytes, cudaStream_t stream);
cudaError_t gdn_rollback_tree_call(int n_layers, float* const* state, const float* const* ckpt, void* const* conv,
                                  const void* const* conv_full, long long state_elems, int node, const int* rows,
                                  int W, int C, cudaStream_t stream);
}  // namespace skinny

namespace {
thread_local int g_last_cuda = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return SKINNY_OK;
  g_last_cuda = static_cast<int>(e);
  return SKINNY_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

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

int skinny_dequant_w4g64(const void* w_tc, int N, int K, void* out, int ldo, void* stream) {
  if (!w_tc || !out) return SKINNY_ERR_INVALID_ARG;
  const int st = check_qmm_shape(N, K);
  if (st != SKINNY_OK) return st;
  if (ldo < K || (ldo % 8) || !aligned16(out) || !aligned16(w_tc)) return SKINNY_ERR_ALIGNMENT;
  return cuda_status(skinny::qmm_dequant_launch(w_tc, N, K, out, ldo, static_cast<cudaStream_t>(stream)));
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

int skinny_qmm_w4g64_noalloc_errors(void* dst, void* stream) {
  if (!dst) return SKINNY_ERR_INVALID_ARG;
  return cuda_status(skinny::qmm_noalloc_error_copy(dst, static_cast<cudaStream_t>(stream)));
}

int skinny_qmm_launch_config(int M, int N, int K, int* token_cols, int* split, int* ctas) {
  if (!token_cols || !split || !ctas) return SKINNY_ERR_INVALID_ARG;
  const int st = check_qmm_shape(N, K);
  if (st != SKINNY_OK) return st;
  if (M < 1 || M > skinny::kMaxTokens) return SKINNY_ERR_TOKENS;
  return cuda_status(skinny::qmm_launch_config(M, N, K, token_cols, split, ctas));
}

// A peer-sync descriptor: absent, or a device epoch with an error word, 1..8 ranks, and for a
// wait the local flag array, for a signal the local counter and one flag address per rank;
// 0..8 mirror destinations, 16-byte aligned.
static bool sync_ok(const skinny_peer_sync* s) {
  if (!s || !s->epoch) return true;
  if (s->n_ranks < 1 || s->n_ranks > 8 || !s->err) return false;
  if (!s->wait_flags && !s->counter) return false;
  if (s->counter)
    for (int r = 0; r < s->n_ranks; ++r)
      if (!s->signal_flags[r]) return false;
  if (s->n_mirror < 0 || s->n_mirror > 8) return false;
  for (int i = 0; i < s->n_mirror; ++i)
    if (!s->mirror[i] || (reinterpret_cast<uintptr_t>(s->mirror[i]) & 15)) return false;
  return true;
}

int skinny_embed_w4g64(const int64_t* ids, int M, const void* w_packed, const void* scales, const void* biases,
                       int V, int K, void* out, int ldo, void* stream) {
  if (!ids || !w_packed || !scales || !biases || !out || V < 1) return SKINNY_ERR_INVALID_ARG;
  if (M < 1 || M > 65535) return SKINNY_ERR_TOKENS;
  if (K < skinny::kGroup || K % skinny::kGroup || ldo < K) return SKINNY_ERR_SHAPE;
  if (!aligned16(out) || (ldo % 8) || (reinterpret_cast<uintptr_t>(w_packed) & 3) ||
      (reinterpret_cast<uintptr_t>(scales) & 1) || (reinterpret_cast<uintptr_t>(biases) & 1) ||
      (reinterpret_cast<uintptr_t>(ids) & 7))
    return SKINNY_ERR_ALIGNMENT;
  return cuda_status(skinny::embed_launch(ids, M, w_packed, scales, biases, V, K, out, ldo,
                                          static_cast<cudaStream_t>(stream)));
}

size_t skinny_xq_bytes(int M, int K) {
  if (M < 1 || M > skinny::kMaxTokens || K < skinny::kGroup || K % skinny::kGroup) return 0;
  return static_cast<size_t>(K / skinny::kGroup) * skinny::xq_block_bytes(M <= 8 ? 8 : 16);
}

int skinny_prep(int mode, const void* x, int ldx, const void* d, int ldd, int dseg_cols, const void* const* dseg,
                void* h_out, int ldh, const float* w, float eps, int M, int K, void* xq, void* a_out,
                const skinny_peer_sync* sync, void* stream) {
  if (!x || !xq || mode < 0 || mode > 2 || (mode == 0 && !w)) return SKINNY_ERR_INVALID_ARG;
  if (M < 1 || M > skinny::kMaxTokens) return SKINNY_ERR_TOKENS;
  if (K < skinny::kGroup || K % skinny::kGroup || (mode == 0 && K > skinny::prep_max_k())) return SKINNY_ERR_SHAPE;
  if (!sync_ok(sync)) return SKINNY_ERR_INVALID_ARG;
  const int need = mode == 1 ? 2 * K : K;
  if (ldx < need || (h_out && ldh < K)) return SKINNY_ERR_INVALID_ARG;
  const bool segd = mode == 0 && dseg_cols > 0;
  if (mode == 0 && dseg_cols < 0) return SKINNY_ERR_INVALID_ARG;
  if (segd && (!dseg || dseg_cols % skinny::kGroup || K % dseg_cols || K / dseg_cols > 8 || ldd < dseg_cols))
    return SKINNY_ERR_INVALID_ARG;
  if (mode == 0 && d && !segd && ldd < K) return SKINNY_ERR_INVALID_ARG;
  const bool has_d = mode == 0 && (d || segd);
  // Outputs are written by one column chunk while other chunks of the row still read the inputs:
  // h_out and a_out must not overlap x or d (or a shard of d).
  const auto span = [M](const void* p, int ld, int width) {
    const uintptr_t b = reinterpret_cast<uintptr_t>(p);
    return std::make_pair(b, b + (static_cast<uintptr_t>(M - 1) * ld + width) * 2);
  };
  const auto overlap = [](std::pair<uintptr_t, uintptr_t> a, std::pair<uintptr_t, uintptr_t> b) {
    return a.first < b.second && b.first < a.second;
  };
  const auto hits_d = [&](std::pair<uintptr_t, uintptr_t> o) {
    if (!has_d) return false;
    if (!segd) return overlap(o, span(d, ldd, K));
    for (int i = 0; i < K / dseg_cols; ++i)
      if (overlap(o, span(dseg[i], ldd, dseg_cols))) return true;
    return false;
  };
  if (mode == 0) {
    const auto xs = span(x, ldx, K);
    if (h_out && has_d && (overlap(span(h_out, ldh, K), xs) || hits_d(span(h_out, ldh, K))))
      return SKINNY_ERR_INVALID_ARG;
    if (a_out && (overlap(span(a_out, K, K), xs) || hits_d(span(a_out, K, K)))) return SKINNY_ERR_INVALID_ARG;
  }
  // bf16 pairs are read and written as 4-byte words; mode 0 reads its row as 16-byte vectors
  if ((ldx % 2) || (has_d && ldd % 2) || (h_out && ldh % 2) || !aligned16(xq) || !aligned4(x) ||
      !aligned4(h_out) || !aligned4(a_out))
    return SKINNY_ERR_ALIGNMENT;
  if (mode == 0 && K > 16384) return SKINNY_ERR_SHAPE;
  if (mode == 0 && ((ldx % 8) || !aligned16(x) || (has_d && (ldd % 8))))
    return SKINNY_ERR_ALIGNMENT;
  if (mode == 0 && has_d && !segd && !aligned16(d)) return SKINNY_ERR_ALIGNMENT;
  if (segd)
    for (int i = 0; i < K / dseg_cols; ++i)
      if (!dseg[i] || !aligned16(dseg[i])) return SKINNY_ERR_ALIGNMENT;
  return cuda_status(skinny::prep_launch(mode, x, ldx, mode == 0 ? d : nullptr, ldd, segd ? dseg_cols : 0, dseg,
                                         h_out, ldh, w, eps, K, M, xq, a_out, sync,
                                         static_cast<cudaStream_t>(stream)));
}

static int gdn_fused_common(const void* proj, int ldp, void* conv, void* conv_full, const float* conv_w,
                            const float* A_log, const float* dt_bias, const float* norm_w, float eps, float* state,
                            float* ckpt, void* xq, void* o_out, int T, int Hv, int Hk, int W, void* err_word,
                            const int32_t* parent, void* stream) {
  if (!proj || !conv || !conv_w || !A_log || !dt_bias || !norm_w || !state || !xq || !err_word)
    return SKINNY_ERR_INVALID_ARG;
  if (T < 1 || T > skinny::kMaxTokens || Hv < 1 || Hk != Hv || W < 1 || W > 4) return SKINNY_ERR_SHAPE;
  const int C = 3 * Hv * 128;
  if (ldp < C + Hv * 128 + 2 * Hv) return SKINNY_ERR_INVALID_ARG;
  if (parent && (!ckpt || !conv_full || !aligned4(parent))) return SKINNY_ERR_INVALID_ARG;
  // conv window and projection rows are read as 16-byte vectors
  if (!aligned16(state) || (ckpt && !aligned16(ckpt)) || !aligned16(xq) || (ldp % 8) || !aligned16(proj) ||
      !aligned16(conv) || !aligned16(conv_full) || !aligned4(o_out) || !aligned4(err_word))
    return SKINNY_ERR_ALIGNMENT;
  skinny::GdnFusedParamsHost prm{proj, ldp, conv, conv_full, conv_w, A_log, dt_bias, norm_w, eps, state,
                             (parent || T > 1) ? ckpt : nullptr, xq, o_out, static_cast<uint32_t*>(err_word),
                             parent, T, Hv, Hk, W};
  return cuda_status(skinny::gdn_fused_call(prm, static_cast<cudaStream_t>(stream)));
}

int skinny_gdn_fused(const void* proj, int ldp, void* conv, void* conv_full, const float* conv_w,
                     const float* A_log, const float* dt_bias, const float* norm_w, float eps, float* state,
                     float* ckpt, void* xq, void* o_out, int T, int Hv, int Hk, int W, void* err_word,
                     void* stream) {
  return gdn_fused_common(proj, ldp, conv, conv_full, conv_w, A_log, dt_bias, norm_w, eps, state, ckpt, xq, o_out,
                          T, Hv, Hk, W, err_word, nullptr, stream);
}

int skinny_gdn_fused_tree(const void* proj, int ldp, void* conv, void* conv_full, const float* conv_w,
                          const float* A_log, const float* dt_bias, const float* norm_w, float eps, const float* state,
                          float* ckpt, void* xq, void* o_out, int T, int Hv, int Hk, int W, void* err_word,
                          const int32_t* parent, void* stream) {
  if (!parent) return SKINNY_ERR_INVALID_ARG;
  return gdn_fused_common(proj, ldp, conv, conv_full, conv_w, A_log, dt_bias, norm_w, eps, const_cast<float*>(state),
                          ckpt, xq, o_out, T, Hv, Hk, W, err_word, parent, stream);
}

size_t skinny_attn_workspace_bytes(int T, int n_heads, int n_kv_heads, int max_len) {
  if (T < 1 || T > skinny::kMaxTokens || max_len < 1 || !skinny::attn_fits(T, n_heads, n_kv_heads)) return 0;
  return skinny::attn_ws_bytes(T, n_heads, n_kv_heads, max_len);
}

static int attn_fused_common(const void* proj, int ldp, const float* q_norm_w, const float* k_norm_w,
                             const float* inv_freq, int rot, int gated, float eps, void* k_cache, void* v_cache,
                             int L0, const int32_t* length_dev, int T, int n_heads, int n_kv_heads, int max_len,
                             void* workspace, size_t workspace_bytes, void* xq, void* o_out,
                             const skinny_peer_sync* sync, const int32_t* parent, void* stream) {
  if (!proj || !q_norm_w || !k_norm_w || !k_cache || !v_cache || !xq || (rot > 0 && !inv_freq))
    return SKINNY_ERR_INVALID_ARG;
  if (T < 1 || T > skinny::kMaxTokens) return SKINNY_ERR_TOKENS;
  // with length_dev the caller guarantees 0 <= *length_dev <= max_len - T when the launch runs
  if (!skinny::attn_fits(T, n_heads, n_kv_heads) || (rot != 0 && rot != 16 && rot != 32 && rot != 64 && rot != 128) ||
      L0 < 0 ||
      (!length_dev && L0 + T > max_len) || max_len < T)
    return SKINNY_ERR_SHAPE;
  if ((gated != 0 && gated != 1) || ldp < ((1 + gated) * n_heads + 2 * n_kv_heads) * 128 || !sync_ok(sync))
    return SKINNY_ERR_INVALID_ARG;
  if (!aligned16(xq) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned4(o_out) || !aligned16(proj) ||
      (ldp % 8) || !aligned4(length_dev) || !aligned4(parent))
    return SKINNY_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < skinny::attn_ws_bytes(T, n_heads, n_kv_heads, max_len) ||
      !aligned16(workspace))
    return SKINNY_ERR_WORKSPACE;
  return cuda_status(skinny::attn_fused_launch(proj, ldp, q_norm_w, k_norm_w, inv_freq, rot, gated, eps, k_cache,
                                               v_cache, L0, length_dev, max_len, T, n_heads, n_kv_heads,
                                               workspace, xq, o_out, sync, parent, static_cast<cudaStream_t>(stream)));
}

int skinny_attn_fused(const void* proj, int ldp, const float* q_norm_w, const float* k_norm_w,
                      const float* inv_freq, int rot, int gated, float eps, void* k_cache, void* v_cache, int L0,
                      const int32_t* length_dev, int T, int n_heads, int n_kv_heads, int max_len, void* workspace,
                      size_t workspace_bytes, void* xq, void* o_out, const skinny_peer_sync* sync, void* stream) {
  return attn_fused_common(proj, ldp, q_norm_w, k_norm_w, inv_freq, rot, gated, eps, k_cache, v_cache, L0, length_dev,
                           T, n_heads, n_kv_heads, max_len, workspace, workspace_bytes, xq, o_out, sync, nullptr,
                           stream);
}

int skinny_attn_fused_tree(const void* proj, int ldp, const float* q_norm_w, const float* k_norm_w,
                           const float* inv_freq, int rot, int gated, float eps, void* k_cache, void* v_cache, int L0,
                           const int32_t* length_dev, int T, int n_heads, int n_kv_heads, int max_len,
                           void* workspace, size_t workspace_bytes, void* xq, void* o_out, const int32_t* parent,
                           void* stream) {
  if (!parent) return SKINNY_ERR_INVALID_ARG;
  return attn_fused_common(proj, ldp, q_norm_w, k_norm_w, inv_freq, rot, gated, eps, k_cache, v_cache, L0, length_dev,
                           T, n_heads, n_kv_heads, max_len, workspace, workspace_bytes, xq, o_out, nullptr, parent,
                           stream);
}

int skinny_qmm_w4g64_prepared(const void* xq, const void* w_tc, void* out, int ldo, int M, int N, int K,
                              void* workspace, size_t workspace_bytes, const void* const* xq_ranks,
                              int xq_groups_per_rank, const skinny_peer_sync* sync, void* stream) {
  if ((!xq && !xq_ranks) || !w_tc || !out) return SKINNY_ERR_INVALID_ARG;
  const int st = check_qmm_shape(N, K);
  if (st != SKINNY_OK) return st;
  if (M < 1 || M > skinny::kMaxTokens) return SKINNY_ERR_TOKENS;
  if (ldo < N) return SKINNY_ERR_INVALID_ARG;
  if (xq_ranks) {
    const int G = K / skinny::kGroup;
    if (xq_groups_per_rank < 1 || G % xq_groups_per_rank || G / xq_groups_per_rank > 8) return SKINNY_ERR_INVALID_ARG;
    for (int r = 0; r < G / xq_groups_per_rank; ++r)
      if (!xq_ranks[r] || !aligned16(xq_ranks[r])) return SKINNY_ERR_ALIGNMENT;
  } else if (!aligned16(xq)) {
    return SKINNY_ERR_ALIGNMENT;
  }
  if (!sync_ok(sync)) return SKINNY_ERR_INVALID_ARG;
  if (!aligned16(w_tc)) return SKINNY_ERR_ALIGNMENT;
  const skinny::WsLayout wl = skinny::ws_layout(skinny::device_sm_count(current_device()));
  if (!workspace || workspace_bytes < wl.total || !aligned16(workspace)) return SKINNY_ERR_WORKSPACE;
  return cuda_status(skinny::qmm_tc_launch_prepared(xq, w_tc, out, ldo, M, N, K, workspace, xq_ranks,
                                                    xq_groups_per_rank, sync, static_cast<cudaStream_t>(stream)));
}

int skinny_qmm_w4g64_swiglu(const void* xq, const void* w_tc, void* xq_out, int M, int N, int K, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!xq || !w_tc || !xq_out) return SKINNY_ERR_INVALID_ARG;
  const int st = check_qmm_shape(N, K);
  if (st != SKINNY_OK) return st;
  if (N % (2 * skinny::kGroup) != 0) return SKINNY_ERR_SHAPE;
  if (M < 1 || M > skinny::kMaxTokens) return SKINNY_ERR_TOKENS;
  if (!aligned16(xq) || !aligned16(w_tc) || !aligned16(xq_out)) return SKINNY_ERR_ALIGNMENT;
  const skinny::WsLayout wl = skinny::ws_layout(skinny::device_sm_count(current_device()));
  if (!workspace || workspace_bytes < wl.total || !aligned16(workspace)) return SKINNY_ERR_WORKSPACE;
  return cuda_status(skinny::qmm_tc_launch_prepared(xq, w_tc, nullptr, N, M, N, K, workspace, nullptr, 0, nullptr,
                                                    static_cast<cudaStream_t>(stream), xq_out));
}

// ---- peer memory (CUDA IPC) ----
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handles");
int skinny_ipc_alloc(size_t bytes, void** ptr, void* handle64) {
  if (!ptr || !handle64 || bytes == 0) return SKINNY_ERR_INVALID_ARG;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_status(e);
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any rank can map it
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle64), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e);
  }
  *ptr = p;
  return SKINNY_OK;
}

int skinny_ipc_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return SKINNY_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int skinny_ipc_close(void* ptr) { return ptr ? cuda_status(cudaIpcCloseMemHandle(ptr)) : SKINNY_ERR_INVALID_ARG; }

int skinny_ipc_free(void* ptr) { return ptr ? cuda_status(cudaFree(ptr)) : SKINNY_ERR_INVALID_ARG; }

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

int skinny_spec_accept_tree(const void* logits, int ld, int rows, int V, const int32_t* tokens,
                            const int32_t* parent, int32_t* result, int32_t* pred, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!logits || !result || !tokens || !parent) return SKINNY_ERR_INVALID_ARG;
  if (!skinny::spec_accept_fits(rows, V) || ld < V) return SKINNY_ERR_SHAPE;
  if (!aligned16(logits) || (ld % 8) != 0 || !aligned4(tokens) || !aligned4(parent)) return SKINNY_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < skinny::spec_accept_ws_bytes() || !aligned16(workspace))
    return SKINNY_ERR_WORKSPACE;
  return cuda_status(skinny::spec_accept_tree_launch(logits, ld, rows, V, tokens, parent, result, pred, workspace,
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

int skinny_kv_compact(int n_layers, void* const* k_caches, void* const* v_caches, int row_bytes, const int32_t* L0,
                      const int32_t* path, int n_path, int max_len, void* stream) {
  if (!k_caches || !v_caches || !L0 || !path || n_path < 1) return SKINNY_ERR_INVALID_ARG;
  if (!skinny::kv_compact_fits(n_layers, n_path - 1, row_bytes) || path[0] != 0) return SKINNY_ERR_SHAPE;
  for (int j = 1; j < n_path; ++j)
    if (path[j] < j || path[j] <= path[j - 1]) return SKINNY_ERR_SHAPE;  // a root-to-node path in a topological tree
  for (int l = 0; l < n_layers; ++l) {
    if (!k_caches[l] || !v_caches[l]) return SKINNY_ERR_INVALID_ARG;
    if (!aligned16(k_caches[l]) || !aligned16(v_caches[l])) return SKINNY_ERR_ALIGNMENT;
    if (L0[l] < 0 || L0[l] + path[n_path - 1] >= max_len) return SKINNY_ERR_SHAPE;
  }
  return cuda_status(skinny::kv_compact_launch(n_layers, k_caches, v_caches, L0, path, n_path - 1, row_bytes,
                                               static_cast<cudaStream_t>(stream)));
}

int skinny_gdn_rollback_tree(int n_layers, float* const* state, const float* const* ckpt, void* const* conv,
                             const void* const* conv_full, long long state_elems, int node, const int32_t* rows,
                             int fed, int W, int C, void* stream) {
  if (n_layers < 1 || n_layers > SKINNY_GDN_MAX_LAYERS || !state || !ckpt || !conv || !conv_full || !rows)
    return SKINNY_ERR_INVALID_ARG;
  if (node < 0 || node >= fed || state_elems < 4 || state_elems % 4 != 0 || W < 1 || W > 4 || C < 1)
    return SKINNY_ERR_SHAPE;
  for (int q = 0; q < W; ++q)
    if (rows[q] < 0 || rows[q] >= W + fed) return SKINNY_ERR_SHAPE;
  for (int l = 0; l < n_layers; ++l) {
    if (!state[l] || !ckpt[l] || !conv[l] || !conv_full[l]) return SKINNY_ERR_INVALID_ARG;
    if (!aligned16(state[l]) || !aligned16(ckpt[l])) return SKINNY_ERR_ALIGNMENT;
  }
  return cuda_status(skinny::gdn_rollback_tree_call(n_layers, state, ckpt, conv, conv_full, state_elems, node, rows,
                                                    W, C, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
