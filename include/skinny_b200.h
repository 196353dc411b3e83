/*
 * skinny_b200 — C ABI of the B200 (sm_100a) flat multi-token verify path.
 *
 * Plain pointers and sizes only; every device pointer is caller-owned CUDA memory, `stream` is a
 * cudaStream_t passed as void*, and every call is stream-ordered on it.  No compute entry point
 * allocates device memory, synchronises the stream, or retains a pointer after it returns.  The
 * exceptions are the peer-memory set-up calls (skinny_ipc_alloc allocates, zero-fills and
 * synchronises the device once, before the buffer is shared; skinny_ipc_free frees), which a
 * sharded step makes once at start-up, never per step.
 *
 * Return value: SKINNY_OK (0) or a negative status (see skinny_strerror).  Argument errors are
 * detected on the host before anything is launched.  Kernel-side errors (a bounded wait that ran
 * out; an out-of-range token id in the embedding lookup) are OR-ed into 32-bit word 0 of the
 * workspace; read it after the stream work completes.  A workspace that recorded an error must
 * be zero-filled again before reuse.  Non-finite activations are not errors: they propagate to
 * the affected outputs as NaN, as f32 arithmetic would.
 *
 * Reference interfaces replaced (paths inside rachittshah/skinny-mlx):
 *   skinny_repack_w4g64  <- skinny_mlx/qmm.py:96  repack_for_skinny(w)
 *   skinny_qmm_w4g64     <- skinny_mlx/qmm.py:132 skinny_qmm(x, w, scales, biases) and the Metal
 *                           kernel it launches, skinny_mlx/qmm.py:21-86; routed to by
 *                           skinny_mlx/patch.py:30-35 _qmm
 */
#ifndef SKINNY_B200_H
#define SKINNY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SKINNY_OK 0
#define SKINNY_ERR_INVALID_ARG -1
#define SKINNY_ERR_SHAPE -2
#define SKINNY_ERR_TOKENS -3
#define SKINNY_ERR_ALIGNMENT -4
#define SKINNY_ERR_WORKSPACE -5
#define SKINNY_ERR_CUDA -6
#define SKINNY_ERR_DEVICE -7
#define SKINNY_ERR_UNSUPPORTED -8
#define SKINNY_ERR_SCRATCH_LIMIT -9

/* Library version, e.g. 100 for 0.1.0. */
int skinny_version(void);

/* Human-readable text for a status code. */
const char* skinny_strerror(int status);

/* The cudaError_t of the most recent failing CUDA call made by this library on this thread. */
int skinny_last_cuda_error(void);

/* ---------------------------------------------------------------------------------------------
 * 4-bit affine group-64 weights (MLX packing: uint32 [N, K/8], element 8j+i at bits 4i of word
 * j; bf16 scales and biases [N, K/64]).
 * ------------------------------------------------------------------------------------------- */

/* Bytes of the relaid weight buffer for an N x K matrix (N rounded up to 128 rows). */
size_t skinny_repack_bytes(int N, int K);

/* One-time relayout of MLX packs + scales + biases into the kernel's unit order.
 * Replaces skinny_mlx/qmm.py:96 repack_for_skinny.  w_tc must hold skinny_repack_bytes(N, K)
 * bytes and be 16-byte aligned.  K % 64 == 0, N >= 1. */
int skinny_repack_w4g64(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                        void* w_tc, int N, int K, void* stream);

/* Workspace bytes a qmm of this shape needs on the current device. */
size_t skinny_qmm_workspace_bytes(int N, int K);

/* out[M, N] (bf16, leading dimension ldo) = x[M, K] (bf16, leading dimension ldx) . W^T for
 * 1 <= M <= 16 tokens, computing sum_g s*sum(x*q) + b*sum(x) in f32 (skinny_mlx/qmm.py:8-9).
 * Products are exact integer dot products (int8 tensor cores) of q with x rounded to 16-bit
 * fixed point per token and 64-column group (relative to the group's largest |x|, at most 2^-16 of
 * it), then scaled and accumulated in f32.  Each token's output depends only on that token's row
 * of x: it is bit-identical for any M.  An x-prep kernel runs first in the same call.
 * x and ldx*2 must be 16-byte aligned.  The workspace must be zero-filled before its first use,
 * hold skinny_qmm_workspace_bytes(N, K) bytes, and not be shared by calls that may run
 * concurrently; calls of different shapes may share it.  Launches use programmatic dependent
 * launch, so the weight stream of a call overlaps the tail of the kernel before it.
 * Replaces skinny_mlx/qmm.py:132 skinny_qmm. */
int skinny_qmm_w4g64(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M, int N,
                     int K, void* workspace, size_t workspace_bytes, void* stream);

/* Limits of one grouped call. */
#define SKINNY_QMM_MAX_GROUP 192       /* matrices per grouped call */
#define SKINNY_QMM_MAX_GROUP_INPUTS 8  /* distinct activation buffers per grouped call */

/* n independent products out[i][M, N[i]] = x[i][M, K[i]] . W_i^T in ONE persistent launch that
 * streams the concatenated weights of all n matrices (same token count M for all).  The launch
 * overhead, pipeline fill and split-K fix-up are paid once for the group instead of per matrix.
 * Same per-matrix contract as skinny_qmm_w4g64; results equal a single call's up to the f32
 * summation order of tiles split between CTAs (the split depends on the whole group), and are
 * deterministic and bit-identical for any M.  This is the B200 form
 * of evaluating a list of quantized matmuls at once, as skinny_mlx/qmm.py:195-196 and
 * bench/model_matmuls.py:188-191 do with mx.eval on a list. */
int skinny_qmm_w4g64_grouped(int n, const void* const* x, const int* ldx, const void* const* w_tc,
                             void* const* out, const int* ldo, const int* N, const int* K, int M,
                             void* workspace, size_t workspace_bytes, void* stream);

/* The relaid weight back as bf16 W[N, K] (row stride ldo, 16-byte aligned rows):
 * W = bf16(q * scale + bias), the f32 product then the f32 sum, each rounded (the dequantisation
 * of skinny_mlx/qmm.py:8-9).  For many-token inputs (a prompt), which a dense GEMM serves
 * better than the token-streaming qmm; skinny_qmm (Python) uses it from 64 tokens.  One launch. */
int skinny_dequant_w4g64(const void* w_tc, int N, int K, void* out, int ldo, void* stream);

/* The launch skinny_qmm_w4g64 makes for M tokens of an N x K weight on the current device:
 * *token_cols = token columns read back per 128 x 64 unit (2, 4, 8 or 16), *split = 0 for the
 * persistent stream-K grid over all units or S >= 1 for S CTAs per 128-row tile (a thread-block
 * cluster summing S K-slices), *ctas = the grid size.  Replaces skinny_mlx/qmm.py:118
 * config_for(m, k) -> (RF, SK), the Metal kernel's row-fragment and K-split choice. */
int skinny_qmm_launch_config(int M, int N, int K, int* token_cols, int* split, int* ctas);

/* ---------------------------------------------------------------------------------------------
 * Peer memory for a sharded step (one GPU per rank): buffers allocated by one rank and opened by
 * the others through CUDA IPC (NVLink loads and stores; no multicast), and the flags that order
 * producers and consumers across ranks.  No counterpart in the reference (it runs on one GPU).
 * ------------------------------------------------------------------------------------------- */

/* cudaMalloc of `bytes` (zero-filled) and its 64-byte IPC handle. */
int skinny_ipc_alloc(size_t bytes, void** ptr, void* handle64);
/* Map another rank's buffer from its handle; unmap with skinny_ipc_close. */
int skinny_ipc_open(const void* handle64, void** ptr);
int skinny_ipc_close(void* ptr);
int skinny_ipc_free(void* ptr);

/* Synchronisation of one launch with the other ranks (all pointers device memory):
 *   wait_flags  != NULL: before reading other ranks' data, wait (bounded, error bit 11) until
 *                        wait_flags[0 .. n_ranks) >= *epoch;
 *   counter     != NULL: after its last write each CTA counts itself on counter (a GPU-scope
 *                        acquire-release atomic), and the last one, after one system-scope fence,
 *                        stores *epoch into signal_flags[r] for every rank r (this rank's word in
 *                        each rank's flags); the counter is zero between launches.
 *   n_mirror > 0:        a launch that writes qmm input digits (skinny_prep, skinny_attn_fused)
 *                        also writes them to mirror[0 .. n_mirror): other ranks' buffers, each
 *                        the address that corresponds to xq there (same block offsets), so that
 *                        consumers read every rank's digits from their own memory; the signal
 *                        above is stored after these writes.
 * epoch is a device counter the caller advances once per step (so a captured graph serves every
 * step); err (required with an epoch) receives the error bits.  A NULL skinny_peer_sync pointer,
 * or epoch == NULL, means no synchronisation. */
typedef struct {
  const uint32_t* epoch;
  const uint32_t* wait_flags;
  uint32_t* counter;
  uint32_t* signal_flags[8];
  uint32_t* err;
  int n_ranks;
  void* mirror[8];
  int n_mirror;
} skinny_peer_sync;

/* Token embedding rows of a 4-bit group-64 table in MLX packing (the embedding lookup of the
 * verify forward, skinny_mlx/spec.py:23-28 via mlx_lm's QuantizedEmbedding; the dequantisation
 * is skinny_mlx/qmm.py:8-9's affine rule):
 *   out[t, k] = bf16(q * scale + bias), q = nibble k % 8 of word k / 8 of row ids[t]
 * (f32 product then f32 sum, each rounded).  ids: M int64 (device), rows outside [0, V) are
 * written as zeros.  w_packed [V, K/8] u32, scales / biases [V, K/64] bf16, out [M, ldo] bf16
 * (16-byte aligned rows).  One launch (programmatic dependent launch). */
int skinny_embed_w4g64(const int64_t* ids, int M, const void* w_packed, const void* scales, const void* biases,
                       int V, int K, void* out, int ldo, void* stream);

/* Bytes of one prepared qmm input (the digit blocks the qmm kernel reads) for M tokens, K columns. */
size_t skinny_xq_bytes(int M, int K);

/* Producers of prepared qmm inputs: compute a bf16 activation row and write it straight in the
 * qmm's input format, so a step's elementwise work and its next matmul need no x-prep launch or
 * activation round trip (the B200 form of the glue between the reference model's projections).
 *   mode 0: h = x (+ d if d != NULL; h written to h_out when given), a = bf16(h / rms(h) * (1 + w))
 *           with w f32 [K] (zero-centred RMSNorm, eps); K <= 8192 (else SKINNY_ERR_SHAPE), x and d (or every shard)
 *           16-byte aligned with leading dimensions multiples of 8
 *   mode 1: a = bf16(silu(g) * u), x = [g | u] with 2K columns (SwiGLU)
 *   mode 2: a = x
 * d may be column-sharded, one [M, dseg_cols] shard per rank (e.g. the per-rank outputs of a
 * column-parallel matmul, in an all-gather buffer or in the ranks' own memory): with
 * dseg_cols > 0 (a multiple of 64 dividing K), column c of token t is read at
 * dseg[c / dseg_cols] + t * ldd + c % dseg_cols (d is then ignored); dseg_cols = 0: plain rows.
 * sync (may be NULL): wait for the shards' producers before reading d; signal after writing
 * xq (a producer of this rank's digit groups).
 * x, d, h_out bf16 rows with leading dimensions ldx, ldd, ldh (even, 4-byte aligned); xq receives
 * skinny_xq_bytes(M, K) bytes (16-byte aligned); a_out (mode 0, may be NULL) receives a as bf16
 * [M, K].  h_out and a_out must not overlap x or d (SKINNY_ERR_INVALID_ARG): column chunks of a
 * row are written while other chunks of it are still being read.  Launched with programmatic
 * dependent launch: the next launch on the stream may start before this one ends. */
int skinny_prep(int mode, const void* x, int ldx, const void* d, int ldd, int dseg_cols, const void* const* dseg,
                void* h_out, int ldh, const float* w, float eps, int M, int K, void* xq, void* a_out,
                const skinny_peer_sync* sync, void* stream);

/* One Gated DeltaNet mixer from its fused input projection to the prepared input of out_proj,
 * in one launch: causal depthwise conv (window W <= 4, weights conv_w [C, W+1] f32) + SiLU,
 * l2-normalised q and k (q / sqrt(128)), g = exp(-exp(A_log) softplus(a + dt_bias)),
 * beta = sigmoid(b), the gated delta recurrence (state [Hv,128,128] f32 updated; ckpt as in
 * skinny_gdn_recurrent), gated RMSNorm rmsnorm(y) (1 + norm_w) * silu(z), written as qmm input
 * digits to xq (K = Hv*128) and, when o_out != NULL, as bf16 [T, Hv*128].  proj [T, ldp] bf16 =
 * q | k | v (the C = 3*Hv*128 conv channels) | z | b | a (16-byte aligned, ldp % 8 == 0); conv
 * [W, C] bf16 (16-byte aligned) is updated in place and conv_full [W+T, C] (may be NULL) records
 * the conv input for skinny_gdn_rollback.  Hk == Hv.  Each head runs on a cluster of 8 CTAs that
 * exchange y through distributed shared memory; a timed-out wait for a peer ORs a bit into the
 * 32-bit error word err_word (required; e.g. word 0 of a qmm workspace).  Launched with
 * programmatic dependent launch.  The layer code this replaces is mlx_lm's (the model the
 * reference patches); skinny_mlx/rollback.py:14-56 records the same state. */
int skinny_gdn_fused(const void* proj, int ldp, void* conv, void* conv_full, const float* conv_w,
                     const float* A_log, const float* dt_bias, const float* norm_w, float eps, float* state,
                     float* ckpt, void* xq, void* o_out, int T, int Hv, int Hk, int W, void* err_word,
                     void* stream);

/* skinny_gdn_fused over a token TREE of T nodes in topological order: parent (device int32 [T])
 * with parent[0] = -1 and parent[t] in [0, t).  Node t's conv window is the W inputs before it on
 * its ancestor path (the cached window above the root) and its recurrence starts from its
 * parent's state.  ckpt [T, Hv, 128, 128] (required) receives the state after EVERY node and
 * conv_full (required) the conv input [W + T, C]; state and conv are only read (the rollback,
 * skinny_gdn_rollback_tree, selects the accepted path).  A malformed parent array sets
 * kErrBitBadInput in err_word and is read as a chain.  Builds the branch-aware recurrence the
 * reference names for tree drafts verified in one pass (docs/flatspec-design.md:64-69). */
int skinny_gdn_fused_tree(const void* proj, int ldp, void* conv, void* conv_full, const float* conv_w,
                          const float* A_log, const float* dt_bias, const float* norm_w, float eps, const float* state,
                          float* ckpt, void* xq, void* o_out, int T, int Hv, int Hk, int W, void* err_word,
                          const int32_t* parent, void* stream);

/* Bytes of the workspace skinny_attn_fused needs for a KV cache of max_len positions (0 when the
 * shape is not supported).  It holds per-chunk partial results between the call's two launches
 * and no state between calls. */
size_t skinny_attn_workspace_bytes(int T, int n_heads, int n_kv_heads, int max_len);

/* One gated full-attention mixer from its fused projection to the prepared input of o_proj, in
 * one launch (the attention layers inside the verify forward of skinny_mlx/spec.py:23-28, which
 * runs the mlx_lm Qwen3.5 model; that layer code is mlx_lm's, not the reference's own):
 *   q, k = RoPE(bf16(rmsnorm(q|k) (1 + w))) on the first rot dims (rot in {0, 16, 32, 64, 128};
 *          inv_freq [rot/2] f32) at
 *          positions L0 .. L0+T-1; k (bf16) and v are appended to k_cache / v_cache
 *          [max_len, n_kv_heads, 128] (16-byte aligned) at L0 .. L0+T-1;
 *   o    = causal (bottom-right) grouped-query softmax(q k^T / sqrt(128)) v over positions
 *          0 .. L0+t, then (gated = 1) bf16(bf16(o) sigmoid(gate)) or (gated = 0) bf16(o),
 *          written as qmm input digits to xq (K = n_heads*128) and, when o_out != NULL, as bf16
 *          [T, n_heads*128].
 * proj [T, ldp] bf16 (16-byte aligned, ldp % 8 == 0) = per query head [q (128) | gate (128)]
 * (gated) or q (128) | k (n_kv*128) | v (n_kv*128).
 * head_dim 128, T * n_heads / n_kv_heads <= 128.  The caller advances its cache length by T.
 * length_dev (may be NULL): when given, the cache length L0 is read from this device int32 when
 * the kernel runs (L0 argument ignored), so that one captured launch (CUDA graph) serves every
 * length; a device length outside [0, max_len - T] makes the launch touch nothing.
 * sync (may be NULL; sharded step): the merge launch signals its completion.
 * Two launches (per-chunk partials, then their merge), both with programmatic dependent launch.
 * No counterpart in the reference's own code. */
int skinny_attn_fused(const void* proj, int ldp, const float* q_norm_w, const float* k_norm_w,
                      const float* inv_freq, int rot, int gated, float eps, void* k_cache, void* v_cache, int L0,
                      const int32_t* length_dev, int T, int n_heads, int n_kv_heads, int max_len, void* workspace,
                      size_t workspace_bytes, void* xq, void* o_out, const skinny_peer_sync* sync, void* stream);

/* skinny_attn_fused over a token TREE (parent as for skinny_gdn_fused_tree): node t is rotated
 * at position L0 + depth(t), attends to the cached positions 0 .. L0-1 and to the new keys of its
 * ancestors and itself, and its key / value are appended at slot L0 + t (after acceptance the
 * caller moves the accepted path's slots to L0 + depth). */
int skinny_attn_fused_tree(const void* proj, int ldp, const float* q_norm_w, const float* k_norm_w,
                           const float* inv_freq, int rot, int gated, float eps, void* k_cache, void* v_cache, int L0,
                           const int32_t* length_dev, int T, int n_heads, int n_kv_heads, int max_len,
                           void* workspace, size_t workspace_bytes, void* xq, void* o_out, const int32_t* parent,
                           void* stream);

/* The gate|up projection of a SwiGLU MLP with its activation in the epilogue: xq is a prepared
 * input (skinny_prep, M tokens, K columns), w_tc a relaid weight of N = 2I rows whose 128-row
 * tile j holds gate rows 64j .. 64j+63 then up rows 64j .. 64j+63 (I % 64 == 0).  Instead of the
 * [M, N] product it writes a = bf16(silu(bf16(g)) bf16(u)) for the I output columns as a prepared
 * input of K = I columns (skinny_xq_bytes(M, I) bytes at xq_out, 16-byte aligned): the same digits
 * as skinny_prep mode 1 on the product's bf16 output, without that launch or the output's round
 * trip.  Workspace as for skinny_qmm_w4g64_prepared.  No counterpart in the reference's own code
 * (its MLP runs gate/up, the activation and down as separate MLX operations). */
int skinny_qmm_w4g64_swiglu(const void* xq, const void* w_tc, void* xq_out, int M, int N, int K, void* workspace,
                            size_t workspace_bytes, void* stream);

/* skinny_qmm_w4g64 on an input prepared by skinny_prep (same result as passing the bf16
 * activation itself), launched without the x-prep kernel.  Sharded step: with xq_ranks != NULL
 * the digit blocks of groups [r * xq_groups_per_rank, (r+1) * xq_groups_per_rank) are read from
 * rank r's buffer xq_ranks[r] (at the offsets of a full K buffer; peer memory over NVLink), after
 * waiting for the ranks' flags (sync), and the launch signals its completion (sync). */
int skinny_qmm_w4g64_prepared(const void* xq, const void* w_tc, void* out, int ldo, int M, int N, int K,
                              void* workspace, size_t workspace_bytes, const void* const* xq_ranks,
                              int xq_groups_per_rank, const skinny_peer_sync* sync, void* stream);

/* Bytes of the workspace skinny_spec_accept needs (zero-filled before first use; reusable). */
size_t skinny_spec_accept_workspace_bytes(void);

/* Greedy acceptance of a verified draft, fused on the device: for the rows = K+1 verified
 * positions, pred[i] = argmax over the V logits of row i (bf16, leading dimension ld; ties to the
 * lowest index, a NaN above every number: numpy's order); n = the longest prefix with
 * draft[i] == pred[i] (i < K); then
 * result[0] = n, result[1 .. n+1] = draft[:n] + [pred[n]], result[n+2 .. rows] = -1.  pred (may be
 * NULL) receives the rows predictions.  rows <= 17, V <= 524,288; logits and ld*2 16-byte aligned.
 * Replaces the verify tail of skinny_mlx/spec.py:136-147 (argmax, the host sync of pred and
 * draft, the Python prefix loop): the host reads back rows + 1 int32 values. */
int skinny_spec_accept(const void* logits, int ld, int rows, int V, const int32_t* draft,
                       int32_t* result, int32_t* pred, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Greedy acceptance of a verified draft TREE of `rows` nodes (node 0 = the last emitted token;
 * tokens int32 [rows] the node tokens, parent int32 [rows] as for skinny_gdn_fused_tree, both
 * device memory): pred as above; from the root, move repeatedly to the first child (lowest index)
 * whose token equals the current node's prediction.  result int32 [2 rows + 1]: result[0] = n
 * accepted nodes, result[1 .. rows] = their tokens + [pred[last]] then -1, result[rows+1 ..
 * 2 rows] = the path 0, p1 .. pn then -1.  The tree form of skinny_mlx/spec.py:136-147. */
int skinny_spec_accept_tree(const void* logits, int ld, int rows, int V, const int32_t* tokens,
                            const int32_t* parent, int32_t* result, int32_t* pred, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Gated DeltaNet verify recurrence with per-token state checkpoints (the B200 form of the
 * recurrence that skinny_mlx/rollback.py:39-42 records and re-runs).  Per value head h and token t
 * (state S [Dv, Dk] f32): S <- g S; S <- S + beta (v - S k) k^T; y = S q, with q, k [T, Hk, 128]
 * bf16 (already normalised and scaled), v [T, Hv, 128] bf16, g (decay) and beta [T, Hv] f32; a k
 * head serves Hv/Hk value heads.  state [Hv, 128, 128] f32 is read and overwritten with the state
 * after the last token; y [T, Hv, 128] bf16; ckpt (may be NULL) [T-1, Hv, 128, 128] f32 receives
 * the state after each of tokens 0 .. T-2 for skinny_gdn_rollback. */
int skinny_gdn_recurrent(const void* q, const void* k, const void* v, const float* g,
                         const float* beta, float* state, void* y, float* ckpt, int T, int Hv, int Hk,
                         int Dk, int Dv, void* stream);

#define SKINNY_GDN_MAX_LAYERS 64

/* Replay-free rollback of all GDN layers after a verify of `fed` tokens that keeps the first
 * `keep`: state[l] <- ckpt[l][keep-1] when keep < fed (each state_elems f32), and, when conv is
 * not NULL, conv[l] [W, C] bf16 <- rows keep .. keep+W-1 of conv_full[l] [W + fed, C] bf16 (the
 * verify step's conv input: old window, then the fed tokens).  One launch for every layer.
 * Replaces skinny_mlx/rollback.py:58-73 (re-running the recurrence over the accepted prefix and
 * re-slicing the conv input); attention KV caches are trimmed on the host (a length update). */
int skinny_gdn_rollback(int n_layers, float* const* state, const float* const* ckpt,
                        void* const* conv, const void* const* conv_full, long long state_elems,
                        int keep, int fed, int W, int C, void* stream);

/* Attention caches after a TREE verify (skinny_attn_fused_tree appends node t at slot L0 + t):
 * in each of n_layers K and V caches ([max_len, ...] rows of row_bytes, 16-byte aligned) rows
 * L0[l] + path[j] move to rows L0[l] + j for j = 1 .. n_path - 1 (path: HOST array, the accepted
 * path 0, p1 .. pn, strictly increasing).  One launch; the caller then sets each length to
 * L0 + n_path.  The tree counterpart of KVCache.trim in skinny_mlx/rollback.py:72-73. */
int skinny_kv_compact(int n_layers, void* const* k_caches, void* const* v_caches, int row_bytes, const int32_t* L0,
                      const int32_t* path, int n_path, int max_len, void* stream);

/* Rollback of all GDN layers after a TREE verify of `fed` nodes whose accepted path ends at node
 * `node`: state[l] <- ckpt[l][node], conv[l] row q <- conv_full[l] row rows[q] for q < W (rows: a
 * HOST array, the last W conv inputs along the path: window rows 0 .. W-1, node t at W + t). */
int skinny_gdn_rollback_tree(int n_layers, float* const* state, const float* const* ckpt, void* const* conv,
                             const void* const* conv_full, long long state_elems, int node, const int32_t* rows,
                             int fed, int W, int C, void* stream);

/* skinny_qmm_w4g64 without a workspace argument and without allocating anything: no cudaMalloc,
 * no cudaFree, no allocating library routine.  It has NO counterpart in the reference; it exists
 * for callers that cannot provide or allocate device memory per call (a plain C FFI host with no
 * device-buffer type, a serving loop with a fixed memory budget, a step where an allocation's
 * implicit device synchronisation is not acceptable).  Its scratch is one static 3,744,000-byte
 * array in the library's device memory per device.  Limits: N <= 262,144 rows (2048 tiles of 128)
 * and K <= 32,768 columns; larger shapes return SKINNY_ERR_SCRATCH_LIMIT before anything is
 * launched.  The first call on a
 * device does the set-up (scratch address lookup, kernel attributes) and should come before any
 * stream capture; what it looks up is cached per device index, i.e. for the device's primary
 * context (the runtime API's): a host that switches driver-API contexts or resets the device
 * between calls is not supported.  Calls that may overlap on one device (other streams or threads without
 * ordering) race on the shared scratch; order them.  Each call clears the scratch's counters on
 * `stream` and then launches, without programmatic dependent launch. */
int skinny_qmm_w4g64_noalloc(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M,
                             int N, int K, void* stream);
/* The device error bits of the latest skinny_qmm_w4g64_noalloc call ordered before this one on
 * `stream` (a bounded wait inside the kernel that ran out; 0 = none), copied as one uint32 to dst
 * (device, pinned or pageable host memory) with a stream-ordered copy: read dst after the stream
 * reaches it (a pageable destination makes the copy wait for the stream).  Enqueue it before the
 * next no-alloc call on the device, which clears the word.  No counterpart in the reference; it
 * allocates nothing. */
int skinny_qmm_w4g64_noalloc_errors(void* dst, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SKINNY_B200_H */
