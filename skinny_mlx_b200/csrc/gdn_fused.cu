// One Gated DeltaNet mixer, from its fused input projection to the prepared input of out_proj,
// in one launch (the B200 form of everything between in_proj and out_proj of the reference
// model's GDN layer; skinny_mlx/rollback.py:14-56 records the same intermediate values):
//
//   full   = [conv window (W rows); qkv of the T new tokens]          (bf16)
//   c[t]   = silu( sum_j conv_w[:, j] * full[t + j] )                  (per channel)
//   q, k   = l2-normalised q and k heads of c (q / sqrt(128)),  v = v heads of c   (-> bf16)
//   g      = exp(-exp(A_log) * softplus(a + dt_bias)),  beta = sigmoid(b)
//   y      = gated delta recurrence over the T tokens (state updated, checkpoints written)
//   o      = bf16( bf16(rmsnorm(y) * (1 + w)) * silu(z) )
//   digits of o for out_proj (the qmm input format, prep.cu)
//
// Work split.  The recurrence is independent per state row (row = value channel): with
// S_t = g_t S_{t-1} + beta_t (v_t - S_{t-1} k_t g_t) k_t^T a row needs only its own v entry and
// the head's shared q_t, k_t.  A head is therefore one cluster of kRanks CTAs, each owning 16
// state rows (16 x 128 f32 in registers: 16 threads per row, 8 columns each), so a layer runs
// on Hv * 8 SMs instead of Hv.  Every CTA recomputes the head's q and k (conv, norm: a few
// hundred channels) rather than exchanging them.  The gated RMSNorm and the digits need whole
// 64-row groups of y, so each CTA pushes its y rows into the shared memory of every CTA
// of the head (distributed shared memory), and rank r finishes tokens r and r + 8.
//
// Token trees (speculative verify of a draft tree in one pass).  With parent != NULL the T inputs
// are the nodes of a tree in topological order (parent[0] = -1, parent[t] < t): node t's conv
// window is the W inputs before it on its ancestor path (the cached window above the root), and
// its recurrence starts from its parent's state -- carried in registers when the parent is node
// t - 1, else reloaded from the parent's checkpoint (which this thread itself wrote).  The state
// after EVERY node goes to ckpt[t]; neither `state` nor the conv window is written (the rollback
// selects the accepted path's last node and gathers the window along the path).
//
// Rounding points follow the unfused model (skinny_mlx_b200/model.py): q, k, v and y to bf16,
// the norm output to bf16, o to bf16.  Launched with programmatic dependent launch: the next
// launch may start at once (it streams weights) and this one waits for the previous grid before
// its first global read.
#include <atomic>
#include <cfloat>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "digits.cuh"
#include "ptx.cuh"
#include "qmm_layout.cuh"
#include "skinny_status.h"

namespace skinny {

constexpr int kGfThreads = 256;
constexpr int kGfD = 128;
constexpr int kGfMaxT = 16;
constexpr int kGfRanks = 8;                    // CTAs (cluster size) per head
constexpr int kGfRows = kGfD / kGfRanks;       // state rows per CTA
constexpr int kGfTpr = kGfThreads / kGfRows;   // threads per row (16)
constexpr int kGfCols = kGfD / kGfTpr;         // state columns per thread (8)
static_assert(kGfTpr == 16 && kGfCols == 8, "thread layout");

struct GdnFusedParams {
  const __nv_bfloat16* proj;  // [T, ldp]: q (Hk*128) | k (Hk*128) | v (Hv*128) | z (Hv*128) | b (Hv) | a (Hv)
  int ldp;
  __nv_bfloat16* conv;        // [W, C] window, updated
  __nv_bfloat16* conv_full;   // [W + T, C] recorded verify input, or null
  const float* conv_w;        // [C, W + 1]
  const float* A_log;         // [Hv]
  const float* dt_bias;       // [Hv]
  const float* norm_w;        // [128]
  float eps;
  float* state;               // [Hv, 128, 128]
  float* ckpt;                // [T - 1, Hv, 128, 128] or null
  uint8_t* xq;                // out_proj input digits (K = Hv * 128)
  __nv_bfloat16* o_out;       // [T, Hv * 128] bf16 copy of o, or null
  uint32_t* err;              // error word (kErrBitWaitCluster, kErrBitBadInput)
  const int32_t* parent;      // [T] tree of the T inputs, or null (a chain)
  int T, Hv, Hk;
};

__device__ __forceinline__ float bf16rf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// 16 bytes into another CTA's shared memory; its mbarrier counts the bytes.
__device__ __forceinline__ void st_async_v4(uint32_t addr, float4 v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   addr),
               "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)),
               "r"(__float_as_uint(v.w)), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

template <int W>
__global__ void __launch_bounds__(kGfThreads) gdn_fused_kernel(const __grid_constant__ GdnFusedParams p) {
  constexpr int kCh = 2 * kGfD + kGfRows;  // conv channels a CTA needs: q, k of its head; its 16 v
  constexpr int kVec = kCh / 8;            // 16-byte vectors per row of them
  constexpr int kRowsMax = W + kGfMaxT;
  constexpr int kStg = (kRowsMax * kVec + kGfThreads - 1) / kGfThreads;
  const int h = blockIdx.x / kGfRanks;
  const uint32_t rank = cluster_ctarank();
  const int r0 = static_cast<int>(rank) * kGfRows;
  const int rep = p.Hv / p.Hk;
  const int hk = h / rep;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.T;
  const int C = (2 * p.Hk + p.Hv) * kGfD;
  const int mpad = T <= 8 ? 8 : 16;
  __shared__ __align__(16) __nv_bfloat16 fw[kRowsMax][kCh];  // [window; new tokens] of the CTA's channels
  __shared__ float qs[kGfMaxT][kGfD], ks[kGfMaxT][kGfD];
  __shared__ float vs[kGfMaxT][kGfRows];
  __shared__ __align__(16) float yl[kGfMaxT][kGfRows];
  __shared__ __align__(16) float yall[kGfMaxT][kGfD];  // the head's y, pushed by every rank
  __shared__ float gs[kGfMaxT], bs[kGfMaxT], kq[kGfMaxT];  // gates; k_t . q_t
  __shared__ int8_t rsel[kGfMaxT][W + 1];  // rows of fw that form node t's conv window
  __shared__ int8_t par_s[kGfMaxT];        // parent node (-1: the root)
  __shared__ __align__(8) uint64_t ybar;
  __shared__ int abort_flag;
  // dynamic: the per-thread partials of S q for every token (summed after the recurrence) and u
  extern __shared__ __align__(16) float gdn_dyn[];
  float* bpart = gdn_dyn;                        // [kGfMaxT][kGfThreads]
  float* ust = gdn_dyn + kGfMaxT * kGfThreads;   // [kGfMaxT][kGfRows]

  // channel of CTA-local conv slot i: q (0..127) and k (128..255) of head hk, v rows r0..r0+15 of h
  const auto chan = [&](int i) {
    return i < kGfD ? hk * kGfD + i : i < 2 * kGfD ? (p.Hk + hk) * kGfD + (i - kGfD) : (2 * p.Hk + h) * kGfD + r0 + (i - 2 * kGfD);
  };

  if (tid == 0) {
    mbar_init(smem_u32(&ybar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  pdl_launch_dependents();
  pdl_wait_prior_grid();
  const bool tree = p.parent != nullptr;

  // ---- every global load, issued together
  const int row = tid / kGfTpr, sub = tid % kGfTpr;  // recurrence: (state row, column phase)
  const size_t srow = (static_cast<size_t>(h) * kGfD + r0 + row) * kGfD + sub;
  float S[kGfCols];
#pragma unroll
  for (int i = 0; i < kGfCols; ++i) S[i] = p.state[srow + kGfTpr * i];
  float ga = 0.f, gb = 0.f, gdt = 0.f, galog = 0.f;
  if (tid < T) {
    const size_t base = static_cast<size_t>(tid) * p.ldp + C + static_cast<size_t>(p.Hv) * kGfD;
    gb = __bfloat162float(p.proj[base + h]);
    ga = __bfloat162float(p.proj[base + p.Hv + h]);
    gdt = p.dt_bias[h];
    galog = p.A_log[h];
  }
  // digit job: warp w of rank r finishes token r + 8 (w / 2), column half w % 2
  const int jt = static_cast<int>(rank) + kGfRanks * (warp >> 1), jhalf = warp & 1;
  const int j0 = jhalf * 64 + 2 * lane;
  float z0 = 0.f, z1 = 0.f, nw0 = 0.f, nw1 = 0.f;
  if (jt < T) {
    const size_t zc = static_cast<size_t>(jt) * p.ldp + C + static_cast<size_t>(h) * kGfD + j0;
    z0 = __bfloat162float(p.proj[zc]);
    z1 = __bfloat162float(p.proj[zc + 1]);
    nw0 = p.norm_w[j0];
    nw1 = p.norm_w[j0 + 1];
  }
  // conv weights: channel tid (a q or k channel) and v channel 2*128 + (tid & 15)
  static_assert(kGfThreads == 2 * kGfD && kGfRows * kGfMaxT == kGfThreads, "conv work split");
  float cw[W + 1], cwv[W + 1];
#pragma unroll
  for (int q = 0; q <= W; ++q) {
    cw[q] = p.conv_w[static_cast<size_t>(chan(tid)) * (W + 1) + q];
    cwv[q] = p.conv_w[static_cast<size_t>(chan(2 * kGfD + (tid & 15))) * (W + 1) + q];
  }
  {
    const int nvec = (W + T) * kVec;
    uint4 stg[kStg];
#pragma unroll
    for (int u = 0; u < kStg; ++u) {
      const int e = tid + u * kGfThreads;
      if (e < nvec) {
        const int r = e / kVec, c = e - (e / kVec) * kVec;
        const int col = chan(8 * c);
        const __nv_bfloat16* src = r < W ? p.conv + static_cast<size_t>(r) * C + col
                                         : p.proj + static_cast<size_t>(r - W) * p.ldp + col;
        stg[u] = *reinterpret_cast<const uint4*>(src);
      }
    }
#pragma unroll
    for (int u = 0; u < kStg; ++u) {
      const int e = tid + u * kGfThreads;
      if (e < nvec) {
        const int r = e / kVec, c = e - (e / kVec) * kVec;
        *reinterpret_cast<uint4*>(&fw[r][8 * c]) = stg[u];
      }
    }
  }
  // Conv window rows and parents of every node.  fw rows: [0, W) the cached window, W + t node
  // t.  The row before node t's row is its parent's row (the last window row for the root), the
  // row before a window row the previous one.  A malformed tree (parent[0] != -1, parent[t] >= t
  // or < 0 for t > 0) is recorded and read as a chain.
  if (tid < T) {
    int pt = tid - 1;
    if (tree) {
      const int v = p.parent[tid];
      const bool ok = tid == 0 ? v == -1 : (v >= 0 && v < tid);
      if (!ok && rank == 0 && (blockIdx.x / kGfRanks) == 0) atomicOr(p.err, kErrBitBadInput);
      if (ok) pt = v;
    }
    par_s[tid] = static_cast<int8_t>(pt);
  }
  __syncthreads();
  if (tid < T) {
    int r = W + tid;
    rsel[tid][W] = static_cast<int8_t>(r);
#pragma unroll
    for (int q = W - 1; q >= 0; --q) {
      r = r >= W ? (par_s[r - W] >= 0 ? W + par_s[r - W] : W - 1) : r - 1;
      rsel[tid][q] = static_cast<int8_t>(r);
    }
  }
  __syncthreads();
  // Arrive once this CTA's mbarrier exists and its reads of the conv window are complete: a peer
  // writes its share of the new window, and stores into this CTA's shared memory, only after the
  // matching wait.
  cluster_arrive_relaxed();

  // ---- conv + silu.  Thread tid: q/k channel tid for every token, and v channel tid & 15 for
  // token tid >> 4, so that no thread has more than T + 1 outputs.
  {
    const int part = tid < kGfD ? 0 : 1;
    const int j = tid - part * kGfD;
#pragma unroll 4
    for (int t = 0; t < T; ++t) {
      float acc = 0.f;
#pragma unroll
      for (int q = 0; q <= W; ++q) acc = fmaf(__bfloat162float(fw[rsel[t][q]][tid]), cw[q], acc);
      const float sv = __fdividef(acc, 1.f + __expf(-acc));
      if (part == 0) qs[t][j] = sv;
      else ks[t][j] = sv;
    }
    const int tv = tid >> 4, jv = tid & 15;
    if (tv < T) {
      float acc = 0.f;
#pragma unroll
      for (int q = 0; q <= W; ++q) acc = fmaf(__bfloat162float(fw[rsel[tv][q]][2 * kGfD + jv]), cwv[q], acc);
      vs[tv][jv] = bf16rf(__fdividef(acc, 1.f + __expf(-acc)));
    }
  }
  __syncthreads();
  // ---- l2-normalised q (/ sqrt(128)) and k, bf16 (warp per token); gates
  for (int t = warp; t < T; t += kGfThreads / 32) {
    float qv[4], kv[4], sq = 0.f, sk = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      qv[u] = qs[t][lane + 32 * u];
      kv[u] = ks[t][lane + 32 * u];
      sq = fmaf(qv[u], qv[u], sq);
      sk = fmaf(kv[u], kv[u], sk);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
      sk += __shfl_xor_sync(0xFFFFFFFFu, sk, o);
    }
    const float nq = rsqrtf(static_cast<float>(kGfD)) / fmaxf(sqrtf(sq), 1e-12f);
    const float nk = 1.f / fmaxf(sqrtf(sk), 1e-12f);
    float c = 0.f;  // k_t . q_t of the rounded vectors (the same for every state row)
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float qr = bf16rf(qv[u] * nq), kr = bf16rf(kv[u] * nk);
      qs[t][lane + 32 * u] = qr;
      ks[t][lane + 32 * u] = kr;
      c = fmaf(kr, qr, c);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
    if (lane == 0) kq[t] = c;
  }
  if (tid < T) {
    const float xa = ga + gdt;
    const float sp = xa > 20.f ? xa : log1pf(expf(xa));
    gs[tid] = expf(-expf(galog) * sp);
    bs[tid] = 1.f / (1.f + expf(-gb));
  }
  __syncthreads();
  // ---- recurrence: thread = (row, sub); columns sub + 8 i in registers.  Per token only a = S k
  // (of the previous state) is reduced across the row's lanes; the partials of b = S q are kept
  // and summed after the loop, and c = k q comes from the norm phase:
  //   u = beta (v - g a),   S <- g S + u k^T,   y = S q = g b + u c.
  // The next token's operands are loaded while the current token's reductions run; the
  // arithmetic per token is the same whatever T is, so a token's results do not depend on how
  // many tokens share the launch.
  float kn[kGfCols], qn[kGfCols], gn = 0.f, bn = 0.f, vn = 0.f;
  const auto load_tok = [&](int t) {
    gn = gs[t];
    bn = bs[t];
    vn = vs[t][row];
#pragma unroll
    for (int i = 0; i < kGfCols; ++i) {
      kn[i] = ks[t][sub + kGfTpr * i];
      qn[i] = qs[t][sub + kGfTpr * i];
    }
  };
  if (T > 0) load_tok(0);
  for (int t = 0; t < T; ++t) {
    const float gt = gn, bt = bn, vt = vn;
    float kk[kGfCols], qq[kGfCols];
#pragma unroll
    for (int i = 0; i < kGfCols; ++i) {
      kk[i] = kn[i];
      qq[i] = qn[i];
    }
    if (t + 1 < T) load_tok(t + 1);
    if (tree && t > 0 && par_s[t] != t - 1) {  // a branch: start from the parent's checkpoint
      const float* cp = p.ckpt + static_cast<size_t>(par_s[t]) * p.Hv * kGfD * kGfD + srow;
#pragma unroll
      for (int i = 0; i < kGfCols; ++i) S[i] = cp[kGfTpr * i];
    }
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
    for (int i = 0; i < kGfCols; i += 2) {
      a0 = fmaf(S[i], kk[i], a0);
      a1 = fmaf(S[i + 1], kk[i + 1], a1);
      b0 = fmaf(S[i], qq[i], b0);
      b1 = fmaf(S[i + 1], qq[i + 1], b1);
    }
    float a = a0 + a1;
    bpart[t * kGfThreads + tid] = b0 + b1;  // reduced after the recurrence: off the token chain
#pragma unroll
    for (int o = 1; o < kGfTpr; o <<= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    const float u = bt * (vt - gt * a);
#pragma unroll
    for (int i = 0; i < kGfCols; ++i) S[i] = fmaf(u, kk[i], gt * S[i]);
    if (sub == 0) ust[t * kGfRows + row] = u;
    if (p.ckpt && (tree || t + 1 < T)) {
      float* cp = p.ckpt + static_cast<size_t>(t) * p.Hv * kGfD * kGfD + srow;
#pragma unroll
      for (int i = 0; i < kGfCols; ++i) cp[kGfTpr * i] = S[i];
    }
  }
  if (!tree) {
#pragma unroll
    for (int i = 0; i < kGfCols; ++i) p.state[srow + kGfTpr * i] = S[i];
  }
  __syncthreads();
  // y = g b + u c per (token, row): b summed from the 16 column partials in the order of the
  // lane butterfly (pairs, then pairs of pairs, ...), which is the same value in every lane
  {
    const int t = tid >> 4, rw = tid & 15;
    if (t < T) {
      const float4* pb = reinterpret_cast<const float4*>(bpart + t * kGfThreads + rw * kGfTpr);
      float pv[16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v = pb[i];
        pv[4 * i] = v.x;
        pv[4 * i + 1] = v.y;
        pv[4 * i + 2] = v.z;
        pv[4 * i + 3] = v.w;
      }
      float s1[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) s1[i] = pv[2 * i] + pv[2 * i + 1];
      const float s2a = s1[0] + s1[1], s2b = s1[2] + s1[3], s2c = s1[4] + s1[5], s2d = s1[6] + s1[7];
      const float b = (s2a + s2b) + (s2c + s2d);
      yl[t][rw] = bf16rf(fmaf(gs[t], b, ust[t * kGfRows + rw] * kq[t]));
    }
  }
  __syncthreads();
  // ---- every rank receives the head's whole y: 16-byte asynchronous stores into each peer's
  // shared memory, counted on the peer's mbarrier (no cluster-wide release of global stores)
  cluster_wait();  // all peers have initialised their mbarriers and read the old window
  // ---- conv_full (the verify's conv input) and the new window (its last W rows), 16-byte
  // stores from the staged rows.  One writer per channel: this CTA's v channels, and q/k
  // channels 16 rank .. 16 rank + 15 when h is the first value head of its k head.
  {
    const int runs = (h % rep) == 0 ? 3 : 1;  // 8-channel vectors per row: 2 per run
    const int per_row = 2 * runs;
    const int n_full = p.conv_full ? (W + T) * per_row : 0;
    const int n_win = tree ? 0 : W * per_row;  // (a tree's window is gathered by the rollback)
    for (int e = tid; e < n_full + n_win; e += kGfThreads) {
      const bool full = e < n_full;
      const int e2 = full ? e : e - n_full;
      const int r = e2 / per_row, v = e2 - r * per_row;
      const int run = runs == 3 ? v >> 1 : 2;  // 0: q, 1: k, 2: v
      const int slot = (run == 2 ? 2 * kGfD : run * kGfD + static_cast<int>(rank) * kGfRows) + (v & 1) * 8;
      const uint4 val = *reinterpret_cast<const uint4*>(&fw[full ? r : T + r][slot]);
      __nv_bfloat16* dst = full ? p.conv_full + static_cast<size_t>(r) * C : p.conv + static_cast<size_t>(r) * C;
      *reinterpret_cast<uint4*>(dst + chan(slot)) = val;
    }
  }
  {
    const uint32_t ybase = smem_u32(&yall[0][0]), ybl = smem_u32(&ybar);
    for (int i = tid; i < T * (kGfRows / 4) * kGfRanks; i += kGfThreads) {
      const int dst = i % kGfRanks, e = i / kGfRanks;
      const int t = e / (kGfRows / 4), r4 = (e % (kGfRows / 4)) * 4;
      const float4 v = *reinterpret_cast<const float4*>(&yl[t][r4]);
      const uint32_t off = static_cast<uint32_t>((t * kGfD + r0 + r4) * 4);
      st_async_v4(map_shared_rank(ybase + off, dst), v, map_shared_rank(ybl, dst));
    }
    if (tid == 0) mbar_arrive_expect_tx(ybl, static_cast<uint32_t>(T * kGfD * 4));
    if (!mbar_wait(ybl, 0, p.err, kErrBitWaitCluster, &abort_flag)) return;
  }
  // ---- gated rmsnorm and digits: warp w of rank r takes token r + 8 (w / 2), column half w % 2
  if (jt < mpad) {
    float a0 = 0.f, a1 = 0.f;
    if (jt < T) {
      float ss = 0.f;
#pragma unroll
      for (int j = lane; j < kGfD; j += 32) ss = fmaf(yall[jt][j], yall[jt][j], ss);
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
      const float rstd = rsqrtf(ss / kGfD + p.eps);
      const float n0 = bf16rf(yall[jt][j0] * rstd * (1.f + nw0));
      const float n1 = bf16rf(yall[jt][j0 + 1] * rstd * (1.f + nw1));
      a0 = bf16rf(n0 * (z0 / (1.f + __expf(-z0))));
      a1 = bf16rf(n1 * (z1 / (1.f + __expf(-z1))));
      if (p.o_out) {
        __nv_bfloat16* op = p.o_out + static_cast<size_t>(jt) * p.Hv * kGfD + h * kGfD + j0;
        op[0] = __float2bfloat16_rn(a0);
        op[1] = __float2bfloat16_rn(a1);
      }
    }
    write_digits(p.xq, mpad, jt, 2 * h + jhalf, lane, a0, a1);
  }
}

// Host-side mirror of the parameter block with untyped pointers (the C-ABI layer's view).
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

constexpr size_t kGfDynBytes = (kGfMaxT * kGfThreads + kGfMaxT * kGfRows) * sizeof(float);

// One or two CTAs per SM.  Under programmatic dependent launch this kernel's CTAs become resident while
// the previous launch (a qmm of one CTA per SM) still holds most SMs, and the block scheduler
// packs them onto the few free SMs, up to four per SM: those CTAs then take about 1.6x as long
// (measured in a verify step with per-CTA %smid / %globaltimer records).  Asking for more than
// half (a third) of an SM's shared memory keeps at most one (two) CTAs on an SM; the padding is
// used only where the GPU can hold every cluster of the launch at once (else the launch would
// run in waves).
template <int W>
static cudaError_t launch_gdn_fused(const GdnFusedParams& prm, cudaStream_t stream) {
  static std::atomic<int> dyn_for[64][65];  // per device and value-head count: the dynamic shared memory used
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(prm.Hv * kGfRanks);
  cfg.blockDim = dim3(kGfThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kGfRanks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  int dyn = dyn_for[dev][min(prm.Hv, 64)].load(std::memory_order_acquire);
  if (dyn == 0) {
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, gdn_fused_kernel<W>);
    int smem_sm = 0;
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (e != cudaSuccess) return e;
    // at most one, else at most two CTAs per SM (more than a half, a third of its shared memory);
    // the kernel's limit stays at the largest size any launch may use
    const int pad1 = max(static_cast<int>(kGfDynBytes), smem_sm / 2 + 1024 - static_cast<int>(fa.sharedSizeBytes));
    e = cudaFuncSetAttribute(gdn_fused_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize, pad1);
    if (e != cudaSuccess) return e;
    dyn = static_cast<int>(kGfDynBytes);
    for (int per_sm = 1; per_sm <= 2; ++per_sm) {
      const int padded = max(static_cast<int>(kGfDynBytes),
                             smem_sm / (per_sm + 1) + 1024 - static_cast<int>(fa.sharedSizeBytes));
      int clusters = 0;
      cfg.dynamicSmemBytes = padded;
      if (cudaOccupancyMaxActiveClusters(&clusters, gdn_fused_kernel<W>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        clusters = 0;
      }
      if (clusters >= prm.Hv) {
        dyn = padded;
        break;
      }
    }
  }
  dyn_for[dev][min(prm.Hv, 64)].store(dyn, std::memory_order_release);  // (the same value from any thread)
  cfg.dynamicSmemBytes = dyn;
  return cudaLaunchKernelEx(&cfg, gdn_fused_kernel<W>, prm);
}

cudaError_t gdn_fused_call(const GdnFusedParamsHost& h, cudaStream_t stream) {
  GdnFusedParams prm{static_cast<const __nv_bfloat16*>(h.proj), h.ldp, static_cast<__nv_bfloat16*>(h.conv),
                     static_cast<__nv_bfloat16*>(h.conv_full), h.conv_w, h.A_log, h.dt_bias, h.norm_w, h.eps,
                     h.state, h.ckpt, static_cast<uint8_t*>(h.xq), static_cast<__nv_bfloat16*>(h.o_out),
                     h.err, h.parent, h.T, h.Hv, h.Hk};
  switch (h.W) {
    case 1: return launch_gdn_fused<1>(prm, stream);
    case 2: return launch_gdn_fused<2>(prm, stream);
    case 3: return launch_gdn_fused<3>(prm, stream);
    case 4: return launch_gdn_fused<4>(prm, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace skinny
