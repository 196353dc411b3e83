// One full-attention mixer, from its fused projection to the prepared input of o_proj (the B200
// form of the attention layers of the model the reference patches, run during a verify step of
// T <= 16 tokens against a KV cache):
//
//   q, k  = RoPE( bf16(rmsnorm(q|k) * (1 + w)) )  on the first `rot` dims, positions L0 .. L0+T-1
//   cache[L0 .. L0+T-1] = bf16(k), v                                (KV append)
//   o     = softmax(q k^T / sqrt(128), causal bottom-right) v        (GQA: rep = n_heads / n_kv)
//   o     = bf16( bf16(o) * sigmoid(gate) )  (gated layers; else bf16(o))  -> digits of o for o_proj
//
// Two launches, split over keys (flash-decode style):
//   attn_chunk_kernel  CTA (128-key chunk, KV head): loads the chunk's keys and values once,
//                      then in passes of up to three 16-row tiles of query rows (row = t * rep +
//                      q head in the group) computes the chunk's row maxima, sums and
//                      unnormalised outputs on bf16 tensor-core tiles and publishes them.  The
//                      new keys of the chunk are normalised, rotated and appended to the cache by
//                      that CTA (positions >= L0 are only written, positions < L0 only read, so
//                      chunks never race).
//   attn_merge_kernel  CTA (one query row, KV head): merges the chunks (a fixed order:
//                      deterministic), applies the gate and writes the digits.
// Token trees: with parent != NULL the T new tokens are the nodes of a draft tree in topological
// order (parent[0] = -1, parent[t] < t).  Node t sits at position L0 + depth(t) (RoPE of its q
// and k) and sees the cached keys plus the new keys of its ancestors and itself; its key and
// value are appended at slot L0 + t (the rollback moves the accepted path's slots into place).
// No CTA waits on another; the merge launch waits for the chunk launch through programmatic
// dependent launch, like every launch of the step (the next launch may start at once; a kernel
// waits for the previous grid before its first global read).
#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "digits.cuh"
#include "mma_bf16.cuh"
#include "peer.cuh"
#include "ptx.cuh"
#include "qmm_layout.cuh"

namespace skinny {

constexpr int kAtD = 128;
constexpr int kAtChunk = 128;        // keys per CTA
constexpr int kAtRG = 16;            // query rows per tensor-core tile
constexpr int kAtThreads = 256;
constexpr int kAtWarps = kAtThreads / 32;
constexpr int kAtStride = kAtD + 8;   // bf16 per shared row: 272 bytes, ldmatrix conflict-free
constexpr int kAtPart = kAtD + 4;     // floats per published row: m, l, (pad), o[128] (16-byte aligned)
constexpr int kAtMaxRG = 8;           // row groups per KV head (rep * T <= 128)
constexpr int kAtMergeRows = 1;       // query rows per merge CTA
constexpr int kAtMergeSub = 16;       // chunk subsets per row (threads per (row, 8 dims))
constexpr int kAtMergePass = 3;       // chunk partials whose loads a merging thread issues together
constexpr int kAtMaxT = 16;

struct AttnParams {
  const __nv_bfloat16* proj;  // [T, ldp]: q heads (q | gate per head when gated) | k (nkv x 128) | v
  int ldp;
  const float* qn_w;          // [128] zero-centred RMSNorm weights
  const float* kn_w;
  const float* inv_freq;      // [rot / 2] rotary frequencies
  float eps;
  __nv_bfloat16* kc;          // [max_len, nkv, 128]
  __nv_bfloat16* vc;
  int T, L0, nh, nkv, rot, nchunks, nrg, max_len;
  int gated;                  // 1: per head [q | gate] and o *= sigmoid(gate); 0: q heads only
  const int* len_dev;         // if set: the cache length is read here (grid sized for max_len)
  const int32_t* parent;      // [T] tree of the new tokens, or null (a chain)
  float* part;                // [nkv, nrg, nchunks, 16, kAtPart]: per row m, l, -, -, o[128]
  uint8_t* xq;                // o_proj input digits (K = nh * 128)
  __nv_bfloat16* o_out;       // [T, nh * 128] or null
  PeerSync sync;              // (sharded step) the merge launch signals its completion
};

constexpr int kAtMaxRows = kAtRG * kAtMaxRG;  // query rows of one KV head (T * rep)

constexpr int kAtPassTiles = 3;                      // 16-row tiles of one pass of a chunk CTA
constexpr int kAtPassRows = kAtRG * kAtPassTiles;    // query rows per pass

struct AttnSmem {
  float cs[kAtMaxT][kAtD / 2][2];            // cos / sin of (position, frequency), computed once
  float qw[kAtD], kw[kAtD];                  // q / k norm weights
  __nv_bfloat16 q[kAtPassRows][kAtStride];   // normalised, rotated query rows of the pass
  __nv_bfloat16 k[kAtChunk][kAtStride];      // keys of the chunk
  __nv_bfloat16 v[kAtChunk][kAtStride];      // values of the chunk
  __nv_bfloat16 pr[kAtPassRows][kAtStride];  // probabilities (bf16, as a flash kernel rounds them)
  float redm[kAtWarps][kAtPassRows];         // per (warp = 16-key block, row): max of the block
  float redl[kAtWarps][kAtPassRows];         //                                sum of its probabilities
  int dep[kAtMaxT];                          // tree: depth of every new token
  uint32_t anc[kAtMaxT];                     //       its ancestors and itself (bit per token)
};

__device__ __forceinline__ float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Loads issued where they stand (volatile: the compiler neither sinks them towards their first
// use nor splits a batch of them into several round trips).  nc: data that no launch writes while
// this one runs; cg: data written by the previous launch (read from L2).
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ float ld_nc_f32(const float* p) {
  float r;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ float4 ld_cg_v4(const float* p) {
  float4 r;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ float2 ld_cg_v2(const float* p) {
  float2 r;
  asm volatile("ld.global.cg.v2.f32 {%0, %1}, [%2];" : "=f"(r.x), "=f"(r.y) : "l"(p));
  return r;
}

// Half-warp collective (16 lanes; lane pc holds dims 8 pc .. 8 pc + 7 of one head row, bf16-exact;
// both halves of the warp call it together, each for its own row): zero-centred RMSNorm (-> bf16)
// and RoPE on the first rot dims (-> bf16), rot in {0, 16, 32, 64, 128}, so the partner dims
// d +- rot/2 sit in lane pc ^ (rot / 16).
__device__ __forceinline__ void norm_rope_hw(float (&x)[8], const float* w, float eps, const float (*cs)[2], int rot,
                                             int pc) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int o = 8; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  const float rstd = rsqrtf(ss / kAtD + eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = bfr(x[i] * rstd * (1.f + w[8 * pc + i]));
  const int half = rot >> 1;
  const int px = rot >= 16 ? rot >> 4 : 0;
  float y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) y[i] = __shfl_xor_sync(0xFFFFFFFFu, x[i], px);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = 8 * pc + i;
    if (d < rot) {
      const int j = d < half ? d : d - half;
      const float c = cs[j][0], sn = cs[j][1];
      x[i] = d < half ? x[i] * c - y[i] * sn : x[i] * c + y[i] * sn;
    }
    x[i] = bfr(x[i]);
  }
}

// The cache length: a kernel argument, or read from device memory so that one captured launch
// serves every length (the chunk grid then covers max_len and the surplus chunks leave).
// Returns -1 for a device length out of range (the launch then touches nothing).
__device__ __forceinline__ int attn_length(const AttnParams& p) {
  const int L0 = p.len_dev ? *p.len_dev : p.L0;
  return (L0 < 0 || L0 + p.T > p.max_len) ? -1 : L0;
}

__device__ __forceinline__ float* part_row(const AttnParams& p, int kvh, int rg, int chunk, int rr) {
  return p.part + (((static_cast<size_t>(kvh) * p.nrg + rg) * p.nchunks + chunk) * kAtRG + rr) * kAtPart;
}

__global__ void __launch_bounds__(kAtThreads, 2) attn_chunk_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint8_t at_smem_raw[];
  AttnSmem& sm = *reinterpret_cast<AttnSmem*>(at_smem_raw);
  const int chunk = blockIdx.x, kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rep = p.nh / p.nkv;
  const int R = p.T * rep;
  const int qstride = p.gated ? 2 * kAtD : kAtD;  // proj columns per query head
  const int qkw = p.nh * qstride;                  // column of k in proj
  pdl_launch_dependents();
  pdl_wait_prior_grid();
  const int L0 = attn_length(p);
  if (L0 < 0) return;
  const int nchunks = (L0 + p.T + kAtChunk - 1) / kAtChunk;
  if (chunk >= nchunks) return;
  const int Ltot = L0 + p.T;
  const int k0 = chunk * kAtChunk;
  const int nk = min(kAtChunk, Ltot - k0);
  const int half = p.rot >> 1;

  // ---- every load of the CTA issued together: cached keys and values of the chunk, the KV head's
  // query rows (kept in registers: thread = (row (tid >> 4) + 16 u, dims 8 (tid & 15) ..)), the
  // norm weights and the rotary frequencies of the position table
  constexpr int kPieces = kAtChunk * (kAtD / 8);  // 16-byte pieces per matrix
  constexpr int kPer = kPieces / kAtThreads;
  constexpr int kQPer = kAtMaxRows * (kAtD / 8) / kAtThreads;
  constexpr int kTabPer = kAtMaxT * (kAtD / 2) / kAtThreads;
  const int pc = tid & 15;
  uint4 qv[kQPer];
  // Query rows of the pass starting at row rbase (ntiles 16-row tiles): normalised and rotated from
  // registers (half-warp per row) into sm.q; rows past R inside the pass's tiles are zero.
  const auto norm_pass = [&](int rbase, int ntiles) {
#pragma unroll
    for (int u = 0; u < kQPer; ++u) {
      const int r = (tid >> 4) + 16 * u;  // rows 16u .. 16u+15 are in one pass: warp-uniform test
      if (r >= rbase && r < rbase + ntiles * kAtRG) {
        if (u >= kAtPassTiles && r < R) {
          const int t = r / rep, hq = kvh * rep + r % rep;
          qv[u] = ld_nc_v4(p.proj + static_cast<size_t>(t) * p.ldp + hq * qstride + 8 * pc);
        }
        float x[8];
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&qv[u]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h2[i]);
          x[2 * i] = f.x;
          x[2 * i + 1] = f.y;
        }
        const int t = min(r / rep, p.T - 1);
        norm_rope_hw(x, sm.qw, p.eps, sm.cs[t], p.rot, pc);
        uint4 packed;
        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          o2[i] = r < R ? __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]) : __floats2bfloat162_rn(0.f, 0.f);
        *reinterpret_cast<uint4*>(&sm.q[r - rbase][8 * pc]) = packed;
      }
    }
  };
  {
    uint4 kw[kPer], vw[kPer];
#pragma unroll
    for (int u = 0; u < kQPer; ++u) {  // rows of the first pass now, the others when their pass starts
      const int r = (tid >> 4) + 16 * u;
      qv[u] = make_uint4(0u, 0u, 0u, 0u);
      if (u < kAtPassTiles && r < R) {
        const int t = r / rep, hq = kvh * rep + r % rep;
        qv[u] = ld_nc_v4(p.proj + static_cast<size_t>(t) * p.ldp + hq * qstride + 8 * pc);
      }
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = tid + u * kAtThreads, j = e >> 4, pce = e & 15;
      const int pos = k0 + j;
      if (j < nk && pos < L0) {
        const size_t off = (static_cast<size_t>(pos) * p.nkv + kvh) * kAtD + 8 * pce;
        kw[u] = ld_nc_v4(p.kc + off);
        vw[u] = ld_nc_v4(p.vc + off);
      } else {
        kw[u] = make_uint4(0u, 0u, 0u, 0u);
        vw[u] = kw[u];
      }
    }
    // the chunk's new keys (positions L0 .. L0+T-1 that fall in it, at most 16): half-warp per key
    const int jnew = max(L0 - k0, 0) + (tid >> 4);
    const bool has_new = jnew < nk;
    uint4 knew = make_uint4(0u, 0u, 0u, 0u), vnew = knew;
    if (has_new) {
      const __nv_bfloat16* src = p.proj + static_cast<size_t>(k0 + jnew - L0) * p.ldp + qkw;
      knew = ld_nc_v4(src + kvh * kAtD + 8 * pc);
      vnew = ld_nc_v4(src + p.nkv * kAtD + kvh * kAtD + 8 * pc);
    }
    const float nwv = ld_nc_f32(tid < kAtD ? p.qn_w + tid : p.kn_w + (tid - kAtD));
    float fr[kTabPer];
#pragma unroll
    for (int u = 0; u < kTabPer; ++u) {
      const int i = tid + u * kAtThreads;
      fr[u] = 0.f;
      if (half > 0 && i < p.T * half) fr[u] = ld_nc_f32(p.inv_freq + i % half);
    }
    if (tid < kAtD) sm.qw[tid] = nwv;
    else sm.kw[tid - kAtD] = nwv;
    if (p.parent) {  // tree: depth and ancestor set of every node (warp 0, by shuffles)
      if (warp == 0) {
        int par = lane - 1;
        if (lane < p.T) {
          const int v = p.parent[lane];
          if (lane == 0 ? v == -1 : (v >= 0 && v < lane)) par = v;  // else read as a chain
        }
        int cur = lane, d = 0;
        uint32_t m = lane < p.T ? 1u << lane : 0u;
#pragma unroll
        for (int it = 0; it < kAtMaxT; ++it) {
          const int pc = __shfl_sync(0xFFFFFFFFu, par, cur & 31);
          if (cur >= 0 && pc >= 0) {
            m |= 1u << pc;
            ++d;
          }
          cur = cur >= 0 ? pc : -1;
        }
        if (lane < p.T) {
          sm.dep[lane] = d;
          sm.anc[lane] = m;
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < kTabPer; ++u) {
      const int i = tid + u * kAtThreads;
      if (half > 0 && i < p.T * half) {
        const int t = i / half, j = i - t * half;
        float sn, c;
        sincosf(static_cast<float>(L0 + (p.parent ? sm.dep[t] : t)) * fr[u], &sn, &c);
        sm.cs[t][j][0] = c;
        sm.cs[t][j][1] = sn;
      }
    }
    __syncthreads();  // the position table and the norm weights
    // the first pass's query rows are normalised while the cached keys and values are still
    // arriving; then those are stored
    norm_pass(0, min(kAtPassTiles, (R + kAtRG - 1) / kAtRG));
    // new keys: normalised, rotated (every warp takes part in the shuffles), appended to the cache
    if (__any_sync(0xFFFFFFFFu, has_new)) {
      float x[8];
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&knew);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
      }
      const int t = has_new ? k0 + jnew - L0 : 0;
      norm_rope_hw(x, sm.kw, p.eps, sm.cs[t], p.rot, pc);
      if (has_new) {
        uint4 kb;
        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&kb);
#pragma unroll
        for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
        *reinterpret_cast<uint4*>(&sm.k[jnew][8 * pc]) = kb;
        *reinterpret_cast<uint4*>(&sm.v[jnew][8 * pc]) = vnew;
        const size_t off = (static_cast<size_t>(k0 + jnew) * p.nkv + kvh) * kAtD + 8 * pc;
        *reinterpret_cast<uint4*>(p.kc + off) = kb;
        *reinterpret_cast<uint4*>(p.vc + off) = vnew;
      }
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = tid + u * kAtThreads, j = e >> 4, pce = e & 15;
      if (j < nk && k0 + j >= L0) continue;  // a new key: written below by its warp
      *reinterpret_cast<uint4*>(&sm.k[j][8 * pce]) = kw[u];
      *reinterpret_cast<uint4*>(&sm.v[j][8 * pce]) = vw[u];
    }
  }
  __syncthreads();
  // ---- passes of up to three 16-row tiles: scores, softmax and outputs of all the pass's rows
  // together (warp w: keys 16w .. 16w+15 for the scores, dims 16w .. 16w+15 for the outputs)
  const int g = lane >> 2, cq = lane & 3;
  const float sc = rsqrtf(static_cast<float>(kAtD)) * 1.4426950408889634f;
  for (int rbase = 0; rbase < R; rbase += kAtPassRows) {
    const int nrows = min(kAtPassRows, R - rbase);
    const int ntiles = (nrows + kAtRG - 1) / kAtRG;
    if (rbase > 0) norm_pass(rbase, ntiles);  // (the first pass's rows were done while staging)
    __syncthreads();
    // scores (log2 domain), masked; each warp's 16-key maximum per row
    float c[kAtPassTiles][2][4];
#pragma unroll
    for (int rt = 0; rt < kAtPassTiles; ++rt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) c[rt][nt][e] = 0.f;
    {
      const uint32_t a_addr =
          smem_u32(&sm.q[0][0]) + (((lane & 7) + 8 * ((lane >> 3) & 1)) * kAtStride + 8 * (lane >> 4)) * 2;
      const uint32_t b_addr =
          smem_u32(&sm.k[0][0]) + ((16 * warp + (lane & 7) + 8 * (lane >> 4)) * kAtStride + 8 * ((lane >> 3) & 1)) * 2;
#pragma unroll
      for (int ks = 0; ks < kAtD / 16; ++ks) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b_addr + ks * 32, b0, b1, b2, b3);
#pragma unroll
        for (int rt = 0; rt < kAtPassTiles; ++rt) {
          if (rt < ntiles) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(a_addr + (rt * kAtRG * kAtStride) * 2 + ks * 32, a0, a1, a2, a3);
            mma_bf16(c[rt][0], a0, a1, a2, a3, b0, b1);
            mma_bf16(c[rt][1], a0, a1, a2, a3, b2, b3);
          }
        }
      }
    }
#pragma unroll
    for (int rt = 0; rt < kAtPassTiles; ++rt) {
      if (rt < ntiles) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int rr = rt * kAtRG + g + 8 * hf;
          const int t = min((rbase + rr) / rep, p.T - 1);
          const uint32_t anc = p.parent ? sm.anc[t] : (2u << t) - 1u;  // new keys row t sees
          float m = -INFINITY;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int j = 16 * warp + 8 * nt + 2 * cq + e;
              const int rel = k0 + j - L0;  // < 0: a cached key
              const bool vis = j < nk && (rel < 0 || ((anc >> rel) & 1u));
              const float v = vis ? c[rt][nt][2 * hf + e] * sc : -INFINITY;
              c[rt][nt][2 * hf + e] = v;
              m = fmaxf(m, v);
            }
          m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
          m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
          if (cq == 0) sm.redm[warp][rr] = m;
        }
      }
    }
    __syncthreads();
    // probabilities (bf16) with the row maximum over the chunk; each warp's partial sums
#pragma unroll
    for (int rt = 0; rt < kAtPassTiles; ++rt) {
      if (rt < ntiles) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int rr = rt * kAtRG + g + 8 * hf;
          float m = sm.redm[0][rr];
#pragma unroll
          for (int w = 1; w < kAtWarps; ++w) m = fmaxf(m, sm.redm[w][rr]);
          float l = 0.f;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const float e0 = m == -INFINITY ? 0.f : exp2f(c[rt][nt][2 * hf] - m);
            const float e1 = m == -INFINITY ? 0.f : exp2f(c[rt][nt][2 * hf + 1] - m);
            const __nv_bfloat162 pb = __floats2bfloat162_rn(e0, e1);
            *reinterpret_cast<__nv_bfloat162*>(&sm.pr[rr][16 * warp + 8 * nt + 2 * cq]) = pb;
            const float2 pf = __bfloat1622float2(pb);  // the probabilities as the products use them
            l += pf.x;
            l += pf.y;
          }
          l += __shfl_xor_sync(0xFFFFFFFFu, l, 1);
          l += __shfl_xor_sync(0xFFFFFFFFu, l, 2);
          if (cq == 0) sm.redl[warp][rr] = l;
        }
      }
    }
    __syncthreads();
    // unnormalised outputs on tensor cores; publish them with each row's (max, sum)
    {
      float o[kAtPassTiles][2][4];
#pragma unroll
      for (int rt = 0; rt < kAtPassTiles; ++rt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) o[rt][nt][e] = 0.f;
      const uint32_t a_addr =
          smem_u32(&sm.pr[0][0]) + (((lane & 7) + 8 * ((lane >> 3) & 1)) * kAtStride + 8 * (lane >> 4)) * 2;
      const uint32_t b_addr =
          smem_u32(&sm.v[0][0]) + (((lane & 7) + 8 * ((lane >> 3) & 1)) * kAtStride + 16 * warp + 8 * (lane >> 4)) * 2;
#pragma unroll
      for (int ks = 0; ks < kAtChunk / 16; ++ks) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(b_addr + ks * 16 * kAtStride * 2, b0, b1, b2, b3);
#pragma unroll
        for (int rt = 0; rt < kAtPassTiles; ++rt) {
          if (rt < ntiles) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(a_addr + (rt * kAtRG * kAtStride) * 2 + ks * 32, a0, a1, a2, a3);
            mma_bf16(o[rt][0], a0, a1, a2, a3, b0, b1);
            mma_bf16(o[rt][1], a0, a1, a2, a3, b2, b3);
          }
        }
      }
#pragma unroll
      for (int rt = 0; rt < kAtPassTiles; ++rt) {
        if (rt < ntiles) {
          const int rg = (rbase + rt * kAtRG) / kAtRG;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              const int rr = g + 8 * hf;
              if (rt * kAtRG + rr < nrows)
                *reinterpret_cast<float2*>(part_row(p, kvh, rg, chunk, rr) + 4 + 16 * warp + 8 * nt + 2 * cq) =
                    make_float2(o[rt][nt][2 * hf], o[rt][nt][2 * hf + 1]);
            }
        }
      }
      if (tid < nrows) {
        float m = sm.redm[0][tid], l = sm.redl[0][tid];
#pragma unroll
        for (int w = 1; w < kAtWarps; ++w) {
          m = fmaxf(m, sm.redm[w][tid]);
          l += sm.redl[w][tid];
        }
        float* row = part_row(p, kvh, (rbase + tid) / kAtRG, chunk, (rbase + tid) % kAtRG);
        row[0] = m;
        row[1] = l;
      }
    }
    __syncthreads();  // q, pr and the reductions are reused by the next pass
  }
}

// Merge: CTA (row, KV head) of 256 threads = 16 dim groups (8 dims each) x 16 chunk subsets: one
// row per CTA spreads the partials' reads over many SMs (with 4 rows per CTA the reads of 96 CTAs
// took ~5 us for 6.7 MB).  Thread subset s merges chunks s, s + 16, ... of its dims, issuing all
// of those loads at once (up to kAtMergePass chunks per pass); the 16 subsets' (max, sum, output)
// are then combined in subset order in shared memory.  The result is a fixed function of the
// partials (deterministic), and chunks past a row's last visible key change nothing.
__global__ void __launch_bounds__(kAtThreads) attn_merge_kernel(const __grid_constant__ AttnParams p) {
  constexpr int kSub = kAtMergeSub, kRowsPer = kAtMergeRows;
  static_assert(kSub * kRowsPer * 16 == kAtThreads, "thread layout");
  constexpr int kQuarters = kAtRG / kRowsPer;  // CTAs per row group
  __shared__ float os[kRowsPer][kAtD];
  __shared__ float red[kSub - 1][kRowsPer][16][10];
  __shared__ int sync_flag;
  const int rq = blockIdx.x % kQuarters, rg = blockIdx.x / kQuarters, kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rep = p.nh / p.nkv;
  const int R = p.T * rep;
  const int r0 = rg * kAtRG + rq * kRowsPer;          // first row of this CTA
  const int nrows = max(0, min(kRowsPer, R - r0));
  const int sub = tid / (16 * kRowsPer), rr = (tid >> 4) % kRowsPer, dg = tid & 15, d0 = dg * 8;
  pdl_launch_dependents();
  pdl_wait_prior_grid();  // the chunk launch's partials (and the gates, written before it)
  const int L0 = attn_length(p);
  const bool work = L0 >= 0 && nrows > 0;  // (no early exit: every CTA counts in the signal)
  const int nchunks = work ? (L0 + p.T + kAtChunk - 1) / kAtChunk : 0;
  const bool live = work && rr < nrows;
  uint4 gw = make_uint4(0u, 0u, 0u, 0u);  // the gate of this (row, dims), loaded with the partials
  if (live && sub == 0 && p.gated) {
    const int r = r0 + rr, t = r / rep, hq = kvh * rep + r % rep;
    gw = ld_nc_v4(p.proj + static_cast<size_t>(t) * p.ldp + hq * 2 * kAtD + kAtD + d0);
  }
  float M = -INFINITY, L = 0.f, acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  if (live) {
    const float* base = part_row(p, kvh, rg, 0, rq * kRowsPer + rr);
    const size_t cstride = static_cast<size_t>(kAtRG) * kAtPart;
    for (int c0 = sub; c0 < nchunks; c0 += kSub * kAtMergePass) {
      float mv[kAtMergePass], lv[kAtMergePass];
      float4 ov[kAtMergePass][2];
#pragma unroll
      for (int u = 0; u < kAtMergePass; ++u) {  // unconditional loads (clamped), masked below
        const float* row = base + min(c0 + kSub * u, nchunks - 1) * cstride;
        const float2 ml = ld_cg_v2(row);
        mv[u] = ml.x;
        lv[u] = ml.y;
        ov[u][0] = ld_cg_v4(row + 4 + d0);
        ov[u][1] = ld_cg_v4(row + 8 + d0);
      }
#pragma unroll
      for (int u = 0; u < kAtMergePass; ++u)
        if (c0 + kSub * u >= nchunks) mv[u] = -INFINITY;
      float Mn = M;
#pragma unroll
      for (int u = 0; u < kAtMergePass; ++u) Mn = fmaxf(Mn, mv[u]);
      const float alpha = M == -INFINITY ? 0.f : exp2f(M - Mn);
      L *= alpha;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= alpha;
#pragma unroll
      for (int u = 0; u < kAtMergePass; ++u) {
        const float wgt = mv[u] == -INFINITY ? 0.f : exp2f(mv[u] - Mn);
        L = fmaf(wgt, lv[u], L);
        acc[0] = fmaf(wgt, ov[u][0].x, acc[0]);
        acc[1] = fmaf(wgt, ov[u][0].y, acc[1]);
        acc[2] = fmaf(wgt, ov[u][0].z, acc[2]);
        acc[3] = fmaf(wgt, ov[u][0].w, acc[3]);
        acc[4] = fmaf(wgt, ov[u][1].x, acc[4]);
        acc[5] = fmaf(wgt, ov[u][1].y, acc[5]);
        acc[6] = fmaf(wgt, ov[u][1].z, acc[6]);
        acc[7] = fmaf(wgt, ov[u][1].w, acc[7]);
      }
      M = Mn;
    }
    if (sub > 0) {
      float* dst = red[sub - 1][rr][dg];
      dst[0] = M;
      dst[1] = L;
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[2 + i] = acc[i];
    }
  }
  __syncthreads();
  if (live && sub == 0) {
    // combine the subsets in order; the gate of this (row, dims)
#pragma unroll
    for (int q = 0; q < kSub - 1; ++q) {
      const float* src = red[q][rr][dg];
      const float Mn = fmaxf(M, src[0]);
      const float a0 = M == -INFINITY ? 0.f : exp2f(M - Mn);
      const float a1 = src[0] == -INFINITY ? 0.f : exp2f(src[0] - Mn);
      L = fmaf(a1, src[1], L * a0);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(a1, src[2 + i], acc[i] * a0);
      M = Mn;
    }
    float gate[8];
    if (p.gated) {
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(g2[i]);
        gate[2 * i] = f.x;
        gate[2 * i + 1] = f.y;
      }
    }
    const float invL = 1.f / L;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float o = bfr(acc[i] * invL);
      os[rr][d0 + i] = p.gated ? bfr(o * (1.f / (1.f + __expf(-gate[i])))) : o;
    }
  }
  __syncthreads();
  // ---- digits (and the optional bf16 copy) of the CTA's rows: warp per (row, 64 columns)
  const int mpad = p.T <= 8 ? 8 : 16;
  if (work && warp < 2 * nrows) {
    const int jr = warp >> 1, hf = warp & 1;
    const int r = r0 + jr, t = r / rep, hq = kvh * rep + r % rep;
    const int d = hf * 64 + 2 * lane;
    const float a0 = os[jr][d], a1 = os[jr][d + 1];
    if (p.o_out) {
      __nv_bfloat16* op = p.o_out + static_cast<size_t>(t) * p.nh * kAtD + hq * kAtD + d;
      *reinterpret_cast<__nv_bfloat162*>(op) = __floats2bfloat162_rn(a0, a1);
    }
    write_digits(p.xq, mpad, t, 2 * hq + hf, lane, a0, a1, p.sync.mirror, p.sync.n_mirror);
  }
  if (work && rg == 0 && rq == 0) {  // padding tokens T .. mpad-1 of this KV head's query heads
    for (int job = warp; job < (mpad - p.T) * rep * 2; job += kAtWarps) {
      const int t = p.T + job / (rep * 2), rem = job % (rep * 2);
      write_digits(p.xq, mpad, t, 2 * (kvh * rep + rem / 2) + (rem & 1), lane, 0.f, 0.f, p.sync.mirror,
                   p.sync.n_mirror);
    }
  }
  peer_signal_done(p.sync, &sync_flag);  // (sharded step) this rank's digit groups are ready
}

// KV slot compaction after a tree verify: in every layer's K and V cache, rows L0 + path[j] move
// to rows L0 + j (j = 1 .. n; path[0] = 0 stays).  One CTA per (layer, K or V): every source row
// is loaded before any destination row is written (a destination may be another copy's source).
constexpr int kKvMaxLayers = 64;
struct KvCompactParams {
  uint8_t* cache[2 * kKvMaxLayers];  // k of layer l at 2l, v at 2l + 1
  int L0[kKvMaxLayers];
  int path[kAtMaxT];
  int n, row_bytes;
};

__global__ void __launch_bounds__(256) kv_compact_kernel(const __grid_constant__ KvCompactParams p) {
  constexpr int kPer = 8;  // 16-byte pieces per thread: 256 * 8 * 16 = 32 KB >= 15 rows of 2 KB
  uint8_t* base = p.cache[blockIdx.x];
  const int L0 = p.L0[blockIdx.x >> 1];
  const int pieces_row = p.row_bytes / 16, total = p.n * pieces_row;
  uint4 v[kPer];
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int e = threadIdx.x + u * 256;
    if (e < total) {
      const int j = e / pieces_row + 1, q = e - (j - 1) * pieces_row;
      v[u] = *reinterpret_cast<const uint4*>(base + static_cast<size_t>(L0 + p.path[j]) * p.row_bytes + 16 * q);
    }
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int e = threadIdx.x + u * 256;
    if (e < total) {
      const int j = e / pieces_row + 1, q = e - (j - 1) * pieces_row;
      *reinterpret_cast<uint4*>(base + static_cast<size_t>(L0 + j) * p.row_bytes + 16 * q) = v[u];
    }
  }
}

bool kv_compact_fits(int n_layers, int n, int row_bytes) {
  return n_layers >= 1 && n_layers <= kKvMaxLayers && n >= 0 && n < kAtMaxT && row_bytes >= 16 &&
         row_bytes % 16 == 0 && static_cast<long long>(n) * (row_bytes / 16) <= 256 * 8;
}

cudaError_t kv_compact_launch(int n_layers, void* const* k, void* const* v, const int* L0, const int* path, int n,
                              int row_bytes, cudaStream_t stream) {
  static thread_local KvCompactParams prm;
  for (int l = 0; l < n_layers; ++l) {
    prm.cache[2 * l] = static_cast<uint8_t*>(k[l]);
    prm.cache[2 * l + 1] = static_cast<uint8_t*>(v[l]);
    prm.L0[l] = L0[l];
  }
  for (int j = 0; j < kAtMaxT; ++j) prm.path[j] = j <= n ? path[j] : 0;
  prm.n = n;
  prm.row_bytes = row_bytes;
  if (n == 0) return cudaSuccess;
  kv_compact_kernel<<<2 * n_layers, 256, 0, stream>>>(prm);
  return cudaGetLastError();
}

size_t attn_ws_bytes(int T, int nh, int nkv, int max_len) {
  const int rep = nh / nkv;
  const int nrg = (T * rep + kAtRG - 1) / kAtRG;
  const int nchunks = (max_len + kAtChunk - 1) / kAtChunk;
  return static_cast<size_t>(nkv) * nrg * nchunks * kAtRG * kAtPart * 4;
}

bool attn_fits(int T, int nh, int nkv) {
  return nkv >= 1 && nkv <= 64 && nh % nkv == 0 && T * (nh / nkv) <= kAtRG * kAtMaxRG;
}

static int device_sm_count_attn(int dev) {
  static std::atomic<int> n[64];
  if (dev < 0 || dev >= 64) return 0;
  int v = n[dev].load(std::memory_order_relaxed);
  if (v == 0 && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
    n[dev].store(v, std::memory_order_relaxed);
  return v;
}

cudaError_t attn_fused_launch(const void* proj, int ldp, const float* qn_w, const float* kn_w,
                              const float* inv_freq, int rot, int gated, float eps, void* kc, void* vc, int L0,
                              const int* len_dev, int max_len, int T, int nh, int nkv, void* ws, void* xq,
                              void* o_out, const skinny_peer_sync* sync, const int32_t* parent, cudaStream_t stream) {
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    const cudaError_t e = cudaFuncSetAttribute(attn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(sizeof(AttnSmem)));
    if (e != cudaSuccess) return e;
    attr_set[dev].store(true, std::memory_order_release);
  }
  const int rep = nh / nkv;
  AttnParams prm;
  prm.proj = static_cast<const __nv_bfloat16*>(proj);
  prm.ldp = ldp;
  prm.qn_w = qn_w;
  prm.kn_w = kn_w;
  prm.inv_freq = inv_freq;
  prm.eps = eps;
  prm.kc = static_cast<__nv_bfloat16*>(kc);
  prm.vc = static_cast<__nv_bfloat16*>(vc);
  prm.T = T;
  prm.L0 = L0;
  prm.nh = nh;
  prm.nkv = nkv;
  prm.rot = rot;
  prm.gated = gated;
  prm.len_dev = len_dev;
  prm.parent = parent;
  prm.max_len = max_len;
  // chunk grid (and the partials' chunk stride): the largest chunk count this cache can need
  // with a device length, else the exact count
  prm.nchunks = ((len_dev ? max_len : L0 + T) + kAtChunk - 1) / kAtChunk;
  prm.nrg = (T * rep + kAtRG - 1) / kAtRG;
  prm.part = static_cast<float*>(ws);
  prm.xq = static_cast<uint8_t*>(xq);
  prm.o_out = static_cast<__nv_bfloat16*>(o_out);
  prm.sync = peer_sync_from(sync);
  // One CTA per SM where the grid fits the GPU: launched early (programmatic dependent launch),
  // CTAs otherwise pile onto the few SMs the previous launch leaves free, two to four per SM.
  // Asking for more than half an SM's shared memory spreads them.
  static std::atomic<int> padded[64][2];  // per device: dynamic bytes of the chunk / merge launch (0: unset)
  if (padded[dev][1].load(std::memory_order_acquire) == 0) {
    int smem_sm = 0;
    cudaFuncAttributes fa{};
    cudaError_t e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, attn_merge_kernel);
    if (e != cudaSuccess) return e;
    const int chunk = std::max(static_cast<int>(sizeof(AttnSmem)), smem_sm / 2 + 1024);
    const int merge = smem_sm / 2 + 1024 - static_cast<int>(fa.sharedSizeBytes);
    e = cudaFuncSetAttribute(attn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, chunk);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, merge);
    if (e != cudaSuccess) return e;
    padded[dev][0].store(chunk, std::memory_order_relaxed);
    padded[dev][1].store(merge, std::memory_order_release);
  }
  const int n_sm = device_sm_count_attn(dev);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(prm.nchunks, nkv);
  cfg.blockDim = dim3(kAtThreads);
  cfg.dynamicSmemBytes = prm.nchunks * nkv <= n_sm ? padded[dev][0].load(std::memory_order_relaxed) : sizeof(AttnSmem);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, attn_chunk_kernel, prm);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t mcfg = {};
  mcfg.gridDim = dim3(prm.nrg * (kAtRG / kAtMergeRows), nkv);  // (rows, row group) x KV head
  mcfg.blockDim = dim3(kAtThreads);
  mcfg.dynamicSmemBytes =
      mcfg.gridDim.x * mcfg.gridDim.y <= static_cast<unsigned>(n_sm) ? padded[dev][1].load(std::memory_order_relaxed) : 0;
  mcfg.stream = stream;
  mcfg.attrs = attr;
  mcfg.numAttrs = 1;
  return cudaLaunchKernelEx(&mcfg, attn_merge_kernel, prm);
}

}  // namespace skinny
