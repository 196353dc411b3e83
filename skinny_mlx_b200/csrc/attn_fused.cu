// One gated full-attention mixer of the hybrid model, from its fused q|gate / k / v projection to
// the prepared input of o_proj (the B200 form of the reference model's attention layer between
// its projections, run during a verify step of T <= 16 tokens against a KV cache):
//
//   q, k  = RoPE( bf16(rmsnorm(q|k) * (1 + w)) )  on the first `rot` dims, positions L0 .. L0+T-1
//   cache[L0 .. L0+T-1] = bf16(k), v                                (KV append)
//   o     = softmax(q k^T / sqrt(128), causal bottom-right) v        (GQA: rep = n_heads / n_kv)
//   o     = bf16( bf16(o) * sigmoid(gate) )  -> digits of o for o_proj (qmm input format)
//
// Split over keys (flash-decode style): CTA (chunk, row group, kv head) takes 128 keys of one KV
// head and up to 16 query rows (row = t * rep + q head within the group), computes the chunk's
// row maxima, sums and unnormalised outputs in f32 and publishes them; the CTA that finishes a
// (row group, kv head) last merges the chunks in chunk order (deterministic) and finishes the
// rows.  There is no waiting on other CTAs: the merge is done by whichever CTA arrives last.
// Every CTA recomputes the normalised, rotated q of its rows and k of the new keys in its chunk;
// the new keys are appended to the cache by the row-group-0 CTA of their chunk (positions >= L0
// are only ever written, positions < L0 only read, so chunks never race).
//
// Launched with programmatic dependent launch (the next launch may start at once; this one waits
// for the previous grid before its first global read).
#include <cfloat>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "digits.cuh"
#include "ptx.cuh"
#include "qmm_layout.cuh"

namespace skinny {

constexpr int kAtD = 128;
constexpr int kAtChunk = 128;        // keys per CTA
constexpr int kAtRG = 16;            // query rows per CTA
constexpr int kAtThreads = 256;
constexpr int kAtWarps = kAtThreads / 32;
constexpr int kAtStride = kAtD + 8;   // bf16 per shared row: 272 bytes, ldmatrix conflict-free
constexpr int kAtPart = kAtD + 4;     // floats per published row: m, l, (pad), o[128] (16-byte aligned)
constexpr int kAtMergePass = 8;       // chunk partials whose loads a merging thread issues together
constexpr int kAtMaxRG = 8;           // row groups per KV head (rep * T <= 128)
constexpr int kAtCntWords = 64 * kAtMaxRG;
constexpr size_t kAtPartOff = kAtCntWords * 4;

struct AttnParams {
  const __nv_bfloat16* proj;  // [T, ldp]: q|gate (nh x 2 x 128, per head q then gate) | k (nkv x 128) | v
  int ldp;
  const float* qn_w;          // [128] zero-centred RMSNorm weights
  const float* kn_w;
  const float* inv_freq;      // [rot / 2] rotary frequencies
  float eps;
  __nv_bfloat16* kc;          // [max_len, nkv, 128]
  __nv_bfloat16* vc;
  int T, L0, nh, nkv, rot, nchunks, nrg, max_len;
  const int* len_dev;         // if set: the cache length is read here (grid sized for max_len)
  float* part;                // [nkv, nrg, nchunks, 16, kAtPart]: per row m, l, -, -, o[128]
  uint32_t* cnt;              // [nkv * kAtMaxRG], zero on entry, left zero
  uint8_t* xq;                // o_proj input digits (K = nh * 128)
  __nv_bfloat16* o_out;       // [T, nh * 128] or null
};

struct AttnSmem {
  __nv_bfloat16 q[kAtRG][kAtStride];      // rotated queries of the row group
  __nv_bfloat16 k[kAtChunk][kAtStride];   // keys of the chunk
  __nv_bfloat16 v[kAtChunk][kAtStride];   // values of the chunk
  __nv_bfloat16 pr[kAtRG][kAtStride];     // probabilities (bf16, as a flash kernel rounds them)
  float s[kAtRG][kAtChunk];               // scores (log2 domain); reused for the merged rows
  float stage[kAtWarps][kAtD];
  float rowm[kAtRG], rowl[kAtRG];
  int last;
};

// ---- warp-level bf16 tensor-core tiles (m16n8k16, f32 accumulate)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Warp-collective: x holds dims lane + 32 i of one head row (bf16-exact).  Returns the row after
// zero-centred RMSNorm (-> bf16) and RoPE at position pos on the first rot dims (-> bf16).
__device__ __forceinline__ void norm_rope(float (&x)[4], const float* w, float eps, const float* inv_freq,
                                          int rot, int pos, float* stage, int lane) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  const float rstd = rsqrtf(ss / kAtD + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane + 32 * i;
    x[i] = bfr(x[i] * rstd * (1.f + w[d]));
    stage[d] = x[i];
  }
  __syncwarp();
  const int half = rot >> 1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane + 32 * i;
    if (d < rot) {
      const int j = d < half ? d : d - half;
      const float ang = static_cast<float>(pos) * inv_freq[j];
      float sn, cs;
      sincosf(ang, &sn, &cs);
      x[i] = d < half ? x[i] * cs - stage[d + half] * sn : x[i] * cs + stage[d - half] * sn;
    }
    x[i] = bfr(x[i]);
  }
  __syncwarp();
}

__global__ void __launch_bounds__(kAtThreads) attn_fused_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint8_t at_smem_raw[];
  AttnSmem& sm = *reinterpret_cast<AttnSmem*>(at_smem_raw);
  const int chunk = blockIdx.x, rg = blockIdx.y, kvh = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rep = p.nh / p.nkv;
  const int R = p.T * rep;
  const int rbase = rg * kAtRG;
  const int nrows = min(kAtRG, R - rbase);
  const int qkw = p.nh * 2 * kAtD;  // column of k in proj
  pdl_launch_dependents();
  pdl_wait_prior_grid();
  // the cache length: a kernel argument, or read from device memory so that one captured
  // launch serves every length (the grid then covers max_len and the surplus chunks leave)
  const int L0 = p.len_dev ? *p.len_dev : p.L0;
  if (L0 < 0 || L0 + p.T > p.max_len) return;  // a device length out of range: no access at all
  const int nchunks = p.len_dev ? (L0 + p.T + kAtChunk - 1) / kAtChunk : p.nchunks;
  if (chunk >= nchunks) return;
  const int Ltot = L0 + p.T;
  const int k0 = chunk * kAtChunk;
  const int nk = min(kAtChunk, Ltot - k0);

  // output gates of the rows this thread finishes if this CTA merges (row tid / 16, 8 dims)
  float gate_pre[8];
  {
    const int rr = tid / 16, d0 = (tid % 16) * 8;
    if (rr < nrows) {
      const int r = rbase + rr, t = r / rep, hq = kvh * rep + r % rep;
      const uint4 gw = *reinterpret_cast<const uint4*>(p.proj + static_cast<size_t>(t) * p.ldp + hq * 2 * kAtD + kAtD + d0);
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(g2[i]);
        gate_pre[2 * i] = f.x;
        gate_pre[2 * i + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) gate_pre[i] = 0.f;
    }
  }

  // ---- cached keys and values of the chunk: every thread issues all its 16-byte loads first
  {
    constexpr int kPieces = kAtChunk * (kAtD / 8);  // 16-byte pieces per matrix
    constexpr int kPer = kPieces / kAtThreads;
    uint4 kw[kPer], vw[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = tid + u * kAtThreads, j = e >> 4, pc = e & 15;
      const int pos = k0 + j;
      if (j < nk && pos < L0) {
        const size_t off = (static_cast<size_t>(pos) * p.nkv + kvh) * kAtD + 8 * pc;
        kw[u] = __ldg(reinterpret_cast<const uint4*>(p.kc + off));
        vw[u] = __ldg(reinterpret_cast<const uint4*>(p.vc + off));
      } else {
        kw[u] = make_uint4(0u, 0u, 0u, 0u);
        vw[u] = kw[u];
      }
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = tid + u * kAtThreads, j = e >> 4, pc = e & 15;
      if (j < nk && k0 + j >= L0) continue;  // a new key: written below by its warp
      *reinterpret_cast<uint4*>(&sm.k[j][8 * pc]) = kw[u];
      *reinterpret_cast<uint4*>(&sm.v[j][8 * pc]) = vw[u];
    }
  }
  // ---- query rows: normalised, rotated, bf16
  for (int rr = warp; rr < nrows; rr += kAtWarps) {
    const int r = rbase + rr, t = r / rep, hq = kvh * rep + r % rep;
    const __nv_bfloat16* src = p.proj + static_cast<size_t>(t) * p.ldp + hq * 2 * kAtD;
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = __bfloat162float(src[lane + 32 * i]);
    norm_rope(x, p.qn_w, p.eps, p.inv_freq, p.rot, L0 + t, sm.stage[warp], lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) sm.q[rr][lane + 32 * i] = __float2bfloat16_rn(x[i]);
  }
  for (int i = tid; i < (kAtRG - nrows) * kAtD; i += kAtThreads)  // rows past the group: zero
    sm.q[nrows + i / kAtD][i % kAtD] = __float2bfloat16_rn(0.f);
  // ---- new keys in the chunk (positions L0 .. L0+T-1): warp per key
  {
    const int jn0 = max(L0 - k0, 0);
    for (int j = jn0 + warp; j < nk; j += kAtWarps) {
      const int pos = k0 + j, t = pos - L0;
      const __nv_bfloat16* src = p.proj + static_cast<size_t>(t) * p.ldp + qkw;
      float x[4];
      __nv_bfloat16 vb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        x[i] = __bfloat162float(src[kvh * kAtD + lane + 32 * i]);
        vb[i] = src[p.nkv * kAtD + kvh * kAtD + lane + 32 * i];
      }
      norm_rope(x, p.kn_w, p.eps, p.inv_freq, p.rot, pos, sm.stage[warp], lane);
      const size_t off = (static_cast<size_t>(pos) * p.nkv + kvh) * kAtD;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int d = lane + 32 * i;
        const __nv_bfloat16 kb = __float2bfloat16_rn(x[i]);
        sm.k[j][d] = kb;
        sm.v[j][d] = vb[i];
        if (rg == 0) {
          p.kc[off + d] = kb;
          p.vc[off + d] = vb[i];
        }
      }
    }
  }
  __syncthreads();
  // ---- scores on tensor cores (log2 domain): warp w takes keys 16w .. 16w+15 for the 16 rows
  {
    const int g = lane >> 2, cq = lane & 3;
    const uint32_t a_addr =
        smem_u32(&sm.q[0][0]) + (((lane & 7) + 8 * ((lane >> 3) & 1)) * kAtStride + 8 * (lane >> 4)) * 2;
    const uint32_t b_addr =
        smem_u32(&sm.k[0][0]) + ((16 * warp + (lane & 7) + 8 * (lane >> 4)) * kAtStride + 8 * ((lane >> 3) & 1)) * 2;
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < kAtD / 16; ++ks) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      ldsm_x4(a_addr + ks * 32, a0, a1, a2, a3);
      ldsm_x4(b_addr + ks * 32, b0, b1, b2, b3);
      mma_bf16(c[0], a0, a1, a2, a3, b0, b1);
      mma_bf16(c[1], a0, a1, a2, a3, b2, b3);
    }
    const float sc = rsqrtf(static_cast<float>(kAtD)) * 1.4426950408889634f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rr = g + 8 * (e >> 1), j = 16 * warp + 8 * nt + 2 * cq + (e & 1);
        if (rr < nrows) {
          const int t = (rbase + rr) / rep;
          const bool vis = j < nk && k0 + j <= L0 + t;
          sm.s[rr][j] = vis ? c[nt][e] * sc : -INFINITY;
        }
      }
  }
  __syncthreads();
  // ---- chunk softmax per row (warp per row)
  for (int rr = warp; rr < nrows; rr += kAtWarps) {
    float sv[4];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sv[i] = sm.s[rr][lane + 32 * i];
      m = fmaxf(m, sv[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    float l = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat16 e = __float2bfloat16_rn(m == -INFINITY ? 0.f : exp2f(sv[i] - m));
      sm.pr[rr][lane + 32 * i] = e;
      l += __bfloat162float(e);  // the sum of the probabilities as the products use them
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
    if (lane == 0) {
      sm.rowm[rr] = m;
      sm.rowl[rr] = l;
    }
  }
  __syncthreads();
  for (int i = tid; i < (kAtRG - nrows) * kAtD; i += kAtThreads)
    sm.pr[nrows + i / kAtD][i % kAtD] = __float2bfloat16_rn(0.f);
  __syncthreads();
  // ---- unnormalised outputs on tensor cores: warp w takes dims 16w .. 16w+15; publish
  {
    const int g = lane >> 2, cq = lane & 3;
    const uint32_t a_addr =
        smem_u32(&sm.pr[0][0]) + (((lane & 7) + 8 * ((lane >> 3) & 1)) * kAtStride + 8 * (lane >> 4)) * 2;
    const uint32_t b_addr =
        smem_u32(&sm.v[0][0]) + (((lane & 7) + 8 * ((lane >> 3) & 1)) * kAtStride + 16 * warp + 8 * (lane >> 4)) * 2;
    float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < kAtChunk / 16; ++ks) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      ldsm_x4(a_addr + ks * 32, a0, a1, a2, a3);
      ldsm_x4_t(b_addr + ks * 16 * kAtStride * 2, b0, b1, b2, b3);
      mma_bf16(o[0], a0, a1, a2, a3, b0, b1);
      mma_bf16(o[1], a0, a1, a2, a3, b2, b3);
    }
    float* base = p.part + ((static_cast<size_t>(kvh) * p.nrg + rg) * nchunks + chunk) * kAtRG * kAtPart;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int rr = g + 8 * hf;
        if (rr < nrows)
          *reinterpret_cast<float2*>(base + static_cast<size_t>(rr) * kAtPart + 4 + 16 * warp + 8 * nt + 2 * cq) =
              make_float2(o[nt][2 * hf], o[nt][2 * hf + 1]);
      }
    if (tid < nrows) {
      base[static_cast<size_t>(tid) * kAtPart] = sm.rowm[tid];
      base[static_cast<size_t>(tid) * kAtPart + 1] = sm.rowl[tid];
    }
  }
  // Publish: the block's writes are ordered before thread 0's release-acquire increment (the
  // barrier makes them visible to thread 0; the release is cumulative), and the last arriver's
  // acquire makes every chunk's partials visible to it.
  __syncthreads();
  if (tid == 0) {
    uint32_t prev;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                 : "=r"(prev)
                 : "l"(p.cnt + kvh * kAtMaxRG + rg)
                 : "memory");
    sm.last = prev == static_cast<uint32_t>(nchunks - 1);
  }
  __syncthreads();
  if (!sm.last) return;
  // ---- merge the chunks (chunk order, passes of kAtMergePass), gate, digits
  {
    const int rr = tid / 16, d0 = (tid % 16) * 8;
    if (rr < nrows) {
      const float* base = p.part + (static_cast<size_t>(kvh) * p.nrg + rg) * nchunks * kAtRG * kAtPart +
                          static_cast<size_t>(rr) * kAtPart;
      const size_t cstride = static_cast<size_t>(kAtRG) * kAtPart;
      float M = -INFINITY, L = 0.f, acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int c0 = 0; c0 < nchunks; c0 += kAtMergePass) {
        float mv[kAtMergePass], lv[kAtMergePass];
        float4 ov[kAtMergePass][2];
#pragma unroll
        for (int u = 0; u < kAtMergePass; ++u) {
          const int c = c0 + u;
          if (c < nchunks) {
            const float* row = base + c * cstride;
            mv[u] = __ldcg(row);
            lv[u] = __ldcg(row + 1);
            ov[u][0] = __ldcg(reinterpret_cast<const float4*>(row + 4 + d0));
            ov[u][1] = __ldcg(reinterpret_cast<const float4*>(row + 8 + d0));
          } else {
            mv[u] = -INFINITY;
            lv[u] = 0.f;
            ov[u][0] = ov[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
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
      const float invL = 1.f / L;
#pragma unroll
      for (int i = 0; i < 8; ++i) sm.s[rr][d0 + i] = bfr(bfr(acc[i] * invL) * (1.f / (1.f + __expf(-gate_pre[i]))));
    }
  }
  __syncthreads();
  const int mpad = p.T <= 8 ? 8 : 16;
  for (int job = warp; job < 2 * nrows; job += kAtWarps) {
    const int rr = job >> 1, hf = job & 1;
    const int r = rbase + rr, t = r / rep, hq = kvh * rep + r % rep;
    const int d = hf * 64 + 2 * lane;
    const float a0 = sm.s[rr][d], a1 = sm.s[rr][d + 1];
    if (p.o_out) {
      __nv_bfloat16* op = p.o_out + static_cast<size_t>(t) * p.nh * kAtD + hq * kAtD + d;
      *reinterpret_cast<__nv_bfloat162*>(op) = __floats2bfloat162_rn(a0, a1);
    }
    write_digits(p.xq, mpad, t, 2 * hq + hf, lane, a0, a1);
  }
  if (rg == 0) {  // padding tokens T .. mpad-1 of this KV head's query heads
    for (int job = warp; job < (mpad - p.T) * rep * 2; job += kAtWarps) {
      const int t = p.T + job / (rep * 2), rem = job % (rep * 2);
      write_digits(p.xq, mpad, t, 2 * (kvh * rep + rem / 2) + (rem & 1), lane, 0.f, 0.f);
    }
  }
  if (tid == 0) p.cnt[kvh * kAtMaxRG + rg] = 0;  // ready for the next launch
}

size_t attn_ws_bytes(int T, int nh, int nkv, int max_len) {
  const int rep = nh / nkv;
  const int nrg = (T * rep + kAtRG - 1) / kAtRG;
  const int nchunks = (max_len + kAtChunk - 1) / kAtChunk;
  return kAtPartOff + static_cast<size_t>(nkv) * nrg * nchunks * kAtRG * kAtPart * 4;
}

bool attn_fits(int T, int nh, int nkv) {
  return nkv >= 1 && nkv <= 64 && nh % nkv == 0 && T * (nh / nkv) <= kAtRG * kAtMaxRG;
}

cudaError_t attn_fused_launch(const void* proj, int ldp, const float* qn_w, const float* kn_w,
                              const float* inv_freq, int rot, float eps, void* kc, void* vc, int L0,
                              const int* len_dev, int max_len, int T, int nh, int nkv, void* ws, void* xq,
                              void* o_out, cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(attn_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(sizeof(AttnSmem)));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
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
  prm.len_dev = len_dev;
  prm.max_len = max_len;
  prm.nchunks = ((len_dev ? max_len : L0 + T) + kAtChunk - 1) / kAtChunk;  // grid; the kernel recomputes it from len_dev
  prm.nrg = (T * rep + kAtRG - 1) / kAtRG;
  prm.cnt = static_cast<uint32_t*>(ws);
  prm.part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kAtPartOff);
  prm.xq = static_cast<uint8_t*>(xq);
  prm.o_out = static_cast<__nv_bfloat16*>(o_out);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(prm.nchunks, prm.nrg, nkv);
  cfg.blockDim = dim3(kAtThreads);
  cfg.dynamicSmemBytes = sizeof(AttnSmem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_fused_kernel, prm);
}

}  // namespace skinny
