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
constexpr int kAtKStride = kAtD + 2;  // bf16 per shared key row: 65 words, conflict-free by key
constexpr int kAtPart = kAtD + 2;     // floats per published row: m, l, o[128]
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
  int T, L0, nh, nkv, rot, nchunks, nrg;
  float* part;                // [nkv, nrg, nchunks, 16, kAtPart]
  uint32_t* cnt;              // [nkv * kAtMaxRG], zero on entry, left zero
  uint8_t* xq;                // o_proj input digits (K = nh * 128)
  __nv_bfloat16* o_out;       // [T, nh * 128] or null
};

struct AttnSmem {
  float q[kAtRG][kAtD];
  float s[kAtRG][kAtChunk];
  __nv_bfloat16 k[kAtChunk][kAtKStride];
  __nv_bfloat16 v[kAtChunk][kAtD];
  float stage[kAtWarps][kAtD];
  float rowm[kAtRG], rowl[kAtRG];
  int last;
};

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
  const int Ltot = p.L0 + p.T;
  const int k0 = chunk * kAtChunk;
  const int nk = min(kAtChunk, Ltot - k0);
  const int qkw = p.nh * 2 * kAtD;  // column of k in proj
  pdl_launch_dependents();
  pdl_wait_prior_grid();

  // ---- cached keys and values of the chunk: every thread issues all its 16-byte loads first
  {
    constexpr int kPieces = kAtChunk * (kAtD / 8);  // 16-byte pieces per matrix
    constexpr int kPer = kPieces / kAtThreads;
    uint4 kw[kPer], vw[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = tid + u * kAtThreads, j = e >> 4, pc = e & 15;
      const int pos = k0 + j;
      if (j < nk && pos < p.L0) {
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
      if (j < nk && k0 + j >= p.L0) continue;  // a new key: written below by its warp
      uint32_t* kd = reinterpret_cast<uint32_t*>(&sm.k[j][8 * pc]);  // 4-byte aligned rows
      kd[0] = kw[u].x;
      kd[1] = kw[u].y;
      kd[2] = kw[u].z;
      kd[3] = kw[u].w;
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
    norm_rope(x, p.qn_w, p.eps, p.inv_freq, p.rot, p.L0 + t, sm.stage[warp], lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) sm.q[rr][lane + 32 * i] = x[i];
  }
  // ---- new keys in the chunk (positions L0 .. L0+T-1): warp per key
  {
    const int jn0 = max(p.L0 - k0, 0);
    for (int j = jn0 + warp; j < nk; j += kAtWarps) {
      const int pos = k0 + j, t = pos - p.L0;
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
  // ---- scores (log2 domain): thread = (key j, row half)
  {
    const int j = tid % kAtChunk, h8 = (tid / kAtChunk) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll 4
    for (int d = 0; d < kAtD; d += 2) {
      const float2 kf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.k[j][d]));
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 qf = *reinterpret_cast<const float2*>(&sm.q[h8 + i][d]);
        acc[i] = fmaf(qf.x, kf.x, fmaf(qf.y, kf.y, acc[i]));
      }
    }
    const float sc = rsqrtf(static_cast<float>(kAtD)) * 1.4426950408889634f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = h8 + i;
      if (rr < nrows) {
        const int t = (rbase + rr) / rep;
        const bool vis = j < nk && k0 + j <= p.L0 + t;
        sm.s[rr][j] = vis ? acc[i] * sc : -INFINITY;
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
      const float e = m == -INFINITY ? 0.f : exp2f(sv[i] - m);
      sm.s[rr][lane + 32 * i] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
    if (lane == 0) {
      sm.rowm[rr] = m;
      sm.rowl[rr] = l;
    }
  }
  __syncthreads();
  // ---- unnormalised outputs: thread = (dim pair, 4 rows); publish
  {
    const int dp = tid % 64, r4 = (tid / 64) * 4;
    float o[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = 0.f;
    for (int j = 0; j < kAtChunk; ++j) {
      const float2 vf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.v[j][2 * dp]));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float pj = sm.s[r4 + i][j];
        o[i][0] = fmaf(pj, vf.x, o[i][0]);
        o[i][1] = fmaf(pj, vf.y, o[i][1]);
      }
    }
    float* base = p.part + ((static_cast<size_t>(kvh) * p.nrg + rg) * p.nchunks + chunk) * kAtRG * kAtPart;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = r4 + i;
      if (rr < nrows) {
        float* row = base + static_cast<size_t>(rr) * kAtPart;
        if (dp == 0) {
          row[0] = sm.rowm[rr];
          row[1] = sm.rowl[rr];
        }
        *reinterpret_cast<float2*>(row + 2 + 2 * dp) = make_float2(o[i][0], o[i][1]);
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t prev = atomicAdd(&p.cnt[kvh * kAtMaxRG + rg], 1u);
    sm.last = prev == static_cast<uint32_t>(p.nchunks - 1);
  }
  __syncthreads();
  if (!sm.last) return;
  __threadfence();
  // ---- merge the chunks (chunk order), gate, digits
  {
    const int rr = tid / 16, d0 = (tid % 16) * 8;
    if (rr < nrows) {
      const float* base = p.part + (static_cast<size_t>(kvh) * p.nrg + rg) * p.nchunks * kAtRG * kAtPart +
                          static_cast<size_t>(rr) * kAtPart;
      const size_t cstride = static_cast<size_t>(kAtRG) * kAtPart;
      float M = -INFINITY;
#pragma unroll 8
      for (int c = 0; c < p.nchunks; ++c) M = fmaxf(M, __ldcg(base + c * cstride));
      float L = 0.f, acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll 4
      for (int c = 0; c < p.nchunks; ++c) {
        const float* row = base + c * cstride;
        const float mc = __ldcg(row);
        const float wgt = mc == -INFINITY ? 0.f : exp2f(mc - M);
        L = fmaf(wgt, __ldcg(row + 1), L);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float2 ov = __ldcg(reinterpret_cast<const float2*>(row + 2 + d0 + i));
          acc[i] = fmaf(wgt, ov.x, acc[i]);
          acc[i + 1] = fmaf(wgt, ov.y, acc[i + 1]);
        }
      }
      const int r = rbase + rr, t = r / rep, hq = kvh * rep + r % rep;
      const __nv_bfloat16* gate = p.proj + static_cast<size_t>(t) * p.ldp + hq * 2 * kAtD + kAtD;
      const float invL = 1.f / L;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float g = __bfloat162float(gate[d0 + i]);
        sm.q[rr][d0 + i] = bfr(bfr(acc[i] * invL) * (1.f / (1.f + __expf(-g))));
      }
    }
  }
  __syncthreads();
  const int mpad = p.T <= 8 ? 8 : 16;
  for (int job = warp; job < 2 * nrows; job += kAtWarps) {
    const int rr = job >> 1, hf = job & 1;
    const int r = rbase + rr, t = r / rep, hq = kvh * rep + r % rep;
    const int d = hf * 64 + 2 * lane;
    const float a0 = sm.q[rr][d], a1 = sm.q[rr][d + 1];
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
                              const float* inv_freq, int rot, float eps, void* kc, void* vc, int L0, int T,
                              int nh, int nkv, void* ws, void* xq, void* o_out, cudaStream_t stream) {
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
  prm.nchunks = (L0 + T + kAtChunk - 1) / kAtChunk;
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
