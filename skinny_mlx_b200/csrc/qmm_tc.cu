// 4-bit affine group-64 quantized matmul for 1..16 tokens on sm_100a (tcgen05 + TMEM + TMA).
//
//   out[t, n] = sum_g ( s[n,g] * sum_{k in g} x[t,k] * q[n,k]  +  b[n,g] * xsum[t,g] )
//
// This is the affine identity of skinny_mlx/qmm.py:8-9 and :64-71 (scale and bias applied once
// per 64-group), computed "swap-AB": weight rows are the 128-row MMA operand A and the tokens are
// the N=16 operand B, so a 1..16-token step reads every weight byte exactly once.
//
// Work split (stream-K): the matrix is cut into units of 128 rows x 64 columns (4608 relaid
// bytes, see qmm_layout.cuh) and each of the C CTAs (one per SM) takes a contiguous range of
// units in tile-major order.  A CTA therefore streams one contiguous byte range of the relaid
// weights.  Tiles that straddle CTAs are finished by whichever contributing CTA arrives last; it
// adds the partial sums in contributor order, so results are deterministic and do not depend on
// the token count (row t of a 16-token call equals the same row of a 1-token call, bit for bit).
//
// Warp roles in a CTA of 320 threads:
//   warp 0 lane 0  TMA producer: bulk-copies weight units and x blocks into a 12-stage ring.
//                  Weight units are prefetched before griddepcontrol.wait (they do not depend on
//                  the previous kernel), so with programmatic dependent launch the weight stream
//                  of this launch overlaps the tail of the previous one.
//   warp 1         allocates TMEM; lane 0 issues 4 tcgen05.mma (128x16x16) per unit, A read from
//                  TMEM, B = x^T from shared memory, D (f32) into a TMEM slot per unit.
//   warps 2..9     two warpgroups; thread <-> weight row (TMEM lane).  Warpgroup h dequantizes
//                  columns 32h..32h+31 of every unit: 0x6400 | nibble gives the f16 1024+q, the
//                  high nibble of each byte gives 1024+16q, and one HSUB2/HFMA2 yields q exactly;
//                  tcgen05.st writes the pairs into the unit's A slot.  One unit later the same
//                  threads read the unit's 16 partial dot products from TMEM and apply scale and
//                  bias in f32 (warpgroup h owns token slots h*NTH .. h*NTH+NTH-1).
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ptx.cuh"
#include "qmm_layout.cuh"
#include "skinny_status.h"

namespace skinny {

constexpr int kStages = 12;
constexpr int kStageBytes = 6784;  // 4608 + 2112 rounded up to 128
constexpr int kNumA = 4;           // TMEM A slots (32 columns each)
constexpr int kNumD = 4;           // TMEM D slots (16 columns each)
constexpr int kTmemCols = 256;
constexpr int kDCol0 = kNumA * 32;
constexpr int kThreads = 320;
constexpr int kEpiThreads = 256;

struct QmmParams {
  const uint8_t* w_tc;  // relaid weight units
  const uint8_t* xw;    // x blocks [G][2112] (workspace)
  __nv_bfloat16* out;   // [M, ldo]
  float* part;          // [C][2][16][128] partial sums (workspace)
  uint32_t* cnt;        // [T] arrival counters (workspace)
  uint32_t* err;        // device error word (workspace)
  int M, N, G, T, C, ldo;
  long long U;
};

struct __align__(8) QmmSmemBarriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t a_full[kNumA];
  uint64_t a_empty[kNumA];
  uint64_t d_full[kNumD];
  uint64_t d_empty[kNumD];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  int last_flag;
};

constexpr size_t kQmmSmemBytes = static_cast<size_t>(kStages) * kStageBytes + 1024;

// 16 nibbles of one row (4 relaid words) -> 8 f16x2 pairs holding q exactly, natural column order.
__device__ __forceinline__ void decode4(const uint4& w, uint32_t (&o)[16]) {
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
  const __half2 k1024 = __half2half2(__ushort_as_half(0x6400));  // 1024
  const __half2 k1_16 = __half2half2(__float2half(0.0625f));
  const __half2 km64 = __half2half2(__float2half(-64.0f));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t v = words[j];
    const uint32_t v8 = v >> 8;
    uint32_t p0 = (v & 0x000F000Fu) | 0x64006400u;   // 1024 + (k0, k1)
    uint32_t p1 = (v & 0x00F000F0u) | 0x64006400u;   // 1024 + 16 (k2, k3)
    uint32_t p2 = (v8 & 0x000F000Fu) | 0x64006400u;  // 1024 + (k4, k5)
    uint32_t p3 = (v8 & 0x00F000F0u) | 0x64006400u;  // 1024 + 16 (k6, k7)
    __half2 h0 = __hsub2(*reinterpret_cast<__half2*>(&p0), k1024);
    __half2 h1 = __hfma2(*reinterpret_cast<__half2*>(&p1), k1_16, km64);
    __half2 h2 = __hsub2(*reinterpret_cast<__half2*>(&p2), k1024);
    __half2 h3 = __hfma2(*reinterpret_cast<__half2*>(&p3), k1_16, km64);
    o[4 * j + 0] = *reinterpret_cast<uint32_t*>(&h0);
    o[4 * j + 1] = *reinterpret_cast<uint32_t*>(&h1);
    o[4 * j + 2] = *reinterpret_cast<uint32_t*>(&h2);
    o[4 * j + 3] = *reinterpret_cast<uint32_t*>(&h3);
  }
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <int NTH>
__global__ void __launch_bounds__(kThreads, 1) qmm_w4g64_tc_kernel(const QmmParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  QmmSmemBarriers* sb = reinterpret_cast<QmmSmemBarriers*>(smem + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const long long u0 = u_begin(c, p.U, p.C);
  const long long u1 = u_begin(c + 1, p.U, p.C);
  const int L = static_cast<int>(u1 - u0);
  volatile int* abort_flag = &sb->abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&sb->full[i]), 1);
      mbar_init(smem_u32(&sb->empty[i]), 1);
    }
    for (int i = 0; i < kNumA; ++i) {
      mbar_init(smem_u32(&sb->a_full[i]), kEpiThreads);
      mbar_init(smem_u32(&sb->a_empty[i]), 1);
    }
    for (int i = 0; i < kNumD; ++i) {
      mbar_init(smem_u32(&sb->d_full[i]), 1);
      mbar_init(smem_u32(&sb->d_empty[i]), kEpiThreads);
    }
    mbar_init(smem_u32(&sb->mma_done), 1);
    sb->abort_flag = 0;
    sb->last_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&sb->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sb->tmem_base;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      const int pre = L < kStages ? L : kStages;
      for (int i = 0; i < pre; ++i) {
        const uint32_t stage = smem_u32(smem + i * kStageBytes);
        mbar_arrive_expect_tx(smem_u32(&sb->full[i]), kUnitWBytes + kUnitXBytes);
        bulk_g2s_hint(stage, p.w_tc + (u0 + i) * kUnitWBytes, kUnitWBytes, smem_u32(&sb->full[i]),
                      pol_w);
      }
      pdl_wait_prior_grid();  // x blocks are written by the x-prep kernel
      for (int i = 0; i < pre; ++i) {
        const uint32_t stage = smem_u32(smem + i * kStageBytes);
        const int g = static_cast<int>((u0 + i) % p.G);
        bulk_g2s_hint(stage + kUnitWBytes, p.xw + static_cast<size_t>(g) * kUnitXBytes, kUnitXBytes,
                      smem_u32(&sb->full[i]), pol_x);
      }
      for (int i = kStages; i < L; ++i) {
        const int s = i % kStages;
        if (!mbar_wait(smem_u32(&sb->empty[s]), ((i / kStages) - 1) & 1, p.err, kErrBitWaitEmpty,
                       abort_flag))
          break;
        const uint32_t stage = smem_u32(smem + s * kStageBytes);
        const int g = static_cast<int>((u0 + i) % p.G);
        mbar_arrive_expect_tx(smem_u32(&sb->full[s]), kUnitWBytes + kUnitXBytes);
        bulk_g2s_hint(stage, p.w_tc + (u0 + i) * kUnitWBytes, kUnitWBytes, smem_u32(&sb->full[s]),
                      pol_w);
        bulk_g2s_hint(stage + kUnitWBytes, p.xw + static_cast<size_t>(g) * kUnitXBytes, kUnitXBytes,
                      smem_u32(&sb->full[s]), pol_x);
      }
      // Never leave the CTA with copies in flight: wait (bounded, ignoring abort) for the last
      // stages issued.  On the normal path they completed long ago.
      int zero = 0;
      for (int i = (L > kStages ? L - kStages : 0); i < L; ++i) {
        const int s = i % kStages;
        mbar_wait(smem_u32(&sb->full[s]), (i / kStages) & 1, p.err, kErrBitWaitDrain, &zero);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------ MMA issuer ------------------------------
      constexpr uint32_t idesc = idesc_f16_f32(128, 16);
      for (int i = 0; i < L; ++i) {
        const int s = i % kStages, a = i % kNumA, d = i % kNumD;
        if (!mbar_wait(smem_u32(&sb->full[s]), (i / kStages) & 1, p.err, kErrBitWaitFull, abort_flag))
          break;
        if (!mbar_wait(smem_u32(&sb->a_full[a]), (i / kNumA) & 1, p.err, kErrBitWaitAFull, abort_flag))
          break;
        if (i >= kNumD &&
            !mbar_wait(smem_u32(&sb->d_empty[d]), ((i / kNumD) - 1) & 1, p.err, kErrBitWaitDEmpty,
                       abort_flag))
          break;
        tc_fence_after();
        const uint32_t xs = smem_u32(smem + s * kStageBytes + kUnitWBytes);
        const uint32_t d_tmem = tmem + kDCol0 + d * 16;
        const uint32_t a_tmem = tmem + a * 32;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t bdesc = smem_desc_noswizzle(xs + j * 512, 128, 256);
          umma_f16_ts(d_tmem, a_tmem + j * 8, bdesc, idesc, j > 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(&sb->empty[s]));
        umma_commit(smem_u32(&sb->a_empty[a]));
        umma_commit(smem_u32(&sb->d_full[d]));
      }
      // All MMAs issued by this thread must be complete before TMEM is released.
      umma_commit(smem_u32(&sb->mma_done));
      int zero = 0;
      mbar_wait(smem_u32(&sb->mma_done), 0, p.err, kErrBitWaitDrain, &zero);
    }
  } else {
    // ------------------------------ dequant + epilogue ------------------------------
    const int e = threadIdx.x - 64;
    const int wg = e >> 7;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    float acc[NTH];
#pragma unroll
    for (int t = 0; t < NTH; ++t) acc[t] = 0.f;
    // pending epilogue (unit i-1)
    float pend_s = 0.f, pend_b = 0.f, pend_xs[NTH];
#pragma unroll
    for (int t = 0; t < NTH; ++t) pend_xs[t] = 0.f;
    bool dep_waited = false;

    auto flush = [&](long long tile, bool full_tile, bool first_seg) {
      const int row_g = static_cast<int>(tile) * kTileRows + r;
      const bool ok = !*abort_flag;
      if (!dep_waited) {
        pdl_wait_prior_grid();
        dep_waited = true;
      }
      if (full_tile) {
        if (ok && row_g < p.N) {
#pragma unroll
          for (int t = 0; t < NTH; ++t) {
            const int tok = wg * NTH + t;
            if (tok < p.M) p.out[static_cast<size_t>(tok) * p.ldo + row_g] = __float2bfloat16_rn(acc[t]);
          }
        }
        return;
      }
      const int slot = first_seg ? 0 : 1;
      float* mine = p.part + (static_cast<size_t>(c) * 2 + slot) * kMaxTokens * kTileRows;
#pragma unroll
      for (int t = 0; t < NTH; ++t) mine[(wg * NTH + t) * kTileRows + r] = acc[t];
      __threadfence();
      named_bar_sync(1, kEpiThreads);
      if (e == 0) {
        const long long cf = cta_of_unit(tile * p.G, p.U, p.C);
        const long long cl = cta_of_unit(tile * p.G + p.G - 1, p.U, p.C);
        const unsigned n_contrib = static_cast<unsigned>(cl - cf + 1);
        const unsigned old = ok ? atomicAdd(&p.cnt[tile], 1u) : 0u;
        sb->last_flag = ok && (old == n_contrib - 1);
      }
      named_bar_sync(1, kEpiThreads);
      if (sb->last_flag) {
        __threadfence();
        const long long cf = cta_of_unit(tile * p.G, p.U, p.C);
        const long long cl = cta_of_unit(tile * p.G + p.G - 1, p.U, p.C);
        float v[NTH];
#pragma unroll
        for (int t = 0; t < NTH; ++t) v[t] = 0.f;
        for (long long cc = cf; cc <= cl; ++cc) {
          const long long cu0 = u_begin(cc, p.U, p.C);
          const int cs = (cu0 / p.G == tile) ? 0 : 1;
          const float* src = p.part + (static_cast<size_t>(cc) * 2 + cs) * kMaxTokens * kTileRows;
#pragma unroll
          for (int t = 0; t < NTH; ++t) v[t] += __ldcg(src + (wg * NTH + t) * kTileRows + r);
        }
        if (row_g < p.N) {
#pragma unroll
          for (int t = 0; t < NTH; ++t) {
            const int tok = wg * NTH + t;
            if (tok < p.M) p.out[static_cast<size_t>(tok) * p.ldo + row_g] = __float2bfloat16_rn(v[t]);
          }
        }
        if (e == 0) p.cnt[tile] = 0u;
      }
      named_bar_sync(1, kEpiThreads);
    };

    auto epilogue = [&](int j) {
      const int d = j % kNumD;
      float gsum[NTH];
      const bool ok = mbar_wait(smem_u32(&sb->d_full[d]), (j / kNumD) & 1, p.err, kErrBitWaitDFull,
                                abort_flag);
      if (ok) {
        tc_fence_after();
        tmem_ld<NTH>(tmem + lane_off + kDCol0 + d * 16 + wg * NTH, gsum);
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(smem_u32(&sb->d_empty[d]));
#pragma unroll
        for (int t = 0; t < NTH; ++t) acc[t] = fmaf(pend_s, gsum[t], fmaf(pend_b, pend_xs[t], acc[t]));
      }
      const long long u = u0 + j;
      const int g = static_cast<int>(u % p.G);
      if (g == p.G - 1 || j == L - 1) {
        const long long tile = u / p.G;
        const long long seg_start = (tile * p.G > u0) ? tile * p.G : u0;
        const bool full_tile = (seg_start == tile * p.G) && (g == p.G - 1);
        const bool first_seg = (seg_start == u0);
        flush(tile, full_tile, first_seg);
#pragma unroll
        for (int t = 0; t < NTH; ++t) acc[t] = 0.f;
      }
    };

    for (int i = 0; i < L; ++i) {
      const int s = i % kStages, a = i % kNumA;
      const uint8_t* stage = smem + s * kStageBytes;
      float sc = 0.f, bi = 0.f, xs[NTH];
#pragma unroll
      for (int t = 0; t < NTH; ++t) xs[t] = 0.f;
      if (mbar_wait(smem_u32(&sb->full[s]), (i / kStages) & 1, p.err, kErrBitWaitFull, abort_flag)) {
        const uint4 w4 = *reinterpret_cast<const uint4*>(stage + wg * 2048 + r * 16);
        const uint32_t sbw = *reinterpret_cast<const uint32_t*>(stage + kUnitNibBytes + r * 4);
        sc = __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(sbw & 0xFFFFu)));
        bi = __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(sbw >> 16)));
        const float* xsum = reinterpret_cast<const float*>(stage + kUnitWBytes + kXsumOffset);
#pragma unroll
        for (int t = 0; t < NTH; ++t) xs[t] = xsum[wg * NTH + t];
        uint32_t q[16];
        decode4(w4, q);
        if (i < kNumA ||
            mbar_wait(smem_u32(&sb->a_empty[a]), ((i / kNumA) - 1) & 1, p.err, kErrBitWaitAEmpty,
                      abort_flag)) {
          tc_fence_after();
          tmem_st_x16(tmem + lane_off + a * 32 + wg * 16, q);
          tc_wait_st();
          tc_fence_before();
          mbar_arrive(smem_u32(&sb->a_full[a]));
        }
      }
      if (i > 0) epilogue(i - 1);
      pend_s = sc;
      pend_b = bi;
#pragma unroll
      for (int t = 0; t < NTH; ++t) pend_xs[t] = xs[t];
    }
    if (L > 0) epilogue(L - 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// x [M, ldx] bf16  ->  per-group blocks of f16 x^T in the canonical B layout + f32 group sums.
// One CTA per 64-column group, 128 threads, each converting 8 consecutive columns of one token.
__global__ void __launch_bounds__(128) qmm_xprep_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                        int M, uint8_t* __restrict__ xw,
                                                        uint32_t* err) {
  __shared__ float red[kMaxTokens][8];
  pdl_launch_dependents();
  pdl_wait_prior_grid();
  const int g = blockIdx.x;
  const int e = threadIdx.x;
  const int tr = e & 7, tb = (e >> 3) & 1, kh = (e >> 4) & 1, j = e >> 5;
  const int t = tb * 8 + tr;
  const int k0 = g * kGroup + j * 16 + kh * 8;
  uint4 packed = make_uint4(0, 0, 0, 0);
  float psum = 0.f;
  if (t < M) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * ldx + k0);
    const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t hw[4];
    bool overflow = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = __uint_as_float(rw[i] << 16);
      const float hi = __uint_as_float(rw[i] & 0xFFFF0000u);
      const __half2 h = __floats2half2_rn(lo, hi);
      const float2 back = __half22float2(h);
      overflow |= (isinf(back.x) && !isinf(lo)) || (isinf(back.y) && !isinf(hi));
      psum += back.x;
      psum += back.y;
      hw[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    if (overflow) atomicOr(err, kErrBitXOverflow);
    packed = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  }
  uint8_t* blk = xw + static_cast<size_t>(g) * kUnitXBytes;
  *reinterpret_cast<uint4*>(blk + j * 512 + tb * 256 + kh * 128 + tr * 16) = packed;
  red[t][j * 2 + kh] = psum;
  __syncthreads();
  if (e < kMaxTokens) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += red[e][i];
    reinterpret_cast<float*>(blk + kXsumOffset)[e] = s;
  }
}

// One-time relayout: MLX packs + bf16 scales/biases -> units (see qmm_layout.cuh).
// One thread per (unit, row).
__global__ void qmm_repack_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ scales,
                                  const uint16_t* __restrict__ biases, uint8_t* __restrict__ w_tc,
                                  int N, int K, long long total) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int G = K / kGroup;
  const int r = static_cast<int>(idx & (kTileRows - 1));
  const long long unit = idx >> 7;
  const long long tile = unit / G;
  const int g = static_cast<int>(unit % G);
  const long long n = tile * kTileRows + r;
  uint8_t* base = w_tc + unit * kUnitWBytes;
  uint32_t outw[8];
  uint32_t sbw = 0;
  if (n < N) {
    const uint32_t* src = w + n * (K / 8) + g * 8;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const uint32_t v = src[jj];
      uint32_t o = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t nib = (v >> (4 * i)) & 0xFu;
        // even columns go to the low half-word, odd ones to the high half-word
        const int slot = (i & 1) ? (4 + (i >> 1)) : (i >> 1);
        o |= nib << (4 * slot);
      }
      outw[jj] = o;
    }
    sbw = static_cast<uint32_t>(scales[n * G + g]) | (static_cast<uint32_t>(biases[n * G + g]) << 16);
  } else {
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) outw[jj] = 0;
  }
  *reinterpret_cast<uint4*>(base + r * 16) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
  *reinterpret_cast<uint4*>(base + 2048 + r * 16) = make_uint4(outw[4], outw[5], outw[6], outw[7]);
  *reinterpret_cast<uint32_t*>(base + kUnitNibBytes + r * 4) = sbw;
}

// Plain CUDA-core cross-check of the relaid format: same decode, same identity, same x rounding.
// One thread per (row, token).  Used by the tests to localise a mismatch; not a product path.
__global__ void qmm_simt_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                const uint8_t* __restrict__ w_tc, __nv_bfloat16* __restrict__ out,
                                int ldo, int M, int N, int K) {
  const int G = K / kGroup;
  const int tile = blockIdx.x;
  const int r = threadIdx.x;
  const int tok = blockIdx.y;
  const int n = tile * kTileRows + r;
  if (n >= N || tok >= M) return;
  float acc = 0.f;
  for (int g = 0; g < G; ++g) {
    const uint8_t* base = w_tc + (static_cast<long long>(tile) * G + g) * kUnitWBytes;
    const uint32_t sbw = *reinterpret_cast<const uint32_t*>(base + kUnitNibBytes + r * 4);
    const float sc = __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(sbw & 0xFFFFu)));
    const float bi = __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(sbw >> 16)));
    float gs = 0.f, xsum = 0.f;
    for (int ch = 0; ch < 2; ++ch) {
      const uint4 w4 = *reinterpret_cast<const uint4*>(base + ch * 2048 + r * 16);
      uint32_t q[16];
      decode4(w4, q);
      for (int pidx = 0; pidx < 16; ++pidx) {
        const __half2 h = *reinterpret_cast<const __half2*>(&q[pidx]);
        const float2 qf = __half22float2(h);
        const int k = g * kGroup + ch * 32 + pidx * 2;
        const float x0 = __half2float(__float2half_rn(__bfloat162float(x[static_cast<size_t>(tok) * ldx + k])));
        const float x1 = __half2float(__float2half_rn(__bfloat162float(x[static_cast<size_t>(tok) * ldx + k + 1])));
        gs = fmaf(qf.x, x0, gs);
        gs = fmaf(qf.y, x1, gs);
        xsum += x0;
        xsum += x1;
      }
    }
    acc = fmaf(sc, gs, fmaf(bi, xsum, acc));
  }
  out[static_cast<size_t>(tok) * ldo + n] = __float2bfloat16_rn(acc);
}

// ---------------------------------------------------------------------------------------------
// Host launchers (called from the C-ABI layer)
// ---------------------------------------------------------------------------------------------
static int g_num_sms[64] = {0};
static bool g_attr_set[64][4] = {};

int device_sm_count(int dev) {
  if (dev < 0 || dev >= 64) return 148;
  if (g_num_sms[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    g_num_sms[dev] = v;
  }
  return g_num_sms[dev];
}

template <int NTH>
static cudaError_t launch_tc(const QmmParams& prm, int dev, cudaStream_t stream, bool pdl) {
  constexpr int slot = NTH == 1 ? 0 : NTH == 2 ? 1 : NTH == 4 ? 2 : 3;
  if (dev >= 0 && dev < 64 && !g_attr_set[dev][slot]) {
    cudaError_t e = cudaFuncSetAttribute(qmm_w4g64_tc_kernel<NTH>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kQmmSmemBytes));
    if (e != cudaSuccess) return e;
    g_attr_set[dev][slot] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(prm.C);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kQmmSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qmm_w4g64_tc_kernel<NTH>, prm);
}

static cudaError_t launch_xprep(const __nv_bfloat16* x, int ldx, int M, int G, uint8_t* xw,
                                uint32_t* err, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qmm_xprep_kernel, x, ldx, M, xw, err);
}

cudaError_t qmm_tc_launch(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M, int N,
                          int K, void* ws, int C, cudaStream_t stream, bool pdl) {
  int dev = 0;
  cudaGetDevice(&dev);
  const QmmShape sh = qmm_shape(N, K);
  const WsLayout wl = ws_layout(N, K, C);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  QmmParams prm;
  prm.w_tc = static_cast<const uint8_t*>(w_tc);
  prm.xw = wsb + wl.x_off;
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.part = reinterpret_cast<float*>(wsb + wl.part_off);
  prm.cnt = reinterpret_cast<uint32_t*>(wsb + wl.cnt_off);
  prm.err = reinterpret_cast<uint32_t*>(wsb);
  prm.M = M;
  prm.N = N;
  prm.G = sh.G;
  prm.T = sh.T;
  prm.C = C;
  prm.ldo = ldo;
  prm.U = sh.U;
  cudaError_t e = launch_xprep(static_cast<const __nv_bfloat16*>(x), ldx, M, sh.G, wsb + wl.x_off,
                               prm.err, stream, pdl);
  if (e != cudaSuccess) return e;
  if (M <= 2) return launch_tc<1>(prm, dev, stream, true);
  if (M <= 4) return launch_tc<2>(prm, dev, stream, true);
  if (M <= 8) return launch_tc<4>(prm, dev, stream, true);
  return launch_tc<8>(prm, dev, stream, true);
}

cudaError_t qmm_repack_launch(const uint32_t* w, const uint16_t* s, const uint16_t* b, void* w_tc,
                              int N, int K, cudaStream_t stream) {
  const QmmShape sh = qmm_shape(N, K);
  const long long total = sh.U * kTileRows;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  qmm_repack_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      w, s, b, static_cast<uint8_t*>(w_tc), N, K, total);
  return cudaGetLastError();
}

cudaError_t qmm_simt_launch(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M,
                            int N, int K, cudaStream_t stream) {
  const QmmShape sh = qmm_shape(N, K);
  dim3 grid(sh.T, M);
  qmm_simt_kernel<<<grid, kTileRows, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), ldx,
                                                   static_cast<const uint8_t*>(w_tc),
                                                   static_cast<__nv_bfloat16*>(out), ldo, M, N, K);
  return cudaGetLastError();
}

}  // namespace skinny
