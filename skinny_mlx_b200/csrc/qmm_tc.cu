// 4-bit affine group-64 quantized matmul for 1..16 tokens on sm_100a (tcgen05 + TMEM + TMA).
//
//   out[t, n] = sum_g ( s[n,g] * sum_{k in g} x[t,k] * q[n,k]  +  b[n,g] * xsum[t,g] )
//
// This is the affine identity of skinny_mlx/qmm.py:8-9 and :64-71: scale and bias are applied
// once per 64-column group, in f32.  It is computed "swap-AB": weight rows are the 128-row MMA
// operand A and the tokens are the N=16 operand B, so a 1..16-token step reads every weight byte
// exactly once.
//
// Operands are bf16.  A nibble q OR-ed into the bf16 0x4300 (= 128) gives 128 + q exactly (the
// bf16 form of the reference's f16 0x6400 "1024 + q" trick, skinny_mlx/qmm.py:57-58), so the MMA
// sees A = 128 + q and x exactly as given, with f32 products exact.  A helper warp sums each x
// tile per token (xsum, f32, fixed reduction tree), and the epilogue folds the offset away:
//   s * sum x (128 + q) + (b - 128 s) * xsum  =  s * sum x q + b * xsum.
//
// Work split (stream-K): the matrix is cut into units of 128 rows x 64 columns (4608 relaid
// bytes, see qmm_layout.cuh) and each of the C CTAs (one per SM) takes a contiguous range of
// units in tile-major order, i.e. one contiguous byte range of the relaid weights.  Tiles that
// straddle CTAs are finished by the contributing CTA that arrives last; it adds the partial sums
// in contributor order, so results are deterministic and independent of the token count (row t
// of a 16-token call equals the same row of a 1-token call bit for bit).
//
// Load stages.  A TMA bulk copy costs a roughly fixed amount of engine time, so small copies cap
// the stream well below HBM bandwidth (measured on B200: 4.6 KB copies ~2.6 TB/s per CTA-per-SM,
// 18 KB copies ~6.6 TB/s).  A stage therefore carries up to 4 consecutive units of one tile:
// one bulk copy of their weights and one tensor-map box per unit for its x tile
// (64 columns x 8 or 16 token rows, SWIZZLE_128B, rows past M zero-filled).  Stages
// alternate between two (dequant warpgroup, MMA issuer) pairs, so each stage is consumed and
// released by exactly one pair plus the xsum warp.
//
// Warp roles in a CTA of 512 threads (16 warps):
//   warp 0 lane 0   TMA producer over a 3-stage ring.  The first stages are issued before
//                   griddepcontrol.wait only for their weights (weights do not depend on the
//                   previous kernel), so under programmatic dependent launch this launch's weight
//                   stream overlaps the tail of the previous one.  Tensor memory is allocated
//                   after that, since the previous kernel's CTA on this SM may still hold it.
//   warps 1, 15     MMA issuers for even / odd stages (warp 1 also allocates TMEM): per unit 4
//                   independent tcgen05.mma 128x16x16 (one per 16-column K slice, A = the unit's
//                   dequantized slot in TMEM, B = its x tile) as two independent 2-deep chains
//                   into two 16-column D sub-slots (long accumulation chains serialise in the
//                   tensor pipe).
//   warps 2..5      epilogue warpgroup, units in order: thread = weight row = TMEM lane; sums
//                   the 4 partial dot products, applies scale/bias with the tile's xsums and
//                   accumulates in f32 registers; writes finished tiles or publishes partials.
//   warps 6..9      dequant warpgroup for even stages, warps 10..13 for odd stages: thread =
//                   weight row; 64 nibbles (two 16-byte shared loads) -> 32 bf16x2 words ->
//                   tcgen05.st into the unit's A slot.
//   warp 14         xsum: per unit sums each token row of its x tile from shared memory.
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "ptx.cuh"
#include "qmm_layout.cuh"
#include "skinny_status.h"

namespace skinny {

constexpr int kStages = 3;
constexpr int kUPS = 4;                            // units per stage (same tile)
constexpr int kXTileBytes = 2048;                  // 16 token rows x 128 B (SWIZZLE_128B)
constexpr int kXStageBytes = kUPS * kXTileBytes;   // 8 KB
constexpr int kWStageBytes = kUPS * kUnitWBytes;   // 18 KB
constexpr int kXRingBytes = kStages * kXStageBytes;
constexpr int kWRingBytes = kStages * kWStageBytes;
constexpr int kNumA = 2 * kUPS;                    // TMEM A slots: 4 per dequant warpgroup
// TMEM D slots (2 x 16 columns each).  The two MMA issuers own alternate 4-unit stages, so one
// issuer's consecutive units can be up to 5 apart; the D ring must be at least that deep or a
// parity wait on d_empty can alias a phase two ahead.
constexpr int kNumD = 8;
constexpr int kTmemCols = 512;
constexpr int kDCol0 = kNumA * 32;                 // 256
constexpr int kThreads = 512;
constexpr int kEpiThreads = 128;
constexpr int kDeqThreads = 128;                   // per warpgroup
constexpr int kXsumWarp = 14;
constexpr int kRS = 16;                            // per-unit scale/bias + xsum ring for the epilogue

// Grouped launch: one persistent grid streams the concatenated units of up to kMaxMats
// independent matrices (same token count), so launch overhead, pipeline fill and the stream-K
// fix-up tail are paid once for the whole group.  A single qmm is a group of one.
constexpr int kMaxMats = 192;
constexpr int kMaxX = 8;

struct QmmMat {
  const uint8_t* w_tc;  // relaid weight units of this matrix
  __nv_bfloat16* out;   // [M, N] (leading dimension N)
  long long unit_off;   // first global unit of this matrix
  int N, G;             // rows, 64-column groups
  int tile_off;         // first global tile (counter index) of this matrix
  int xi;               // index of this matrix's activation tensor map
  int ldo;              // leading dimension of out (>= N)
};

struct QmmParams {
  float* part;          // [C_dev][2][16][128] partial sums (workspace)
  uint32_t* cnt;        // [kMaxTiles] arrival counters (workspace)
  uint32_t* err;        // device error word (workspace)
  int M, C, x_rows, n_mats;
  long long U;          // total units
  QmmMat mats[kMaxMats];
};

struct XMaps {
  CUtensorMap m[kMaxX];
};

// Matrix holding global unit u (largest m with unit_off <= u).
__device__ __forceinline__ int mat_of(const QmmParams& p, long long u) {
  int lo = 0, hi = p.n_mats - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.mats[mid].unit_off <= u) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// The epilogue, which trails the MMA, reads each unit's scale/bias words and xsums from a
// kRS-deep ring, so a load stage is released as soon as its dequant warpgroup, the xsum warp and
// its MMA issuer are done with it and the epilogue's lag never throttles the TMA stream.
struct __align__(16) QmmSmemBarriers {
  uint32_t sbr[kRS][kTileRows];        // per-unit (bf16 scale, bf16 bias) of each row
  float xsr[kRS][kMaxTokens];          // per-unit xsum of each token
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t a_full[kNumA];
  uint64_t a_empty[kNumA];
  uint64_t d_full[kNumD];
  uint64_t d_empty[kNumD];
  uint64_t sb_full[kRS];
  uint64_t xs_full[kRS];
  uint64_t ep_empty[kRS];
  uint64_t mma_done[2];
  uint32_t tmem_base;
  int abort_flag;
  int last_flag;
};

constexpr int kBarBytes = 12288;
constexpr size_t kQmmSmemBytes = static_cast<size_t>(kXRingBytes) + kWRingBytes + kBarBytes + 1024;
static_assert(sizeof(QmmSmemBarriers) <= kBarBytes, "barrier block");

// Units of the next stage starting at global unit u: at most kUPS, never past the CTA's range
// end or the end of u's tile (hence never across matrices).
__device__ __forceinline__ int stage_units(const QmmParams& p, long long u, long long u1) {
  const QmmMat& mt = p.mats[mat_of(p, u)];
  long long n = u1 - u;
  const int to_tile_end = mt.G - static_cast<int>((u - mt.unit_off) % mt.G);
  if (n > to_tile_end) n = to_tile_end;
  return n < kUPS ? static_cast<int>(n) : kUPS;
}

// 64 nibbles of one row (8 relaid words) -> 32 bf16x2 words holding (128 + q) exactly, in
// natural column order: pair j of word w covers columns 8w + 2j, 8w + 2j + 1.
__device__ __forceinline__ void decode8(const uint4& lo, const uint4& hi, uint32_t (&o)[32]) {
  const uint32_t words[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t v = words[j];
    o[4 * j + 0] = (v & 0x000F000Fu) | 0x43004300u;
    o[4 * j + 1] = ((v >> 4) & 0x000F000Fu) | 0x43004300u;
    o[4 * j + 2] = ((v >> 8) & 0x000F000Fu) | 0x43004300u;
    o[4 * j + 3] = ((v >> 12) & 0x000F000Fu) | 0x43004300u;
  }
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// NT: token columns read back per unit (2, 4, 8 or 16).
template <int NT>
__global__ void __launch_bounds__(kThreads, NT == 16 ? 1 : 2)
    qmm_w4g64_tc_kernel(const __grid_constant__ QmmParams p, const __grid_constant__ XMaps xmaps) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the SWIZZLE_128B x tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xring = smem;
  uint8_t* wring = smem + kXRingBytes;
  QmmSmemBarriers* sb = reinterpret_cast<QmmSmemBarriers*>(wring + kWRingBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const long long u0 = u_begin(c, p.U, p.C);
  const long long u1 = u_begin(c + 1, p.U, p.C);
  const int L = static_cast<int>(u1 - u0);
  const int xtile = p.x_rows * 128;  // bytes of one x tile in shared memory
  volatile int* abort_flag = &sb->abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&sb->full[i]), 1);
      mbar_init(smem_u32(&sb->empty[i]), 1 + kDeqThreads + 32);  // MMA commit + dequant wg + xsum warp
    }
    for (int i = 0; i < kNumA; ++i) {
      mbar_init(smem_u32(&sb->a_full[i]), kDeqThreads);
      mbar_init(smem_u32(&sb->a_empty[i]), 1);
    }
    for (int i = 0; i < kNumD; ++i) {
      mbar_init(smem_u32(&sb->d_full[i]), 1);
      mbar_init(smem_u32(&sb->d_empty[i]), kEpiThreads);
    }
    for (int i = 0; i < kRS; ++i) {
      mbar_init(smem_u32(&sb->sb_full[i]), kDeqThreads);
      mbar_init(smem_u32(&sb->xs_full[i]), 32);
      mbar_init(smem_u32(&sb->ep_empty[i]), kEpiThreads);
    }
    mbar_init(smem_u32(&sb->mma_done[0]), 1);
    mbar_init(smem_u32(&sb->mma_done[1]), 1);
    sb->abort_flag = 0;
    sb->last_flag = 0;
    fence_mbar_init();
    for (int q = 0; q < kMaxX; ++q) prefetch_tmap(&xmaps.m[q]);
  }
  __syncthreads();
  pdl_launch_dependents();
  // The producer starts streaming before tensor memory is allocated: under programmatic
  // dependent launch the CTA of the previous kernel on this SM may still hold its columns.
  uint32_t tmem = 0;
  if (warp != 0) {
    if (warp == 1) {
      tmem_alloc(smem_u32(&sb->tmem_base), kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
    named_bar_sync(2, kThreads - 32);
    tc_fence_after();
    tmem = sb->tmem_base;
  }

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      const uint64_t pol_w = policy_evict_first();
      const uint32_t xbytes = static_cast<uint32_t>(xtile);
      long long u = u0;
      int k = 0;
      // first stages: weights before griddepcontrol.wait, x tiles after
      long long first_u[kStages];
      int nfirst = 0;
      while (u < u1 && k < kStages) {
        const int n = stage_units(p, u, u1);
        const QmmMat& mt = p.mats[mat_of(p, u)];
        mbar_arrive_expect_tx(smem_u32(&sb->full[k]), static_cast<uint32_t>(n) * (kUnitWBytes + xbytes));
        bulk_g2s_hint(smem_u32(wring + k * kWStageBytes), mt.w_tc + (u - mt.unit_off) * kUnitWBytes,
                      static_cast<uint32_t>(n) * kUnitWBytes, smem_u32(&sb->full[k]), pol_w);
        first_u[k] = u;
        u += n;
        ++k;
        ++nfirst;
      }
      pdl_wait_prior_grid();  // x is produced by the previous kernel
      for (int f = 0; f < nfirst; ++f) {
        const QmmMat& mt = p.mats[mat_of(p, first_u[f])];
        const int g = static_cast<int>((first_u[f] - mt.unit_off) % mt.G);
        const int n = stage_units(p, first_u[f], u1);
        for (int j = 0; j < n; ++j)
          tma_load_2d(smem_u32(xring + f * kXStageBytes + j * xtile), &xmaps.m[mt.xi], (g + j) * kGroup, 0,
                      smem_u32(&sb->full[f]));
      }
      while (u < u1) {
        const int s = k % kStages;
        if (!mbar_wait(smem_u32(&sb->empty[s]), ((k / kStages) - 1) & 1, p.err, kErrBitWaitEmpty,
                       abort_flag))
          break;
        const int n = stage_units(p, u, u1);
        const QmmMat& mt = p.mats[mat_of(p, u)];
        const int g = static_cast<int>((u - mt.unit_off) % mt.G);
        mbar_arrive_expect_tx(smem_u32(&sb->full[s]), static_cast<uint32_t>(n) * (kUnitWBytes + xbytes));
        bulk_g2s_hint(smem_u32(wring + s * kWStageBytes), mt.w_tc + (u - mt.unit_off) * kUnitWBytes,
                      static_cast<uint32_t>(n) * kUnitWBytes, smem_u32(&sb->full[s]), pol_w);
        for (int j = 0; j < n; ++j)
          tma_load_2d(smem_u32(xring + s * kXStageBytes + j * xtile), &xmaps.m[mt.xi], (g + j) * kGroup, 0,
                      smem_u32(&sb->full[s]));
        u += n;
        ++k;
      }
      // Never leave the CTA with copies in flight: wait (bounded, ignoring abort) for the last
      // stages issued.  On the normal path they completed long ago.
      int zero = 0;
      for (int kk = (k > kStages ? k - kStages : 0); kk < k; ++kk)
        mbar_wait(smem_u32(&sb->full[kk % kStages]), (kk / kStages) & 1, p.err, kErrBitWaitDrain, &zero);
    }
  } else if (warp == 1 || warp == 15) {
    if (lane == 0) {
      // ------------------------------ MMA issuers (stages alternate) ---------------------------
      const int w = warp == 1 ? 0 : 1;
      constexpr uint32_t idesc = idesc_bf16_f32(128, 16);
      const uint64_t desc0 = smem_desc_sw128(smem_u32(xring));
      uint32_t a_uses[kUPS] = {0, 0, 0, 0};
      long long u = u0;
      int i = 0;  // unit index within this CTA
      bool live = true;
      for (int k = 0; u < u1 && live; ++k) {
        const int n = stage_units(p, u, u1);
        if ((k & 1) == w) {
          const int s = k % kStages;
          if (!mbar_wait(smem_u32(&sb->full[s]), (k / kStages) & 1, p.err, kErrBitWaitFull, abort_flag))
            break;
          for (int j = 0; j < n; ++j) {
            const int a = w * kUPS + j;
            const int d = (i + j) % kNumD;
            if (!mbar_wait(smem_u32(&sb->a_full[a]), a_uses[j] & 1, p.err, kErrBitWaitAFull, abort_flag) ||
                (i + j >= kNumD &&
                 !mbar_wait(smem_u32(&sb->d_empty[d]), (((i + j) / kNumD) - 1) & 1, p.err,
                            kErrBitWaitDEmpty, abort_flag))) {
              live = false;
              break;
            }
            ++a_uses[j];
            tc_fence_after();
            // start-address field: stage base + j x-tile + 32 bytes per 16-column K slice
            const uint64_t bdesc = desc0 + static_cast<uint64_t>((s * kXStageBytes + j * xtile) >> 4);
            const uint32_t d_dot = tmem + kDCol0 + d * 32;
            const uint32_t a_tmem = tmem + a * 32;
            umma_f16_ts(d_dot, a_tmem, bdesc, idesc, 0u);                 // columns 0-15
            umma_f16_ts(d_dot + 16, a_tmem + 16, bdesc + 4, idesc, 0u);   // columns 32-47
            umma_f16_ts(d_dot, a_tmem + 8, bdesc + 2, idesc, 1u);         // columns 16-31
            umma_f16_ts(d_dot + 16, a_tmem + 24, bdesc + 6, idesc, 1u);   // columns 48-63
            umma_commit(smem_u32(&sb->a_empty[a]));
            umma_commit(smem_u32(&sb->d_full[d]));
          }
          if (!live) break;
          umma_commit(smem_u32(&sb->empty[s]));
        }
        u += n;
        i += n;
      }
      // Every MMA issued by this thread completes before TMEM is released.
      umma_commit(smem_u32(&sb->mma_done[w]));
      int zero = 0;
      mbar_wait(smem_u32(&sb->mma_done[w]), 0, p.err, kErrBitWaitDrain, &zero);
    }
  } else if (warp == kXsumWarp) {
    // ------------------------------ xsum of each x tile ------------------------------
    // lane = (token t = lane / 2, half h = lane % 2); chunk sums are combined in the same tree
    // for every token count, so a token's xsum is bit-identical for any M.
    const int t = lane >> 1, h = lane & 1;
    long long u = u0;
    int i = 0;
    bool live = true;
    for (int k = 0; u < u1 && live; ++k) {
      const int n = stage_units(p, u, u1);
      const int s = k % kStages;
      if (!mbar_wait(smem_u32(&sb->full[s]), (k / kStages) & 1, p.err, kErrBitWaitFull, abort_flag))
        break;
      float part[kUPS];
      for (int j = 0; j < n; ++j) {
        // rows >= x_rows of a tile belong to the next tile (or are stale): their sums are unused
        const uint8_t* row = xring + s * kXStageBytes + j * xtile + t * 128;
        float cs[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int cch = 4 * h + q;  // 16-byte chunk = 8 columns; SWIZZLE_128B permutes chunks by row
          const uint4 v = *reinterpret_cast<const uint4*>(row + ((cch ^ (t & 7)) << 4));
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
          float acc = 0.f;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            acc += __uint_as_float(wv[kk] << 16);
            acc += __uint_as_float(wv[kk] & 0xFFFF0000u);
          }
          cs[q] = acc;
        }
        float pt = (cs[0] + cs[1]) + (cs[2] + cs[3]);
        pt += __shfl_xor_sync(0xFFFFFFFFu, pt, 1);
        part[j] = pt;
      }
      mbar_arrive(smem_u32(&sb->empty[s]));  // this warp is done with the stage's x tiles
      for (int j = 0; j < n; ++j) {
        const int jr = (i + j) % kRS;
        if (i + j >= kRS && !mbar_wait(smem_u32(&sb->ep_empty[jr]), (((i + j) / kRS) - 1) & 1, p.err,
                                       kErrBitWaitEmpty, abort_flag)) {
          live = false;
          break;
        }
        if (h == 0) sb->xsr[jr][t] = part[j];
        __syncwarp();
        mbar_arrive(smem_u32(&sb->xs_full[jr]));
      }
      u += n;
      i += n;
    }
  } else if (warp >= 6 && warp < 14) {
    // ------------------------------ dequant (two warpgroups, stages alternate) ----------------
    const int w = (warp - 6) >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t a_uses[kUPS] = {0, 0, 0, 0};
    long long u = u0;
    int i = 0;
    bool live = true;
    for (int k = 0; u < u1 && live; ++k) {
      const int n = stage_units(p, u, u1);
      if ((k & 1) == w) {
        const int s = k % kStages;
        if (!mbar_wait(smem_u32(&sb->full[s]), (k / kStages) & 1, p.err, kErrBitWaitFull, abort_flag))
          break;
        for (int j = 0; j < n; ++j) {
          const uint8_t* wu = wring + s * kWStageBytes + j * kUnitWBytes;
          const uint4 lo = *reinterpret_cast<const uint4*>(wu + r * 16);
          const uint4 hi = *reinterpret_cast<const uint4*>(wu + 2048 + r * 16);
          const uint32_t sbw = *reinterpret_cast<const uint32_t*>(wu + kUnitNibBytes + r * 4);
          if (j == n - 1) mbar_arrive(smem_u32(&sb->empty[s]));  // done reading the weight stage
          const int jr = (i + j) % kRS;
          if (i + j >= kRS && !mbar_wait(smem_u32(&sb->ep_empty[jr]), (((i + j) / kRS) - 1) & 1,
                                         p.err, kErrBitWaitEmpty, abort_flag)) {
            live = false;
            break;
          }
          sb->sbr[jr][r] = sbw;
          mbar_arrive(smem_u32(&sb->sb_full[jr]));
          uint32_t q[32];
          decode8(lo, hi, q);
          const int a = w * kUPS + j;
          if (a_uses[j] > 0 &&
              !mbar_wait(smem_u32(&sb->a_empty[a]), (a_uses[j] - 1) & 1, p.err, kErrBitWaitAEmpty,
                         abort_flag)) {
            live = false;
            break;
          }
          ++a_uses[j];
          tc_fence_after();
          tmem_st_x32(tmem + lane_off + a * 32, q);
          tc_wait_st();
          tc_fence_before();
          mbar_arrive(smem_u32(&sb->a_full[a]));
        }
      }
      u += n;
      i += n;
    }
  } else {
    // ------------------------------ epilogue (warps 2..5), units in order ----------------------
    const int e = threadIdx.x - 64;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    bool dep_waited = false;

    for (int i = 0; i < L; ++i) {
      const int d = i % kNumD;
      const int jr = i % kRS;
      const uint32_t ph = (i / kRS) & 1;
      const bool ok = mbar_wait(smem_u32(&sb->xs_full[jr]), ph, p.err, kErrBitWaitFull, abort_flag) &&
                      mbar_wait(smem_u32(&sb->sb_full[jr]), ph, p.err, kErrBitWaitFull, abort_flag) &&
                      mbar_wait(smem_u32(&sb->d_full[d]), (i / kNumD) & 1, p.err, kErrBitWaitDFull,
                                abort_flag);
      if (ok) {
        const uint32_t sbw = sb->sbr[jr][r];
        const float sc = __uint_as_float(sbw << 16);
        const float bi = __uint_as_float(sbw & 0xFFFF0000u);
        const float bo = fmaf(-128.0f, sc, bi);  // bias with the +128 operand offset folded in
        // acc += (b - 128 s) * xsum, then acc += s * dot  (same order for every NT)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = fmaf(bo, sb->xsr[jr][t], acc[t]);
        mbar_arrive(smem_u32(&sb->ep_empty[jr]));
        // dot = (columns 0-31 partial) + (columns 32-63 partial)
        const uint32_t dbase = tmem + lane_off + kDCol0 + d * 32;
        float s01[NT], v[NT];
        tc_fence_after();
        tmem_ld<NT>(dbase, s01);
        tmem_ld<NT>(dbase + 16, v);
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(smem_u32(&sb->d_empty[d]));
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = fmaf(sc, s01[t] + v[t], acc[t]);
      }
      const long long u = u0 + i;
      const QmmMat& mt = p.mats[mat_of(p, u)];
      const long long lu = u - mt.unit_off;
      const int g = static_cast<int>(lu % mt.G);
      if (g != mt.G - 1 && i != L - 1) continue;
      // ---- end of a tile segment: write the tile, or publish a partial and maybe finish it
      const long long ltile = lu / mt.G;                     // tile within the matrix
      const long long tile_u0 = mt.unit_off + ltile * mt.G;  // its first global unit
      const long long tile = mt.tile_off + ltile;            // global tile (counter index)
      const long long seg_start = (tile_u0 > u0) ? tile_u0 : u0;
      const bool full_tile = (seg_start == tile_u0) && (g == mt.G - 1);
      const bool first_seg = (seg_start == u0);
      const int row_g = static_cast<int>(ltile) * kTileRows + r;
      const bool live = !*abort_flag;
      if (!dep_waited) {
        pdl_wait_prior_grid();  // outputs may alias buffers the previous kernel still reads
        dep_waited = true;
      }
      if (full_tile) {
        if (live && row_g < mt.N) {
#pragma unroll
          for (int t = 0; t < NT; ++t)
            if (t < p.M) mt.out[static_cast<size_t>(t) * mt.ldo + row_g] = __float2bfloat16_rn(acc[t]);
        }
      } else {
        float* mine = p.part + (static_cast<size_t>(c) * 2 + (first_seg ? 0 : 1)) * kMaxTokens * kTileRows;
#pragma unroll
        for (int t = 0; t < NT; ++t) mine[t * kTileRows + r] = acc[t];
        __threadfence();
        named_bar_sync(1, kEpiThreads);
        const long long cf = cta_of_unit(tile_u0, p.U, p.C);
        const long long cl = cta_of_unit(tile_u0 + mt.G - 1, p.U, p.C);
        if (e == 0) {
          const unsigned n_contrib = static_cast<unsigned>(cl - cf + 1);
          const unsigned old = live ? atomicAdd(&p.cnt[tile], 1u) : 0u;
          sb->last_flag = live && (old == n_contrib - 1);
        }
        named_bar_sync(1, kEpiThreads);
        if (sb->last_flag) {
          __threadfence();
          float v[NT];
#pragma unroll
          for (int t = 0; t < NT; ++t) v[t] = 0.f;
          for (long long cc = cf; cc <= cl; ++cc) {
            const long long cu0 = u_begin(cc, p.U, p.C);
            const int cs = (cu0 >= tile_u0) ? 0 : 1;  // the tile is this contributor's first segment
            const float* src = p.part + (static_cast<size_t>(cc) * 2 + cs) * kMaxTokens * kTileRows;
#pragma unroll
            for (int t = 0; t < NT; ++t) v[t] += __ldcg(src + t * kTileRows + r);
          }
          if (row_g < mt.N) {
#pragma unroll
            for (int t = 0; t < NT; ++t)
              if (t < p.M) mt.out[static_cast<size_t>(t) * mt.ldo + row_g] = __float2bfloat16_rn(v[t]);
          }
          if (e == 0) p.cnt[tile] = 0u;
        }
        named_bar_sync(1, kEpiThreads);
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
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

// Plain CUDA-core cross-check of the relaid format: decodes the same units and computes
// sum_g s * sum(x q) + b * sum(x) in f32.  One thread per (row, token); tests only.
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
    const float sc = __uint_as_float(sbw << 16);
    const float bi = __uint_as_float(sbw & 0xFFFF0000u);
    const uint4 lo = *reinterpret_cast<const uint4*>(base + r * 16);
    const uint4 hi = *reinterpret_cast<const uint4*>(base + 2048 + r * 16);
    uint32_t q[32];
    decode8(lo, hi, q);
    float gs = 0.f, xsum = 0.f;
    for (int pidx = 0; pidx < 32; ++pidx) {
      const int k = g * kGroup + pidx * 2;
      const float x0 = __bfloat162float(x[static_cast<size_t>(tok) * ldx + k]);
      const float x1 = __bfloat162float(x[static_cast<size_t>(tok) * ldx + k + 1]);
      const float q0 = static_cast<float>(q[pidx] & 0xFu);
      const float q1 = static_cast<float>((q[pidx] >> 16) & 0xFu);
      gs = fmaf(q0, x0, gs);
      gs = fmaf(q1, x1, gs);
      xsum += x0;
      xsum += x1;
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
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

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

static cudaError_t get_encoder() {
  if (g_encode) return cudaSuccess;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess) return e;
  if (q != cudaDriverEntryPointSuccess || fn == nullptr) return cudaErrorNotSupported;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return cudaSuccess;
}

// x [M rows, K columns] bf16, row stride ldx elements; box 64 columns x `rows` rows, 128B swizzle.
// (A 3-D view {64, rows, groups} would need a group stride below the row stride, which tensor maps
// do not support: each stride must include the previous dimension's.)
static cudaError_t encode_x_map(CUtensorMap* map, const void* x, int M, int K, int ldx, int rows) {
  cudaError_t e = get_encoder();
  if (e != cudaSuccess) return e;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldx) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kGroup), static_cast<cuuint32_t>(rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int NT>
static cudaError_t launch_tc(const QmmParams& prm, const XMaps& maps, int dev, cudaStream_t stream,
                             bool pdl) {
  constexpr int slot = NT == 2 ? 0 : NT == 4 ? 1 : NT == 8 ? 2 : 3;
  if (dev >= 0 && dev < 64 && !g_attr_set[dev][slot]) {
    cudaError_t e = cudaFuncSetAttribute(qmm_w4g64_tc_kernel<NT>,
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
  return cudaLaunchKernelEx(&cfg, qmm_w4g64_tc_kernel<NT>, prm, maps);
}

// Grouped launch over n matrices sharing the token count M.  Shapes and pointers were validated
// by the caller; distinct (x, K, ldx) inputs share tensor maps (at most kMaxX of them).  The
// scratch is given as its three parts: error word, per-tile counters (zero on entry, left zero)
// and partial sums for up to `C_cap` CTAs.
static cudaError_t launch_grouped_on(int n, const void* const* x, const int* ldx,
                                     const void* const* w_tc, void* const* out, const int* ldo,
                                     const int* N, const int* K, int M, uint32_t* err,
                                     uint32_t* cnt, float* part, int C_cap, int dev,
                                     cudaStream_t stream, bool pdl) {
  if (n < 1 || n > kMaxMats) return cudaErrorInvalidValue;
  const int C_dev = C_cap;
  static thread_local QmmParams prm;  // ~10 KB: keep it off the stack
  static thread_local XMaps maps;
  prm.part = part;
  prm.cnt = cnt;
  prm.err = err;
  prm.M = M;
  prm.x_rows = M <= 8 ? 8 : 16;
  prm.n_mats = n;
  const void* xkey[kMaxX];
  int kkey[kMaxX], lkey[kMaxX];
  int nx = 0;
  long long U = 0;
  long long T = 0;
  for (int i = 0; i < n; ++i) {
    const QmmShape sh = qmm_shape(N[i], K[i]);
    int xi = -1;
    for (int q = 0; q < nx; ++q)
      if (xkey[q] == x[i] && kkey[q] == K[i] && lkey[q] == ldx[i]) xi = q;
    if (xi < 0) {
      if (nx == kMaxX) return cudaErrorInvalidValue;
      xi = nx++;
      xkey[xi] = x[i];
      kkey[xi] = K[i];
      lkey[xi] = ldx[i];
      cudaError_t e = encode_x_map(&maps.m[xi], x[i], M, K[i], ldx[i], prm.x_rows);
      if (e != cudaSuccess) return e;
    }
    QmmMat& mt = prm.mats[i];
    mt.w_tc = static_cast<const uint8_t*>(w_tc[i]);
    mt.out = static_cast<__nv_bfloat16*>(out[i]);
    mt.unit_off = U;
    mt.N = N[i];
    mt.G = sh.G;
    mt.tile_off = static_cast<int>(T);
    mt.xi = xi;
    mt.ldo = ldo[i];
    U += sh.U;
    T += sh.T;
  }
  if (T > kMaxTiles) return cudaErrorInvalidValue;
  for (int q = nx; q < kMaxX; ++q) maps.m[q] = maps.m[0];
  prm.U = U;
  prm.C = static_cast<int>(U < C_dev ? U : C_dev);
  if (M <= 2) return launch_tc<2>(prm, maps, dev, stream, pdl);
  if (M <= 4) return launch_tc<4>(prm, maps, dev, stream, pdl);
  if (M <= 8) return launch_tc<8>(prm, maps, dev, stream, pdl);
  return launch_tc<16>(prm, maps, dev, stream, pdl);
}

cudaError_t qmm_tc_launch_grouped(int n, const void* const* x, const int* ldx, const void* const* w_tc,
                                  void* const* out, const int* ldo, const int* N, const int* K, int M,
                                  void* ws, cudaStream_t stream, bool pdl) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int C_dev = device_sm_count(dev);
  const WsLayout wl = ws_layout(0, 0, C_dev);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  return launch_grouped_on(n, x, ldx, w_tc, out, ldo, N, K, M, reinterpret_cast<uint32_t*>(wsb),
                           reinterpret_cast<uint32_t*>(wsb + wl.cnt_off),
                           reinterpret_cast<float*>(wsb + wl.part_off), C_dev, dev, stream, pdl);
}

// ---------------------------------------------------------------------------------------------
// No-allocation variant: the scratch is a fixed array in this module's device memory.
//
// Some callers have no way to hand us device memory for the workspace: a host runtime reached
// through a plain C FFI that owns no CUDA allocator and carries no device-buffer type, a serving
// loop whose memory budget is fixed when it starts and which must not grow it per request, or a
// step that must never call cudaMalloc/cudaFree because those calls can synchronise the whole
// device and stall the other streams sharing it.  For them the scratch lives in a file-scope
// __device__ array, sized once for the largest call it accepts, and its address is looked up
// with cudaGetSymbolAddress; nothing is allocated by this path, by the CUDA runtime on its behalf,
// or by any library.
//
// Limits: N <= kNoAllocMaxTiles * 128 rows (tail tiles count whole) and at most kNoAllocMaxCtas
// CTAs (a device with more SMs uses kNoAllocMaxCtas of them).  There is ONE scratch per device,
// so two calls that may run at the same time on one device (different streams, threads without
// ordering) race on it and corrupt each other's results; calls must be ordered, e.g. on a single
// stream.  The first call on a device does the set-up (symbol lookup, kernel attributes, tensor-
// map encoder lookup) and should come before any stream capture.
// ---------------------------------------------------------------------------------------------
constexpr int kNoAllocMaxTiles = 2048;  // N <= 262,144 rows
constexpr int kNoAllocMaxCtas = 160;
constexpr size_t kNoAllocCntOff = 256;
constexpr size_t kNoAllocPartOff = kNoAllocCntOff + static_cast<size_t>(kNoAllocMaxTiles) * 4;
constexpr size_t kNoAllocScratchBytes =
    kNoAllocPartOff + static_cast<size_t>(kNoAllocMaxCtas) * 2 * kMaxTokens * kTileRows * 4;
static_assert(kNoAllocScratchBytes == 2629888, "2.5 MiB of static scratch per device");
static_assert(kNoAllocPartOff % 256 == 0, "partials start on a 256-byte boundary");

// [0, 256) error word + padding | [256, 8448) tile counters | [8448, ...) partial sums
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mutex;
static uint8_t* g_noalloc_ptr[64] = {};

// Looks the scratch up on the current device (once per device).
static cudaError_t noalloc_scratch(int dev, uint8_t** out) {
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 255u) != 0) return cudaErrorInvalidValue;
    g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

bool qmm_noalloc_fits(int N, int K) {
  return qmm_shape(N, K).T <= kNoAllocMaxTiles;
}

// The error word and the counters must be zero when the kernel starts.  A launch that completes
// leaves the counters at zero, but one that stopped on a timed-out wait may not, so both are
// cleared on the stream before every launch (a memset node: no allocation).  The launch does not
// use programmatic dependent launch, so it cannot start before that clear has finished.
cudaError_t qmm_tc_launch_noalloc(const void* x, int ldx, const void* w_tc, void* out, int ldo,
                                  int M, int N, int K, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  uint8_t* scratch = nullptr;
  e = noalloc_scratch(dev, &scratch);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(scratch, 0, kNoAllocPartOff, stream);
  if (e != cudaSuccess) return e;
  const int sms = device_sm_count(dev);
  const int C_cap = sms < kNoAllocMaxCtas ? sms : kNoAllocMaxCtas;
  void* o = out;
  return launch_grouped_on(1, &x, &ldx, &w_tc, &o, &ldo, &N, &K, M,
                           reinterpret_cast<uint32_t*>(scratch),
                           reinterpret_cast<uint32_t*>(scratch + kNoAllocCntOff),
                           reinterpret_cast<float*>(scratch + kNoAllocPartOff), C_cap, dev, stream,
                           false);
}

cudaError_t qmm_tc_launch(const void* x, int ldx, const void* w_tc, void* out, int ldo, int M, int N,
                          int K, void* ws, int /*C*/, cudaStream_t stream, bool pdl) {
  void* o = out;
  return qmm_tc_launch_grouped(1, &x, &ldx, &w_tc, &o, &ldo, &N, &K, M, ws, stream, pdl);
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
