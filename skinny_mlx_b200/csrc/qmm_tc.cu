// 4-bit affine group-64 quantized matmul for 1..16 tokens on sm_100a (tcgen05 + TMEM + TMA).
//
//   out[t, n] = sum_g ( s[n,g] * sum_{k in g} x[t,k] * q[n,k]  +  b[n,g] * xsum[t,g] )
//
// This is the affine identity of skinny_mlx/qmm.py:8-9 and :64-71: scale and bias are applied
// once per 64-column group, in f32.  It is computed "swap-AB": weight rows are the 128-row MMA
// operand A and the tokens are the narrow operand B, so a 1..16-token step reads every weight
// byte exactly once.
//
// Integer tensor cores (tcgen05.mma kind::i8).  The relaid nibble q ^ 8 shifted into the high
// half of a byte is the signed 8-bit value 16 (q - 8): two ALU ops per eight weights produce the
// A operand.  x is given to the tensor core as 16-bit fixed point per (token, group): with the
// power-of-two exponent e chosen so that |v| <= 32639, v = rint(x 2^-e) = 256 hi + lo with
// signed 8-bit digits hi, lo, which an x-prep kernel writes once per call.  B holds the hi
// digits of every token in its first rows and the lo digits in the next, so one MMA gives both
// integer dot products exactly (s32 accumulators).  The epilogue computes, per group,
//   G = 256 dot(hi) + dot(lo) = sum v * 16 (q - 8)
//   out += (s 2^(e-4)) * G + (b + 8 s) * (2^e sum v)  =  s * sum x q + b * sum x   (x := v 2^e)
// The only rounding before the f32 accumulation is that of x to 16 significant bits relative
// to its group maximum (at most 2^-16 of it), far below the bf16 output rounding.
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
// 18 KB copies ~6.6 TB/s).  A stage therefore carries up to 4 consecutive units of one tile: one
// bulk copy of their weights and one of their x-prep blocks (consecutive groups are adjacent).
// Stages alternate between two "lanes", each with its own dequant warpgroup, MMA issuer,
// tensor-memory slots and epilogue warpgroup, so every step of one stage overlaps the same step
// of the other.  The hand-offs between the roles are per stage, not per unit: one mbarrier phase
// per lane and stage.
//
// Warp roles in a CTA of 640 threads (20 warps), one CTA per SM:
//   warp 0 lane 0   TMA producer over an 8-stage ring (6 for M > 8).  The first stages are issued before
//                   griddepcontrol.wait only for their weights (weights do not depend on the
//                   previous kernel), so under programmatic dependent launch this launch's weight
//                   stream overlaps the tail of the previous one.  Tensor memory is allocated
//                   after that, since the previous kernel's CTA on this SM may still hold it.
//   warps 1, 2      MMA issuers of lane 0 / lane 1 (warp 1 also allocates TMEM): per stage two
//                   chained tcgen05.mma 128 x (2 mpad) x 32 per unit into the unit's D slot.
//   warps 4..7      dequant warpgroup of lane 0, warps 8..11 of lane 1: thread = weight row;
//                   per unit 64 nibbles (two 16-byte shared loads) -> 16 int8x4 words ->
//                   tcgen05.st into the unit's A slot; also copies the units' scale/bias and x
//                   scales to a small ring read by the epilogue, so a load stage is released early.
//   warps 12..15    epilogue warpgroup of lane 0, warps 16..19 of lane 1: thread = weight row =
//                   TMEM lane; combines the digit dot products, applies scale/bias once per group
//                   and accumulates in f32 registers; at each tile end the two lanes' sums are
//                   added in a fixed order and the tile is written or its partial published.
//   warp 3          allocation helper only.
#include <algorithm>
#include <cfloat>
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "digits.cuh"
#include "peer.cuh"
#include "ptx.cuh"
#include "qmm_layout.cuh"
#include "skinny_status.h"

namespace skinny {

// Load stages in flight: as many as shared memory holds (one CTA per SM), since the stream is
// bounded by (load latency + processing) / stages.  Even, so stage slot s is always used by lane
// s % 2 (a role then only ever waits on slots its own lane used before).
__host__ __device__ constexpr int stages_for(int NT) { return NT <= 8 ? 8 : 6; }
constexpr int kMaxStages = 8;
constexpr int kUPS = 4;                            // units per stage (same tile)
constexpr int kWStageBytes = kUPS * kUnitWBytes;   // 18 KB
constexpr int kThreads = 640;
constexpr int kDeqWarp0 = 4;                       // warps 4..7 lane 0, 8..11 lane 1
constexpr int kEpiWarp0 = 12;                      // warps 12..15 lane 0, 16..19 lane 1
constexpr int kEpiThreads = 128;
constexpr int kACols = 16;                         // TMEM columns of one unit's int8 A operand
// Slot sets: stage k runs on lane k % 2 (dequant warpgroup, MMA issuer, epilogue warpgroup) and
// uses A-set k % kSetsA (its units' A operands in TMEM and meta slots in shared memory, free once
// its MMAs completed and the epilogue read the meta) and D-set k % setsD (accumulators in TMEM,
// free once the epilogue read them).  Both counts are even, so a set always belongs to one lane,
// and with several sets per lane the decode, MMAs and epilogue of consecutive stages of a lane
// overlap instead of forming one chain.  Tensor memory bounds them: 4 A-sets x 4 units x 16
// columns plus 4 D-sets x 4 units x 16 columns for M <= 8 (32 D columns per unit, 2 D-sets, for
// M > 8) = 512 columns.
constexpr int kSetsA = 4;
__host__ __device__ constexpr int sets_d_for(int NT) { return NT <= 8 ? 4 : 2; }
constexpr int kMaxSets = 4;

// Grouped launch: one persistent grid streams the concatenated units of up to kMaxMats
// independent matrices (same token count), so launch overhead, pipeline fill and the stream-K
// fix-up tail are paid once for the whole group.  A single qmm is a group of one.
constexpr int kMaxMats = 192;
constexpr int kMaxX = 8;

// Unit indices fit in 32 bits: at most kMaxTiles tiles of at most kMaxXGroups groups (2^25).
struct QmmMat {
  const uint8_t* w_tc;  // relaid weight units of this matrix
  __nv_bfloat16* out;   // [M, N] (leading dimension ldo)
  int unit_off;         // first global unit of this matrix
  int N, G;             // rows, 64-column groups
  int tile_off;         // first global tile (counter index) of this matrix
  int xg_off;           // first x-prep block of this matrix's input
  int ldo;              // leading dimension of out (>= N)
};

struct QmmParams {
  float* part;          // [C][2][16][128] partial sums (workspace)
  uint32_t* cnt;        // [kMaxTiles] arrival counters (workspace)
  uint32_t* err;        // device error word (workspace)
  const uint8_t* xq;    // x-prep blocks (workspace)
  int M, C, n_mats;
  int U;                // total units
  int split;            // 0: stream-K over all units; S >= 1: one matrix, S CTAs (a cluster) per tile
  // One-matrix calls of a sharded step: the x-prep blocks of groups [r * xq_gpr, (r+1) * xq_gpr)
  // are read from rank r's buffer xq_rank[r] (at the same offsets as in a full buffer) after
  // waiting for the ranks' flags; the launch signals its completion (sync).  xq_gpr = 0: xq.
  const uint8_t* xq_rank[kMaxPeers];
  int xq_gpr;
  PeerSync sync;
  // SwiGLU epilogue (one-matrix prepared calls): with swiglu_xq set, the weight's tile j holds the
  // gate rows 64j .. 64j+63 then the up rows 64j .. 64j+63, and instead of the bf16 output a
  // finished tile writes group j of the qmm input digits of a = bf16(silu(g) u) to swiglu_xq.
  uint8_t* swiglu_xq;
  QmmMat mats[kMaxMats];
};

struct XPrepIn {
  const __nv_bfloat16* x;
  int ldx, G, xg_off, pad_;
};

struct XPrepParams {
  XPrepIn in[kMaxX];
  uint8_t* xq;
  int n_in, M, mpad, total_groups;
};

// Per-unit data the epilogue needs after the load stage is gone: each row's (scale, bias) and
// the tokens' xs / xsum.  One slot per (lane, unit of the stage), like the D slots.
struct __align__(16) QmmMeta {
  uint32_t sb[kTileRows];
  float x[2 * kMaxTokens];  // xs[0..15] then xsum[0..15]
};

struct __align__(16) QmmSmem {
  QmmMeta meta[kSetsA][kUPS];
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  // Per lane, one phase per stage of that lane ("lane-stage"):
  // Per slot set, one phase per use (one stage):
  uint64_t a_full[kSetsA];    // dequant -> MMA/epilogue: A slots stored, meta slots written
  uint64_t a_free[kSetsA];    // MMA commit + epilogue (meta read) -> dequant
  uint64_t d_full[kMaxSets];  // MMA -> epilogue: accumulators ready
  uint64_t d_free[kMaxSets];  // epilogue -> MMA: accumulators read
  uint64_t mma_done[2];
  uint32_t tmem_base;
  int abort_flag;
  int last_flag[2];
  int pre_xg[kMaxStages], pre_n[kMaxStages];  // producer: the prefetched stages' x-prep groups and unit counts
};
// followed by the epilogue's partial-sum exchange, float [2][NT][128]

__host__ __device__ constexpr int mpad_of(int NT) { return NT <= 8 ? 8 : 16; }
__host__ __device__ constexpr int xstage_bytes(int NT) { return kUPS * xq_block_bytes(mpad_of(NT)); }
__host__ __device__ constexpr size_t qmm_smem_bytes(int NT) {
  return static_cast<size_t>(stages_for(NT)) * (xstage_bytes(NT) + kWStageBytes) + sizeof(QmmSmem) +
         static_cast<size_t>(2) * NT * kTileRows * 4 + 128;
}
// One CTA per SM: the register budget (up to 128 per thread) keeps each warp's working set of
// a whole stage in registers, which matters more than co-residency with the next launch.
static_assert(qmm_smem_bytes(8) <= 227 * 1024 && qmm_smem_bytes(16) <= 227 * 1024,
              "shared memory of one CTA");
static_assert(stages_for(8) % 2 == 0 && stages_for(16) % 2 == 0 && stages_for(16) <= kMaxStages,
              "stage ring");

// Walks a CTA's unit range in stages, tracking the matrix, the tile within it and the group
// within the tile incrementally (no division per unit).  A stage never crosses a tile end.  The
// current matrix's fields are held in registers and reloaded only when the walk enters the next
// matrix: indexed reads of the kernel-parameter table cost hundreds of cycles each, which every
// role would otherwise pay on every stage.
struct UnitWalk {
  int u;         // global unit at the start of the current stage
  int mi;        // matrix of unit u
  int lt;        // tile of unit u within its matrix
  int g;         // group of unit u within its tile
  int G;         // groups per tile of matrix mi
  int uoff;      // first global unit of matrix mi
  int next_off;  // first global unit of matrix mi + 1 (INT_MAX for the last)
  __device__ __forceinline__ void load(const QmmParams& p) {
    G = p.mats[mi].G;
    uoff = p.mats[mi].unit_off;
    next_off = mi + 1 < p.n_mats ? p.mats[mi + 1].unit_off : 0x7FFFFFFF;
  }
  __device__ __forceinline__ void init(const QmmParams& p, int u0) {
    int lo = 0, hi = p.n_mats - 1;  // largest m with unit_off <= u0
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.mats[mid].unit_off <= u0) lo = mid; else hi = mid - 1;
    }
    mi = lo;
    load(p);
    const int lu = u0 - uoff;
    lt = lu / G;
    g = lu - lt * G;
    u = u0;
  }
  // Units of the stage starting at u: at most kUPS, never past u1 or the end of u's tile.
  __device__ __forceinline__ int stage_n(int u1) const {
    int n = u1 - u;
    if (n > G - g) n = G - g;
    return n < kUPS ? n : kUPS;
  }
  __device__ __forceinline__ void advance(const QmmParams& p, int n) {
    u += n;
    g += n;
    if (g == G) {
      g = 0;
      ++lt;
      if (u == next_off) {
        ++mi;
        lt = 0;
        load(p);
      }
    }
  }
};

// 64 relaid nibbles of one row -> 16 words of four int8 values 16 (q - 8), in column order.
__device__ __forceinline__ void decode_i8(const uint4& c0, const uint4& c1, uint32_t (&o)[16]) {
  const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    o[2 * j] = w[j] & 0xF0F0F0F0u;
    o[2 * j + 1] = (w[j] << 4) & 0xF0F0F0F0u;
  }
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------------------------
// x-prep: one warp per (token, group).  Lane l holds columns 2l, 2l+1 of the group.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) qmm_xprep_kernel(const __grid_constant__ XPrepParams p) {
  pdl_launch_dependents();  // the qmm kernel may start streaming weights now
  pdl_wait_prior_grid();    // x is written by the previous kernel
  const int wid = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int mpad = p.mpad;
  if (wid >= p.total_groups * mpad) return;
  const int gg = wid / mpad;  // global x-prep block
  const int t = wid - gg * mpad;
  int i = 0;
  while (i + 1 < p.n_in && gg >= p.in[i + 1].xg_off) ++i;
  const XPrepIn& in = p.in[i];
  const int g = gg - in.xg_off;

  float x0 = 0.f, x1 = 0.f;
  if (t < p.M) {
    const uint32_t w2 = *reinterpret_cast<const uint32_t*>(in.x + static_cast<size_t>(t) * in.ldx +
                                                           g * kGroup + 2 * lane);
    x0 = __uint_as_float(w2 << 16);
    x1 = __uint_as_float(w2 & 0xFFFF0000u);
  }
  float amax = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  // fmaxf drops a NaN operand: detect non-finite values separately
  const bool bad = __any_sync(0xFFFFFFFFu, !(fabsf(x0) <= FLT_MAX) || !(fabsf(x1) <= FLT_MAX));

  int v0 = 0, v1 = 0;
  float xs = 0.f, xsum = 0.f;
  if (bad) {
    xs = __int_as_float(0x7FC00000);  // the group's products become NaN, as in f32 arithmetic
    xsum = xs;
  } else if (amax > 0.f) {
    int e2;
    frexpf(amax, &e2);                 // amax = m 2^e2, m in [0.5, 1)
    int e = e2 - 15;                   // smallest e with amax <= 32639 2^e is e2-15 or e2-14
    if (ldexpf(amax, -e) > 32639.f) e += 1;
    v0 = __float2int_rn(ldexpf(x0, -e));  // exact scaling, round half to even
    v1 = __float2int_rn(ldexpf(x1, -e));
    int vs = v0 + v1;
#pragma unroll
    for (int o = 16; o; o >>= 1) vs += __shfl_xor_sync(0xFFFFFFFFu, vs, o);
    xs = ldexpf(1.f, e - 4);
    xsum = ldexpf(static_cast<float>(vs), e);  // |vs| < 2^21: exact
  }
  const int hi0 = (v0 + 128) >> 8, hi1 = (v1 + 128) >> 8;
  const int lo0 = v0 - 256 * hi0, lo1 = v1 - 256 * hi1;
  uint8_t* blk = p.xq + static_cast<size_t>(gg) * xq_block_bytes(mpad);
  const int k = 2 * lane;
  const int kofs = (k >> 5) * (mpad * 64) + ((k >> 4) & 1) * 128 + (k & 15);
  const int rh = t, rl = mpad + t;
  *reinterpret_cast<uint16_t*>(blk + kofs + (rh >> 3) * 256 + (rh & 7) * 16) =
      static_cast<uint16_t>((hi0 & 0xFF) | ((hi1 & 0xFF) << 8));
  *reinterpret_cast<uint16_t*>(blk + kofs + (rl >> 3) * 256 + (rl & 7) * 16) =
      static_cast<uint16_t>((lo0 & 0xFF) | ((lo1 & 0xFF) << 8));
  if (lane == 0) {
    float* xf = reinterpret_cast<float*>(blk + 2 * mpad * 64);
    xf[t] = xs;
    xf[mpad + t] = xsum;
  }
}

// x-prep blocks of n consecutive groups starting at global group `g` into one stage: one bulk
// copy, or (sharded step) one per rank whose slice the groups cross.
__device__ __forceinline__ void copy_x_blocks(const QmmParams& p, uint32_t dst, int g, int n, uint32_t xb,
                                              uint32_t bar) {
  if (p.xq_gpr == 0) {
    bulk_g2s(dst, p.xq + static_cast<size_t>(g) * xb, static_cast<uint32_t>(n) * xb, bar);
    return;
  }
  while (n > 0) {
    const int r = g / p.xq_gpr;
    const int m = min(n, (r + 1) * p.xq_gpr - g);
    bulk_g2s(dst, p.xq_rank[r] + static_cast<size_t>(g) * xb, static_cast<uint32_t>(m) * xb, bar);
    dst += static_cast<uint32_t>(m) * xb;
    g += m;
    n -= m;
  }
}

// The finished tile lt of an interleaved gate|up weight, as the 128 threads of one epilogue lane
// hold it (thread r: row r's sum for every token): g = bf16(rows 0-63), u = bf16(rows 64-127),
// a = bf16(silu(g) u) for output columns 64 lt .. 64 lt + 63 (the rounding of a gate|up output
// followed by the SwiGLU producer), written as x-prep group lt of swiglu_xq (tokens >= M zero).
// sc: 2 * NT * 64 floats of shared scratch; bar: the lane's named barrier.
template <int NT>
__device__ __forceinline__ void swiglu_digits(const QmmParams& p, int lt, int r, int lane, int wq, int bar,
                                              const float (&val)[NT], float* sc) {
  constexpr int MP = mpad_of(NT);
  float* us = sc;            // [NT][64] up values
  float* as = sc + NT * 64;  // [NT][64] outputs
  if (r >= 64) {
#pragma unroll
    for (int t = 0; t < NT; ++t) us[t * 64 + (r - 64)] = __bfloat162float(__float2bfloat16_rn(val[t]));
  }
  named_bar_sync(bar, kEpiThreads);
  if (r < 64) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float g = __bfloat162float(__float2bfloat16_rn(val[t]));
      as[t * 64 + r] = __bfloat162float(__float2bfloat16_rn(g / (1.f + __expf(-g)) * us[t * 64 + r]));
    }
  }
  named_bar_sync(bar, kEpiThreads);
#pragma unroll
  for (int t = wq; t < MP; t += 4) {  // (unrolled: the warp's token jobs are independent chains)
    const bool live = t < NT && t < p.M;
    const float a0 = live ? as[t * 64 + 2 * lane] : 0.f, a1 = live ? as[t * 64 + 2 * lane + 1] : 0.f;
    write_digits(p.swiglu_xq, MP, t, lt, lane, a0, a1);
  }
  named_bar_sync(bar, kEpiThreads);  // the scratch is the lanes' exchange buffer
}

// ---------------------------------------------------------------------------------------------
// The qmm kernel.  NT: token columns read back per unit (2, 4, 8 or 16).
// ---------------------------------------------------------------------------------------------
template <int NT, bool SWIGLU = false>
__global__ void __launch_bounds__(kThreads, 1)
    qmm_w4g64_tc_kernel(const __grid_constant__ QmmParams p) {
  constexpr int MP = mpad_of(NT);
  constexpr int XB = xq_block_bytes(MP);
  constexpr int XSTAGE = xstage_bytes(NT);
  constexpr int DW = 2 * MP;                          // D columns per unit (hi rows, lo rows)
  constexpr int kTmemCols = 512;
  constexpr int kStages = stages_for(NT);
  constexpr int kSetsD = sets_d_for(NT);
  constexpr int kDCol0 = kSetsA * kUPS * kACols;       // D slots follow the A slots
  static_assert(kDCol0 + kSetsD * kUPS * DW <= kTmemCols, "tensor memory budget");
  static_assert(kSetsA % 2 == 0 && kSetsD % 2 == 0, "a set belongs to one lane");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint8_t* xring = smem;                              // kStages x XSTAGE
  uint8_t* wring = smem + kStages * XSTAGE;           // kStages x kWStageBytes
  QmmSmem* sb = reinterpret_cast<QmmSmem*>(wring + kStages * kWStageBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  int u0, u1;
  if (p.split > 0) {  // tile c / S, K slice c % S (the CTA's rank in its cluster)
    const int S = p.split, tile = c / S, rk = c - tile * S, G = p.mats[0].G;
    u0 = tile * G + (rk * G) / S;
    u1 = tile * G + ((rk + 1) * G) / S;
  } else {
    u0 = static_cast<int>(u_begin(c, p.U, p.C));
    u1 = static_cast<int>(u_begin(c + 1, p.U, p.C));
  }
  volatile int* abort_flag = &sb->abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&sb->full[i]), 1);
      mbar_init(smem_u32(&sb->empty[i]), 1 + 4);  // MMA commit + the 4 dequant warps of the lane
    }
    for (int q = 0; q < kSetsA; ++q) {
      mbar_init(smem_u32(&sb->a_full[q]), 4);  // the 4 dequant warps of the set's lane
      mbar_init(smem_u32(&sb->a_free[q]), 5);  // MMA commit + the 4 epilogue warps of the lane
    }
    for (int q = 0; q < kSetsD; ++q) {
      mbar_init(smem_u32(&sb->d_full[q]), 1);  // MMA commit
      mbar_init(smem_u32(&sb->d_free[q]), 4);  // the 4 epilogue warps of the lane
    }
    mbar_init(smem_u32(&sb->mma_done[0]), 1);
    mbar_init(smem_u32(&sb->mma_done[1]), 1);
    sb->abort_flag = 0;
    sb->last_flag[0] = sb->last_flag[1] = 0;
    fence_mbar_init();
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
    // ------------------------------ TMA producer (lane 0) ------------------------------
    // (the whole warp waits for the other ranks' flags of a sharded step, a lane per rank)
    uint64_t pol_w = 0;
    UnitWalk wk;
    int cmi = 0;  // matrix whose weight pointer and x-prep offset are cached
    const uint8_t* w_tc = nullptr;
    int xg_off = 0;
    int k = 0;
    if (lane == 0) {
      pol_w = policy_evict_first();
      wk.init(p, u0);
      cmi = wk.mi;
      w_tc = p.mats[cmi].w_tc;
      xg_off = p.mats[cmi].xg_off;
      // First stages: weights before griddepcontrol.wait, x blocks after.  Each stage's x-prep
      // group and unit count are noted (in shared memory) as its weights are issued, so that
      // after the wait only the x copies are issued: the walk's kernel-parameter reads, about a
      // microsecond for a full ring, stay off the dependency's critical path.
      while (wk.u < u1 && k < kStages) {
        if (wk.mi != cmi) {
          cmi = wk.mi;
          w_tc = p.mats[cmi].w_tc;
          xg_off = p.mats[cmi].xg_off;
        }
        const int n = wk.stage_n(u1);
        mbar_arrive_expect_tx(smem_u32(&sb->full[k]), static_cast<uint32_t>(n) * (kUnitWBytes + XB));
        bulk_g2s_hint(smem_u32(wring + k * kWStageBytes),
                      w_tc + static_cast<size_t>(wk.u - wk.uoff) * kUnitWBytes,
                      static_cast<uint32_t>(n) * kUnitWBytes, smem_u32(&sb->full[k]), pol_w);
        sb->pre_xg[k] = xg_off + wk.g;
        sb->pre_n[k] = n;
        wk.advance(p, n);
        ++k;
      }
    }
    __syncwarp();
    if (lane == 0 || p.sync.wait_flags) pdl_wait_prior_grid();  // the x-prep blocks are written by the previous kernel
    if (p.sync.wait_flags) {  // (sharded step) and by the other ranks; a timeout is recorded
      peer_wait_flags_warp(p.sync, lane);
      if (lane == 0) fence_proxy_async_global();  // the bulk copies below read what the acquires made visible
    }
    if (lane == 0) {
      for (int f = 0; f < k; ++f)
        copy_x_blocks(p, smem_u32(xring + f * XSTAGE), sb->pre_xg[f], sb->pre_n[f], XB, smem_u32(&sb->full[f]));
      cmi = wk.mi;
      w_tc = p.mats[cmi].w_tc;
      xg_off = p.mats[cmi].xg_off;
      while (wk.u < u1) {
        const int s = k % kStages;
        if (!mbar_wait(smem_u32(&sb->empty[s]), ((k / kStages) - 1) & 1, p.err, kErrBitWaitEmpty,
                       abort_flag))
          break;
        if (wk.mi != cmi) {
          cmi = wk.mi;
          w_tc = p.mats[cmi].w_tc;
          xg_off = p.mats[cmi].xg_off;
        }
        const int n = wk.stage_n(u1);
        mbar_arrive_expect_tx(smem_u32(&sb->full[s]), static_cast<uint32_t>(n) * (kUnitWBytes + XB));
        bulk_g2s_hint(smem_u32(wring + s * kWStageBytes),
                      w_tc + static_cast<size_t>(wk.u - wk.uoff) * kUnitWBytes,
                      static_cast<uint32_t>(n) * kUnitWBytes, smem_u32(&sb->full[s]), pol_w);
        copy_x_blocks(p, smem_u32(xring + s * XSTAGE), xg_off + wk.g, n, XB, smem_u32(&sb->full[s]));
        wk.advance(p, n);
        ++k;
      }
      // Never leave the CTA with copies in flight: wait (bounded, ignoring abort) for the last
      // stages issued.  On the normal path they completed long ago.
      int zero = 0;
      for (int kk = (k > kStages ? k - kStages : 0); kk < k; ++kk)
        mbar_wait(smem_u32(&sb->full[kk % kStages]), (kk / kStages) & 1, p.err, kErrBitWaitDrain, &zero);
    }
  } else if (warp == 1 || warp == 2) {
    if (lane == 0) {
      // ------------------------------ MMA issuers (lane = stage parity) ------------------------
      const int L = warp - 1;
      constexpr uint32_t idesc = idesc_s8_s32(128, DW);
      UnitWalk wk;
      wk.init(p, u0);
      for (int k = 0; wk.u < u1; ++k) {
        const int n = wk.stage_n(u1);
        if ((k & 1) == L) {
          const int s = k % kStages;
          const int qa = k % kSetsA, qd = k % kSetsD, used = k / kSetsD;
          if (!mbar_wait(smem_u32(&sb->full[s]), (k / kStages) & 1, p.err, kErrBitWaitFull, abort_flag) ||
              !mbar_wait(smem_u32(&sb->a_full[qa]), (k / kSetsA) & 1, p.err, kErrBitWaitAFull, abort_flag) ||
              (used > 0 && !mbar_wait(smem_u32(&sb->d_free[qd]), (used - 1) & 1, p.err, kErrBitWaitDEmpty,
                                      abort_flag)))
            break;
          tc_fence_after();
          for (int j = 0; j < n; ++j) {
            const uint32_t xb = smem_u32(xring + s * XSTAGE + j * XB);
            const uint32_t a_tmem = tmem + (qa * kUPS + j) * kACols;
            const uint32_t d_tmem = tmem + kDCol0 + (qd * kUPS + j) * DW;
            umma_i8_ts(d_tmem, a_tmem, smem_desc_noswizzle(xb, 128, 256), idesc, 0u);               // k 0-31
            umma_i8_ts(d_tmem, a_tmem + 8, smem_desc_noswizzle(xb + MP * 64, 128, 256), idesc, 1u);  // k 32-63
          }
          umma_commit(smem_u32(&sb->d_full[qd]));
          umma_commit(smem_u32(&sb->a_free[qa]));
          umma_commit(smem_u32(&sb->empty[s]));
        }
        wk.advance(p, n);
      }
      // Every MMA issued by this thread completes before TMEM is released.
      umma_commit(smem_u32(&sb->mma_done[L]));
      int zero = 0;
      mbar_wait(smem_u32(&sb->mma_done[L]), 0, p.err, kErrBitWaitDrain, &zero);
    }
  } else if (warp >= kDeqWarp0 && warp < kEpiWarp0) {
    // ------------------------------ dequant: one warpgroup per lane ---------------------------
    // Per stage of its lane: one wait for the stage and one for the lane's slots; all shared
    // loads of the stage issued together; decode + tensor-memory store of every unit
    // (asynchronous); one wait for the stores and one arrival for the whole stage.
    const int L = (warp - kDeqWarp0) >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    UnitWalk wk;
    wk.init(p, u0);
    for (int k = 0; wk.u < u1; ++k) {
      const int n = wk.stage_n(u1);
      if ((k & 1) == L) {
        const int s = k % kStages;
        const int q = k % kSetsA, use = k / kSetsA;
        // Every wait result is made warp-uniform: a lane that left the loop alone would strand
        // the others at __syncwarp or at a .sync.aligned tensor-memory store.
        const bool ok =
            mbar_wait(smem_u32(&sb->full[s]), (k / kStages) & 1, p.err, kErrBitWaitFull, abort_flag) &&
            (use == 0 ||
             mbar_wait(smem_u32(&sb->a_free[q]), (use - 1) & 1, p.err, kErrBitWaitAEmpty, abort_flag));
        if (!__all_sync(0xFFFFFFFFu, ok)) break;
        const uint8_t* wst = wring + s * kWStageBytes;
        const uint8_t* xst = xring + s * XSTAGE + 2 * MP * 64;
        uint4 c0[kUPS], c1[kUPS];
        uint32_t sbw[kUPS];
        float xm[kUPS];
#pragma unroll
        for (int j = 0; j < kUPS; ++j) {
          if (j < n) {
            const uint8_t* wu = wst + j * kUnitWBytes;
            c0[j] = *reinterpret_cast<const uint4*>(wu + r * 16);
            c1[j] = *reinterpret_cast<const uint4*>(wu + 2048 + r * 16);
            sbw[j] = *reinterpret_cast<const uint32_t*>(wu + kUnitNibBytes + r * 4);
            xm[j] = r < 2 * MP ? *reinterpret_cast<const float*>(xst + j * XB + r * 4) : 0.f;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sb->empty[s]));  // this warp's shared loads are done
#pragma unroll
        for (int j = 0; j < kUPS; ++j) {
          if (j < n) {
            QmmMeta& mm = sb->meta[q][j];
            mm.sb[r] = sbw[j];
            if (r < 2 * MP) mm.x[r < MP ? r : kMaxTokens + r - MP] = xm[j];
          }
        }
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < kUPS; ++j) {
          if (j < n) {
            uint32_t a[16];
            decode_i8(c0[j], c1[j], a);
            tmem_st_x16(tmem + lane_off + (q * kUPS + j) * kACols, a);
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sb->a_full[q]));
      }
      wk.advance(p, n);
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------ epilogue: one warpgroup per lane --------------------------
    // Warpgroup L accumulates the units of the stages of lane L.  At the end of each tile
    // segment the two partial sums are added in a fixed order (lane 0's + lane 1's) by the
    // warpgroup that holds the segment's last stage, which then writes or publishes the tile.
    const int L = (warp - kEpiWarp0) >> 2;
    const int e = threadIdx.x - kEpiWarp0 * 32 - L * kEpiThreads;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    float* xchg = reinterpret_cast<float*>(sb + 1);  // [2][NT][128] partial-sum exchange
    // f32 sums of the segment's groups, token pairs packed (2i, 2i + 1) for f32x2 arithmetic
    uint64_t acc2[NT / 2];
#pragma unroll
    for (int i = 0; i < NT / 2; ++i) acc2[i] = 0ull;
    bool dep_waited = false;
    int seg = 0;  // tile segments finished by this CTA
    UnitWalk wk;
    wk.init(p, u0);
    for (int k = 0; wk.u < u1; ++k) {
      const int n = wk.stage_n(u1);
      if ((k & 1) == L) {
        // a_full: the meta slots this stage reads were written (and d_full: the MMAs are done)
        const int qa = k % kSetsA, qd = k % kSetsD;
        const bool ok = __all_sync(
            0xFFFFFFFFu,
            mbar_wait(smem_u32(&sb->a_full[qa]), (k / kSetsA) & 1, p.err, kErrBitWaitAFull, abort_flag) &&
                mbar_wait(smem_u32(&sb->d_full[qd]), (k / kSetsD) & 1, p.err, kErrBitWaitDFull, abort_flag));
        if (ok) tc_fence_after();
        for (int j = 0; j < n && ok; ++j) {
          {
            const QmmMeta& mm = sb->meta[qa][j];
            const uint32_t sbw = mm.sb[r];
            // (xs, xsum) of token pairs, read as packed pairs
            const uint64_t* xs2 = reinterpret_cast<const uint64_t*>(mm.x);
            const uint64_t* xsum2 = reinterpret_cast<const uint64_t*>(mm.x + kMaxTokens);
            float dh[NT], dl[NT];
            const uint32_t dbase = tmem + lane_off + kDCol0 + (qd * kUPS + j) * DW;
            if constexpr (NT == MP && NT == 8) {
              float d[2 * NT];  // hi columns then lo columns: one load
              tmem_ld<2 * NT>(dbase, d);
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                dh[t] = d[t];
                dl[t] = d[NT + t];
              }
            } else {
              tmem_ld<NT>(dbase, dh);
              tmem_ld<NT>(dbase + MP, dl);
            }
            tc_wait_ld();
            const float sc = __uint_as_float(sbw << 16);
            const float bo = fmaf(8.0f, sc, __uint_as_float(sbw & 0xFFFF0000u));  // b + 8 s
            const uint64_t sc2 = f2_pack(sc, sc), bo2 = f2_pack(bo, bo);
            // acc += (s xs) G + (b + 8 s) xsum per token, as fmaf(s * xs, G, fmaf(bo, xsum, acc))
#pragma unroll
            for (int i = 0; i < NT / 2; ++i) {
              const float g0 = static_cast<float>(__float_as_int(dh[2 * i]) * 256 + __float_as_int(dl[2 * i]));
              const float g1 =
                  static_cast<float>(__float_as_int(dh[2 * i + 1]) * 256 + __float_as_int(dl[2 * i + 1]));
              const uint64_t part = f2_fma(bo2, xsum2[i], acc2[i]);
              acc2[i] = f2_fma(f2_mul(sc2, xs2[i]), f2_pack(g0, g1), part);
            }
          }
        }
        if (ok) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {  // D and meta slots read
            mbar_arrive(smem_u32(&sb->d_free[qd]));
            mbar_arrive(smem_u32(&sb->a_free[qa]));
          }
        }
      }
      const int g = wk.g + n - 1;  // group of the stage's last unit
      if (g == wk.G - 1 || wk.u + n == u1) {
        // ---- end of a tile segment: combine the lanes, then write the tile or publish a partial
        float acc[NT];
#pragma unroll
        for (int i = 0; i < NT / 2; ++i) f2_unpack(acc2[i], acc[2 * i], acc[2 * i + 1]);
        const int own = k & 1;  // the warpgroup that holds the segment's last stage finishes it
        float* xb = xchg + (seg & 1) * NT * kTileRows;
        if (L != own) {
#pragma unroll
          for (int t = 0; t < NT; ++t) xb[t * kTileRows + r] = acc[t];
        }
        named_bar_sync(3, 2 * kEpiThreads);
        if (L == own) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const float o = xb[t * kTileRows + r];
            acc[t] = L == 0 ? acc[t] + o : o + acc[t];
          }
          if (p.split > 1) {
            // cluster split: the slice's sum stays in shared memory; rank 0 adds the ranks' sums
            // after the cluster barrier at the end of the kernel
#pragma unroll
            for (int t = 0; t < NT; ++t) xb[t * kTileRows + r] = acc[t];
          } else {
          const QmmMat& mt = p.mats[wk.mi];                     // read once per tile segment
          const int tile_u0 = mt.unit_off + wk.lt * mt.G;        // the tile's first global unit
          const int tile = mt.tile_off + wk.lt;                  // global tile (counter index)
          const int seg_start = (tile_u0 > u0) ? tile_u0 : u0;
          const bool full_tile = (seg_start == tile_u0) && (g == mt.G - 1);
          const bool first_seg = (seg_start == u0);
          const int row_g = wk.lt * kTileRows + r;
          const bool live = !*abort_flag;
          if (!dep_waited) {
            pdl_wait_prior_grid();  // outputs may alias buffers an earlier kernel still reads
            dep_waited = true;
          }
          if (full_tile) {
            if constexpr (SWIGLU) {
              // The scratch overlaps the exchange slots this warpgroup's other threads may still
              // be reading for the lane combine above: every thread's read first.
              named_bar_sync(4 + L, kEpiThreads);
              swiglu_digits<NT>(p, wk.lt, r, lane, warp & 3, 4 + L, acc, xb);  // (barriers: every thread)
            } else if (live && row_g < mt.N) {
#pragma unroll
              for (int t = 0; t < NT; ++t)
                if (t < p.M) mt.out[static_cast<size_t>(t) * mt.ldo + row_g] = __float2bfloat16_rn(acc[t]);
            }
          } else {
            const int bar = 4 + L;
            const long long cf = cta_of_unit(tile_u0, p.U, p.C);
            const long long cl = cta_of_unit(tile_u0 + mt.G - 1, p.U, p.C);
            const unsigned n_contrib = static_cast<unsigned>(cl - cf + 1);
            // A CTA whose last segment this is usually arrives last (the others published the
            // tile's other parts early in their ranges): it peeks at the counter first and, when
            // every other contributor has arrived, finishes the tile from its own registers and
            // their partials without publishing its own (one write, fence and atomic fewer on
            // the launch's critical path).  Otherwise: publish, count, and the last arriver sums.
            if (e == 0) {
              unsigned seen = 0u;
              if (live && wk.u + n == u1)
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(p.cnt + tile) : "memory");
              sb->last_flag[L] = (live && wk.u + n == u1 && seen == n_contrib - 1) ? 2 : 0;
            }
            named_bar_sync(bar, kEpiThreads);
            const bool early = sb->last_flag[L] == 2;
            if (!early) {
              float* mine = p.part + (static_cast<size_t>(c) * 2 + (first_seg ? 0 : 1)) * kMaxTokens * kTileRows;
#pragma unroll
              for (int t = 0; t < NT; ++t) mine[t * kTileRows + r] = acc[t];
              __threadfence();
              named_bar_sync(bar, kEpiThreads);
              if (e == 0) {
                const unsigned old = live ? atomicAdd(&p.cnt[tile], 1u) : 0u;
                sb->last_flag[L] = live && (old == n_contrib - 1);
              }
              named_bar_sync(bar, kEpiThreads);
            }
            if (sb->last_flag[L]) {
              __threadfence();
              float v[NT];
#pragma unroll
              for (int t = 0; t < NT; ++t) v[t] = 0.f;
              for (long long cc = cf; cc <= cl; ++cc) {  // contributor order, whoever finishes
                if (early && cc == c) {
#pragma unroll
                  for (int t = 0; t < NT; ++t) v[t] += acc[t];
                  continue;
                }
                const long long cu0 = u_begin(cc, p.U, p.C);
                const int cs = (cu0 >= tile_u0) ? 0 : 1;  // the tile is this contributor's first segment
                const float* src = p.part + (static_cast<size_t>(cc) * 2 + cs) * kMaxTokens * kTileRows;
#pragma unroll
                for (int t = 0; t < NT; ++t) v[t] += __ldcg(src + t * kTileRows + r);
              }
              if constexpr (SWIGLU) {
                swiglu_digits<NT>(p, wk.lt, r, lane, warp & 3, bar, v, xb);
              } else if (row_g < mt.N) {
#pragma unroll
                for (int t = 0; t < NT; ++t)
                  if (t < p.M) mt.out[static_cast<size_t>(t) * mt.ldo + row_g] = __float2bfloat16_rn(v[t]);
              }
              if (e == 0) p.cnt[tile] = 0u;
            }
            named_bar_sync(bar, kEpiThreads);
          }
          }  // stream-K / whole tile
        }
#pragma unroll
        for (int i = 0; i < NT / 2; ++i) acc2[i] = 0ull;
        ++seg;
      }
      wk.advance(p, n);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (p.split > 1) {
    // Cluster split-K: every rank's slice sum is in its exchange buffer (slot 0).  After a
    // cluster barrier each rank's epilogue threads add one S-th of the tile's M x 128 outputs
    // over the S ranks (rank order, distributed shared memory; all remote loads of a thread issued
    // before the adds) and write them; the second barrier keeps the peers' shared memory alive.
    // (Config-3 step with the reduction spread over the ranks: 1.927 -> 1.894 ms at M = 8.)
    cluster_arrive_release();
    cluster_wait_acquire();
    const int S = p.split;
    if (warp >= kEpiWarp0) {
      const QmmMat& mt = p.mats[0];
      const int tile = c / S, qr = static_cast<int>(cluster_ctarank());
      const uint32_t xloc = smem_u32(reinterpret_cast<float*>(sb + 1));
      pdl_wait_prior_grid();  // outputs may alias buffers an earlier kernel still reads
      const bool live = !*abort_flag;
      // (one or two tokens: rank 0 alone, the other ranks go on to the barrier -- measured faster)
      const int E = p.M * kTileRows;  // outputs of the tile, token-major
      const bool spread = p.M > 2;
      const int e0 = spread ? E * qr / S : 0, e1 = spread ? E * (qr + 1) / S : (qr == 0 ? E : 0);
      constexpr int kPer = (NT <= 2 ? NT * kTileRows : NT * kTileRows / 2 + 2 * kEpiThreads - 1) / (2 * kEpiThreads);
      const int i0 = threadIdx.x - kEpiWarp0 * 32;
      float part[kPer][8];
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int idx = e0 + i0 + u * 2 * kEpiThreads;
        const uint32_t a = xloc + idx * 4;
#pragma unroll
        for (int q = 0; q < 8; ++q) part[u][q] = (q < S && idx < e1) ? ld_cluster_f32(map_shared_rank(a, q)) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int idx = e0 + i0 + u * 2 * kEpiThreads;
        const int t = idx / kTileRows, row_g = tile * kTileRows + (idx - t * kTileRows);
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < S) v += part[u][q];  // rank order
        if (live && idx < e1 && row_g < mt.N) mt.out[static_cast<size_t>(t) * mt.ldo + row_g] = __float2bfloat16_rn(v);
      }
    }
    cluster_arrive_relaxed();
    cluster_wait_acquire();
  }
  peer_signal_done(p.sync, &sb->last_flag[0]);  // (sharded step) this rank's output is complete
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
        const uint32_t nib = ((v >> (4 * i)) & 0xFu) ^ 0x8u;
        // columns 0-3 -> high nibbles of bytes 0-3, columns 4-7 -> low nibbles
        const int shift = i < 4 ? 8 * i + 4 : 8 * (i - 4);
        o |= nib << shift;
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

// ---------------------------------------------------------------------------------------------
// Host launchers (called from the C-ABI layer)
// ---------------------------------------------------------------------------------------------
// Per-device caches, filled on first use.  Several host threads may fill an entry at once; they
// store the same value, and the entries are atomics so that this is not a data race.  They are
// keyed by device index and so assume the device's primary context (the one the CUDA runtime
// API uses); a host that switches between driver-API contexts on one device must not share them.
static std::atomic<int> g_num_sms[64];
static std::atomic<bool> g_attr_set[64][8];  // per device: [token-column variant + 4 for the SwiGLU epilogue]

int device_sm_count(int dev) {
  if (dev < 0 || dev >= 64) return 148;
  int v = g_num_sms[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    g_num_sms[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

static void pdl_config(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr, bool pdl) {
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
}

template <int NT, bool SWIGLU = false>
static cudaError_t set_smem_attr(int dev) {
  constexpr int slot = (NT == 2 ? 0 : NT == 4 ? 1 : NT == 8 ? 2 : 3) + (SWIGLU ? 4 : 0);
  if (dev >= 0 && dev < 64 && !g_attr_set[dev][slot].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(qmm_w4g64_tc_kernel<NT, SWIGLU>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(qmm_smem_bytes(NT)));
    if (e != cudaSuccess) return e;
    g_attr_set[dev][slot].store(true, std::memory_order_release);
  }
  return cudaSuccess;
}

template <int NT, bool SWIGLU = false>
static cudaError_t launch_tc(const QmmParams& prm, int dev, cudaStream_t stream, bool pdl) {
  const cudaError_t e = set_smem_attr<NT, SWIGLU>(dev);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(prm.C);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = qmm_smem_bytes(NT);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  pdl_config(cfg, attr, pdl);
  if (prm.split > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(prm.split);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, qmm_w4g64_tc_kernel<NT, SWIGLU>, prm);
}

// Clusters of S CTAs of the qmm kernel that can be resident at once on device `dev`: the
// minimum over the four token-count variants, so that the split chosen from it is the same for
// every M (the per-token results stay independent of M).  Cached per (device, S).
static std::atomic<int> g_max_clusters[64][9];

template <int NT>
static int clusters_of(int S) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = qmm_smem_bytes(NT);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(S);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, qmm_w4g64_tc_kernel<NT>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

static int max_active_clusters(int dev, int S) {
  if (dev < 0 || dev >= 64 || S < 2 || S > 8) return 0;
  int cached = g_max_clusters[dev][S].load(std::memory_order_relaxed);
  if (cached == 0) {
    if (set_smem_attr<2>(dev) != cudaSuccess || set_smem_attr<4>(dev) != cudaSuccess ||
        set_smem_attr<8>(dev) != cudaSuccess || set_smem_attr<16>(dev) != cudaSuccess)
      return 0;
    int n = clusters_of<2>(S);
    n = std::min(n, clusters_of<4>(S));
    n = std::min(n, clusters_of<8>(S));
    n = std::min(n, clusters_of<16>(S));
    cached = n > 0 ? n : -1;
    g_max_clusters[dev][S].store(cached, std::memory_order_relaxed);
  }
  return cached;
}

// Work split of a single-matrix call with `tiles` 128-row tiles of G groups on C CTAs.
//   0      stream-K over all units (tiles >= C: every CTA streams whole tiles plus at most two
//          partial ones; the split-K fix-up through global memory is paid a few times)
//   S >= 1 S CTAs per tile, each a contiguous K slice; S > 1 CTAs form a cluster and rank 0 adds
//          the slices over distributed shared memory (no global partials, atomics or fences).
//          S is the largest split (<= 8) whose clusters are all resident at once.
static int choose_split(int dev, int tiles, int G, int C) {
  if (tiles >= C) return 0;
  int S = std::min(std::min(C / tiles, 8), G);
  for (; S > 1; --S)
    if (max_active_clusters(dev, S) >= tiles) return S;
  return 1;
}

// What a single-matrix call (skinny_qmm_w4g64) launches for M tokens on the current device: the
// token columns read back per unit, the split (0 = persistent stream-K over all units, S >= 1 =
// S CTAs per 128-row tile) and the qmm grid size.
cudaError_t qmm_launch_config(int M, int N, int K, int* token_cols, int* split, int* ctas) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int C = device_sm_count(dev);
  const QmmShape sh = qmm_shape(N, K);
  const int S = choose_split(dev, static_cast<int>(sh.T), sh.G, C);
  *token_cols = M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16;
  *split = S;
  *ctas = S > 0 ? static_cast<int>(sh.T) * S : static_cast<int>(sh.U < C ? sh.U : C);
  return cudaSuccess;
}

static cudaError_t launch_xprep(const XPrepParams& xp, cudaStream_t stream, bool pdl) {
  const long long warps = static_cast<long long>(xp.total_groups) * xp.mpad;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((warps + 7) / 8));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, pdl);
  return cudaLaunchKernelEx(&cfg, qmm_xprep_kernel, xp);
}

// Grouped launch over n matrices sharing the token count M: an x-prep launch over the distinct
// (x, K, ldx) inputs (at most kMaxX, sum of K/64 at most xq_groups), then the qmm launch.
// Shapes and pointers were validated by the caller.  The scratch is given as its parts: error
// word, per-tile counters (zero on entry, left zero), partial sums for up to `C_cap` CTAs and
// the x-prep blocks.  `pdl` applies to the x-prep launch (towards the caller's previous work);
// the qmm launch always overlaps the x-prep launch.
static cudaError_t launch_grouped_on(int n, const void* const* x, const int* ldx,
                                     const void* const* w_tc, void* const* out, const int* ldo,
                                     const int* N, const int* K, int M, uint32_t* err,
                                     uint32_t* cnt, float* part, uint8_t* xq, int xq_groups,
                                     int C_cap, int dev, cudaStream_t stream, bool pdl) {
  if (n < 1 || n > kMaxMats) return cudaErrorInvalidValue;
  static thread_local QmmParams prm;  // ~9 KB: keep it off the stack
  static thread_local XPrepParams xp;
  const int mpad = M <= 8 ? 8 : 16;
  prm.part = part;
  prm.cnt = cnt;
  prm.err = err;
  prm.xq = xq;
  prm.M = M;
  prm.n_mats = n;
  prm.xq_gpr = 0;
  prm.sync = PeerSync{};
  prm.swiglu_xq = nullptr;
  xp.xq = xq;
  xp.M = M;
  xp.mpad = mpad;
  int nx = 0, groups = 0;
  long long U = 0;
  long long T = 0;
  for (int i = 0; i < n; ++i) {
    const QmmShape sh = qmm_shape(N[i], K[i]);
    int xi = -1;
    for (int q = 0; q < nx; ++q)
      if (xp.in[q].x == x[i] && xp.in[q].G == sh.G && xp.in[q].ldx == ldx[i]) xi = q;
    if (xi < 0) {
      if (nx == kMaxX || groups + sh.G > xq_groups) return cudaErrorInvalidValue;
      xi = nx++;
      xp.in[xi].x = static_cast<const __nv_bfloat16*>(x[i]);
      xp.in[xi].ldx = ldx[i];
      xp.in[xi].G = sh.G;
      xp.in[xi].xg_off = groups;
      groups += sh.G;
    }
    QmmMat& mt = prm.mats[i];
    mt.w_tc = static_cast<const uint8_t*>(w_tc[i]);
    mt.out = static_cast<__nv_bfloat16*>(out[i]);
    mt.unit_off = static_cast<int>(U);
    mt.N = N[i];
    mt.G = sh.G;
    mt.tile_off = static_cast<int>(T);
    mt.xg_off = xp.in[xi].xg_off;
    mt.ldo = ldo[i];
    U += sh.U;
    T += sh.T;
  }
  if (T > kMaxTiles) return cudaErrorInvalidValue;
  xp.n_in = nx;
  xp.total_groups = groups;
  prm.U = static_cast<int>(U);
  prm.C = static_cast<int>(U < C_cap ? U : C_cap);
  prm.split = n == 1 ? choose_split(dev, static_cast<int>(T), prm.mats[0].G, C_cap) : 0;
  if (prm.split > 0) prm.C = static_cast<int>(T) * prm.split;
  cudaError_t e = launch_xprep(xp, stream, pdl);
  if (e != cudaSuccess) return e;
  if (M <= 2) return launch_tc<2>(prm, dev, stream, true);
  if (M <= 4) return launch_tc<4>(prm, dev, stream, true);
  if (M <= 8) return launch_tc<8>(prm, dev, stream, true);
  return launch_tc<16>(prm, dev, stream, true);
}

// One matrix whose input was already written in the x-prep block format by a producer kernel
// (prep.cu): no x-prep launch.  xq holds K/64 blocks for mpad(M) token rows.
cudaError_t qmm_tc_launch_prepared(const void* xq, const void* w_tc, void* out, int ldo, int M, int N, int K,
                                   void* ws, const void* const* xq_ranks, int xq_gpr, const skinny_peer_sync* sync,
                                   cudaStream_t stream, void* swiglu_xq) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int C_dev = device_sm_count(dev);
  const WsLayout wl = ws_layout(C_dev);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  static thread_local QmmParams prm;
  const QmmShape sh = qmm_shape(N, K);
  prm.part = reinterpret_cast<float*>(wsb + wl.part_off);
  prm.cnt = reinterpret_cast<uint32_t*>(wsb + wl.cnt_off);
  prm.err = reinterpret_cast<uint32_t*>(wsb);
  prm.xq = static_cast<const uint8_t*>(xq);
  prm.M = M;
  prm.n_mats = 1;
  prm.xq_gpr = xq_ranks ? xq_gpr : 0;
  for (int r = 0; r < kMaxPeers; ++r) prm.xq_rank[r] = nullptr;
  if (xq_ranks)
    for (int r = 0; r < kMaxPeers && r * xq_gpr < K / kGroup; ++r) prm.xq_rank[r] = static_cast<const uint8_t*>(xq_ranks[r]);
  prm.sync = peer_sync_from(sync);
  QmmMat& mt = prm.mats[0];
  mt.w_tc = static_cast<const uint8_t*>(w_tc);
  mt.out = static_cast<__nv_bfloat16*>(out);
  mt.unit_off = 0;
  mt.N = N;
  mt.G = sh.G;
  mt.tile_off = 0;
  mt.xg_off = 0;
  mt.ldo = ldo;
  prm.U = static_cast<int>(sh.U);
  prm.C = static_cast<int>(sh.U < C_dev ? sh.U : C_dev);
  prm.swiglu_xq = static_cast<uint8_t*>(swiglu_xq);
  if (swiglu_xq) {  // (a separate kernel variant; its epilogue finishes tiles in the stream-K paths only)
    prm.split = 0;
    if (M <= 2) return launch_tc<2, true>(prm, dev, stream, true);
    if (M <= 4) return launch_tc<4, true>(prm, dev, stream, true);
    if (M <= 8) return launch_tc<8, true>(prm, dev, stream, true);
    return launch_tc<16, true>(prm, dev, stream, true);
  }
  prm.split = choose_split(dev, static_cast<int>(sh.T), sh.G, C_dev);
  if (prm.split > 0) prm.C = static_cast<int>(sh.T) * prm.split;
  if (M <= 2) return launch_tc<2>(prm, dev, stream, true);
  if (M <= 4) return launch_tc<4>(prm, dev, stream, true);
  if (M <= 8) return launch_tc<8>(prm, dev, stream, true);
  return launch_tc<16>(prm, dev, stream, true);
}

cudaError_t qmm_tc_launch_grouped(int n, const void* const* x, const int* ldx, const void* const* w_tc,
                                  void* const* out, const int* ldo, const int* N, const int* K, int M,
                                  void* ws, cudaStream_t stream, bool pdl) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int C_dev = device_sm_count(dev);
  const WsLayout wl = ws_layout(C_dev);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  return launch_grouped_on(n, x, ldx, w_tc, out, ldo, N, K, M, reinterpret_cast<uint32_t*>(wsb),
                           reinterpret_cast<uint32_t*>(wsb + wl.cnt_off),
                           reinterpret_cast<float*>(wsb + wl.part_off), wsb + wl.xq_off, kMaxXGroups,
                           C_dev, dev, stream, pdl);
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
// Limits: N <= kNoAllocMaxTiles * 128 rows (tail tiles count whole), K <= kNoAllocMaxGroups * 64
// columns, and at most kNoAllocMaxCtas CTAs (a device with more SMs uses kNoAllocMaxCtas of
// them).  There is ONE scratch per device, so two calls that may run at the same time on one
// device (different streams, threads without ordering) race on it and corrupt each other's
// results; calls must be ordered, e.g. on a single stream.  The first call on a device does the
// set-up (symbol lookup, kernel attributes) and should come before any stream capture.
// ---------------------------------------------------------------------------------------------
constexpr int kNoAllocMaxTiles = 2048;   // N <= 262,144 rows
constexpr int kNoAllocMaxGroups = 512;   // K <= 32,768 columns
constexpr int kNoAllocMaxCtas = 160;
constexpr size_t kNoAllocCntOff = 256;
constexpr size_t kNoAllocPartOff = kNoAllocCntOff + static_cast<size_t>(kNoAllocMaxTiles) * 4;
constexpr size_t kNoAllocXqOff =
    kNoAllocPartOff + static_cast<size_t>(kNoAllocMaxCtas) * 2 * kMaxTokens * kTileRows * 4;
constexpr size_t kNoAllocScratchBytes =
    kNoAllocXqOff + static_cast<size_t>(kNoAllocMaxGroups) * xq_block_bytes(16);
static_assert(kNoAllocScratchBytes == 3744000, "3.6 MiB of static scratch per device");
static_assert(kNoAllocPartOff % 256 == 0 && kNoAllocXqOff % 256 == 0, "256-byte aligned regions");

// [0, 256) error word + padding | [256, 8448) tile counters | partial sums | x-prep blocks
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
  const QmmShape sh = qmm_shape(N, K);
  return sh.T <= kNoAllocMaxTiles && sh.G <= kNoAllocMaxGroups;
}

// The error word and the counters must be zero when the kernel starts.  A launch that completes
// leaves the counters at zero, but one that stopped on a timed-out wait may not, so both are
// cleared on the stream before every call (a memset node: no allocation).  The x-prep launch
// does not use programmatic dependent launch, so neither kernel can start before that clear.
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
                           reinterpret_cast<float*>(scratch + kNoAllocPartOff),
                           scratch + kNoAllocXqOff, kNoAllocMaxGroups, C_cap, dev, stream, false);
}

// Copies the static scratch's error word (the device error bits of the latest no-alloc call
// ordered before it on `stream`) to `dst` (device, pinned or pageable host memory), stream-ordered.
cudaError_t qmm_noalloc_error_copy(void* dst, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  uint8_t* scratch = nullptr;
  e = noalloc_scratch(dev, &scratch);
  if (e != cudaSuccess) return e;
  return cudaMemcpyAsync(dst, scratch, sizeof(uint32_t), cudaMemcpyDefault, stream);
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

// Relaid units -> bf16 W[N, K] (row stride ldo): w = bf16(q * s + b), the f32 product then the f32
// sum, each rounded (the MLX dequantisation).  CTA per unit, thread per (row, 32-column chunk):
// one 16-byte load of 32 nibbles, four 16-byte stores.  For callers that hand many tokens to a
// dense GEMM instead of the token-streaming qmm.
__global__ void __launch_bounds__(256) qmm_dequant_kernel(const uint8_t* __restrict__ w_tc, int N, int K,
                                                         __nv_bfloat16* __restrict__ out, int ldo) {
  const int G = K / kGroup;
  const long long u = blockIdx.x;
  const int tile = static_cast<int>(u / G), g = static_cast<int>(u % G);
  const int r = threadIdx.x & (kTileRows - 1), c = threadIdx.x >> 7;
  const int n = tile * kTileRows + r;
  if (n >= N) return;
  const uint8_t* unit = w_tc + u * kUnitWBytes;
  const uint4 nib = *reinterpret_cast<const uint4*>(unit + c * 2048 + r * 16);
  const uint32_t sb = *reinterpret_cast<const uint32_t*>(unit + kUnitNibBytes + r * 4);
  const float s = __uint_as_float(sb << 16), b = __uint_as_float(sb & 0xFFFF0000u);
  const uint32_t words[4] = {nib.x, nib.y, nib.z, nib.w};
  // nibble of column k0 + i inside a word: i = 0..3 at bits 4 + 8i, i = 4..7 at bits 8(i - 4)
  __nv_bfloat16* dst = out + static_cast<size_t>(n) * ldo + g * kGroup + 32 * c;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const int sh0 = i < 4 ? 4 + 8 * i : 8 * (i - 4), sh1 = i + 1 < 4 ? 4 + 8 * (i + 1) : 8 * (i - 3);
      const float q0 = static_cast<float>(((words[j] >> sh0) & 0xF) ^ 8);
      const float q1 = static_cast<float>(((words[j] >> sh1) & 0xF) ^ 8);
      o2[i / 2] = __floats2bfloat162_rn(__fadd_rn(__fmul_rn(q0, s), b), __fadd_rn(__fmul_rn(q1, s), b));
    }
    *reinterpret_cast<uint4*>(dst + 8 * j) = o;
  }
}

cudaError_t qmm_dequant_launch(const void* w_tc, int N, int K, void* out, int ldo, cudaStream_t stream) {
  const QmmShape sh = qmm_shape(N, K);
  qmm_dequant_kernel<<<static_cast<unsigned>(sh.U), 256, 0, stream>>>(static_cast<const uint8_t*>(w_tc), N, K,
                                                                    static_cast<__nv_bfloat16*>(out), ldo);
  return cudaGetLastError();
}

}  // namespace skinny
