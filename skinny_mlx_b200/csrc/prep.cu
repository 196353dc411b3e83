// Producers of qmm inputs: each computes a bf16 activation row and writes it directly in the
// x-prep block format the qmm kernel reads (qmm_layout.cuh), so that no separate x-prep launch
// and no bf16 activation round trip sit between a step's elementwise work and its next matmul.
//
//   prep_rmsnorm : h = x (+ d)  [written to h_out as the next residual stream when d is given;
//                  d may be in the column-sharded layout of an all-gather, see d_off],
//                  a = bf16( h / rms(h) * (1 + w) )            -> digits of a
//   prep_swiglu  : a = bf16( silu(g) * u ) for gu = [g | u]     -> digits of a
//   prep_plain   : a = x                                         -> digits of a
//
// Digits: per (token, 64-column group) v = rint(a 2^-e) with the smallest e such that
// |v| <= 32639, v = 256 hi + lo (signed 8-bit), xs = 2^(e-4), xsum = 2^e sum v; tokens >= M of the
// mpad rows are zero.  This is the same rule as the standalone x-prep kernel, so a prepared call
// and an unprepared call on the same bf16 activations give bit-identical qmm results.
//
// Grid: (ceil(G / 8) column chunks, mpad token rows), 256 threads; warp w of chunk c handles
// group 8c + w, lane l holds its columns 2l, 2l+1.  These launches sit on the latency-bound
// critical path of a verify step (a few KB of work each), so the grid is wide and every load of a
// thread is issued before the first one is used.  The RMSNorm needs the whole row: every chunk of
// a row computes the row's sum of squares itself (the same fixed-order reduction in every chunk,
// so all chunks use the same rstd), reading the row from L2 rather than waiting for a second
// launch.  As a consequence h_out must not alias x or d: a chunk writes its columns of h_out
// while other chunks of the row are still reading x and d.
//
// Launched with programmatic dependent launch: a CTA allows the next launch to start at once
// (the next qmm then streams its weights during this kernel) and waits for the previous grid
// before its first global read.
#include <atomic>
#include <cfloat>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "digits.cuh"
#include "peer.cuh"
#include "ptx.cuh"
#include "qmm_layout.cuh"

namespace skinny {

// CTAs of 64 threads and at most 64 registers (4096 per CTA): a prep CTA fits on an SM beside a
// qmm CTA (640 threads x 96 registers = 61440 of the SM's 65536), so the next qmm's CTAs become
// resident and stream their weights while the prep runs.  (An RMSNorm row longer than 2560
// columns takes 128-thread CTAs without that bound.)
constexpr int kPrepThreads = 128;                  // the embedding gather's CTA
constexpr int kPrepLeanThreads = 64;
constexpr int kPrepMaxK = 8 * 8 * 128;             // mode 0 row length: 16-byte vectors per thread <= 8

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float2 ld_bf2(const __nv_bfloat16* p) {
  const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(p);
  return make_float2(__low2float(v), __high2float(v));
}

// d(t, c): plain rows, or column-sharded with one [M, seg_cols] shard per rank (column c of
// token t in shard c / seg_cols at t * ldd + c % seg_cols): the per-rank outputs of a
// column-parallel matmul, in an all-gather buffer or read in place from the ranks' memory.
struct DSegs {
  const __nv_bfloat16* p[kMaxPeers];
};
__device__ __forceinline__ const __nv_bfloat16* d_at(const __nv_bfloat16* d, const DSegs& segs, int t, int c, int ldd,
                                                     int seg_cols) {
  if (seg_cols == 0) return d + static_cast<size_t>(t) * ldd + c;
  const int sh = c / seg_cols;
  return segs.p[sh] + static_cast<size_t>(t) * ldd + (c - sh * seg_cols);
}

// mode 0: rmsnorm (optional residual add), 1: swiglu, 2: plain.  NTHR threads; LEAN: at most
// 4096 registers per CTA.
template <int MODE, int NTHR, bool LEAN>
__global__ void __launch_bounds__(NTHR, LEAN ? 65536 / 4096 : 1) prep_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                            const __nv_bfloat16* __restrict__ d, int ldd,
                                                            int dseg_cols, const __grid_constant__ DSegs segs,
                                                            __nv_bfloat16* __restrict__ h_out, int ldh,
                                                            const float* __restrict__ w, float eps, int K, int M,
                                                            int mpad, uint8_t* __restrict__ xq,
                                                            __nv_bfloat16* __restrict__ a_out,
                                                            const __grid_constant__ PeerSync sync) {
  const int t = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = K / 64;
  constexpr int kWarps = NTHR / 32;
  const int g = blockIdx.x * kWarps + warp;
  const bool live = t < M;
  __shared__ float red[kWarps];
  __shared__ int sync_flag;
  pdl_launch_dependents();
  pdl_wait_prior_grid();  // x, d (and the buffers written below) belong to earlier launches
  peer_wait_all(sync, &sync_flag);  // d's shards from the other ranks (a timeout is recorded)
  const __nv_bfloat16* xr = x + static_cast<size_t>(t) * ldx;
  const bool has_d = d != nullptr || dseg_cols > 0;
  // mode 0: h = bf16(x + d) of the whole row, staged in shared memory by one round of 16-byte
  // loads (the row's sum of squares and this chunk's groups both read it there)
  extern __shared__ __align__(16) uint8_t prep_smem[];
  float* hrow = reinterpret_cast<float*>(prep_smem);
  float rstd = 1.f;
  if (MODE == 0 && live) {
    constexpr int kMaxPer = LEAN ? 5 : 8;  // 16-byte vectors per thread and tensor: K <= kMaxPer * 8 * NTHR
    const int nvec = K / 8;
    uint4 xv[kMaxPer], dv[kMaxPer];
#pragma unroll
    for (int u = 0; u < kMaxPer; ++u) {
      const int v = tid + u * NTHR;
      if (v < nvec) {
        xv[u] = *reinterpret_cast<const uint4*>(xr + 8 * v);
        if (has_d) dv[u] = *reinterpret_cast<const uint4*>(d_at(d, segs, t, 8 * v, ldd, dseg_cols));
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < kMaxPer; ++u) {
      const int v = tid + u * NTHR;
      if (v < nvec) {
        const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv[u]);
        const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&dv[u]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 h = __bfloat1622float2(x2[i]);
          if (has_d) {
            const float2 dd = __bfloat1622float2(d2[i]);
            h.x = bf16r(h.x + dd.x);
            h.y = bf16r(h.y + dd.y);
          }
          hrow[8 * v + 2 * i] = h.x;
          hrow[8 * v + 2 * i + 1] = h.y;
          ss = fmaf(h.x, h.x, fmaf(h.y, h.y, ss));
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) tot += red[i];  // fixed order, the same in every chunk
    rstd = rsqrtf(tot / static_cast<float>(K) + eps);
  }
  if (g < G) {
  const int c = g * 64 + 2 * lane;
  float a0 = 0.f, a1 = 0.f;
  if (live) {
    if (MODE == 0) {
      const float2 hv = make_float2(hrow[c], hrow[c + 1]);
      if (has_d && h_out)
        *reinterpret_cast<__nv_bfloat162*>(h_out + static_cast<size_t>(t) * ldh + c) = __floats2bfloat162_rn(hv.x, hv.y);
      a0 = bf16r(hv.x * rstd * (1.f + w[c]));
      a1 = bf16r(hv.y * rstd * (1.f + w[c + 1]));
      if (a_out)
        *reinterpret_cast<__nv_bfloat162*>(a_out + static_cast<size_t>(t) * K + c) = __floats2bfloat162_rn(a0, a1);
    } else if (MODE == 1) {
      const float2 gv = ld_bf2(xr + c), uv = ld_bf2(xr + K + c);
      a0 = bf16r(gv.x / (1.f + __expf(-gv.x)) * uv.x);
      a1 = bf16r(gv.y / (1.f + __expf(-gv.y)) * uv.y);
    } else {
      const float2 xv = ld_bf2(xr + c);
      a0 = xv.x;
      a1 = xv.y;
    }
  }
  write_digits(xq, mpad, t, g, lane, a0, a1, sync.mirror, sync.n_mirror);
  }
  peer_signal_done(sync, &sync_flag);  // this rank's digit groups are ready for the other ranks
}

static cudaError_t launch_pdl(void (*kern)(const __nv_bfloat16*, int, const __nv_bfloat16*, int, int, DSegs,
                                           __nv_bfloat16*, int, const float*, float, int, int, int, uint8_t*,
                                           __nv_bfloat16*, PeerSync),
                              int nthr, dim3 grid, size_t smem, cudaStream_t stream, const __nv_bfloat16* x, int ldx,
                              const __nv_bfloat16* d, int ldd, int dseg_cols, const DSegs& segs, __nv_bfloat16* h,
                              int ldh, const float* w, float eps, int K, int M, int mpad, uint8_t* xq,
                              __nv_bfloat16* a_out, const PeerSync& sync) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(nthr);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, x, ldx, d, ldd, dseg_cols, segs, h, ldh, w, eps, K, M, mpad, xq, a_out, sync);
}

int prep_max_k() { return kPrepMaxK; }

cudaError_t prep_launch(int mode, const void* x, int ldx, const void* d, int ldd, int dseg_cols,
                        const void* const* dseg, void* h_out, int ldh, const float* w, float eps, int K, int M,
                        void* xq, void* a_out, const skinny_peer_sync* sync, cudaStream_t stream) {
  const int mpad = M <= 8 ? 8 : 16;
  const int G = K / 64;
  const bool lean = mode != 0 || K <= 5 * 8 * kPrepLeanThreads;
  const int nthr = lean ? kPrepLeanThreads : 128;
  const dim3 grid((G + nthr / 32 - 1) / (nthr / 32), mpad);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* q = static_cast<uint8_t*>(xq);
  DSegs segs{};
  if (dseg_cols > 0)
    for (int i = 0; i < K / dseg_cols && i < kMaxPeers; ++i) segs.p[i] = static_cast<const __nv_bfloat16*>(dseg[i]);
  const PeerSync ps = peer_sync_from(sync);
  if (mode == 0) {
    const auto kern = lean ? prep_kernel<0, kPrepLeanThreads, true> : prep_kernel<0, 128, false>;
    static std::atomic<bool> attr_set[2][64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[lean][dev].load(std::memory_order_acquire)) {
      const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(kPrepMaxK * sizeof(float)));
      if (e != cudaSuccess) return e;
      attr_set[lean][dev].store(true, std::memory_order_release);
    }
    return launch_pdl(kern, nthr, grid, static_cast<size_t>(K) * sizeof(float), stream, xb, ldx,
                      static_cast<const __nv_bfloat16*>(d), ldd, dseg_cols, segs, static_cast<__nv_bfloat16*>(h_out),
                      ldh, w, eps, K, M, mpad, q, static_cast<__nv_bfloat16*>(a_out), ps);
  }
  if (mode == 1)
    return launch_pdl(prep_kernel<1, kPrepLeanThreads, true>, nthr, grid, 0, stream, xb, ldx, nullptr, 0, 0, segs,
                      nullptr, 0, nullptr, 0.f, K, M, mpad, q, nullptr, ps);
  return launch_pdl(prep_kernel<2, kPrepLeanThreads, true>, nthr, grid, 0, stream, xb, ldx, nullptr, 0, 0, segs,
                    nullptr, 0, nullptr, 0.f, K, M, mpad, q, nullptr, ps);
}

// Token embedding rows of a 4-bit group-64 table (MLX packing: word j of a row holds columns
// 8j .. 8j+7, nibble i = column 8j + i; bf16 scale and bias per 64 columns):
//   out[t, k] = bf16( q * s + b )  (f32 product, then f32 sum, each rounded: the same two
//   operations as the reference's dequantize), rows of ids outside [0, V) written as zeros.
// CTA per token, thread per packed word: one 4-byte load, eight values, one 16-byte store.
__global__ void __launch_bounds__(kPrepThreads) embed_w4g64_kernel(const int64_t* __restrict__ ids,
                                                                   const uint32_t* __restrict__ w,
                                                                   const __nv_bfloat16* __restrict__ sc,
                                                                   const __nv_bfloat16* __restrict__ bi, int V, int K,
                                                                   __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_launch_dependents();
  pdl_wait_prior_grid();  // the ids (and the rows this launch overwrites) belong to earlier work
  const int t = blockIdx.x;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < V;
  const int nw = K / 8;
  const size_t row = ok ? static_cast<size_t>(id) : 0;
  for (int j = threadIdx.x; j < nw; j += kPrepThreads) {
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (ok) {
      const uint32_t word = w[row * nw + j];
      const float s = __bfloat162float(sc[row * (K / 64) + j / 8]);
      const float b = __bfloat162float(bi[row * (K / 64) + j / 8]);
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float q0 = static_cast<float>((word >> (8 * i)) & 0xF);
        const float q1 = static_cast<float>((word >> (8 * i + 4)) & 0xF);
        o2[i] = __floats2bfloat162_rn(__fadd_rn(__fmul_rn(q0, s), b), __fadd_rn(__fmul_rn(q1, s), b));
      }
    }
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * ldo + 8 * j) = o;
  }
}

cudaError_t embed_launch(const int64_t* ids, int M, const void* w, const void* sc, const void* bi, int V, int K,
                         void* out, int ldo, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M);
  cfg.blockDim = dim3(kPrepThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, embed_w4g64_kernel, ids, static_cast<const uint32_t*>(w),
                            static_cast<const __nv_bfloat16*>(sc), static_cast<const __nv_bfloat16*>(bi), V, K,
                            static_cast<__nv_bfloat16*>(out), ldo);
}

}  // namespace skinny
