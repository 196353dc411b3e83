// Gated DeltaNet verify recurrence with per-token state checkpoints, and the rollback that
// selects a checkpoint (skinny_mlx/rollback.py:19-73 on B200).
//
// Recurrence (the gated delta rule as mlx_lm's gated_delta_update computes it, restated in
// bench/reversal_check.py:21-25 of the reference), per value head h and token t, with the state
// S [Dv, Dk] in f32:
//     S  <- g_t S
//     u  <- beta_t (v_t - S k_t)
//     S  <- S + u k_t^T
//     y_t = S q_t
// q and k are taken as given (the model has already L2-normalised them and folded the 1/sqrt(Dk)
// scale into q); a k head serves Hv/Hk consecutive value heads.
//
// The reference keeps the verify inputs and, on rollback, reruns the recurrence over the accepted
// prefix.  Here the verify pass writes the state after each of the first T-1 tokens to a
// checkpoint buffer, so rollback is a copy: state <- checkpoint[keep-1] (or nothing when every
// token is kept), one launch for all layers together with the conv-window update.
//
// Layout: every row v of S is independent given (g, beta, k, q, v[v]), so the rows of a head are
// spread over kGdnSplit CTAs of 128 threads: 4 threads per row, 32 columns each, state held in
// registers for the whole pass; k and q of each token are staged in shared memory.
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace skinny {

constexpr int kGdnDk = 128;
constexpr int kGdnDv = 128;
constexpr int kGdnThreads = 128;
constexpr int kGdnRowsPerCta = kGdnThreads / 4;  // 32
constexpr int kGdnSplit = kGdnDv / kGdnRowsPerCta;  // 4 CTAs per head

// q, k: [T, Hk, Dk] bf16; v: [T, Hv, Dv] bf16; g, beta: [T, Hv] f32; state: [Hv, Dv, Dk] f32
// (read, then overwritten with the state after token T-1); y: [T, Hv, Dv] bf16;
// ckpt: [T-1, Hv, Dv, Dk] f32 or null.
__global__ void __launch_bounds__(kGdnThreads) gdn_recurrent_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, const float* __restrict__ g, const float* __restrict__ beta,
    float* __restrict__ state, __nv_bfloat16* __restrict__ y, float* __restrict__ ckpt, int T, int Hv,
    int Hk) {
  const int h = blockIdx.y;
  const int hk = h / (Hv / Hk);
  const int tid = threadIdx.x;
  const int row = blockIdx.x * kGdnRowsPerCta + (tid >> 2);
  const int c0 = (tid & 3) * 32;
  __shared__ float ks[kGdnDk], qs[kGdnDk];
  float S[32];
  float* srow = state + (static_cast<size_t>(h) * kGdnDv + row) * kGdnDk + c0;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const float4 w = *reinterpret_cast<const float4*>(srow + j);
    S[j] = w.x; S[j + 1] = w.y; S[j + 2] = w.z; S[j + 3] = w.w;
  }
  for (int t = 0; t < T; ++t) {
    __syncthreads();  // previous token's ks/qs no longer read
    ks[tid] = __bfloat162float(k[(static_cast<size_t>(t) * Hk + hk) * kGdnDk + tid]);
    qs[tid] = __bfloat162float(q[(static_cast<size_t>(t) * Hk + hk) * kGdnDk + tid]);
    __syncthreads();
    const float gt = g[static_cast<size_t>(t) * Hv + h];
    const float bt = beta[static_cast<size_t>(t) * Hv + h];
    const float vt = __bfloat162float(v[(static_cast<size_t>(t) * Hv + h) * kGdnDv + row]);
    float sk = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      S[j] *= gt;
      sk = fmaf(S[j], ks[c0 + j], sk);
    }
    sk += __shfl_xor_sync(0xFFFFFFFFu, sk, 1);
    sk += __shfl_xor_sync(0xFFFFFFFFu, sk, 2);
    const float u = bt * (vt - sk);
    float yt = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      S[j] = fmaf(u, ks[c0 + j], S[j]);
      yt = fmaf(S[j], qs[c0 + j], yt);
    }
    yt += __shfl_xor_sync(0xFFFFFFFFu, yt, 1);
    yt += __shfl_xor_sync(0xFFFFFFFFu, yt, 2);
    if ((tid & 3) == 0) y[(static_cast<size_t>(t) * Hv + h) * kGdnDv + row] = __float2bfloat16_rn(yt);
    if (ckpt && t + 1 < T) {
      float* cp = ckpt + ((static_cast<size_t>(t) * Hv + h) * kGdnDv + row) * kGdnDk + c0;
#pragma unroll
      for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(cp + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
    }
  }
#pragma unroll
  for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(srow + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
}

cudaError_t gdn_recurrent_launch(const void* q, const void* k, const void* v, const float* g,
                                 const float* beta, float* state, void* y, float* ckpt, int T, int Hv,
                                 int Hk, cudaStream_t stream) {
  dim3 grid(kGdnSplit, Hv);
  gdn_recurrent_kernel<<<grid, kGdnThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(v), g, beta, state, static_cast<__nv_bfloat16*>(y), ckpt, T, Hv,
      Hk);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Rollback after a verify of `fed` tokens that keeps the first `keep` (1 <= keep <= fed):
//   state[l] <- ckpt[l][keep-1]                   (if keep < fed)
//   conv[l]  <- rows [keep, keep + W) of conv_full[l]
// for every layer l in one launch.  conv: [W, C] bf16, the previous inputs the causal conv still
// needs; conv_full: [W + fed, C] bf16, the conv input of the verify step (the old window followed
// by the fed tokens' inputs).  The reference re-slices its recorded conv input the same way
// (skinny_mlx/rollback.py:70-71).
// ---------------------------------------------------------------------------------------------
constexpr int kGdnMaxLayers = 64;
struct GdnRollbackParams {
  float* state[kGdnMaxLayers];
  const float* ckpt[kGdnMaxLayers];
  __nv_bfloat16* conv[kGdnMaxLayers];
  const __nv_bfloat16* conv_full[kGdnMaxLayers];
  long long state_elems;  // Hv * Dv * Dk
  int n_layers, keep, fed, W, C;
};

__global__ void __launch_bounds__(256) gdn_rollback_kernel(const __grid_constant__ GdnRollbackParams p) {
  const int l = blockIdx.y;
  if (p.keep < p.fed) {
    const float4* src = reinterpret_cast<const float4*>(p.ckpt[l] + static_cast<size_t>(p.keep - 1) * p.state_elems);
    float4* dst = reinterpret_cast<float4*>(p.state[l]);
    const long long n4 = p.state_elems / 4;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
      dst[i] = src[i];
  }
  if (p.conv[l]) {
    const long long n = static_cast<long long>(p.W) * p.C;
    const __nv_bfloat16* src = p.conv_full[l] + static_cast<size_t>(p.keep) * p.C;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
      p.conv[l][i] = src[i];
  }
}

// Tree rollback: the accepted path ends at node `node`; state[l] <- ckpt[l][node] and conv[l] row
// q <- conv_full[l] row rows[q] (q < W): the last W conv inputs along the path.
struct GdnRollbackTreeParams {
  float* state[kGdnMaxLayers];
  const float* ckpt[kGdnMaxLayers];
  __nv_bfloat16* conv[kGdnMaxLayers];
  const __nv_bfloat16* conv_full[kGdnMaxLayers];
  long long state_elems;
  int rows[4];
  int n_layers, node, W, C;
};

__global__ void __launch_bounds__(256) gdn_rollback_tree_kernel(const __grid_constant__ GdnRollbackTreeParams p) {
  const int l = blockIdx.y;
  const float4* src = reinterpret_cast<const float4*>(p.ckpt[l] + static_cast<size_t>(p.node) * p.state_elems);
  float4* dst = reinterpret_cast<float4*>(p.state[l]);
  const long long n4 = p.state_elems / 4;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
  const long long n = static_cast<long long>(p.W) * p.C;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int q = static_cast<int>(i / p.C);
    const long long c = i - static_cast<long long>(q) * p.C;
    p.conv[l][i] = p.conv_full[l][static_cast<size_t>(p.rows[q]) * p.C + c];
  }
}

cudaError_t gdn_rollback_tree_call(int n_layers, float* const* state, const float* const* ckpt, void* const* conv,
                                  const void* const* conv_full, long long state_elems, int node, const int* rows,
                                  int W, int C, cudaStream_t stream) {
  static thread_local GdnRollbackTreeParams prm;
  prm.n_layers = n_layers;
  prm.node = node;
  prm.W = W;
  prm.C = C;
  prm.state_elems = state_elems;
  for (int q = 0; q < 4; ++q) prm.rows[q] = q < W ? rows[q] : 0;
  for (int l = 0; l < n_layers; ++l) {
    prm.state[l] = state[l];
    prm.ckpt[l] = ckpt[l];
    prm.conv[l] = static_cast<__nv_bfloat16*>(conv[l]);
    prm.conv_full[l] = static_cast<const __nv_bfloat16*>(conv_full[l]);
  }
  dim3 grid(32, n_layers);
  gdn_rollback_tree_kernel<<<grid, 256, 0, stream>>>(prm);
  return cudaGetLastError();
}

cudaError_t gdn_rollback_call(int n_layers, float* const* state, const float* const* ckpt,
                             void* const* conv, const void* const* conv_full, long long state_elems,
                             int keep, int fed, int W, int C, cudaStream_t stream) {
  static thread_local GdnRollbackParams prm;
  prm.n_layers = n_layers;
  prm.keep = keep;
  prm.fed = fed;
  prm.W = W;
  prm.C = C;
  prm.state_elems = state_elems;
  for (int l = 0; l < n_layers; ++l) {
    prm.state[l] = state[l];
    prm.ckpt[l] = ckpt[l];
    prm.conv[l] = conv ? static_cast<__nv_bfloat16*>(conv[l]) : nullptr;
    prm.conv_full[l] = conv ? static_cast<const __nv_bfloat16*>(conv_full[l]) : nullptr;
  }
  dim3 grid(32, n_layers);  // 32 x 256 threads per layer: a 1 MiB state is 256 float4 per thread
  gdn_rollback_kernel<<<grid, 256, 0, stream>>>(prm);
  return cudaGetLastError();
}

}  // namespace skinny
