// Greedy speculative acceptance in one launch (skinny_mlx/spec.py:134-147 on B200):
//
//   pred[i] = argmax_v logits[i, v]            for the K+1 verified positions
//   n       = longest prefix with draft[i] == pred[i], i < K
//   emitted = draft[:n] + [pred[n]]
//
// The reference computes pred on the GPU, copies all K+1 predictions and the draft to the host
// (`.tolist()`, its one host sync per step) and runs the prefix loop in Python.  Here the argmax,
// the comparison and the prefix run on the device; the host reads back 1 + (K+1) int32 values.
//
// Work split: the vocabulary of every row is cut into chunks of kChunk logits, one CTA per
// (chunk, row).  Each CTA reduces its chunk to (max value, lowest index attaining it) and publishes
// it; the CTA that arrives last (global counter in the workspace) reduces the partials of every
// row in chunk order, runs the prefix comparison, writes the result and re-arms the counter.
// Ties resolve to the lowest vocabulary index (first occurrence), and a NaN counts as larger than
// every number, so the first NaN of a row wins: the order numpy's argmax uses (the reference's
// `.tolist()` of mx.argmax is compared with numpy's in its own checks).
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "skinny_status.h"

namespace skinny {

constexpr int kSpecThreads = 256;
constexpr int kSpecChunk = 8192;   // logits per CTA (16 KB of bf16)
constexpr int kSpecMaxRows = 17;   // K <= 16 draft tokens
constexpr int kSpecMaxChunks = 64; // V <= 524,288

struct SpecWs {
  unsigned int counter;    // CTAs arrived (re-armed to 0 by the last one)
  unsigned int pad[63];
  float val[kSpecMaxRows * kSpecMaxChunks];
  int idx[kSpecMaxRows * kSpecMaxChunks];
};

size_t spec_accept_ws_bytes() { return sizeof(SpecWs); }

// (a, ia) better than (b, ib): larger value, or equal value and lower index; NaN above every
// number, the lower index among NaNs.
__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  const bool an = a != a, bn = b != b;
  if (an || bn) return an && (!bn || ia < ib);
  return a > b || (a == b && ia < ib);
}

__device__ __forceinline__ void consider(float v, int i, float& bv, int& bi) {
  if (better(v, i, bv, bi)) {
    bv = v;
    bi = i;
  }
}

// The acceptance after the argmax of every row.  Chain (parent == null): n = the longest prefix
// with draft[i] == pred[i]; result = [n, draft[:n] + [pred[n]], -1 ...].  Tree (parent != null,
// tokens[i] the token of node i, node 0 the last emitted token): from the root, repeatedly move to
// the first child (lowest index) whose token equals the current node's prediction; result = [n,
// the n accepted tokens + [pred[last]], -1 ... (rows entries), the path 0, p1 .. pn, -1 ... (rows
// entries)].  A malformed tree (parent[0] != -1 or parent[i] outside [0, i)) has no children.
__device__ void accept_tail(const int* pred, int rows, const int32_t* draft, const int32_t* tokens,
                            const int32_t* parent, int32_t* result) {
  if (!parent) {
    int n = 0;
    while (n < rows - 1 && draft[n] == pred[n]) ++n;
    result[0] = n;
    for (int i = 0; i < rows; ++i) result[1 + i] = i < n ? draft[i] : (i == n ? pred[n] : -1);
    return;
  }
  const bool root_ok = parent[0] == -1;
  int cur = 0, n = 0;
  int path[kSpecMaxRows];
  path[0] = 0;
  while (root_ok) {
    int next = -1;
    for (int c = cur + 1; c < rows; ++c)
      if (parent[c] == cur && tokens[c] == pred[cur]) {
        next = c;
        break;
      }
    if (next < 0) break;
    path[++n] = next;
    cur = next;
  }
  result[0] = n;
  for (int i = 0; i < rows; ++i) {
    result[1 + i] = i < n ? tokens[path[i + 1]] : (i == n ? pred[cur] : -1);
    result[1 + rows + i] = i <= n ? path[i] : -1;
  }
}

__global__ void __launch_bounds__(kSpecThreads) spec_accept_kernel(
    const __nv_bfloat16* __restrict__ logits, int ld, int rows, int V, int chunks,
    const int32_t* __restrict__ draft, const int32_t* __restrict__ tokens, const int32_t* __restrict__ parent,
    int32_t* __restrict__ result, int32_t* __restrict__ pred_out, SpecWs* __restrict__ ws) {
  const int chunk = blockIdx.x;
  const int row = blockIdx.y;
  const int tid = threadIdx.x;
  const __nv_bfloat16* rp = logits + static_cast<size_t>(row) * ld;
  const int c0 = chunk * kSpecChunk;
  const int c1 = min(c0 + kSpecChunk, V);
  float bv = -__int_as_float(0x7F800000);  // -inf
  int bi = 0x7FFFFFFF;
  // 8 consecutive logits per thread and step (16-byte loads), 2048 per CTA step
  for (int base = c0 + tid * 8; base < c1; base += kSpecThreads * 8) {
    if (base + 8 <= c1) {
      const uint4 w = *reinterpret_cast<const uint4*>(rp + base);
      const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        consider(__uint_as_float(u[q] << 16), base + 2 * q, bv, bi);
        consider(__uint_as_float(u[q] & 0xFFFF0000u), base + 2 * q + 1, bv, bi);
      }
    } else {
      for (int i = base; i < c1; ++i) consider(__bfloat162float(rp[i]), i, bv, bi);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
    consider(ov, oi, bv, bi);
  }
  __shared__ float sv[kSpecThreads / 32];
  __shared__ int si[kSpecThreads / 32];
  __shared__ bool last;
  if ((tid & 31) == 0) {
    sv[tid >> 5] = bv;
    si[tid >> 5] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kSpecThreads / 32; ++w) consider(sv[w], si[w], bv, bi);
    ws->val[row * kSpecMaxChunks + chunk] = bv;
    ws->idx[row * kSpecMaxChunks + chunk] = bi;
    __threadfence();
    const unsigned int total = static_cast<unsigned int>(chunks) * rows;
    last = atomicAdd(&ws->counter, 1u) == total - 1;
  }
  __syncthreads();
  if (!last) return;
  // ---- the last CTA: row predictions, prefix comparison, emitted tokens
  __threadfence();
  __shared__ int pred[kSpecMaxRows];
  if (tid < rows) {
    float v = -__int_as_float(0x7F800000);
    int i = 0x7FFFFFFF;
    for (int c = 0; c < chunks; ++c)
      consider(__ldcg(&ws->val[tid * kSpecMaxChunks + c]), __ldcg(&ws->idx[tid * kSpecMaxChunks + c]), v, i);
    pred[tid] = i == 0x7FFFFFFF ? 0 : i;  // an all-NaN row predicts token 0
  }
  __syncthreads();
  if (tid == 0) {
    accept_tail(pred, rows, draft, tokens, parent, result);
    if (pred_out)
      for (int i = 0; i < rows; ++i) pred_out[i] = pred[i];
    ws->counter = 0u;
  }
}

cudaError_t spec_accept_launch(const void* logits, int ld, int rows, int V, const int32_t* draft,
                               int32_t* result, int32_t* pred, void* ws, cudaStream_t stream) {
  const int chunks = (V + kSpecChunk - 1) / kSpecChunk;
  dim3 grid(chunks, rows);
  spec_accept_kernel<<<grid, kSpecThreads, 0, stream>>>(static_cast<const __nv_bfloat16*>(logits), ld,
                                                        rows, V, chunks, draft, nullptr, nullptr, result, pred,
                                                        static_cast<SpecWs*>(ws));
  return cudaGetLastError();
}

cudaError_t spec_accept_tree_launch(const void* logits, int ld, int rows, int V, const int32_t* tokens,
                                    const int32_t* parent, int32_t* result, int32_t* pred, void* ws,
                                    cudaStream_t stream) {
  const int chunks = (V + kSpecChunk - 1) / kSpecChunk;
  dim3 grid(chunks, rows);
  spec_accept_kernel<<<grid, kSpecThreads, 0, stream>>>(static_cast<const __nv_bfloat16*>(logits), ld,
                                                        rows, V, chunks, nullptr, tokens, parent, result, pred,
                                                        static_cast<SpecWs*>(ws));
  return cudaGetLastError();
}

bool spec_accept_fits(int rows, int V) {
  return rows >= 1 && rows <= kSpecMaxRows && V >= 1 && (V + kSpecChunk - 1) / kSpecChunk <= kSpecMaxChunks;
}

}  // namespace skinny
