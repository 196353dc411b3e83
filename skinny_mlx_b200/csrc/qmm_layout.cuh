// Layout constants shared by the relayout, x-prep and qmm kernels and by the host code.
//
// Weights.  MLX's affine 4-bit packing (skinny_mlx/qmm.py:96-104 decodes it the same way) stores
// W[N, K] as uint32 words [N, K/8], element k = 8j + i at bits 4i..4i+3 of word j, with bf16
// scales and biases [N, K/64] (one per 64-column group).  At load the relayout kernel rewrites
// them into "units": one unit = 128 weight rows x one 64-column group, 4608 contiguous bytes:
//
//   [chunk c in {0,1}][row r in 0..127][16 bytes]   4096 B: row r's columns 32c .. 32c+31
//   [row r in 0..127][bf16 scale, bf16 bias]          512 B
//
// Units are ordered tile-major (tile = 128-row block, rows padded with zeros up to a multiple
// of 128), group-minor, so any contiguous range of units is one contiguous byte range.
// Inside each 32-bit word the eight nibbles of columns k0..k7 are placed so that two masks
// and one shift produce f16 pairs in natural column order (the 0x6400 "1024 + q" trick):
//   bits 0-3 k0 | 4-7 k2 | 8-11 k4 | 12-15 k6 | 16-19 k1 | 20-23 k3 | 24-27 k5 | 28-31 k7
//
// Activations.  For each 64-column group the x-prep kernel writes one 2112-byte block:
//   2048 B: x^T as f16 for 16 token slots in the tcgen05 K-major no-swizzle canonical layout,
//           four 16-column MMA slices of 512 B, each [token-block tb][k-half kh][8 tok][8 col],
//           so LBO (k-half stride) = 128 B and SBO (token-block stride) = 256 B;
//     64 B: xsum[16] f32 = sum of the group's 64 f16-rounded activations per token slot.
#pragma once
#include <cstddef>
#include <cstdint>

namespace skinny {

constexpr int kTileRows = 128;
constexpr int kGroup = 64;
constexpr int kMaxTokens = 16;
constexpr int kUnitWBytes = 4608;   // 4096 nibble bytes + 512 scale/bias bytes
constexpr int kUnitNibBytes = 4096;
constexpr int kUnitXBytes = 2112;   // 2048 f16 bytes + 64 xsum bytes
constexpr int kUnitXMatBytes = 2048;
constexpr int kXsumOffset = 2048;

// Stream-K CTA partition: CTA c owns units [u_begin(c), u_begin(c+1)).
__host__ __device__ inline long long u_begin(long long c, long long U, long long C) {
  return (c * U) / C;
}
// Largest c with u_begin(c) <= u  (i.e. the CTA that owns unit u).
__host__ __device__ inline long long cta_of_unit(long long u, long long U, long long C) {
  return ((u + 1) * C - 1) / U;
}

struct QmmShape {
  int N, K, G, T;  // rows, columns, groups (K/64), row tiles (ceil(N/128))
  long long U;     // units = T * G
};

__host__ __device__ inline QmmShape qmm_shape(int N, int K) {
  QmmShape s;
  s.N = N;
  s.K = K;
  s.G = K / kGroup;
  s.T = (N + kTileRows - 1) / kTileRows;
  s.U = static_cast<long long>(s.T) * s.G;
  return s;
}

inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Workspace layout for one qmm call (caller-owned, zero-filled before its first use):
//   [0, 256)            header; word 0 = device error bits
//   [256, +T*4)         per-tile arrival counters (every launch leaves them at zero)
//   partials            C x 2 slots x 16 tokens x 128 rows f32
//   x blocks            G x 2112 bytes
struct WsLayout {
  size_t cnt_off, part_off, x_off, total;
};
inline WsLayout ws_layout(int N, int K, int C) {
  QmmShape s = qmm_shape(N, K);
  WsLayout w;
  w.cnt_off = 256;
  w.part_off = round_up(w.cnt_off + static_cast<size_t>(s.T) * 4, 256);
  w.x_off = round_up(w.part_off + static_cast<size_t>(C) * 2 * kMaxTokens * kTileRows * 4, 256);
  w.total = round_up(w.x_off + static_cast<size_t>(s.G) * kUnitXBytes, 256);
  return w;
}

}  // namespace skinny
