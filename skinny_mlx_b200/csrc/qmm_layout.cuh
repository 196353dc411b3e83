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
// Activations are read as given (bf16 [M, K], row stride ldx) through a TMA tensor map: one box
// of 64 columns x 8 or 16 token rows per unit, 128-byte swizzled, rows past M zero-filled.
#pragma once
#include <cstddef>
#include <cstdint>

namespace skinny {

constexpr int kTileRows = 128;
constexpr int kGroup = 64;
constexpr int kMaxTokens = 16;
constexpr int kUnitWBytes = 4608;   // 4096 nibble bytes + 512 scale/bias bytes
constexpr int kUnitNibBytes = 4096;

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

// Workspace layout (caller-owned, zero-filled before its first use).  The counter region has a
// fixed offset and capacity so that calls of different shapes can share one workspace: only the
// counters must persist between launches (each launch leaves them at zero); partials are
// rewritten by every launch before they are read.
//   [0, 256)                      header; word 0 = device error bits
//   [256, 256 + 4*kMaxTiles)      per-tile arrival counters
//   partials                      C_dev x 2 slots x 16 tokens x 128 rows f32
constexpr int kMaxTiles = 16384;  // N <= 2,097,152 rows
struct WsLayout {
  size_t cnt_off, part_off, total;
};
inline WsLayout ws_layout(int /*N*/, int /*K*/, int C_dev) {
  WsLayout w;
  w.cnt_off = 256;
  w.part_off = w.cnt_off + static_cast<size_t>(kMaxTiles) * 4;
  w.total = round_up(w.part_off + static_cast<size_t>(C_dev) * 2 * kMaxTokens * kTileRows * 4, 256);
  return w;
}

}  // namespace skinny
