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
// Units are ordered tile-major (tile = 128-row block, rows padded with zero bytes up to a
// multiple of 128), group-minor, so any contiguous range of units is one contiguous byte range.
// Each nibble is stored as q ^ 8, i.e. q - 8 in 4-bit two's complement, and inside the 32-bit
// word of columns k0..k7 the nibbles sit at
//   bits 0-3 k4 | 4-7 k0 | 8-11 k5 | 12-15 k1 | 16-19 k6 | 20-23 k2 | 24-27 k7 | 28-31 k3
// so that  w & 0xF0F0F0F0  is the int8 quadruple 16*(q-8) of k0..k3 and
//  (w << 4) & 0xF0F0F0F0  that of k4..k7: the tensor-core A operand in one or two ALU ops.
//
// Activations.  An x-prep kernel turns x (bf16 [M, K], row stride ldx) into one block per
// 64-column group (xq_block_bytes(mpad) bytes, mpad = 8 for M <= 8 else 16):
//   int8 digits  [2 MMA steps of 32 columns][mpad/4 row groups][2 halves of 16 columns][8 rows][16 B]
//   f32 xs[mpad]    2^(e-4) for the token's power-of-two exponent e in this group (0 if all zero)
//   f32 xsum[mpad]  2^e * sum(v), the exact sum of the fixed-point values
// Digit row t < mpad holds hi(t), row mpad + t holds lo(t), where v = rint(x * 2^-e) has
// |v| <= 32639 = 127 * 256 + 127 and v = 256 hi + lo with hi, lo signed 8-bit.  Tokens >= M are
// zero.  Per MMA step the digits form a K-major, no-swizzle operand of 8-row x 16-byte core
// matrices: 128 bytes between the two 16-column halves, 256 bytes between 8-row groups.
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

// Bytes of one x-prep block for `mpad` (8 or 16) token rows.
__host__ __device__ constexpr int xq_block_bytes(int mpad) { return 2 * mpad * 64 + 8 * mpad; }

// Workspace layout (caller-owned, zero-filled before its first use).  Every region has a fixed
// offset and capacity so that calls of different shapes can share one workspace: only the
// counters must persist between launches (each launch leaves them at zero); partials and x-prep
// blocks are rewritten by every launch before they are read.
//   [0, 256)                      header; word 0 = device error bits
//   [256, 256 + 4*kMaxTiles)      per-tile arrival counters
//   partials                      C_dev x 2 slots x 16 tokens x 128 rows f32
//   x-prep blocks                 kMaxXGroups x xq_block_bytes(16)
constexpr int kMaxTiles = 16384;   // N <= 2,097,152 rows per call (all matrices of a group)
constexpr int kMaxXGroups = 2048;  // sum over distinct inputs of K/64 (K <= 131,072)
struct WsLayout {
  size_t cnt_off, part_off, xq_off, total;
};
inline WsLayout ws_layout(int C_dev) {
  WsLayout w;
  w.cnt_off = 256;
  w.part_off = w.cnt_off + static_cast<size_t>(kMaxTiles) * 4;
  w.xq_off = round_up(w.part_off + static_cast<size_t>(C_dev) * 2 * kMaxTokens * kTileRows * 4, 256);
  w.total = round_up(w.xq_off + static_cast<size_t>(kMaxXGroups) * xq_block_bytes(16), 256);
  return w;
}

}  // namespace skinny
