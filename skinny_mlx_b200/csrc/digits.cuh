// Writing one prepared qmm input (the x-prep block format of qmm_layout.cuh) from device code:
// shared by the producer kernels (prep.cu, gdn_fused.cu).
#pragma once
#include <cfloat>
#include <cstdint>

#include "qmm_layout.cuh"

namespace skinny {

// Writes the digits of two values (columns 2*lane, 2*lane+1 of group g, token t) and, from lane 0,
// the group's xs and xsum.  a0, a1 are bf16-exact floats.  Warp-collective.  The same words are
// also written to mirror[0 .. n_mirror) (other ranks' copies of xq, same layout), if any.
__device__ __forceinline__ void write_digits(uint8_t* xq, int mpad, int t, int g, int lane, float a0, float a1,
                                             uint8_t* const* mirror = nullptr, int n_mirror = 0) {
  float amax = fmaxf(fabsf(a0), fabsf(a1));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  const bool bad = __any_sync(0xFFFFFFFFu, !(fabsf(a0) <= FLT_MAX) || !(fabsf(a1) <= FLT_MAX));
  int v0 = 0, v1 = 0;
  float xs = 0.f, xsum = 0.f;
  if (bad) {
    xs = __int_as_float(0x7FC00000);
    xsum = xs;
  } else if (amax > 0.f) {
    int e2;
    frexpf(amax, &e2);
    int e = e2 - 15;
    if (ldexpf(amax, -e) > 32639.f) e += 1;
    v0 = __float2int_rn(ldexpf(a0, -e));
    v1 = __float2int_rn(ldexpf(a1, -e));
    int vs = v0 + v1;
#pragma unroll
    for (int o = 16; o; o >>= 1) vs += __shfl_xor_sync(0xFFFFFFFFu, vs, o);
    xs = ldexpf(1.f, e - 4);
    xsum = ldexpf(static_cast<float>(vs), e);
  }
  const int hi0 = (v0 + 128) >> 8, hi1 = (v1 + 128) >> 8;
  const int lo0 = v0 - 256 * hi0, lo1 = v1 - 256 * hi1;
  const size_t boff = static_cast<size_t>(g) * xq_block_bytes(mpad);
  const int k = 2 * lane;
  const int kofs = (k >> 5) * (mpad * 64) + ((k >> 4) & 1) * 128 + (k & 15);
  const int rh = t, rl = mpad + t;
  const uint16_t whi = static_cast<uint16_t>((hi0 & 0xFF) | ((hi1 & 0xFF) << 8));
  const uint16_t wlo = static_cast<uint16_t>((lo0 & 0xFF) | ((lo1 & 0xFF) << 8));
  for (int d = -1; d < n_mirror; ++d) {
    uint8_t* blk = (d < 0 ? xq : mirror[d]) + boff;
    *reinterpret_cast<uint16_t*>(blk + kofs + (rh >> 3) * 256 + (rh & 7) * 16) = whi;
    *reinterpret_cast<uint16_t*>(blk + kofs + (rl >> 3) * 256 + (rl & 7) * 16) = wlo;
    if (lane == 0) {
      float* xf = reinterpret_cast<float*>(blk + 2 * mpad * 64);
      xf[t] = xs;
      xf[mpad + t] = xsum;
    }
  }
}

}  // namespace skinny
