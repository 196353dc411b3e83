"""CPU restatement of MLX affine 4-bit group-64 quantization and quantized matmul.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows:
  * the packing decode of skinny_mlx/qmm.py:104 (element k = 8j + i at bits 4i of word j);
  * the quantizer stated for BASELINE config 1: per 64-column group scale = (max - min) / 15,
    bias = min, bf16 scale/bias, q = clamp(round((w - bias) / scale), 0, 15);
  * mx.quantized_matmul(x, w, s, b, transpose=True, group_size=64, bits=4) as called at
    skinny_mlx/qmm.py:183 and skinny_mlx/patch.py:35: y = x @ (q * s + b)^T;
  * the reference kernel's affine identity sum_k x (q s + b) = s sum_k x q + b sum_k x with x
    rounded to f16 (skinny_mlx/qmm.py:8-9, 64-71, 136, 143).
"""

from __future__ import annotations

import numpy as np

GROUP = 64


# ------------------------------------------------------------------------------------------------
# bf16 / f16 helpers (round-to-nearest-even, as the hardware conversions do)
# ------------------------------------------------------------------------------------------------
def f32_to_bf16_bits(a) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(a, dtype=np.float32))
    if nan.any():
        out = np.where(nan, np.uint16(0x7FC0), out)
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(a) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


def round_f16(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


# ------------------------------------------------------------------------------------------------
# quantize / pack / dequantize
# ------------------------------------------------------------------------------------------------
def quantize(w: np.ndarray):
    """w [N, K] float32 -> (packed uint32 [N, K/8], scales bf16 bits [N, K/64], biases bf16 bits)."""
    n, k = w.shape
    assert k % GROUP == 0, k
    wg = np.asarray(w, dtype=np.float32).reshape(n, k // GROUP, GROUP)
    wmax = wg.max(-1)
    wmin = wg.min(-1)
    s_bits = f32_to_bf16_bits((wmax - wmin) / np.float32(15.0))
    b_bits = f32_to_bf16_bits(wmin)
    s = bf16_bits_to_f32(s_bits)[..., None]
    b = bf16_bits_to_f32(b_bits)[..., None]
    safe = np.where(s == 0, np.float32(1.0), s)
    q = np.clip(np.rint((wg - b) / safe), 0, 15)
    q = np.where(s == 0, 0, q).astype(np.uint32).reshape(n, k // 8, 8)
    packed = np.zeros((n, k // 8), dtype=np.uint32)
    for i in range(8):
        packed |= q[..., i] << np.uint32(4 * i)
    return packed, s_bits, b_bits


def unpack(packed: np.ndarray) -> np.ndarray:
    """uint32 [N, K/8] -> uint8 nibbles [N, K] (element 8j + i = bits 4i of word j)."""
    n, kw = packed.shape
    q = np.stack([(packed >> np.uint32(4 * i)) & np.uint32(0xF) for i in range(8)], axis=-1)
    return q.reshape(n, kw * 8).astype(np.uint8)


def dequantize(packed, s_bits, b_bits) -> np.ndarray:
    q = unpack(packed).astype(np.float64)
    s = np.repeat(bf16_bits_to_f32(s_bits).astype(np.float64), GROUP, axis=1)
    b = np.repeat(bf16_bits_to_f32(b_bits).astype(np.float64), GROUP, axis=1)
    return q * s + b


# ------------------------------------------------------------------------------------------------
# quantized matmul
# ------------------------------------------------------------------------------------------------
def qmm_ref(x: np.ndarray, packed, s_bits, b_bits) -> np.ndarray:
    """MLX quantized_matmul semantics in float64: x [M, K] @ (q s + b)^T -> [M, N]."""
    return np.asarray(x, dtype=np.float64) @ dequantize(packed, s_bits, b_bits).T


def qmm_identity(x: np.ndarray, packed, s_bits, b_bits) -> np.ndarray:
    """The reference kernel's arithmetic in float64: x rounded to f16, then per 64-group
    s * sum(x q) + b * sum(x) (skinny_mlx/qmm.py:64-71, 143)."""
    xf = round_f16(x).astype(np.float64)
    m, k = xf.shape
    q = unpack(packed).astype(np.float64)
    n = q.shape[0]
    g = k // GROUP
    s = bf16_bits_to_f32(s_bits).astype(np.float64)
    b = bf16_bits_to_f32(b_bits).astype(np.float64)
    xg = xf.reshape(m, g, GROUP)
    qg = q.reshape(n, g, GROUP)
    dots = np.einsum("mgk,ngk->mng", xg, qg)
    xsum = xg.sum(-1)  # [m, g]
    return (dots * s[None] + xsum[:, None, :] * b[None]).sum(-1)


def rel_err(ref, got) -> float:
    """max |ref - got| / max |ref| (the metric of skinny_mlx/qmm.py:185)."""
    ref = np.asarray(ref, dtype=np.float64)
    got = np.asarray(got, dtype=np.float64)
    den = np.abs(ref).max()
    return float(np.abs(ref - got).max() / (den if den > 0 else 1.0))


# ------------------------------------------------------------------------------------------------
# the reference's Metal lane-order relayout, restated (pinned against the reference's own code)
# ------------------------------------------------------------------------------------------------
def _lane_maps():
    lane = np.arange(32)
    qid = lane // 4
    fm = (qid & 4) + ((lane // 2) % 4)  # skinny_mlx/qmm.py:35, :107
    fn = (qid & 2) * 2 + (lane % 2) * 2  # skinny_mlx/qmm.py:36, :108
    return fm, fn


def repack_metal_order(packed: np.ndarray) -> np.ndarray:
    """skinny_mlx/qmm.py:96-115: [N, K/8] -> [N/8, K/64, 32 lanes, 2 words] (same bytes)."""
    n, kw = packed.shape
    kg = kw // 8
    q = unpack(packed).reshape(n // 8, 8, kg, 8, 8)  # [R, row-in-fragment, g, step, col]
    fm, fn = _lane_maps()
    out = np.zeros((n // 8, kg, 32, 2), dtype=np.uint32)
    for lane in range(32):
        e0 = q[:, fm[lane], :, :, fn[lane]].astype(np.uint32)      # [R, g, step]
        e1 = q[:, fm[lane], :, :, fn[lane] + 1].astype(np.uint32)
        for h in range(2):
            for i in range(4):
                out[:, :, lane, h] |= (e0[..., 4 * h + i] << np.uint32(4 * i)) | (
                    e1[..., 4 * h + i] << np.uint32(16 + 4 * i))
    return out.reshape(n, kw)


def qmm_metal_order(x: np.ndarray, relaid: np.ndarray, s_bits, b_bits) -> np.ndarray:
    """The reference kernel's inner loop restated over its own relaid layout
    (skinny_mlx/qmm.py:42-71): lane (fm, fn) of fragment R, group g, step s holds
    W[8R + fm, 64g + 8s + fn + {0, 1}] at bits (4(s%4), 16 + 4(s%4)) of word s // 4."""
    xf = round_f16(x).astype(np.float64)
    m, k = xf.shape
    n = relaid.shape[0]
    kg = k // GROUP
    words = relaid.reshape(n // 8, kg, 32, 2)
    fm, fn = _lane_maps()
    q = np.zeros((n, k), dtype=np.float64)
    for lane in range(32):
        for s in range(8):
            wv = words[:, :, lane, s // 4]
            bits = (wv >> np.uint32(4 * (s % 4))) & np.uint32(0x000F000F)
            lo = (bits & 0xF).astype(np.float64)
            hi = ((bits >> 16) & 0xF).astype(np.float64)
            rows = np.arange(n // 8) * 8 + fm[lane]
            for g in range(kg):
                col = 64 * g + 8 * s + fn[lane]
                q[rows, col] = lo[:, g]
                q[rows, col + 1] = hi[:, g]
    s = bf16_bits_to_f32(s_bits).astype(np.float64)
    b = bf16_bits_to_f32(b_bits).astype(np.float64)
    xg = xf.reshape(m, kg, GROUP)
    qg = q.reshape(n, kg, GROUP)
    dots = np.einsum("mgk,ngk->mng", xg, qg)
    return (dots * s[None] + xg.sum(-1)[:, None, :] * b[None]).sum(-1)


# ------------------------------------------------------------------------------------------------
# the B200 unit layout (byte-exact statement of what skinny_repack_w4g64 must produce)
# ------------------------------------------------------------------------------------------------
TILE = 128
UNIT_BYTES = 4608


def repack_tc(packed: np.ndarray, s_bits, b_bits) -> np.ndarray:
    """MLX packs -> the kernel's unit order as uint8 bytes (see csrc/qmm_layout.cuh).

    Each nibble is stored as q ^ 8 (q - 8 in 4-bit two's complement).  Within the 32-bit word of
    columns c0..c7: c0..c3 sit in the high nibbles of bytes 0..3 and c4..c7 in the low nibbles,
    so `w & 0xF0F0F0F0` and `(w << 4) & 0xF0F0F0F0` are four int8 values 16 * (q - 8) each."""
    n, kw = packed.shape
    k = kw * 8
    g = k // GROUP
    t = (n + TILE - 1) // TILE
    npad = t * TILE
    q = np.zeros((npad, k), dtype=np.uint32)
    q[:n] = unpack(packed)
    sb = np.zeros((npad, g), dtype=np.uint32)
    sb[:n] = s_bits.astype(np.uint32) | (b_bits.astype(np.uint32) << np.uint32(16))
    q8 = q.reshape(npad, k // 8, 8) ^ np.uint32(8)
    shift = [4, 12, 20, 28, 0, 8, 16, 24]  # column i -> bit position
    words = np.zeros((npad, k // 8), dtype=np.uint32)
    for i in range(8):
        words |= q8[..., i] << np.uint32(shift[i])
    if n < npad:
        words[n:] = 0  # padding rows hold zero bytes, not the q ^ 8 of q = 0
    # [tile, row, group, chunk, 4 words] -> [tile, group, chunk, row, 4 words]
    w5 = words.reshape(t, TILE, g, 2, 4).transpose(0, 2, 3, 1, 4)
    nib = np.ascontiguousarray(w5).reshape(t, g, 2 * TILE * 4).view(np.uint8).reshape(t, g, 4096)
    sbu = np.ascontiguousarray(sb.reshape(t, TILE, g).transpose(0, 2, 1)).view(np.uint8).reshape(t, g, 512)
    return np.concatenate([nib, sbu], axis=-1).reshape(-1)


def unit_int8(unit_bytes: np.ndarray) -> np.ndarray:
    """Decode one relaid unit's nibble bytes as the kernel does -> int8 [128 rows, 64 columns]
    holding 16 * (q - 8)."""
    words = unit_bytes[:4096].view(np.uint32).reshape(2, TILE, 4).transpose(1, 0, 2).reshape(TILE, 8)
    lo = words & np.uint32(0xF0F0F0F0)
    hi = (words << np.uint32(4)) & np.uint32(0xF0F0F0F0)
    out = np.stack([lo, hi], axis=-1).reshape(TILE, 16)  # word order: k 0-3, 4-7, 8-11, ...
    return out.view(np.int8).reshape(TILE, 64)


# ------------------------------------------------------------------------------------------------
# 16-bit fixed-point activations as two int8 digits (the B200 kernel's B operand)
# ------------------------------------------------------------------------------------------------
XQ_MAXINT = 32639  # 127 * 256 + 127: the largest value two signed int8 digits (hi*256 + lo) hold


def xq_digits(x: np.ndarray):
    """x [M, K] float32 (bf16 values) -> per (token, 64-group) power-of-two scale, int16 value,
    hi/lo int8 digits and exact group sum, as the x-prep kernel computes them:
      e = smallest integer with max|x_g| <= 32639 * 2^e (e = -133 for an all-zero group),
      v = rint(x * 2^-e) (|v| <= 32639), hi = (v + 128) >> 8, lo = v - 256 hi, xsum = sum(v) * 2^e.
    """
    m, k = x.shape
    g = k // GROUP
    xg = np.asarray(x, dtype=np.float64).reshape(m, g, GROUP)
    amax = np.abs(xg).max(-1)
    e = np.full((m, g), -133, dtype=np.int64)
    nz = amax > 0
    # smallest e with amax <= 32639 * 2^e
    e_nz = np.ceil(np.log2(amax[nz] / XQ_MAXINT)).astype(np.int64)
    # fix float rounding of log2 at exact powers
    e_nz = np.where(amax[nz] <= XQ_MAXINT * np.exp2(e_nz - 1), e_nz - 1, e_nz)
    e_nz = np.where(amax[nz] > XQ_MAXINT * np.exp2(e_nz), e_nz + 1, e_nz)
    e[nz] = e_nz
    v = np.rint(xg * np.exp2(-e)[..., None]).astype(np.int64)
    assert np.abs(v).max() <= XQ_MAXINT
    hi = (v + 128) >> 8
    lo = v - 256 * hi
    xsum = v.sum(-1).astype(np.float64) * np.exp2(e)
    return e, v, hi.astype(np.int8), lo.astype(np.int8), xsum


def qmm_xq(x: np.ndarray, packed, s_bits, b_bits) -> np.ndarray:
    """The B200 kernel's arithmetic: integer dot products of nibbles with the 16-bit fixed-point x,
    then per group s * 2^e * dot + b * xsum (float64 here)."""
    e, v, hi, lo, xsum = xq_digits(x)
    q = unpack(packed).astype(np.int64)
    n = q.shape[0]
    m, g = e.shape
    qg = q.reshape(n, g, GROUP)
    dot = np.einsum("mgk,ngk->mng", hi.astype(np.int64), qg) * 256 + np.einsum("mgk,ngk->mng", lo.astype(np.int64), qg)
    s = bf16_bits_to_f32(s_bits).astype(np.float64)
    b = bf16_bits_to_f32(b_bits).astype(np.float64)
    return (dot * np.exp2(e)[:, None, :] * s[None] + xsum[:, None, :] * b[None]).sum(-1)


def xq_block_bytes(mpad: int) -> int:
    """Bytes of one x-prep block: int8 digits [2 MMAs][mpad/4 row groups][2][8 rows][16 B], then
    f32 xs[mpad] and f32 xsum[mpad]."""
    return 2 * mpad * 64 + 8 * mpad


def xq_blocks(x: np.ndarray, mpad: int) -> np.ndarray:
    """The x-prep kernel's output for x [M, K] (bf16 values as float32), as bytes [G, block].

    Digit rows 0..mpad-1 are the hi digits of tokens 0..mpad-1, rows mpad..2*mpad-1 the lo digits;
    byte (row r, column k) of a group sits at
      (k >> 5) * (mpad * 64) + (r >> 3) * 256 + ((k >> 4) & 1) * 128 + (r & 7) * 16 + (k & 15),
    i.e. per 32-column MMA step a K-major no-swizzle layout of 8-row x 16-byte core matrices with
    128 bytes between the two K halves (leading offset) and 256 between 8-row groups (stride
    offset).  xs = 2^(e-4) (0 for an all-zero group), xsum = 2^e * sum(v); tokens >= M are zero."""
    m, k = x.shape
    g = k // GROUP
    e, v, hi, lo, xsum = xq_digits(x)
    nz = np.abs(np.asarray(x, np.float64).reshape(m, g, GROUP)).max(-1) > 0
    dig = np.zeros((g, 2 * mpad, GROUP), np.int8)
    dig[:, :m] = hi.transpose(1, 0, 2)
    dig[:, mpad:mpad + m] = lo.transpose(1, 0, 2)
    rr, kk = np.meshgrid(np.arange(2 * mpad), np.arange(GROUP), indexing="ij")
    off = (kk >> 5) * (mpad * 64) + (rr >> 3) * 256 + ((kk >> 4) & 1) * 128 + (rr & 7) * 16 + (kk & 15)
    blk = np.zeros((g, xq_block_bytes(mpad)), np.uint8)
    blk[:, off.reshape(-1)] = dig.reshape(g, -1).view(np.uint8)
    xs = np.zeros((g, mpad), np.float32)
    xs[:, :m] = np.where(nz, np.exp2(e - 4.0), 0.0).T.astype(np.float32)
    xsm = np.zeros((g, mpad), np.float32)
    xsm[:, :m] = np.where(nz, xsum, 0.0).T.astype(np.float32)
    blk[:, 2 * mpad * 64: 2 * mpad * 64 + 4 * mpad] = xs.view(np.uint8)
    blk[:, 2 * mpad * 64 + 4 * mpad:] = xsm.view(np.uint8)
    return blk


def qmm_kernel_arith(x: np.ndarray, packed, s_bits, b_bits) -> np.ndarray:
    """The B200 kernel's arithmetic restated in float64 over its own operands: int8 weights
    16 * (q - 8), int8 x digits, integer dot products G = 256 * dot(hi) + dot(lo), then per group
    out += s * xs * G + (b + 8 s) * xsum.  Equals qmm_xq up to float rounding."""
    e, v, hi, lo, xsum = xq_digits(x)
    q = unpack(packed).astype(np.int64)
    n = q.shape[0]
    m, g = e.shape
    a = 16 * (q.reshape(n, g, GROUP) - 8)
    G = (np.einsum("mgk,ngk->mng", hi.astype(np.int64), a) * 256
         + np.einsum("mgk,ngk->mng", lo.astype(np.int64), a))
    s = bf16_bits_to_f32(s_bits).astype(np.float64)
    b = bf16_bits_to_f32(b_bits).astype(np.float64)
    xs = np.exp2(e - 4.0)
    return (G * xs[:, None, :] * s[None] + xsum[:, None, :] * (b + 8 * s)[None]).sum(-1)
