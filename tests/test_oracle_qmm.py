"""CPU tests: the qmm oracle against the reference's own golden vectors, and host-side logic."""

import json

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import quant


def test_metal_relayout_matches_reference_code():
    """oracle.repack_metal_order restates skinny_mlx/qmm.py:96-115; the fixture is that
    function's own output (tests/golden/make_golden.py)."""
    d = np.load(golden("qmm_repack_ref.npz"))
    for i in range(3):
        assert np.array_equal(quant.repack_metal_order(d[f"w{i}"]), d[f"r{i}"])


def test_reference_kernel_arithmetic_equals_identity_form():
    """The reference kernel's decode over its own lane-order layout (qmm.py:42-71) computes the
    same numbers as the affine identity over the natural MLX order."""
    rng = np.random.default_rng(3)
    n, k, m = 64, 256, 5
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    packed, s, b = quant.quantize(w)
    x = quant.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    relaid = quant.repack_metal_order(packed)
    a = quant.qmm_metal_order(x, relaid, s, b)
    bb = quant.qmm_identity(x, packed, s, b)
    assert np.allclose(a, bb, rtol=0, atol=1e-9)
    # the f16 rounding of x keeps the identity form within bf16-level error of MLX semantics
    assert quant.rel_err(quant.qmm_ref(x, packed, s, b), a) < 2e-3


def test_quantizer_rule_and_roundtrip():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((32, 128)) * 0.02).astype(np.float32)
    packed, s, b = quant.quantize(w)
    wg = w.reshape(32, 2, 64)
    assert np.array_equal(s, quant.f32_to_bf16_bits((wg.max(-1) - wg.min(-1)) / np.float32(15)))
    assert np.array_equal(b, quant.f32_to_bf16_bits(wg.min(-1)))
    deq = quant.dequantize(packed, s, b)
    step = np.repeat(quant.bf16_bits_to_f32(s), 64, axis=1)
    assert np.all(np.abs(deq - w) <= 0.5 * step + 2e-3 * np.abs(w).max())
    q = quant.unpack(packed)
    assert q.max() <= 15
    # element k = 8j + i at bits 4i of word j (skinny_mlx/qmm.py:104)
    assert ((packed[3, 5] >> np.uint32(4 * 6)) & 0xF) == q[3, 8 * 5 + 6]


def test_constant_group_quantizes_to_zero_scale():
    w = np.zeros((2, 64), np.float32)
    w[1] = 0.25
    packed, s, b = quant.quantize(w)
    assert np.all(quant.bf16_bits_to_f32(s) == 0)
    assert np.allclose(quant.dequantize(packed, s, b), w)


def test_product_quantizer_matches_oracle():
    """skinny_mlx_b200.qmm.quantize (torch) packs exactly what the oracle packs."""
    from skinny_mlx_b200.qmm import quantize, dequantize

    rng = np.random.default_rng(11)
    w = (rng.standard_normal((200, 320)) * 0.02).astype(np.float32)
    p_t, s_t, b_t = quantize(torch.from_numpy(w))
    p_o, s_o, b_o = quant.quantize(w)
    assert np.array_equal(p_t.numpy().view(np.uint32), p_o)
    assert np.array_equal(s_t.view(torch.int16).numpy().view(np.uint16), s_o)
    assert np.array_equal(b_t.view(torch.int16).numpy().view(np.uint16), b_o)
    assert np.allclose(dequantize(p_t, s_t, b_t).numpy(), quant.dequantize(p_o, s_o, b_o), atol=1e-6)


def test_golden_small_fixture_consistent():
    d = np.load(golden("qmm_small.npz"))
    for m in (1, 3, 8, 16):
        x = quant.bf16_bits_to_f32(d[f"x{m}"])
        y = quant.qmm_ref(x, d["packed"], d["s_bits"], d["b_bits"])
        assert np.allclose(y, d[f"y{m}"], rtol=1e-6, atol=1e-6)


def test_config_for_fixture_is_reference_table():
    """The reference's tile heuristic (qmm.py:118-126) recorded from its own code."""
    table = json.loads(golden("config_for_ref.json").read_text())
    for key, (rf, sk) in table.items():
        m, k = map(int, key.split(","))
        assert (rf, sk) == ((2, 8) if m <= 8 else (1, 4)) or (k // 64) % 8 != 0
        assert (k // 64) % sk == 0


def test_unit_relayout_is_a_permutation():
    """The B200 unit order holds the same nibbles (as int8 16 * (q - 8)), scales and biases;
    padding rows are zero."""
    rng = np.random.default_rng(5)
    n, k = 200, 192
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    packed, s, b = quant.quantize(w)
    tc = quant.repack_tc(packed, s, b)
    t, g = 2, 3
    assert tc.size == t * g * quant.UNIT_BYTES
    units = tc.reshape(t, g, quant.UNIT_BYTES)
    q = quant.unpack(packed).astype(np.int32)
    for tile in range(t):
        for grp in range(g):
            a = quant.unit_int8(units[tile, grp]).astype(np.int32)
            rows = min(128, n - 128 * tile)
            assert np.array_equal(a[:rows], 16 * (q[128 * tile: 128 * tile + rows, 64 * grp: 64 * grp + 64] - 8))
            assert not a[rows:].any()
    row, tile, grp = 7, 1, 2
    sbw = units[tile, grp, 4096 + 4 * row: 4096 + 4 * row + 4].view(np.uint32)[0]
    assert sbw & 0xFFFF == s[128 + row, grp] and sbw >> 16 == b[128 + row, grp]


def test_kernel_arithmetic_matches_mlx_semantics():
    rng = np.random.default_rng(8)
    w = (rng.standard_normal((96, 256)) * 0.02).astype(np.float32)
    packed, s, b = quant.quantize(w)
    x = quant.round_bf16(rng.standard_normal((6, 256)).astype(np.float32))
    ref = quant.qmm_ref(x, packed, s, b)
    got = quant.qmm_kernel_arith(x, packed, s, b)
    assert np.allclose(got, quant.qmm_xq(x, packed, s, b), rtol=1e-9, atol=1e-12)
    assert quant.rel_err(ref, got) < 1e-3


@pytest.mark.parametrize("mpad", [8, 16])
def test_xq_blocks_layout(mpad):
    """Reading the digits back through the documented offsets gives v = 256 hi + lo."""
    rng = np.random.default_rng(9)
    m = 5 if mpad == 8 else 13
    x = quant.round_bf16(rng.standard_normal((m, 192)).astype(np.float32))
    x[1, 64:128] = 0
    blk = quant.xq_blocks(x, mpad)
    assert blk.shape == (3, quant.xq_block_bytes(mpad))
    e, v, hi, lo, xsum = quant.xq_digits(x)
    for grp in range(3):
        for r in (0, m - 1, mpad, mpad + m - 1):
            for kk in (0, 17, 31, 32, 63):
                off = (kk >> 5) * (mpad * 64) + (r >> 3) * 256 + ((kk >> 4) & 1) * 128 + (r & 7) * 16 + (kk & 15)
                d = blk[grp, off].astype(np.int8)
                want = hi[r, grp, kk] if r < mpad else lo[r - mpad, grp, kk]
                assert d == want
    xs = blk[:, 2 * mpad * 64: 2 * mpad * 64 + 4 * mpad].view(np.float32)
    assert xs[1, 1] == 0 and xs[0, m:].max() == 0
    assert xs[0, 0] == np.float32(2.0 ** (e[0, 0] - 4))


@pytest.mark.parametrize("U,C", [(10, 3), (7, 3), (3040, 148), (47480, 148), (5, 5), (641, 148), (8, 1)])
def test_stream_k_partition(U, C):
    """Host mirror of u_begin / cta_of_unit (csrc/qmm_layout.cuh)."""
    def u_begin(c):
        return (c * U) // C

    def cta_of(u):
        return ((u + 1) * C - 1) // U

    for c in range(C):
        assert u_begin(c + 1) > u_begin(c)
    for u in range(U):
        c = cta_of(u)
        assert u_begin(c) <= u < u_begin(c + 1)


def test_xq_digits_exact_and_accurate():
    """The kernel's B operand: per (token, group) power-of-two scale, two int8 digits holding a
    16-bit fixed-point value; integer dot products, then s * 2^e * dot + b * xsum."""
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((192, 640)) * 0.02).astype(np.float32)
    packed, s, b = quant.quantize(w)
    for scale in (1.0, 1e-4, 500.0):
        x = quant.round_bf16((rng.standard_normal((5, 640)) * scale).astype(np.float32))
        x[0, :64] = 0.0
        x[2, 70] = 1000.0 * scale
        e, v, hi, lo, xsum = quant.xq_digits(x)
        assert np.array_equal(hi.astype(np.int64) * 256 + lo, v)
        assert np.abs(v).max() <= quant.XQ_MAXINT and hi.min() >= -128 and lo.max() <= 127
        assert quant.rel_err(quant.qmm_ref(x, packed, s, b), quant.qmm_xq(x, packed, s, b)) < 1e-3
