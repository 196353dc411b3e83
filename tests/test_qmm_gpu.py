"""GPU parity tests for the tcgen05 qmm path, through the C-ABI, against the CPU oracle.

Tolerance: max|ref - got| / max|ref| <= 1.5e-2 (skinny_mlx/qmm.py:185 metric, BASELINE bound);
the kernel is expected to sit near bf16 output rounding, so most cases also assert 6e-3.
"""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import quant

pytestmark = pytest.mark.gpu

TOL = 1.5e-2
TIGHT = 6e-3


def make_weight(n, k, seed, dev):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    packed, s, b = quant.quantize(w)
    tw = torch.from_numpy(packed.view(np.int32)).to(dev)
    ts = torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).to(dev)
    tb = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).to(dev)
    return (packed, s, b), (tw, ts, tb)


def make_x(m, k, seed, dev):
    rng = np.random.default_rng(seed)
    xb = quant.f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(dev)
    return quant.bf16_bits_to_f32(xb), x


@pytest.mark.parametrize("n,k", [(9728, 2560), (8224, 2560), (200, 192), (2560, 9728), (32, 64), (1, 64)])
def test_repack_bytes_match_oracle(cuda_lib, dev, n, k):
    from skinny_mlx_b200.qmm import repack_for_skinny

    (packed, s, b), (tw, ts, tb) = make_weight(n, k, 1, dev)
    sw = repack_for_skinny(tw, ts, tb)
    torch.cuda.synchronize()
    got = sw.w_tc.cpu().numpy()
    assert np.array_equal(got, quant.repack_tc(packed, s, b))


@pytest.mark.parametrize("m", [1, 2, 4, 6, 8, 12, 16])
def test_qmm_config1_every_m(cuda_lib, dev, m):
    """x [M, 2560] ~N(0,1), W [9728, 2560] ~N(0, 0.02)."""
    from skinny_mlx_b200.qmm import repack_for_skinny, skinny_qmm, device_errors

    (packed, s, b), (tw, ts, tb) = make_weight(9728, 2560, 0, dev)
    sw = repack_for_skinny(tw, ts, tb)
    xf, x = make_x(m, 2560, 100 + m, dev)
    y = skinny_qmm(x, sw).float().cpu().numpy()
    ref = quant.qmm_ref(xf, packed, s, b)
    err = quant.rel_err(ref, y)
    assert err <= TOL and err <= TIGHT, err
    assert device_errors(dev) == 0


def test_qmm_golden_fixture(cuda_lib, dev):
    from skinny_mlx_b200.qmm import repack_for_skinny, skinny_qmm

    d = np.load(golden("qmm_small.npz"))
    tw = torch.from_numpy(d["packed"].view(np.int32)).to(dev)
    ts = torch.from_numpy(d["s_bits"].view(np.int16)).view(torch.bfloat16).to(dev)
    tb = torch.from_numpy(d["b_bits"].view(np.int16)).view(torch.bfloat16).to(dev)
    sw = repack_for_skinny(tw, ts, tb)
    for m in (1, 3, 8, 16):
        x = torch.from_numpy(d[f"x{m}"].view(np.int16)).view(torch.bfloat16).to(dev)
        y = skinny_qmm(x, sw).float().cpu().numpy()
        assert quant.rel_err(d[f"y{m}"], y) <= TIGHT


@pytest.mark.parametrize("n,k,m", [(8224, 2560, 8), (2560, 4096, 8), (2560, 2048, 16), (2560, 9728, 4),
                                   (200, 192, 3), (32, 64, 1), (1, 64, 16), (384, 25600, 8),
                                   (151936 // 8, 2560, 8)])
def test_qmm_shapes_and_tails(cuda_lib, dev, n, k, m):
    from skinny_mlx_b200.qmm import repack_for_skinny, skinny_qmm

    (packed, s, b), (tw, ts, tb) = make_weight(n, k, n + k, dev)
    sw = repack_for_skinny(tw, ts, tb)
    xf, x = make_x(m, k, 7, dev)
    y = skinny_qmm(x, sw).float().cpu().numpy()
    assert quant.rel_err(quant.qmm_ref(xf, packed, s, b), y) <= TIGHT


def test_config_for_is_the_launch_and_output_dtype_follows_x(cuda_lib, dev):
    """config_for (the reference's (RF, SK) heuristic, skinny_mlx/qmm.py:118) reports the launch
    the library makes: token columns by M, a K-split per tile for matrices with fewer tiles than
    SMs (S CTAs per tile, S <= 8) and the persistent stream-K grid (split 0) for larger ones.
    skinny_qmm and qmm return x's dtype (skinny_mlx/qmm.py:135,151)."""
    from skinny_mlx_b200.qmm import config_for, qmm, repack_for_skinny, skinny_qmm

    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    for m, cols in ((1, 2), (2, 2), (3, 4), (4, 4), (6, 8), (8, 8), (12, 16), (16, 16)):
        assert config_for(m, 2560)[0] == cols
    for n, k in ((9728, 2560), (2560, 9728), (5120, 2560), (2560, 2048)):
        tiles = (n + 127) // 128
        _, split = config_for(8, k, n)
        assert 1 <= split <= min(8, max(1, sms // tiles)), (n, k, split)
    assert config_for(8, 2560, 151936)[1] == 0  # more tiles than SMs: stream-K
    with pytest.raises(Exception):
        config_for(17, 2560)
    (packed, s, b), (tw, ts, tb) = make_weight(1024, 1024, 9, dev)
    sw = repack_for_skinny(tw, ts, tb)
    xf, x = make_x(8, 1024, 10, dev)
    ref = quant.qmm_ref(xf, packed, s, b)
    for dt in (torch.float16, torch.float32):
        y = skinny_qmm(x.to(dt), sw)
        assert y.dtype == dt
        assert quant.rel_err(ref, y.float().cpu().numpy()) <= TIGHT
        y2 = qmm(x.to(dt), tw, ts, tb)
        assert y2.dtype == dt
        assert torch.equal(y2, y)


def test_qmm_token_count_invariance(cuda_lib, dev):
    """Row t of a 16-token call equals a 1-token call on x[t], bit for bit (the stream-K split
    and the reduction order do not depend on M), so verify and greedy logits agree exactly."""
    from skinny_mlx_b200.qmm import repack_for_skinny, skinny_qmm

    _, (tw, ts, tb) = make_weight(9728, 2560, 2, dev)
    sw = repack_for_skinny(tw, ts, tb)
    _, x = make_x(16, 2560, 3, dev)
    full = skinny_qmm(x, sw)
    for m in (1, 3, 5, 8, 9, 13):
        part = skinny_qmm(x[:m].clone(), sw)
        assert torch.equal(part, full[:m])
    for t in (0, 7, 15):
        one = skinny_qmm(x[t:t + 1].clone(), sw)
        assert torch.equal(one[0], full[t])


def test_qmm_repeatable_and_workspace_reset(cuda_lib, dev):
    from skinny_mlx_b200.qmm import repack_for_skinny, skinny_qmm, device_errors

    _, (tw, ts, tb) = make_weight(4096, 2560, 4, dev)
    sw = repack_for_skinny(tw, ts, tb)
    _, x = make_x(8, 2560, 5, dev)
    a = skinny_qmm(x, sw)
    for _ in range(5):
        assert torch.equal(skinny_qmm(x, sw), a)
    assert device_errors(dev) == 0


def test_qmm_mlx_style_entry_and_chunking(cuda_lib, dev):
    """qmm(x, w_packed, scales, biases) on MLX packs; M > 16 runs in 16-token chunks."""
    from skinny_mlx_b200.qmm import qmm

    (packed, s, b), (tw, ts, tb) = make_weight(512, 640, 12, dev)
    xf, x = make_x(40, 640, 13, dev)
    y = qmm(x.reshape(2, 20, 640), tw, ts, tb, group_size=64, bits=4)
    assert y.shape == (2, 20, 512)
    ref = quant.qmm_ref(xf, packed, s, b)
    assert quant.rel_err(ref, y.reshape(40, 512).float().cpu().numpy()) <= TIGHT
    with pytest.raises(ValueError):
        qmm(x, tw, ts, tb, group_size=32)


def test_qmm_argument_errors(cuda_lib, dev):
    from skinny_mlx_b200 import _lib

    L = _lib.lib()
    x = torch.zeros(17, 128, dtype=torch.bfloat16, device=dev)
    w = torch.zeros(L.skinny_repack_bytes(128, 128), dtype=torch.uint8, device=dev)
    out = torch.zeros(17, 128, dtype=torch.bfloat16, device=dev)
    ws = torch.zeros(L.skinny_qmm_workspace_bytes(128, 128), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    args = lambda m, k, xp=x.data_ptr(), wsb=ws.numel(): (xp, k, w.data_ptr(), out.data_ptr(), 128, m, 128, k,
                                                         ws.data_ptr(), wsb, st)
    assert L.skinny_qmm_w4g64(*args(17, 128)) == -3
    assert L.skinny_qmm_w4g64(*args(0, 128)) == -3
    assert L.skinny_qmm_w4g64(*args(4, 100)) == -2
    assert L.skinny_qmm_w4g64(*args(4, 128, xp=x.data_ptr() + 2)) == -4
    assert L.skinny_qmm_w4g64(*args(4, 128, wsb=16)) == -5
    assert L.skinny_qmm_w4g64(*args(4, 128)) == 0
    torch.cuda.synchronize()


@pytest.mark.parametrize("m", [1, 8, 16])
def test_qmm_grouped_matches_single_calls(cuda_lib, dev, m):
    """One grouped launch over matrices of different shapes and inputs matches the single-call
    results within bf16 rounding (the stream-K split points differ, so the f32 summation order of a
    straddling tile differs) and is itself deterministic and token-count invariant."""
    from skinny_mlx_b200.qmm import repack_for_skinny, skinny_qmm, skinny_qmm_grouped, device_errors

    shapes = [(5120, 2560), (2560, 4096), (8224, 2560), (2560, 2048), (19456 // 4, 2560), (2560, 9728),
              (200, 192), (1, 64)]
    ws, xs, refs = [], [], []
    xcache = {}
    for i, (n, k) in enumerate(shapes):
        (packed, s, b), (tw, ts, tb) = make_weight(n, k, 50 + i, dev)
        ws.append(repack_for_skinny(tw, ts, tb))
        if k not in xcache:
            xcache[k] = make_x(m, k, 60 + k, dev)
        xf, x = xcache[k]
        xs.append(x)
        refs.append(quant.qmm_ref(xf, packed, s, b))
    outs = skinny_qmm_grouped(xs, ws)
    again = skinny_qmm_grouped(xs, ws)
    one_token = skinny_qmm_grouped([x[:1].clone() for x in xs], ws)
    for o, o2, o1, x, w, ref in zip(outs, again, one_token, xs, ws, refs):
        assert torch.equal(o, o2)
        assert torch.equal(o1[0], o[0])
        single = skinny_qmm(x, w).float().cpu().numpy()
        assert quant.rel_err(single, o.float().cpu().numpy()) <= TIGHT
        assert quant.rel_err(ref, o.float().cpu().numpy()) <= TIGHT
    assert device_errors(dev) == 0


def test_dequant_and_many_token_path(cuda_lib, dev):
    """skinny_dequant_w4g64 gives the MLX dequantisation bit for bit (bf16 of q * s + b), and
    skinny_qmm from PREFILL_TOKENS tokens (dequantise + dense GEMM) agrees with the f32 reference
    and with the token-streaming kernel within the bf16 tolerance."""
    import ctypes

    from skinny_mlx_b200.qmm import PREFILL_TOKENS, dequantize, quantize, repack_for_skinny, skinny_qmm

    torch.manual_seed(7)
    N, K = 8224, 1024  # a partial last row tile
    wp, s, b = quantize(torch.randn(N, K, device=dev) * 0.02)
    sw = repack_for_skinny(wp, s, b)
    wd = torch.empty(N, K, dtype=torch.bfloat16, device=dev)
    assert cuda_lib.skinny_dequant_w4g64(ctypes.c_void_p(sw.w_tc.data_ptr()), N, K, ctypes.c_void_p(wd.data_ptr()), K,
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    ref_w = dequantize(wp, s, b)
    assert torch.equal(wd, ref_w.to(torch.bfloat16))
    m = PREFILL_TOKENS + 8
    x = torch.randn(m, K, device=dev).to(torch.bfloat16)
    y = skinny_qmm(x, sw).float()
    ref = x.float() @ ref_w.t()
    assert ((y - ref).abs().max() / ref.abs().max()).item() <= 1e-2
    small = torch.cat([skinny_qmm(x[i:i + 16], sw) for i in range(0, m, 16)]).float()
    assert ((y - small).abs().max() / small.abs().max()).item() <= 1e-2
