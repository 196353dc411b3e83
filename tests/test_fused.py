"""Fused step kernels (prep producers, prepared qmm, fused GDN mixer) and the fused verify step
against the module-by-module path and the oracle."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import quant
from oracle.checks import argmax_violations
from skinny_mlx_b200.model import SMALL, HybridModel

pytestmark = pytest.mark.gpu
PROMPT = [int(x) for x in np.random.default_rng(5).integers(0, SMALL.vocab, 24)]


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _bf16(a, dev):
    return torch.from_numpy(quant.f32_to_bf16_bits(np.asarray(a, np.float32)).view(np.int16)).view(torch.bfloat16).to(dev)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m", [1, 5, 8, 13])
def test_prep_plain_is_the_xprep_format(cuda_lib, dev, m):
    rng = np.random.default_rng(m)
    x = quant.round_bf16(rng.standard_normal((m, 640)).astype(np.float32) * 3)
    x[0, 64:128] = 0
    xq = torch.zeros(int(cuda_lib.skinny_xq_bytes(m, 640)), dtype=torch.uint8, device=dev)
    xt = _bf16(x, dev)
    assert cuda_lib.skinny_prep(2, _p(xt), 640, None, 0, 0, None, None, 0, None, ctypes.c_float(0), m, 640, _p(xq),
                                None, None, _stream()) == 0
    mpad = 8 if m <= 8 else 16
    assert np.array_equal(xq.cpu().numpy().reshape(10, -1), quant.xq_blocks(x, mpad))


@pytest.mark.parametrize("m", [1, 3, 8, 13, 16])
@pytest.mark.parametrize("K,I", [(2560, 9728), (512, 256)])
def test_swiglu_epilogue_equals_product_then_swiglu_prep(cuda_lib, dev, m, K, I):
    """skinny_qmm_w4g64_swiglu on an interleaved gate|up weight writes byte for byte the digits that
    the prepared product (same weight) followed by skinny_prep mode 1 on the de-interleaved bf16
    output writes.  (2560, 9728): the config-3 MLP, whole tiles and stream-K partial tiles;
    (512, 256): 32 units on 32 CTAs, every tile finished by the fix-up."""
    from skinny_mlx_b200.patch import _interleave64
    from skinny_mlx_b200.qmm import get_workspace, quantize, repack_for_skinny

    torch.manual_seed(7 * m + K)
    wq, sq, bq = quantize(torch.randn(2 * I, K, device=dev) * 0.03)
    g, u = (wq[:I], sq[:I], bq[:I]), (wq[I:], sq[I:], bq[I:])
    w = repack_for_skinny(*(_interleave64(a, b) for a, b in zip(g, u)))
    ws = get_workspace(dev, int(cuda_lib.skinny_qmm_workspace_bytes(2 * I, K)))
    x = (torch.randn(m, K, device=dev) * 2).to(torch.bfloat16)
    xq = torch.zeros(int(cuda_lib.skinny_xq_bytes(m, K)), dtype=torch.uint8, device=dev)
    assert cuda_lib.skinny_prep(2, _p(x), K, None, 0, 0, None, None, 0, None, ctypes.c_float(0), m, K, _p(xq), None,
                                None, _stream()) == 0
    got = torch.full((int(cuda_lib.skinny_xq_bytes(m, I)),), 0x5A, dtype=torch.uint8, device=dev)
    assert cuda_lib.skinny_qmm_w4g64_swiglu(_p(xq), _p(w.w_tc), _p(got), m, 2 * I, K, _p(ws), ws.numel(), _stream()) == 0
    gu = torch.empty(m, 2 * I, dtype=torch.bfloat16, device=dev)
    assert cuda_lib.skinny_qmm_w4g64_prepared(_p(xq), _p(w.w_tc), _p(gu), 2 * I, m, 2 * I, K, _p(ws), ws.numel(),
                                              None, 0, None, _stream()) == 0
    gu = gu.unflatten(-1, (-1, 2, 64)).transpose(1, 2).reshape(m, 2 * I).contiguous()  # [gate | up]
    ref = torch.full_like(got, 0x5A)
    assert cuda_lib.skinny_prep(1, _p(gu), 2 * I, None, 0, 0, None, None, 0, None, ctypes.c_float(0), m, I, _p(ref),
                                None, None, _stream()) == 0
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 0
    assert torch.equal(got, ref)
    # argument checks: N not a whole number of 128-row tiles; misaligned output
    assert cuda_lib.skinny_qmm_w4g64_swiglu(_p(xq), _p(w.w_tc), _p(got), m, 2 * I - 64, K, _p(ws), ws.numel(),
                                            _stream()) == -2
    assert cuda_lib.skinny_qmm_w4g64_swiglu(_p(xq), _p(w.w_tc), ctypes.c_void_p(got.data_ptr() + 4), m, 2 * I, K,
                                            _p(ws), ws.numel(), _stream()) == -4


@pytest.mark.parametrize("m", [1, 8, 16])
def test_prep_norm_and_swiglu_feed_the_prepared_qmm(cuda_lib, dev, m):
    from skinny_mlx_b200.qmm import get_workspace, quantize, repack_for_skinny, skinny_qmm

    torch.manual_seed(m)
    K, N = 1024, 768
    w = repack_for_skinny(*quantize(torch.randn(N, K, device=dev) * 0.02))
    ws = get_workspace(dev, int(cuda_lib.skinny_qmm_workspace_bytes(N, K)))
    x = torch.randn(m, K, device=dev).to(torch.bfloat16)
    d = torch.randn(m, K, device=dev).to(torch.bfloat16)
    gw = torch.randn(K, device=dev) * 0.1
    xq = torch.empty(int(cuda_lib.skinny_xq_bytes(m, K)), dtype=torch.uint8, device=dev)
    h = torch.empty_like(x)
    a = torch.empty(m, K, dtype=torch.bfloat16, device=dev)
    # outputs overlapping the inputs are refused (chunks of a row are written while others read it)
    assert cuda_lib.skinny_prep(0, _p(x), K, _p(d), K, 0, None, _p(x), K, _p(gw), ctypes.c_float(1e-6), m, K, _p(xq),
                                _p(a), None, _stream()) == -1
    assert cuda_lib.skinny_prep(0, _p(x), K, _p(d), K, 0, None, _p(h), K, _p(gw), ctypes.c_float(1e-6), m, K, _p(xq),
                                _p(d), None, _stream()) == -1
    assert cuda_lib.skinny_prep(0, _p(x), K, _p(d), K, 0, None, _p(h), K, _p(gw), ctypes.c_float(1e-6), m, K, _p(xq),
                                _p(a), None, _stream()) == 0
    y = torch.empty(m, N, dtype=torch.bfloat16, device=dev)
    assert cuda_lib.skinny_qmm_w4g64_prepared(_p(xq), _p(w.w_tc), _p(y), N, m, N, K, _p(ws), ws.numel(), None, 0, None,
                                                 _stream()) == 0
    href = (x.float() + d.float()).to(torch.bfloat16)
    assert torch.equal(h, href)
    hf = href.float()
    aref = (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + gw)).to(torch.bfloat16)
    assert (a.float() - aref.float()).abs().max().item() <= 2 ** -7 * aref.float().abs().max().item()
    yref = skinny_qmm(a, w)  # same activation through the unprepared path: bit-identical
    assert torch.equal(y, yref)
    # SwiGLU
    gu = torch.randn(m, 2 * K, device=dev).to(torch.bfloat16)
    assert cuda_lib.skinny_prep(1, _p(gu), 2 * K, None, 0, 0, None, None, 0, None, ctypes.c_float(0), m, K, _p(xq), None,
                                None, _stream()) == 0
    assert cuda_lib.skinny_qmm_w4g64_prepared(_p(xq), _p(w.w_tc), _p(y), N, m, N, K, _p(ws), ws.numel(), None, 0, None,
                                                 _stream()) == 0
    sref = (torch.nn.functional.silu(gu[:, :K].float()) * gu[:, K:].float()).to(torch.bfloat16)
    yref = skinny_qmm(sref, w).float()
    assert ((y.float() - yref).abs().max() / yref.abs().max()).item() <= 1e-2


@pytest.mark.parametrize("T", [1, 4, 8, 16])
def test_gdn_fused_matches_module_mixer(cuda_lib, dev, T):
    from skinny_mlx_b200.model import GDNCache

    m = HybridModel(SMALL, seed=0, device=dev)
    g = m.layers[0].linear_attn
    cfg = SMALL
    torch.manual_seed(T)
    proj = (torch.randn(T, 3 * cfg.gdn_value_dim + cfg.gdn_value_dim + 2 * cfg.gdn_v_heads, device=dev) * 0.5).to(torch.bfloat16)
    C = 3 * cfg.gdn_value_dim
    ca, cb = GDNCache(cfg, 17, dev), GDNCache(cfg, 17, dev)
    for c in (ca, cb):
        c.conv.copy_((torch.randn_like(c.conv.float()) * 0.5).to(torch.bfloat16))
        c.state.normal_().mul_(0.1)
        c.recording = True
    cb.conv.copy_(ca.conv)
    cb.state.copy_(ca.state)
    Hv = cfg.gdn_v_heads
    ref = g.mix(proj[:, :C], proj[:, C:C + cfg.gdn_value_dim], proj[:, C + cfg.gdn_value_dim:C + cfg.gdn_value_dim + Hv],
                proj[:, C + cfg.gdn_value_dim + Hv:], ca)
    xq = torch.empty(int(cuda_lib.skinny_xq_bytes(T, cfg.gdn_value_dim)), dtype=torch.uint8, device=dev)
    o = torch.empty(T, cfg.gdn_value_dim, dtype=torch.bfloat16, device=dev)
    errw = torch.zeros(1, dtype=torch.int32, device=dev)
    st = cuda_lib.skinny_gdn_fused(_p(proj), proj.stride(0), _p(cb.conv), _p(cb.conv_full), _p(g.conv_weight.float().contiguous()),
                                   _p(g.A_log), _p(g.dt_bias), _p(g.norm.weight), ctypes.c_float(cfg.rms_eps),
                                   _p(cb.state), _p(cb.ckpt), _p(xq), _p(o), T, Hv, cfg.gdn_k_heads, cfg.conv_kernel - 1,
                                   _p(errw), _stream())
    assert st == 0
    torch.cuda.synchronize()
    assert int(errw.item()) == 0
    rel = lambda a, b: ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()
    assert rel(o, ref) <= 2e-2, rel(o, ref)
    assert rel(cb.state, ca.state) <= 1e-2
    assert torch.equal(cb.conv, ca.conv)
    assert torch.equal(cb.conv_full[:3 + T], ca.conv_full[:3 + T])
    if T > 1:
        assert rel(cb.ckpt[:T - 1], ca.ckpt[:T - 1]) <= 1e-2


def test_gdn_fused_prefix_reproduces_checkpoints(cuda_lib, dev):
    """Rollback through the fused mixer: a verify of the first n of 12 tokens from the same state
    yields the 12-token verify's checkpoint n - 1 as its state, and the same outputs, bit for bit;
    so do n single-token steps (a token's results depend only on the tokens before it, not on
    how many tokens share the launch: speculative decoding then reproduces greedy decoding)."""
    from skinny_mlx_b200.model import GDNCache

    m = HybridModel(SMALL, seed=0, device=dev)
    g = m.layers[0].linear_attn
    cfg = SMALL
    torch.manual_seed(12)
    Tl, Hv = 12, cfg.gdn_v_heads
    proj = (torch.randn(Tl, 4 * cfg.gdn_value_dim + 2 * Hv, device=dev) * 0.5).to(torch.bfloat16)
    base = GDNCache(cfg, 17, dev)
    base.conv.copy_((torch.randn_like(base.conv.float()) * 0.5).to(torch.bfloat16))
    base.state.normal_().mul_(0.1)

    def run(T, c=None, row=0):
        if c is None:
            c = GDNCache(cfg, 17, dev)
            c.conv.copy_(base.conv)
            c.state.copy_(base.state)
        xq = torch.empty(int(cuda_lib.skinny_xq_bytes(T, cfg.gdn_value_dim)), dtype=torch.uint8, device=dev)
        o = torch.empty(T, cfg.gdn_value_dim, dtype=torch.bfloat16, device=dev)
        errw = torch.zeros(1, dtype=torch.int32, device=dev)
        assert cuda_lib.skinny_gdn_fused(_p(proj[row:]), proj.stride(0), _p(c.conv), _p(c.conv_full),
                                         _p(g.conv_weight.float().contiguous()), _p(g.A_log), _p(g.dt_bias),
                                         _p(g.norm.weight), ctypes.c_float(cfg.rms_eps), _p(c.state), _p(c.ckpt),
                                         _p(xq), _p(o), T, Hv, cfg.gdn_k_heads, cfg.conv_kernel - 1, _p(errw),
                                         _stream()) == 0
        torch.cuda.synchronize()
        assert int(errw.item()) == 0
        return c, o

    full, o_full = run(Tl)
    for n in (1, 3, 7, 11):
        c, o = run(n)
        assert torch.equal(c.state, full.ckpt[n - 1])
        assert torch.equal(o, o_full[:n])
    c = None
    for t in range(4):  # single-token steps
        c, o = run(1, c, t)
        assert torch.equal(c.state, full.ckpt[t])
        assert torch.equal(o, o_full[t:t + 1])


def test_fused_step_matches_patched_model_and_keeps_spec_exact(cuda_lib, dev):
    from skinny_mlx_b200.fused import FusedStep
    from skinny_mlx_b200.patch import patch_model
    from skinny_mlx_b200.spec import greedy, speculative
    from test_model_patch import ReplayDrafter, _exact_or_near_tie

    m = HybridModel(SMALL, seed=0, device=dev)
    patch_model(m)
    f = FusedStep(m)
    ids = torch.tensor(PROMPT[:16], device=dev)
    x = torch.tensor(PROMPT[16:24], device=dev)
    ca, cb = m.make_cache(), m.make_cache()
    m(ids, ca)
    m(ids, cb)
    ref = m(x, ca)[1].float()
    got = f(x, cb)[1].float()
    assert ((ref - got).abs().max() / ref.abs().max()).item() <= 1.5e-2
    assert not argmax_violations(ref.cpu().numpy(), got.cpu().numpy())  # M = 8: every row, or a near-tie
    gaps = []
    gref = greedy(f, PROMPT, 24, gaps)
    d = ReplayDrafter(gref)
    d.device = dev
    st = {}
    assert _exact_or_near_tie(gref, speculative(f, PROMPT, 24, d, 3, st), gaps)
    assert st["accepted"] > 0


@pytest.mark.parametrize("T,L0", [(1, 0), (1, 300), (5, 37), (8, 129), (16, 0), (16, 250)])
def test_attn_fused_matches_module_attention(cuda_lib, dev, T, L0):
    """Fused attention (norm, RoPE, KV append, split-KV softmax, gate, digits) against the module
    path (torch RMSNorm/RoPE + SDPA) on the same projection output and cache."""
    from skinny_mlx_b200.model import AttnCache

    cfg = SMALL
    m = HybridModel(cfg, seed=0, device=dev)
    a = m.layers[cfg.attn_every - 1].self_attn
    torch.manual_seed(T * 1000 + L0)
    D, nh, nkv = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    a.q_norm.weight.normal_().mul_(0.1)
    a.k_norm.weight.normal_().mul_(0.1)
    width = 2 * nh * D + 2 * nkv * D
    proj = (torch.randn(T, width + 8, device=dev) * 2).to(torch.bfloat16)[:, :width]  # ldp > width
    max_len = 400
    ca, cb = AttnCache(cfg, max_len, dev), AttnCache(cfg, max_len, dev)
    ca.k[:L0] = torch.randn(L0, nkv, D, device=dev).to(torch.bfloat16)
    ca.v[:L0] = torch.randn(L0, nkv, D, device=dev).to(torch.bfloat16)
    cb.k.copy_(ca.k)
    cb.v.copy_(ca.v)
    ca.length = cb.length = L0
    q1, k1 = 2 * nh * D, 2 * nh * D + nkv * D
    ref = a.attend(proj[:, :q1], proj[:, q1:k1], proj[:, k1:], ca)
    half = cfg.rotary_dim // 2
    inv = cfg.rope_theta ** (-torch.arange(0, half, device=dev, dtype=torch.float32) / half)
    ws = torch.zeros(int(cuda_lib.skinny_attn_workspace_bytes(T, nh, nkv, max_len)), dtype=torch.uint8, device=dev)
    xq = torch.empty(int(cuda_lib.skinny_xq_bytes(T, nh * D)), dtype=torch.uint8, device=dev)
    o = torch.empty(T, nh * D, dtype=torch.bfloat16, device=dev)
    len_dev = torch.tensor([L0], dtype=torch.int32, device=dev)
    for rep in range(2):  # twice (the workspace is reused); the second call reads L0 on the device
        cb.k[L0:].zero_()
        cb.v[L0:].zero_()
        st = cuda_lib.skinny_attn_fused(_p(proj), proj.stride(0), _p(a.q_norm.weight), _p(a.k_norm.weight), _p(inv),
                                        cfg.rotary_dim, 1, ctypes.c_float(cfg.rms_eps), _p(cb.k), _p(cb.v), L0,
                                        _p(len_dev) if rep == 1 else None, T, nh, nkv, max_len, _p(ws), ws.numel(),
                                        _p(xq), _p(o), None, _stream())
        assert st == 0
        torch.cuda.synchronize()
        err = ((o.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
        assert err <= 2e-2, err
        assert torch.equal(cb.v[:L0 + T], ca.v[:L0 + T])
        assert torch.equal(cb.k[:L0], ca.k[:L0])
        kd = (cb.k[L0:L0 + T].float() - ca.k[L0:L0 + T].float()).abs()
        assert (kd <= ca.k[L0:L0 + T].float().abs() * 2 ** -7 + 1e-6).all()  # within one bf16 ulp
        mpad = 8 if T <= 8 else 16
        got = xq.cpu().numpy().reshape(nh * D // 64, -1)
        assert np.array_equal(got, quant.xq_blocks(o.float().cpu().numpy(), mpad))


def test_graphed_step_equals_eager_and_keeps_spec_exact(cuda_lib, dev):
    """The CUDA-graph replay of the fused step (device-side cache lengths) reproduces the eager
    fused step bit for bit over a greedy run, and speculative decoding through it equals greedy."""
    from skinny_mlx_b200.fused import FusedStep, GraphedStep
    from skinny_mlx_b200.patch import patch_model
    from skinny_mlx_b200.spec import ScriptedDrafter, greedy, speculative
    from test_model_patch import _exact_or_near_tie

    m = HybridModel(SMALL, seed=0, device=dev)
    patch_model(m)
    f = FusedStep(m)
    gs = GraphedStep(f)
    gaps = []
    ref = greedy(f, PROMPT, 24, gaps)
    cache = gs.make_cache()
    assert greedy(gs, PROMPT, 24, cache=cache) == ref
    assert greedy(gs, PROMPT, 24, cache=cache) == ref  # same cache reset and replayed again
    for k, p in ((2, 0.8), (3, 0.6)):
        st = {}
        got = speculative(gs, PROMPT, 24, ScriptedDrafter(ref, p, SMALL.vocab, dev, seed=k), k, st, cache=cache)
        assert _exact_or_near_tie(ref, got, gaps)
        assert st["accepted"] > 0


def test_attn_fused_ungated_dense_shape(cuda_lib, dev):
    """The dense model's attention layout (no gate, RoPE on all 128 dims, 5 query heads per KV
    head, a 4096-token cache) against torch: zero-centred RMSNorm, rotate-half RoPE, causal GQA
    softmax attention in f32."""
    torch.manual_seed(1)
    T, nh, nkv, L0, D = 8, 40, 8, 4096, 128
    max_len = L0 + 32
    qn = (torch.randn(D, device=dev) * 0.1).contiguous()
    kn = (torch.randn(D, device=dev) * 0.1).contiguous()
    proj = torch.randn(T, (nh + 2 * nkv) * D, device=dev).to(torch.bfloat16)
    kc = torch.randn(max_len, nkv, D, device=dev).to(torch.bfloat16)
    vc = torch.randn(max_len, nkv, D, device=dev).to(torch.bfloat16)
    inv = (1e6 ** (-torch.arange(0, 64, device=dev, dtype=torch.float32) / 64)).contiguous()

    def norm(x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + w)).to(torch.bfloat16).float()

    def rope(x, pos):
        ang = pos.float()[:, None] * inv[None]
        c, s = ang.cos()[:, None, :], ang.sin()[:, None, :]
        x1, x2 = x[..., :64], x[..., 64:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)

    pos = torch.arange(L0, L0 + T, device=dev)
    q = rope(norm(proj[:, :nh * D].reshape(T, nh, D), qn), pos).to(torch.bfloat16).float()
    k_new = rope(norm(proj[:, nh * D:(nh + nkv) * D].reshape(T, nkv, D), kn), pos).to(torch.bfloat16)
    v_new = proj[:, (nh + nkv) * D:].reshape(T, nkv, D)
    kr, vr = kc.clone(), vc.clone()
    kr[L0:L0 + T], vr[L0:L0 + T] = k_new, v_new
    K = kr[:L0 + T].float().repeat_interleave(nh // nkv, 1)  # [L, nh, D]
    V = vr[:L0 + T].float().repeat_interleave(nh // nkv, 1)
    sc = torch.einsum("thd,lhd->thl", q, K) / D ** 0.5
    mask = pos[:, None] >= torch.arange(L0 + T, device=dev)[None, :]
    sc = sc.masked_fill(~mask[:, None, :], float("-inf"))
    ref = torch.einsum("thl,lhd->thd", sc.softmax(-1), V).reshape(T, nh * D)

    ws = torch.empty(int(cuda_lib.skinny_attn_workspace_bytes(16, nh, nkv, max_len)), dtype=torch.uint8, device=dev)
    xq = torch.empty(int(cuda_lib.skinny_xq_bytes(T, nh * D)), dtype=torch.uint8, device=dev)
    o = torch.empty(T, nh * D, dtype=torch.bfloat16, device=dev)
    st = cuda_lib.skinny_attn_fused(_p(proj), proj.stride(0), _p(qn), _p(kn), _p(inv), 128, 0, ctypes.c_float(1e-6),
                                    _p(kc), _p(vc), L0, None, T, nh, nkv, max_len, _p(ws), ws.numel(), _p(xq), _p(o),
                                    None, _stream())
    assert st == 0
    torch.cuda.synchronize()
    err = ((o.float() - ref).abs().max() / ref.abs().max()).item()
    assert err <= 2e-2, err
    assert torch.equal(vc[L0:L0 + T], v_new)
    assert ((kc[L0:L0 + T].float() - k_new.float()).abs() <= k_new.float().abs() * 2 ** -7 + 1e-6).all()


def test_fused_mtp_head_matches_module_head(cuda_lib, dev):
    """The MTP draft head on the fused kernels against its patched module forward: a 20-token
    prompt through the module path into both caches, then draft steps of 1, 3 and 1 tokens."""
    from skinny_mlx_b200.mtp import FusedMTPHead, MTPHead
    from skinny_mlx_b200.patch import patch_model

    m = HybridModel(SMALL, seed=0, device=dev)
    patch_model(m)
    head = MTPHead(m, seed=13)
    patch_model(head)
    fused = FusedMTPHead(head)
    ca, cb = head.make_cache(64), fused.make_cache(64)
    g = torch.Generator(device="cpu").manual_seed(3)
    ids = torch.randint(0, SMALL.vocab, (25,), generator=g).to(dev)
    hid = (torch.randn(25, SMALL.hidden, generator=g) * 2).to(torch.bfloat16).to(dev)
    emb = m.embed_tokens(ids)
    ref = head(emb[:20], hid[:20], ca)
    got = fused(emb[:20], hid[:20], cb)  # more than 16 tokens: the module forward
    assert torch.equal(ref, got)
    rel = lambda a, b: ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()
    for a, b in ((20, 21), (21, 24), (24, 25)):
        ref = head(emb[a:b], hid[a:b], ca)
        got = fused(emb[a:b], hid[a:b], cb).clone()
        assert rel(got, ref) <= 2e-2, (a, b, rel(got, ref))
        assert ca.length == cb.length == b


def test_embedding_gather_matches_module_lookup(cuda_lib, dev):
    """skinny_embed_w4g64 against the module embedding (dequantise then bf16), bit for bit, with
    repeated ids; an id outside the table gives a zero row."""
    m = HybridModel(SMALL, seed=0, device=dev)
    emb = m.embed_tokens
    V, H = emb.weight.shape[0], SMALL.hidden
    ids = torch.tensor([3, 0, V - 1, 3, 77, 1000 % V, 5, 6, 7], device=dev)
    out = torch.full((ids.numel() + 1, H), 7.0, dtype=torch.bfloat16, device=dev)
    ids_bad = torch.cat([ids, torch.tensor([V], device=dev)])
    assert cuda_lib.skinny_embed_w4g64(_p(ids_bad), ids_bad.numel(), _p(emb.weight), _p(emb.scales), _p(emb.biases), V,
                                       H, _p(out), H, _stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(out[:-1], emb(ids))
    assert torch.count_nonzero(out[-1]).item() == 0


def test_graphed_mtp_drafter_equals_eager_drafter(cuda_lib, dev):
    """The MTP drafter replayed from CUDA graphs proposes the same tokens as the eager drafter on
    the fused kernels through begin, draft and update steps, and speculative decoding with it
    reproduces greedy decoding."""
    from skinny_mlx_b200.fused import FusedStep, GraphedStep
    from skinny_mlx_b200.mtp import MTPHead
    from skinny_mlx_b200.patch import patch_model
    from skinny_mlx_b200.spec import GraphedMTPDrafter, MTPDrafter, greedy, speculative
    from test_model_patch import _exact_or_near_tie

    m = HybridModel(SMALL, seed=0, device=dev)
    patch_model(m)
    head = MTPHead(m, seed=13)
    patch_model(head)
    f = FusedStep(m)
    cache = f.make_cache()
    h, _ = f(torch.tensor(PROMPT, device=dev), cache)
    eager, graphed = MTPDrafter(m, head, vocab=None), GraphedMTPDrafter(m, head, vocab=None)
    for d in (eager, graphed):
        d.begin(PROMPT, h, 5)
    g = torch.Generator(device="cpu").manual_seed(1)
    for k, keep in ((2, 1), (3, 3), (2, 2), (3, 1)):
        a, b = eager.draft(k).clone(), graphed.draft(k).clone()
        assert torch.equal(a, b), (k, a, b)
        hk = (torch.randn(keep, SMALL.hidden, generator=g) * 2).to(torch.bfloat16).to(dev)
        new = torch.randint(0, SMALL.vocab, (keep,), generator=g).tolist()
        eager.update(hk, new)
        graphed.update(hk, new)
        assert eager.cache.length == graphed.cache.length
    gs = GraphedStep(f)
    gaps = []
    ref = greedy(f, PROMPT, 20, gaps)
    got = speculative(gs, PROMPT, 20, GraphedMTPDrafter(m, head, vocab=None), 2, cache=gs.make_cache())
    assert _exact_or_near_tie(ref, got, gaps)


def test_prompt_lookup_speculation_reproduces_greedy(cuda_lib, dev):
    """Speculative decoding with the model-free prompt-lookup drafter (drafts of any length,
    including none) through the graph-replayed fused step reproduces greedy decoding, on a
    prompt with repeats so that drafts are proposed."""
    from skinny_mlx_b200.fused import FusedStep, GraphedStep
    from skinny_mlx_b200.patch import patch_model
    from skinny_mlx_b200.spec import PromptLookupDrafter, greedy, speculative
    from test_model_patch import _exact_or_near_tie

    m = HybridModel(SMALL, seed=0, device=dev)
    patch_model(m)
    f = FusedStep(m)
    gs = GraphedStep(f)
    prompt = (PROMPT[:8] * 3)[:20]
    gaps = []
    ref = greedy(f, prompt, 24, gaps)
    st = {}
    got = speculative(gs, prompt, 24, PromptLookupDrafter(3), 3, st, cache=gs.make_cache())
    assert _exact_or_near_tie(ref, got, gaps)
    assert st["steps"] > 0
