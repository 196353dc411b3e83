"""Full-size parity of the config-3 verify step on one B200.

The fused step (skinny_mlx_b200.fused.FusedStep: prep producers, prepared qmm, fused GDN and
attention mixers) on the full 32-layer hybrid model (hidden 2560, 16 query / 4 KV heads with a
gated query and 32-dim partial RoPE, 24 GDN layers of 16 heads x 128, vocab 151936) against the
UNPATCHED module forward of the same model: dequantised weights with f32 matmuls (the semantics of
mx.quantized_matmul), torch SDPA attention and the gated-delta recurrence in torch, so no kernel of
this library is on the reference side.  2048 cached tokens in every attention layer and live GDN
states, checkpoints recorded as in speculative verify.

Bar (north star): logits rel err max|d| / max|ref| <= 1.5e-2 and 100 % argmax agreement at every
M, a difference allowed only at a checked near-tie (top-1 vs the fused choice within 2 bf16 ulps).
"""

import ctypes

import pytest
import torch

from oracle.checks import argmax_violations, rel_err

pytestmark = pytest.mark.gpu

KV = 2048
MS = (1, 6, 8, 16)


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


@pytest.mark.parametrize("T", [1, 8, 16])
def test_attn_fused_hybrid_shape(cuda_lib, dev, T):
    """The config-3 attention layer (16 gated query heads, 4 KV heads, RoPE on the first 32 of
    128 dims) over 2048 cached tokens: the fused mixer against the module path's torch norm /
    RoPE / SDPA / gate on the same projection output and cache."""
    from skinny_mlx_b200.model import AttnCache, Attention, config3

    cfg = config3()
    gen = torch.Generator(device=dev).manual_seed(40 + T)
    a = Attention(cfg, gen, dev)
    a.q_norm.weight.normal_(generator=gen).mul_(0.1)
    a.k_norm.weight.normal_(generator=gen).mul_(0.1)
    D, nh, nkv = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    width = 2 * nh * D + 2 * nkv * D
    proj = (torch.randn(T, width, device=dev, generator=gen) * 2).to(torch.bfloat16)
    max_len = KV + 32
    ca, cb = AttnCache(cfg, max_len, dev), AttnCache(cfg, max_len, dev)
    ca.k[:KV] = torch.randn(KV, nkv, D, device=dev, generator=gen).to(torch.bfloat16)
    ca.v[:KV] = torch.randn(KV, nkv, D, device=dev, generator=gen).to(torch.bfloat16)
    cb.k.copy_(ca.k)
    cb.v.copy_(ca.v)
    ca.length = cb.length = KV
    q1, k1 = 2 * nh * D, 2 * nh * D + nkv * D
    ref = a.attend(proj[:, :q1], proj[:, q1:k1], proj[:, k1:], ca)
    half = cfg.rotary_dim // 2
    inv = (cfg.rope_theta ** (-torch.arange(0, half, device=dev, dtype=torch.float32) / half)).contiguous()
    ws = torch.zeros(int(cuda_lib.skinny_attn_workspace_bytes(16, nh, nkv, max_len)), dtype=torch.uint8, device=dev)
    xq = torch.empty(int(cuda_lib.skinny_xq_bytes(T, nh * D)), dtype=torch.uint8, device=dev)
    o = torch.empty(T, nh * D, dtype=torch.bfloat16, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = cuda_lib.skinny_attn_fused(_p(proj), proj.stride(0), _p(a.q_norm.weight), _p(a.k_norm.weight), _p(inv),
                                    cfg.rotary_dim, 1, ctypes.c_float(cfg.rms_eps), _p(cb.k), _p(cb.v), KV, None, T,
                                    nh, nkv, max_len, _p(ws), ws.numel(), _p(xq), _p(o), None, stream)
    assert st == 0
    torch.cuda.synchronize()
    err = rel_err(ref.float().cpu().numpy(), o.float().cpu().numpy())
    assert err <= 2e-2, err
    assert torch.equal(cb.v[:KV + T], ca.v[:KV + T])
    assert torch.equal(cb.k[:KV], ca.k[:KV])
    kd = (cb.k[KV:KV + T].float() - ca.k[KV:KV + T].float()).abs()
    assert (kd <= ca.k[KV:KV + T].float().abs() * 2 ** -7 + 1e-6).all()  # within one bf16 ulp


def _snapshot(cache):
    out = []
    for c in cache.layers:
        if hasattr(c, "k"):
            out.append(("attn", c.k.clone(), c.v.clone(), c.length))
        else:
            out.append(("gdn", c.conv.clone(), c.state.clone()))
    return out


def _restore(cache, snap):
    for c, s in zip(cache.layers, snap):
        if s[0] == "attn":
            c.k.copy_(s[1])
            c.v.copy_(s[2])
            c.length = s[3]
        else:
            c.conv.copy_(s[1])
            c.state.copy_(s[2])
            c.recording = True
            c.fed = 0


def test_config3_fused_step_matches_unpatched_full_model(cuda_lib, dev):
    from skinny_mlx_b200.fused import FusedStep
    from skinny_mlx_b200.model import AttnCache, GatedDeltaNet, HybridModel, QuantizedLinear, config3
    from skinny_mlx_b200.patch import patch_model

    cfg = config3()
    model = HybridModel(cfg, seed=11, device=dev)
    gen = torch.Generator(device=dev).manual_seed(5)
    cache = model.make_cache(max_len=KV + 32, max_verify=17)
    for c in cache.layers:
        if isinstance(c, AttnCache):
            c.k.normal_(generator=gen)
            c.v.normal_(generator=gen)
            c.length = KV
        else:
            c.state.normal_(generator=gen).mul_(0.05)
            c.conv.copy_((torch.randn(c.conv.shape, device=dev, generator=gen) * 0.5).to(torch.bfloat16))
    snap = _snapshot(cache)
    ids = {m: torch.randint(0, cfg.vocab, (m,), generator=gen, device=dev) for m in MS}

    refs, ref_states = {}, {}
    GatedDeltaNet.torch_recurrence = True
    try:
        for m in MS:
            _restore(cache, snap)
            refs[m] = model(ids[m], cache)[1].float().cpu()
            ref_states[m] = [c.state.clone() for c in cache.layers if not isinstance(c, AttnCache)]
    finally:
        GatedDeltaNet.torch_recurrence = False
    for mod in model.modules():  # drop the f32 dequantised copies of the reference path
        if isinstance(mod, QuantizedLinear):
            mod._deq = None
    model.embed_tokens.__dict__["_deq"] = None
    torch.cuda.empty_cache()

    patch_model(model)
    f = FusedStep(model)
    report = {}
    for m in MS:
        _restore(cache, snap)
        got = f(ids[m], cache)[1].float().cpu()
        torch.cuda.synchronize()
        err = rel_err(refs[m].numpy(), got.numpy())
        bad = argmax_violations(refs[m].numpy(), got.numpy())
        ties = int((refs[m].argmax(-1) != got.argmax(-1)).sum())
        states = [c.state for c in cache.layers if not isinstance(c, AttnCache)]
        s_err = max(rel_err(r.cpu().numpy(), g.cpu().numpy()) for r, g in zip(ref_states[m], states))
        report[m] = (round(err, 5), ties, round(s_err, 5))
        assert err <= 1.5e-2, (m, err)
        assert not bad, (m, bad)
        assert s_err <= 1e-2, (m, s_err)
        assert all(c.length == KV + m for c in cache.layers if isinstance(c, AttnCache))
    print("config-3 full-size parity (rel err, near-tie argmax differences, GDN state rel err):", report)
