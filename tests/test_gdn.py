"""Gated DeltaNet recurrence with checkpoints and rollback: oracle checks on CPU (including against
transformers' own gated-delta reference) and the CUDA kernels against the oracle."""

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from oracle import quant


def _inputs(rng, T, Hv, Hk, d=128):
    q = rng.standard_normal((T, Hk, d))
    k = rng.standard_normal((T, Hk, d))
    q /= np.linalg.norm(q, axis=-1, keepdims=True) * np.sqrt(d)  # l2-normalised, scaled
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, Hv, d))
    g = np.exp(-rng.uniform(0.01, 2.0, (T, Hv)))
    beta = 1 / (1 + np.exp(-rng.standard_normal((T, Hv))))
    s0 = rng.standard_normal((Hv, d, d)) * 0.1
    bf = lambda a: quant.round_bf16(a.astype(np.float32))
    return bf(q), bf(k), bf(v), g.astype(np.float32), beta.astype(np.float32), s0.astype(np.float32)


def test_oracle_matches_transformers_reference():
    """transformers' torch_recurrent_gated_delta_rule (state [Dk, Dv]) computes the same rule."""
    from transformers.models.qwen3_next.modeling_qwen3_next import torch_recurrent_gated_delta_rule

    rng = np.random.default_rng(0)
    T, H, d = 5, 3, 128
    q, k, v, g, beta, s0 = _inputs(rng, T, H, H, d)
    y, sT, _ = ogdn.recurrent(q, k, v, g, beta, s0)
    tq = lambda a: torch.from_numpy(np.ascontiguousarray(a)).double()
    # transformers scales q by 1/sqrt(Dk) itself: pass q * sqrt(Dk); takes log-decay g
    out, fin = torch_recurrent_gated_delta_rule(
        tq(q * np.sqrt(d)).permute(1, 0, 2)[None].transpose(1, 2), tq(k).permute(1, 0, 2)[None].transpose(1, 2),
        tq(v).permute(1, 0, 2)[None].transpose(1, 2), tq(np.log(g))[None], tq(beta)[None],
        tq(s0).transpose(-1, -2)[None], True)
    # transformers computes in f32 whatever the input dtype
    assert np.abs(out[0].numpy() - y).max() <= 1e-5 * np.abs(y).max()
    assert np.abs(fin[0].transpose(-1, -2).numpy() - sT).max() <= 1e-5 * np.abs(sT).max()


def test_oracle_rollback_is_prefix_replay():
    """State after keeping `keep` tokens equals running the recurrence on those tokens only."""
    rng = np.random.default_rng(1)
    q, k, v, g, beta, s0 = _inputs(rng, 6, 4, 2)
    _, _, states = ogdn.recurrent(q, k, v, g, beta, s0)
    for keep in range(1, 7):
        _, s_keep, _ = ogdn.recurrent(q[:keep], k[:keep], v[:keep], g[:keep], beta[:keep], s0)
        conv_full = np.arange(3 + 6)
        st, cw = ogdn.rollback(states, conv_full, keep, 6, 3)
        assert np.allclose(st, s_keep) and list(cw) == [keep, keep + 1, keep + 2]


def _dev(a, dt, dev):
    if dt == torch.bfloat16:
        return torch.from_numpy(quant.f32_to_bf16_bits(a).view(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("T,Hv,Hk", [(1, 16, 16), (4, 16, 16), (8, 16, 16), (16, 16, 16), (5, 32, 16)])
def test_recurrent_matches_oracle(cuda_lib, dev, T, Hv, Hk):
    from skinny_mlx_b200.gdn import recurrent

    rng = np.random.default_rng(T * 100 + Hv)
    q, k, v, g, beta, s0 = _inputs(rng, T, Hv, Hk)
    y_ref, s_ref, st_ref = ogdn.recurrent(q, k, v, g, beta, s0)
    state = _dev(s0, torch.float32, dev)
    ckpt = torch.zeros(max(T - 1, 1), Hv, 128, 128, device=dev)
    y = recurrent(_dev(q, torch.bfloat16, dev), _dev(k, torch.bfloat16, dev), _dev(v, torch.bfloat16, dev),
                  _dev(g, torch.float32, dev), _dev(beta, torch.float32, dev), state, ckpt)
    torch.cuda.synchronize()
    assert np.abs(y.float().cpu().numpy() - y_ref).max() <= 1e-2 * np.abs(y_ref).max() + 1e-6
    assert np.allclose(state.cpu().numpy(), s_ref, rtol=1e-4, atol=1e-4)
    if T > 1:
        assert np.allclose(ckpt[:T - 1].cpu().numpy(), st_ref[:T - 1], rtol=1e-4, atol=1e-4)


@pytest.mark.gpu
def test_rollback_restores_prefix_state_and_conv(cuda_lib, dev):
    from skinny_mlx_b200.gdn import recurrent, rollback

    rng = np.random.default_rng(7)
    T, Hv, W, C, L = 6, 16, 3, 256, 3
    layers = []
    for l in range(L):
        q, k, v, g, beta, s0 = _inputs(rng, T, Hv, Hv)
        _, _, st_ref = ogdn.recurrent(q, k, v, g, beta, s0)
        state = _dev(s0, torch.float32, dev)
        ckpt = torch.zeros(T - 1, Hv, 128, 128, device=dev)
        recurrent(_dev(q, torch.bfloat16, dev), _dev(k, torch.bfloat16, dev), _dev(v, torch.bfloat16, dev),
                  _dev(g, torch.float32, dev), _dev(beta, torch.float32, dev), state, ckpt)
        conv_full = quant.round_bf16(rng.standard_normal((W + T, C)).astype(np.float32))
        conv = torch.zeros(W, C, dtype=torch.bfloat16, device=dev)
        layers.append((state, ckpt, conv, _dev(conv_full, torch.bfloat16, dev), st_ref, conv_full))
    for keep in (T, 4, 1):
        snap = [(s.clone(), c.clone()) for s, _, c, *_ in layers]
        rollback([x[0] for x in layers], [x[1] for x in layers], keep, T, [x[2] for x in layers],
                 [x[3] for x in layers])
        torch.cuda.synchronize()
        for (state, ckpt, conv, _, st_ref, conv_full) in layers:
            s_want, c_want = ogdn.rollback(st_ref, conv_full, keep, T, W)
            assert np.allclose(state.cpu().numpy(), s_want, rtol=1e-4, atol=1e-4)
            assert np.array_equal(conv.float().cpu().numpy(), c_want)
        for (s, c), x in zip(snap, layers):  # restore the after-verify state for the next keep
            x[0].copy_(s)


@pytest.mark.gpu
def test_rollback_tree_selects_node_state_and_path_window(cuda_lib, dev):
    """Tree rollback: every layer's state becomes its checkpoint of the accepted path's last node
    and its conv window the given conv_full rows, bit for bit, in one launch."""
    from skinny_mlx_b200.gdn import rollback_tree
    from skinny_mlx_b200.model import tree_rows

    torch.manual_seed(3)
    T, Hv, W, C, L = 7, 4, 3, 192, 2
    parent = [-1, 0, 0, 1, 1, 3, 3]
    states = [torch.randn(Hv, 128, 128, device=dev) for _ in range(L)]
    ckpts = [torch.randn(T, Hv, 128, 128, device=dev) for _ in range(L)]
    convs = [torch.zeros(W, C, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    fulls = [torch.randn(W + T, C, device=dev).to(torch.bfloat16) for _ in range(L)]
    for path in ([0], [0, 2], [0, 1, 4], [0, 1, 3, 6]):
        node = path[-1]
        rows = tree_rows(parent, node, W)[1:]  # the window after the node: its last W inputs
        assert rows == ([*range(W)] + [W + j for j in path])[-W:]
        rollback_tree(states, ckpts, node, rows, T, convs, fulls)
        torch.cuda.synchronize()
        for s, ck, cv, cf in zip(states, ckpts, convs, fulls):
            assert torch.equal(s, ck[node])
            assert torch.equal(cv, cf[rows])


@pytest.mark.gpu
def test_kv_compaction_moves_the_path_rows(cuda_lib, dev):
    """After a tree verify, rows L0 + path[j] of every K and V cache move to L0 + j (a moved row
    may be another move's source), one launch for all layers; other rows are untouched."""
    from skinny_mlx_b200.model import AttnCache, SMALL
    from skinny_mlx_b200.spec import HybridRollback

    torch.manual_seed(5)
    caches = [AttnCache(SMALL, 64, dev) for _ in range(3)]
    for c in caches:
        c.k.normal_()
        c.v.normal_()
    for path, fed in (([0, 2, 3], 7), ([0, 1, 4, 6], 7), ([0, 1, 2], 5), ([0], 3)):
        for c in caches:
            c.length = 20 + fed
        before = [(c.k.clone(), c.v.clone()) for c in caches]

        class C:
            layers = caches

        HybridRollback().rollback_tree(C(), fed, path)
        torch.cuda.synchronize()
        for c, (k0, v0) in zip(caches, before):
            n = len(path)
            assert c.length == 20 + n
            want_k, want_v = k0.clone(), v0.clone()
            want_k[20:20 + n] = k0[[20 + j for j in path]]
            want_v[20:20 + n] = v0[[20 + j for j in path]]
            assert torch.equal(c.k, want_k) and torch.equal(c.v, want_v)
