"""The decode loops against the reference's own loops.

tests/golden/spec_streams.json holds token streams produced by the reference's own Python --
skinny_mlx/spec.py `greedy` / `speculative` (with its `MTPDrafter` and `PromptLookupDrafter`) and
skinny_mlx/rollback.py `HybridRollback` -- run over the float64 oracle model (oracle/model.py) of
the seeded small hybrid model (tests/golden/make_golden.py).  Here this repository's loops
(skinny_mlx_b200.spec) must reproduce those streams token for token, except at a checked
near-tie of the reference run (top1 - top2 within 2 bf16 ulps), after which the runs may
legitimately differ: on the CPU (torch module path, host acceptance and rollback) and on the GPU
(patched module path, the fused step eagerly and replayed from CUDA graphs, device acceptance,
checkpoint-select rollback, the eager and graphed MTP drafters, prompt lookup).
"""

import json

import numpy as np
import pytest
import torch

from conftest import golden
from oracle.checks import stream_matches

G = json.loads(golden("spec_streams.json").read_text())
PROMPT, N = G["prompt"], G["tokens"]


def _model(dev):
    from skinny_mlx_b200.model import SMALL, HybridModel

    return HybridModel(SMALL, seed=0, device=dev, init_device="cpu")


def _check(name, got, ref=None, gaps=None, steps=None, st=None):
    ref = G["greedy"] if ref is None else ref
    gaps = G["gaps"] if gaps is None else gaps
    ok, j = stream_matches(ref, got, gaps)
    assert ok, (name, j, ref, got)
    if j is None and steps is not None and st is not None:
        assert st["steps"] == steps, (name, st["steps"], steps)  # same acceptance pattern as the reference
    return j


def test_fixture_is_self_consistent():
    """Every reference speculative run reproduced the reference greedy stream exactly."""
    for name, run in G["runs"].items():
        ref = G["greedy_repeat"] if run.get("prompt") == "repeat" else G["greedy"]
        assert run["tokens"] == ref, name
    assert len(G["greedy"]) == len(G["gaps"]) == N


def test_oracle_greedy_reproduces_the_fixture():
    """The oracle model driven by a plain greedy loop gives the stream the reference's loop gave
    over it (the fixture is a function of the oracle and the committed seeds)."""
    from oracle import model as om

    m = om.HybridModel(om.weights_from_torch(_model("cpu")))
    cache = m.make_cache()
    logits = m(np.array([PROMPT]), cache)
    out = []
    for _ in range(N):
        y = int(np.argmax(logits[0, -1]))
        out.append(y)
        logits = m(np.array([[y]]), cache)
    assert out == G["greedy"]


def test_cpu_module_loops_match_reference_streams():
    from skinny_mlx_b200.spec import PromptLookupDrafter, greedy, speculative
    from test_model_patch import ReplayDrafter

    m = _model("cpu")
    _check("greedy", greedy(m, PROMPT, N))
    for name, bad in (("scripted_k2_bad3", 3), ("scripted_k3_bad2", 2), ("scripted_k4_bad5", 5)):
        run = G["runs"][name]
        d = ReplayDrafter(G["greedy"], bad=bad)
        d.device = "cpu"
        st = {}
        _check(name, speculative(m, PROMPT, N, d, run["k"], st), steps=run["steps"], st=st)
    rep = G["repeat_prompt"]
    st = {}
    _check("prompt_lookup", speculative(m, rep, N, PromptLookupDrafter(3, device="cpu"), 3, st), G["greedy_repeat"],
           G["gaps_repeat"])


@pytest.mark.gpu
def test_gpu_loops_match_reference_streams(cuda_lib, dev):
    from skinny_mlx_b200.fused import FusedStep, GraphedStep
    from skinny_mlx_b200.mtp import MTPHead
    from skinny_mlx_b200.patch import patch_model
    from skinny_mlx_b200.spec import GraphedMTPDrafter, MTPDrafter, PromptLookupDrafter, greedy, speculative
    from test_model_patch import ReplayDrafter

    m = _model(dev)
    head = MTPHead(m, seed=13, init_device="cpu")
    patch_model(m)
    patch_model(head)
    f = FusedStep(m)
    gs = GraphedStep(f)
    cache = gs.make_cache()
    _check("greedy patched module path", greedy(m, PROMPT, N))
    _check("greedy fused", greedy(f, PROMPT, N))
    _check("greedy graphed", greedy(gs, PROMPT, N, cache=cache))
    for name, bad in (("scripted_k2_bad3", 3), ("scripted_k3_bad2", 2), ("scripted_k4_bad5", 5)):
        run = G["runs"][name]
        for label, model, kw in (("fused", f, {}), ("graphed", gs, {"cache": cache})):
            d = ReplayDrafter(G["greedy"], bad=bad)
            d.device = dev
            st = {}
            _check(f"{name} {label}", speculative(model, PROMPT, N, d, run["k"], st, **kw), steps=run["steps"], st=st)
    for label, d in (("mtp eager", MTPDrafter(m, head, vocab=None)),
                     ("mtp graphed", GraphedMTPDrafter(m, head, vocab=None))):
        _check(label, speculative(gs, PROMPT, N, d, 2, cache=cache))
    torch.cuda.synchronize()
    rep = G["repeat_prompt"]
    _check("prompt_lookup graphed", speculative(gs, rep, N, PromptLookupDrafter(3), 3, cache=cache),
           G["greedy_repeat"], G["gaps_repeat"])
    from skinny_mlx_b200.qmm import device_errors

    assert device_errors(dev) == 0


@pytest.mark.gpu
def test_mtp_head_matches_oracle(cuda_lib, dev):
    """The MTP draft head (skinny_mlx/mtp.py:64-67) on the GPU -- unpatched module forward,
    patched module forward and the fused kernels (FusedMTPHead) -- against the float64 oracle
    head on the same weights: a 20-token prompt, then draft steps of 1, 3 and 1 tokens on the
    head's KV cache."""
    from oracle import model as om
    from oracle.checks import rel_err
    from skinny_mlx_b200.mtp import FusedMTPHead, MTPHead
    from skinny_mlx_b200.patch import patch_model

    m = _model(dev)
    head = MTPHead(m, seed=13, init_device="cpu")
    oh = om.MTPHead(om.head_weights_from_torch(head))
    g = torch.Generator(device="cpu").manual_seed(3)
    ids = torch.randint(0, m.cfg.vocab, (25,), generator=g)
    emb = m.embed_tokens(ids.to(dev))
    hid = (torch.randn(25, m.cfg.hidden, generator=g) * 2).to(torch.bfloat16).to(dev)
    spans = ((0, 20), (20, 21), (21, 24), (24, 25))
    oc = om.KVCache()
    ref = [oh(emb[a:b].float().cpu().numpy()[None], hid[a:b].float().cpu().numpy()[None], oc)[0] for a, b in spans]
    c0 = head.make_cache(64)
    unpatched = [head(emb[a:b], hid[a:b], c0).float().cpu().numpy() for a, b in spans]
    patch_model(head)
    fused = FusedMTPHead(head)
    c1, c2 = head.make_cache(64), fused.make_cache(64)
    patched = [head(emb[a:b], hid[a:b], c1).float().cpu().numpy() for a, b in spans]
    fz = [fused(emb[a:b], hid[a:b], c2).float().cpu().numpy().copy() for a, b in spans]
    for i, (a, b) in enumerate(spans):
        for label, got in (("unpatched", unpatched[i]), ("patched", patched[i]), ("fused", fz[i])):
            err = rel_err(ref[i], got)
            assert err <= 1.5e-2, (label, a, b, err)
    assert oc.offset == c1.length == c2.length == 25


def test_cpu_mtp_head_matches_oracle():
    """The torch MTP head's module forward on the CPU against the float64 oracle head."""
    from oracle import model as om
    from oracle.checks import rel_err
    from skinny_mlx_b200.mtp import MTPHead

    m = _model("cpu")
    head = MTPHead(m, seed=13, init_device="cpu")
    oh = om.MTPHead(om.head_weights_from_torch(head))
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, m.cfg.vocab, (24,), generator=g)
    emb = m.embed_tokens(ids)
    hid = (torch.randn(24, m.cfg.hidden, generator=g) * 2).to(torch.bfloat16)
    oc, c = om.KVCache(), head.make_cache(64)
    for a, b in ((0, 20), (20, 21), (21, 24)):
        ref = oh(emb[a:b].float().numpy()[None], hid[a:b].float().numpy()[None], oc)[0]
        assert rel_err(ref, head(emb[a:b], hid[a:b], c).float().numpy()) <= 1.5e-2


def _tree_vs_paths(model, cache_factory, ids_prompt, nodes, parent, dev):
    """Logits of a tree verify, and for every node t the logits of a chain verify of t's path
    from the same cache (the reference for tree attention and the branch-aware recurrence)."""
    from skinny_mlx_b200.model import tree_paths
    from skinny_mlx_b200.spec import HybridRollback

    rb = HybridRollback()
    c = cache_factory()
    model(ids_prompt, c)
    rb.record(c)
    tree_logits = model(nodes, c, tree=parent)[1].float().cpu().clone()
    rows = []
    for t, path in enumerate(tree_paths(parent)):
        c = cache_factory()
        model(ids_prompt, c)
        rb.record(c)
        rows.append(model(nodes[path], c)[1][-1].float().cpu().clone())
    return tree_logits, torch.stack(rows)


def test_cpu_tree_verify_equals_path_verifies():
    """Module path on the CPU: each node's logits in a tree verify (tree mask, positions by depth,
    branch-aware conv and recurrence) equal those of verifying its ancestor path as a chain."""
    from oracle.checks import rel_err
    from skinny_mlx_b200.spec import chain_tree

    m = _model("cpu")
    parent = chain_tree(3)
    nodes = torch.tensor(G["greedy"][:7])
    got, want = _tree_vs_paths(m, m.make_cache, torch.tensor(PROMPT), nodes, parent, "cpu")
    assert rel_err(want.numpy(), got.numpy()) <= 1e-2


def test_cpu_tree_speculation_matches_reference_stream():
    """speculative_tree (top-2 chain trees from a scripted drafter; host acceptance and tree
    rollback) on the CPU module path reproduces the reference's greedy stream."""
    from skinny_mlx_b200.spec import ScriptedTreeDrafter, speculative_tree

    m = _model("cpu")
    for k, p in ((2, 0.5), (3, 0.7)):
        st = {}
        got = speculative_tree(m, PROMPT, N, ScriptedTreeDrafter(G["greedy"], p, m.cfg.vocab, "cpu", seed=k), k, st)
        _check(f"tree k{k}", got)
        assert st["accepted"] > 0


@pytest.mark.gpu
def test_gpu_tree_verify_equals_path_verifies(cuda_lib, dev):
    """Fused kernels (tree attention, branch-aware GDN mixer), eager and graph-replayed: each
    node's logits in one tree verify equal the logits of verifying its ancestor path as a chain
    on the same kernels (a token's arithmetic does not depend on its batch), and equal the torch
    module path's tree verify within the bf16 tolerance."""
    from oracle.checks import argmax_violations, rel_err
    from skinny_mlx_b200.fused import FusedStep, GraphedStep
    from skinny_mlx_b200.patch import patch_model
    from skinny_mlx_b200.spec import chain_tree

    m = _model(dev)
    patch_model(m)
    f = FusedStep(m)
    gs = GraphedStep(f)
    ids = torch.tensor(PROMPT, device=dev)
    for k, parent in ((3, chain_tree(3)), (2, [-1, 0, 0, 1, 1]), (7, [-1, 0, 1, 1, 0, 4, 2, 3, 7, 8, 6, 10, 11, 12, 9])):
        nodes = torch.tensor(G["greedy"][:len(parent)], device=dev)
        got, want = _tree_vs_paths(f, f.make_cache, ids, nodes, parent, dev)
        assert rel_err(want.numpy(), got.numpy()) <= 1.5e-2, k
        assert not argmax_violations(want.numpy(), got.numpy())
        gcache = gs.make_cache()
        got_g, _ = _tree_vs_paths(gs, lambda: (gcache.reset(), gcache)[1], ids, nodes, parent, dev)
        assert torch.equal(got_g, got)
        mod, _ = _tree_vs_paths(m, m.make_cache, ids, nodes, parent, dev)
        assert rel_err(mod.numpy(), got.numpy()) <= 1.5e-2
    from skinny_mlx_b200.qmm import device_errors

    assert device_errors(dev) == 0


@pytest.mark.gpu
def test_gpu_tree_speculation_matches_reference_stream(cuda_lib, dev):
    """speculative_tree on the fused step (eager and graph-replayed) with scripted top-2 trees and
    the MTP head's top-2 chain tree reproduces the reference's greedy stream."""
    from skinny_mlx_b200.fused import FusedStep, GraphedStep
    from skinny_mlx_b200.mtp import MTPHead
    from skinny_mlx_b200.patch import patch_model
    from skinny_mlx_b200.spec import MTPDrafter, ScriptedTreeDrafter, speculative_tree

    m = _model(dev)
    head = MTPHead(m, seed=13, init_device="cpu")
    patch_model(m)
    patch_model(head)
    f = FusedStep(m)
    gs = GraphedStep(f)
    cache = gs.make_cache()
    for k, p in ((2, 0.5), (3, 0.7), (4, 0.8)):
        for label, model, kw in (("fused", f, {}), ("graphed", gs, {"cache": cache})):
            st = {}
            d = ScriptedTreeDrafter(G["greedy"], p, m.cfg.vocab, dev, seed=k)
            _check(f"tree k{k} {label}", speculative_tree(model, PROMPT, N, d, k, st, **kw))
            assert st["accepted"] > 0
    _check("mtp tree", speculative_tree(gs, PROMPT, N, MTPDrafter(m, head, vocab=None), 3, cache=cache))
    from skinny_mlx_b200.qmm import device_errors

    assert device_errors(dev) == 0
