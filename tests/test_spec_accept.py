"""Fused greedy acceptance (skinny_mlx/spec.py:136-147) against the CPU oracle."""

import numpy as np
import pytest
import torch

from oracle import quant, spec as ospec


def test_oracle_acceptance_rule():
    lg = np.full((4, 10), -1.0, np.float32)
    for i, t in enumerate([3, 5, 7, 9]):
        lg[i, t] = 2.0
    assert ospec.accept(lg, [3, 5, 1]) == (2, [3, 5, 7], [3, 5, 7, 9])
    assert ospec.accept(lg, [3, 5, 7]) == (3, [3, 5, 7, 9], [3, 5, 7, 9])
    assert ospec.accept(lg, [0, 5, 7]) == (0, [3], [3, 5, 7, 9])
    lg[0, 1] = 2.0  # tie between 1 and 3: first occurrence wins
    assert ospec.accept(lg, [1, 5, 7])[0] == 3
    assert ospec.accept(lg[:1], [])[1] == [1]
    lg[1, 8] = np.nan  # a NaN is above every number (numpy's argmax)
    assert ospec.accept(lg, [1, 8, 7]) == (3, [1, 8, 7, 9], [1, 8, 7, 9])


def test_oracle_tree_acceptance_rule():
    par = [-1, 0, 0, 1, 1, 3, 3]        # top-2 chain tree of depth 3
    tok = [9, 4, 5, 6, 7, 8, 1]
    lg = np.zeros((7, 10), np.float32)
    for i, t in enumerate([5, 6, 3, 8, 2, 4, 0]):  # node predictions
        lg[i, t] = 1.0
    # root predicts 5 -> node 2 (the sibling); node 2 has no children: stop, bonus = pred[2] = 3
    assert ospec.accept_tree(lg, tok, par) == (1, [5, 3], [0, 2])
    lg[0] = 0
    lg[0, 4] = 1.0                       # root -> node 1 (4); node 1 predicts 6 -> node 3; node 3 -> 8 -> node 5
    assert ospec.accept_tree(lg, tok, par) == (3, [4, 6, 8, 4], [0, 1, 3, 5])
    lg[0] = 0
    lg[0, 0] = 1.0                       # no child carries 0: nothing accepted
    assert ospec.accept_tree(lg, tok, par) == (0, [0], [0])
    chain = [-1, 0, 1, 2]
    lgc = np.zeros((4, 10), np.float32)
    for i, t in enumerate([3, 5, 7, 2]):
        lgc[i, t] = 1.0
    n, toks, _ = ospec.accept(lgc, [3, 5, 1])
    assert ospec.accept_tree(lgc, [0, 3, 5, 1], chain)[:2] == (n, toks)  # a chain tree is the chain rule


def _random_tree(rng, rows):
    return [-1] + [int(rng.integers(0, t)) for t in range(1, rows)]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,v", [(7, 151936), (9, 151936), (17, 32768), (1, 1000), (5, 8)])
def test_device_tree_acceptance_matches_oracle(cuda_lib, dev, rows, v):
    from skinny_mlx_b200.spec import accept_tree

    rng = np.random.default_rng(rows * 31 + v)
    for trial in range(6):
        par = _random_tree(rng, rows) if trial % 2 else ([-1] + [max(0, 2 * ((t + 1) // 2) - 3) for t in range(1, rows)])
        x = quant.round_bf16(rng.standard_normal((rows, v)).astype(np.float32))
        pred = ospec.argmax_rows(x)
        tok = [int(rng.integers(0, v))]
        for t in range(1, rows):  # about half of the nodes carry their parent's prediction
            tok.append(int(pred[par[t]]) if rng.random() < 0.5 else int(rng.integers(0, v)))
        want = ospec.accept_tree(x, tok, par)
        lg = torch.from_numpy(quant.f32_to_bf16_bits(x).view(np.int16)).view(torch.bfloat16).to(dev)
        got = accept_tree(lg, torch.tensor(tok, dtype=torch.int32, device=dev),
                          torch.tensor(par, dtype=torch.int32, device=dev))
        assert got == want, (par, tok, got, want)


def _case(rng, rows, v, n_match, tie=False):
    x = rng.standard_normal((rows, v)).astype(np.float32) * 3
    pred = rng.integers(0, v, rows)
    x[np.arange(rows), pred] = 20.0
    if tie:
        alt = (pred + 1 + rng.integers(0, v - 1, rows)) % v
        x[np.arange(rows), alt] = 20.0
    xb = quant.round_bf16(x)
    truth = ospec.argmax_rows(xb)
    draft = [int(truth[i]) if i < n_match else int((truth[i] + 1) % v) for i in range(rows - 1)]
    return xb, draft


@pytest.mark.gpu
@pytest.mark.parametrize("rows,v", [(4, 151936), (3, 151936), (9, 151936), (17, 151936), (1, 151936),
                                    (5, 1000), (2, 8), (16, 32768), (6, 8200)])
def test_device_acceptance_matches_oracle(cuda_lib, dev, rows, v):
    from skinny_mlx_b200.spec import accept, accept_device

    rng = np.random.default_rng(rows * 7919 + v)
    for n_match in sorted({0, (rows - 1) // 2, rows - 1}):
        for tie in (False, True):
            xb, draft = _case(rng, rows, v, n_match, tie)
            lg = torch.from_numpy(quant.f32_to_bf16_bits(xb).view(np.int16)).view(torch.bfloat16).to(dev)
            dr = torch.tensor(draft, dtype=torch.int32, device=dev)
            n, toks, pred = ospec.accept(xb, draft)
            got_n, got = accept(lg, dr)
            assert (got_n, got) == (n, toks)
            pr = torch.empty(rows, dtype=torch.int32, device=dev)
            r = accept_device(lg, dr, pred=pr)
            assert pr.cpu().tolist() == pred
            assert r.cpu().tolist()[n + 2:] == [-1] * (rows - 1 - n)


@pytest.mark.gpu
def test_device_acceptance_special_values(cuda_lib, dev):
    from skinny_mlx_b200.spec import accept

    v = 4096
    x = np.full((3, v), -np.inf, np.float32)
    x[0, 17] = 1.0
    x[1, :] = np.nan
    x[2, 4095] = -1e30
    x[2, :5] = np.nan
    lg = torch.from_numpy(quant.f32_to_bf16_bits(x).view(np.int16)).view(torch.bfloat16).to(dev)
    draft = [17, 0]
    n, toks, pred = ospec.accept(quant.bf16_bits_to_f32(quant.f32_to_bf16_bits(x)), draft)
    assert pred == [17, 0, 0]  # numpy's order: the first NaN of a row wins
    assert accept(lg, torch.tensor(draft, dtype=torch.int32, device=dev)) == (n, toks)
    x[2, :5] = -np.inf
    x[2, 100] = np.nan
    lg = torch.from_numpy(quant.f32_to_bf16_bits(x).view(np.int16)).view(torch.bfloat16).to(dev)
    n, toks, pred = ospec.accept(quant.bf16_bits_to_f32(quant.f32_to_bf16_bits(x)), draft)
    assert pred == [17, 0, 100]
    assert accept(lg, torch.tensor(draft, dtype=torch.int32, device=dev)) == (n, toks)
