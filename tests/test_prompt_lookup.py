"""CPU test: the prompt-lookup drafter's indexed search proposes what a direct scan of the
context (the rule of skinny_mlx/spec.py:40-47: the latest earlier occurrence of the trailing
n-gram, longest n first, then the tokens that followed it) proposes."""

import random

import torch

from skinny_mlx_b200.spec import PromptLookupDrafter


def _scan(ctx, ngram, k):
    for n in range(ngram, 0, -1):
        tail = ctx[-n:]
        for start in range(len(ctx) - n - 1, -1, -1):
            if ctx[start:start + n] == tail:
                return ctx[start + n:start + n + k]
    return []


def test_indexed_lookup_equals_scan():
    rng = random.Random(0)
    for trial in range(40):
        vocab = rng.choice([3, 5, 12, 50])
        ngram = rng.choice([1, 2, 3, 4])
        prompt = [rng.randrange(vocab) for _ in range(rng.randrange(0, 30))]
        d = PromptLookupDrafter(ngram, device="cpu")
        first = rng.randrange(vocab)
        d.begin(prompt, None, first)
        ctx = prompt + [first]
        for step in range(25):
            k = rng.choice([1, 2, 3, 5])
            got = d.draft(k).tolist()
            assert got == _scan(ctx, ngram, k), (trial, step, ctx, got)
            new = [rng.randrange(vocab) for _ in range(rng.randrange(1, 4))]
            d.update(None, new)
            ctx += new
    assert d.draft(2).dtype == torch.int32
