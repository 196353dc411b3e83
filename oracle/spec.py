"""TEST INFRASTRUCTURE ONLY -- CPU restatement of the reference's greedy speculative acceptance.

skinny_mlx/spec.py:136-147 (speculative):
    pred = argmax(logits[0], axis=-1)                       # K+1 verified positions
    n = 0; while n < len(draft) and draft[n] == pred[n]: n += 1
    new = draft[:n] + [pred[n]]
numpy's argmax returns the first maximal index and treats NaN as larger than every number (the
first NaN of a row wins); the device kernel follows the same order.
"""

from __future__ import annotations

import numpy as np


def argmax_rows(logits: np.ndarray) -> np.ndarray:
    """Row argmax as numpy computes it: first occurrence of the maximum, a NaN above every number."""
    return np.argmax(np.asarray(logits, np.float64), axis=-1).astype(np.int64)


def accept(logits: np.ndarray, draft) -> tuple[int, list[int], list[int]]:
    """logits [K+1, V] (float values), draft K ids -> (n, emitted tokens, predictions)."""
    pred = [int(v) for v in argmax_rows(np.asarray(logits))]
    draft = [int(d) for d in draft]
    n = 0
    while n < len(draft) and draft[n] == pred[n]:
        n += 1
    return n, draft[:n] + [pred[n]], pred


def accept_tree(logits: np.ndarray, tokens, parent) -> tuple[int, list[int], list[int]]:
    """The tree form of the acceptance (the draft tree the reference proposes for flat verify,
    docs/flatspec-design.md:64-69): logits [M, V] of the M nodes (node 0 = the last emitted
    token), tokens [M], parent [M] (parent[0] = -1, parent[t] < t).  From the root, move to the
    first child (lowest index) whose token equals the current node's prediction while one
    exists.  Returns (n, the accepted tokens + [pred of the last node], the path 0, p1 .. pn)."""
    pred = [int(v) for v in argmax_rows(np.asarray(logits))]
    tokens = [int(t) for t in tokens]
    parent = [int(p) for p in parent]
    cur, path = 0, [0]
    if parent[0] == -1:
        while True:
            nxt = next((c for c in range(cur + 1, len(parent)) if parent[c] == cur and tokens[c] == pred[cur]), None)
            if nxt is None:
                break
            path.append(nxt)
            cur = nxt
    return len(path) - 1, [tokens[c] for c in path[1:]] + [pred[cur]], path
