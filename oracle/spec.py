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
