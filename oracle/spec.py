"""TEST INFRASTRUCTURE ONLY -- CPU restatement of the reference's greedy speculative acceptance.

skinny_mlx/spec.py:136-147 (speculative):
    pred = argmax(logits[0], axis=-1)                       # K+1 verified positions
    n = 0; while n < len(draft) and draft[n] == pred[n]: n += 1
    new = draft[:n] + [pred[n]]
numpy's argmax returns the first maximal index, as MLX's does; NaN is treated here as never
winning (the device kernel's rule), which only matters for logits that contain NaN.
"""

from __future__ import annotations

import numpy as np


def argmax_rows(logits: np.ndarray) -> np.ndarray:
    """Row argmax, first occurrence of the maximum, NaN ignored (an all-NaN row gives 0)."""
    x = np.where(np.isnan(logits), -np.inf, logits.astype(np.float64))
    out = np.argmax(x, axis=-1)
    allnan = np.isnan(logits).all(axis=-1)
    out[allnan] = 0
    return out.astype(np.int64)


def accept(logits: np.ndarray, draft) -> tuple[int, list[int], list[int]]:
    """logits [K+1, V] (float values), draft K ids -> (n, emitted tokens, predictions)."""
    pred = [int(v) for v in argmax_rows(np.asarray(logits))]
    draft = [int(d) for d in draft]
    n = 0
    while n < len(draft) and draft[n] == pred[n]:
        n += 1
    return n, draft[:n] + [pred[n]], pred
