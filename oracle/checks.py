"""TEST INFRASTRUCTURE ONLY -- the parity rules the tests and the smoke check apply.

BASELINE's bar for the verify path: relative error max|d| / max|ref| <= 1.5e-2 on bf16 outputs
(the reference's own metric, skinny_mlx/qmm.py:185), 100 % argmax agreement at M = 8, and greedy
output identical token for token except at checked bf16 near-ties: a disagreement is allowed only
where the reference's top-1 and the other side's choice are within 2 bf16 ulps of each other at
the top logit's magnitude (the reference prints the same gap, skinny_mlx/patch.py:136-142).
"""

from __future__ import annotations

import math

import numpy as np


def bf16_ulp(v: float) -> float:
    """Spacing of bf16 values at |v| (8 significant bits)."""
    return 2.0 ** (math.floor(math.log2(max(abs(float(v)), 1e-30))) - 7)


def rel_err(ref, got) -> float:
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(ref - got).max() / den) if den > 0 else float(np.abs(got).max())


def argmax_violations(ref, got, ulps: float = 2.0) -> list[tuple[int, float, float]]:
    """Rows whose argmax differs between `ref` and `got` ([M, V] logits) by more than a near-tie:
    (row, ref[top_ref] - ref[top_got], allowed gap).  Empty list = the contract holds."""
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    a_ref, a_got = ref.argmax(-1), got.argmax(-1)
    bad = []
    for i in np.nonzero(a_ref != a_got)[0].tolist():
        top = ref[i, a_ref[i]]
        gap = float(top - ref[i, a_got[i]])
        allowed = ulps * bf16_ulp(top)
        if gap > allowed:
            bad.append((i, gap, allowed))
    return bad


def top2_gap(logits_row) -> tuple[float, float]:
    """(top1 - top2, top1) of one row of logits."""
    r = np.sort(np.asarray(logits_row, np.float64))
    return float(r[-1] - r[-2]), float(r[-1])


def first_divergence(a, b):
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), None)


def stream_matches(ref, got, gaps, ulps: float = 2.0) -> tuple[bool, int | None]:
    """Token streams: identical, or the first difference sits at a near-tie of the reference run
    (gaps[j] = (top1 - top2, top1) of the logits that chose ref[j]); after a near-tie the two
    runs legitimately continue differently.  Returns (ok, first divergence or None)."""
    j = first_divergence(ref, got)
    if j is None:
        return len(ref) == len(got), None
    gap, top = gaps[j]
    return gap <= ulps * bf16_ulp(top), j
