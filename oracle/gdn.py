"""TEST INFRASTRUCTURE ONLY -- CPU restatement of the Gated DeltaNet recurrence and of the
reference's replay-free rollback.

Recurrence (mlx_lm's gated_delta_update, restated by the reference in bench/reversal_check.py:21-25
as S_{t+1} = g_t S_t (I - b_t k_t k_t^T) + b_t v_t k_t^T), per value head with S [Dv, Dk]:
    S <- g S;  S <- S + beta (v - S k) k^T;  y = S q
Rollback (skinny_mlx/rollback.py:58-73): after a verify of `fed` tokens keeping `keep`, the state
is the one after token keep-1 (the reference re-runs the recurrence over the kept prefix from the
pre-verify state), the conv window is rows [keep, keep + W) of the recorded conv input, and
attention caches are trimmed by fed - keep.
"""

from __future__ import annotations

import numpy as np


def recurrent(q, k, v, g, beta, state):
    """q, k [T, Hk, Dk]; v [T, Hv, Dv]; g, beta [T, Hv]; state [Hv, Dv, Dk] -> (y [T, Hv, Dv],
    final state, states after every token [T, Hv, Dv, Dk]), float64."""
    q, k, v, g, beta = (np.asarray(a, np.float64) for a in (q, k, v, g, beta))
    S = np.array(state, np.float64)
    T, Hk, _ = q.shape
    Hv = v.shape[1]
    rep = Hv // Hk
    y = np.zeros((T, Hv, v.shape[2]))
    states = np.zeros((T,) + S.shape)
    for t in range(T):
        kt = np.repeat(k[t], rep, axis=0)
        qt = np.repeat(q[t], rep, axis=0)
        S = g[t][:, None, None] * S
        sk = np.einsum("hvk,hk->hv", S, kt)
        S = S + np.einsum("hv,hk->hvk", beta[t][:, None] * (v[t] - sk), kt)
        y[t] = np.einsum("hvk,hk->hv", S, qt)
        states[t] = S
    return y, S, states


def rollback(states_after, conv_full, keep: int, fed: int, W: int):
    """The state and conv window a rollback to `keep` of `fed` tokens leaves."""
    assert 1 <= keep <= fed
    return states_after[keep - 1], np.asarray(conv_full)[keep: keep + W]
