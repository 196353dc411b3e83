"""Gated DeltaNet verify recurrence with state checkpoints and replay-free rollback on B200
(the hooks of skinny_mlx/rollback.py:19-73: record during verify, roll back to the kept prefix).

`recurrent` runs the verify pass of one GDN layer and, given a checkpoint buffer, keeps the
state after every token but the last; `rollback` then restores the state after token keep-1 and
re-slices the conv window for every layer in one launch; `rollback_tree` does the same after a
tree verify (the state of the accepted path's last node, the window gathered along the path).
Attention KV caches need no device work for a chain: trimming them is a length update.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


def _stream(dev: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _p(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def recurrent(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
              state: torch.Tensor, ckpt: torch.Tensor | None = None, y: torch.Tensor | None = None) -> torch.Tensor:
    """q, k [T, Hk, 128] bf16; v [T, Hv, 128] bf16; g (decay), beta [T, Hv] f32; state [Hv, 128, 128]
    f32 (updated in place); ckpt [>= T-1, Hv, 128, 128] f32 or None.  Returns y [T, Hv, 128] bf16."""
    T, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    for t, dt in ((q, torch.bfloat16), (k, torch.bfloat16), (v, torch.bfloat16), (g, torch.float32),
                  (beta, torch.float32), (state, torch.float32)):
        if t.dtype != dt or not t.is_contiguous():
            raise ValueError("gdn.recurrent: wrong dtype or non-contiguous tensor")
    if ckpt is not None and (ckpt.dtype != torch.float32 or not ckpt.is_contiguous() or ckpt.shape[0] < T - 1):
        raise ValueError("gdn.recurrent: checkpoint buffer must be f32 [>= T-1, Hv, 128, 128]")
    if y is None:
        y = torch.empty(T, Hv, dv, dtype=torch.bfloat16, device=q.device)
    _lib.call("skinny_gdn_recurrent", _p(q), _p(k), _p(v), _p(g), _p(beta), _p(state), _p(y),
              _p(ckpt if T > 1 else None), T, Hv, Hk, dk, dv, _stream(q.device))
    return y


def rollback(states: list[torch.Tensor], ckpts: list[torch.Tensor], keep: int, fed: int,
             convs: list[torch.Tensor] | None = None, conv_fulls: list[torch.Tensor] | None = None) -> None:
    """Keep the first `keep` of `fed` verified tokens in every GDN layer (one launch)."""
    n = len(states)
    arr = ctypes.c_void_p * n
    st = arr(*[s.data_ptr() for s in states])
    ck = arr(*[c.data_ptr() for c in ckpts])
    W = C = 0
    cv = cf = None
    if convs is not None:
        W, C = convs[0].shape
        cv = arr(*[c.data_ptr() for c in convs])
        cf = arr(*[c.data_ptr() for c in conv_fulls])
    _lib.call("skinny_gdn_rollback", n, st, ck, cv, cf, states[0].numel(), keep, fed, W, C,
              _stream(states[0].device))


def rollback_tree(states: list[torch.Tensor], ckpts: list[torch.Tensor], node: int, rows: list[int], fed: int,
                  convs: list[torch.Tensor], conv_fulls: list[torch.Tensor]) -> None:
    """After a tree verify of `fed` nodes whose accepted path ends at `node`: every GDN layer's
    state <- its checkpoint of `node`, its conv window <- conv_full rows `rows` (one launch)."""
    n = len(states)
    arr = ctypes.c_void_p * n
    W, C = convs[0].shape
    if len(rows) != W:
        raise ValueError("one conv_full row per window row")
    _lib.call("skinny_gdn_rollback_tree", n, arr(*[s.data_ptr() for s in states]), arr(*[c.data_ptr() for c in ckpts]),
              arr(*[c.data_ptr() for c in convs]), arr(*[c.data_ptr() for c in conv_fulls]), states[0].numel(), node,
              (ctypes.c_int32 * W)(*rows), fed, W, C, _stream(states[0].device))


__all__ = ["recurrent", "rollback", "rollback_tree"]
