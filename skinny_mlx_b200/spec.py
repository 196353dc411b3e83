"""Greedy speculative acceptance on the device (skinny_mlx/spec.py:136-147).

`accept(logits, draft)` replaces the reference's verify tail -- argmax over the K+1 verified
logits, `.tolist()` of predictions and draft (its one host sync per step) and the Python prefix
loop -- with one kernel launch and a read-back of K+2 int32 values.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_ws: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(dev: torch.device) -> torch.Tensor:
    key = (dev.index if dev.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(dev).cuda_stream)
    ws = _ws.get(key)
    if ws is None:
        ws = torch.zeros(int(_lib.lib().skinny_spec_accept_workspace_bytes()), dtype=torch.uint8, device=dev)
        _ws[key] = ws
    return ws


def accept_device(logits: torch.Tensor, draft: torch.Tensor, result: torch.Tensor | None = None,
                  pred: torch.Tensor | None = None) -> torch.Tensor:
    """Stream-ordered, no host sync.  logits bf16 [K+1, V] (rows contiguous), draft int32 [K] on
    the same device.  Returns result int32 [K+2]: [n, draft[:n] + [pred[n]], -1 ...]."""
    if logits.dtype != torch.bfloat16 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a bf16 [K+1, V] tensor with unit column stride")
    rows, v = logits.shape
    if draft.numel() != rows - 1 or draft.dtype != torch.int32:
        raise ValueError("draft must be int32 with K = rows - 1 entries")
    dev = logits.device
    if result is None:
        result = torch.empty(rows + 1, dtype=torch.int32, device=dev)
    ws = _workspace(dev)
    _lib.call("skinny_spec_accept", ctypes.c_void_p(logits.data_ptr()), logits.stride(0), rows, v,
              ctypes.c_void_p(draft.data_ptr() if rows > 1 else 0), ctypes.c_void_p(result.data_ptr()),
              ctypes.c_void_p(pred.data_ptr() if pred is not None else 0), ctypes.c_void_p(ws.data_ptr()),
              ws.numel(), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    return result


def accept(logits: torch.Tensor, draft: torch.Tensor) -> tuple[int, list[int]]:
    """(n accepted draft tokens, emitted tokens draft[:n] + [pred[n]]); one small D2H."""
    r = accept_device(logits, draft).cpu().tolist()
    n = r[0]
    return n, r[1:n + 2]


__all__ = ["accept", "accept_device"]
