"""Drop-in patch of a hybrid model for the B200 qmm kernel (skinny_mlx/patch.py on B200).

1. Routing: every quantized projection runs the sm_100a kernel for any token count (the
   reference keeps MLX's qmv for M = 1..5 and uses its Metal kernel for M = 6..16,
   patch.py:22,30-35; the B200 kernel is bandwidth-bound from M = 1, and larger M runs in
   16-token chunks).
2. Horizontal fusion: projections that read the same input (FUSE_GROUPS, patch.py:23-27) are
   concatenated along N at load time and run as ONE qmm; the siblings return slices of a
   one-entry result cache matched by input identity (patch.py:52-77), so the model code is
   untouched.
3. The tied LM head (`embed_tokens.as_linear`) runs on the same kernel (patch.py:84-87).

Unlike the reference prototype, a patched module keeps only the relaid weights (the MLX copy is
dropped), so weight memory is not doubled.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .model import QuantizedEmbedding, QuantizedLinear
from .qmm import SkinnyWeight, repack_for_skinny, skinny_qmm

SKINNY_RANGE = (1, 16)
FUSE_GROUPS = [
    ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a"),  # Gated DeltaNet mixer
    ("q_proj", "k_proj", "v_proj"),                          # full attention
    ("gate_proj", "up_proj"),                                # MLP
]


def _qmm(x: torch.Tensor, w: SkinnyWeight) -> torch.Tensor:
    k = x.shape[-1]
    m = x.numel() // k
    y = skinny_qmm(x.reshape(m, k).to(torch.bfloat16).contiguous(), w)
    return y.reshape(*x.shape[:-1], w.N)


class SkinnyQuantizedLinear(nn.Module):
    """A single projection on the B200 kernel (patch.py:38-49)."""

    def __init__(self, ql: QuantizedLinear):
        super().__init__()
        self.group_size, self.bits = ql.group_size, ql.bits
        self.rweight = repack_for_skinny(ql.weight, ql.scales, ql.biases)

    @property
    def out_features(self) -> int:
        return self.rweight.N

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _qmm(x, self.rweight)


def _interleave64(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Rows of a and b (same shape, rows % 64 == 0) in blocks of 64: a[0:64], b[0:64], a[64:128], ..."""
    n = a.shape[0]
    return torch.stack([a.reshape(n // 64, 64, *a.shape[1:]), b.reshape(n // 64, 64, *b.shape[1:])], 1).reshape(
        2 * n, *a.shape[1:])


class _FusedGroup:
    """Concatenated weights of same-input projections + a one-entry result cache (patch.py:52-68).

    A SwiGLU pair (gate_proj, up_proj of equal size, a multiple of 64 rows) is stored with its rows
    interleaved in blocks of 64 (gate 0-63, up 0-63, gate 64-127, ...): each 128-row tile of the
    relaid weight then holds matching gate and up rows, so the fused step's gate|up launch can
    apply the activation in its epilogue (skinny_qmm_w4g64_swiglu).  The slices return the
    projections' outputs in their own column order either way."""

    def __init__(self, qls: list[QuantizedLinear], swiglu: bool = False):
        self.interleaved = (swiglu and len(qls) == 2 and qls[0].weight.shape == qls[1].weight.shape
                            and qls[0].weight.shape[0] % 64 == 0)
        if self.interleaved:
            g, u = qls
            self.rw = repack_for_skinny(_interleave64(g.weight, u.weight), _interleave64(g.scales, u.scales),
                                        _interleave64(g.biases, u.biases))
        else:
            self.rw = repack_for_skinny(torch.cat([q.weight for q in qls]), torch.cat([q.scales for q in qls]),
                                        torch.cat([q.biases for q in qls]))
        sizes = [q.weight.shape[0] for q in qls]
        self.bounds = [(sum(sizes[:i]), sum(sizes[: i + 1])) for i in range(len(sizes))]
        self.x = self.y = None

    def output(self, x: torch.Tensor) -> torch.Tensor:
        if self.x is not x:  # strong reference held, so the identity cannot be recycled
            self.x, self.y = x, _qmm(x, self.rw)
        return self.y

    def slice(self, x: torch.Tensor, idx: int) -> torch.Tensor:
        y = self.output(x)
        if self.interleaved:  # [..., I / 64, (gate | up), 64] -> projection idx
            return y.unflatten(-1, (-1, 2, 64))[..., idx, :].flatten(-2)
        lo, hi = self.bounds[idx]
        return y[..., lo:hi]


class FusedSliceLinear(nn.Module):
    def __init__(self, group: _FusedGroup, idx: int):
        super().__init__()
        self._group, self._idx = group, idx
        self._lo, self._hi = group.bounds[idx]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._group.slice(x, self._idx)


def _ok(m) -> bool:
    return isinstance(m, QuantizedLinear) and m.bits == 4 and m.group_size == 64


def _patch_tied_head(emb: QuantizedEmbedding) -> None:
    rw = repack_for_skinny(emb.weight, emb.scales, emb.biases)
    emb.skinny_head = rw
    emb.as_linear = lambda x: _qmm(x, rw)


@torch.no_grad()
def patch_model(model: nn.Module, fuse: bool = True) -> dict:
    """Patch in place (patch.py:90-115).  Returns counts of fused groups, single swaps, heads."""
    stats = {"fused_groups": 0, "single": 0, "heads": 0}
    fused_ids = set()
    if fuse:
        for _, parent in list(model.named_modules()):
            children = dict(parent.named_children())
            for names in FUSE_GROUPS:
                if all(_ok(children.get(n)) for n in names):
                    group = _FusedGroup([children[n] for n in names], swiglu=names == ("gate_proj", "up_proj"))
                    for i, n in enumerate(names):
                        fused_ids.add(id(children[n]))
                        setattr(parent, n, FusedSliceLinear(group, i))
                    stats["fused_groups"] += 1
    for _, parent in list(model.named_modules()):
        for n, child in list(parent.named_children()):
            if _ok(child) and id(child) not in fused_ids:
                setattr(parent, n, SkinnyQuantizedLinear(child))
                stats["single"] += 1
    for _, m in model.named_modules():
        if isinstance(m, QuantizedEmbedding) and m.bits == 4 and m.group_size == 64:
            _patch_tied_head(m)
            stats["heads"] += 1
    torch.cuda.synchronize()
    return stats


__all__ = ["patch_model", "FUSE_GROUPS", "SKINNY_RANGE", "SkinnyQuantizedLinear", "FusedSliceLinear"]
