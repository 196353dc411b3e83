"""skinny_mlx_b200 — skinny-mlx's flat multi-token verify path, rebuilt for NVIDIA B200 (sm_100a).

Drop-in API of rachittshah/skinny-mlx on PyTorch tensors:
  qmm / skinny_qmm / repack_for_skinny / quantize   (skinny_mlx/qmm.py)
The CUDA work runs in the in-tree C-ABI library `_skinny_b200.so` (include/skinny_b200.h).
"""

from .qmm import (GROUP, BITS, MAX_TOKENS, SkinnyWeight, config_for, dequantize, qmm, quantize,
                  repack_for_skinny, skinny_qmm)

__all__ = ["GROUP", "BITS", "MAX_TOKENS", "SkinnyWeight", "config_for", "dequantize", "qmm",
           "quantize", "repack_for_skinny", "skinny_qmm"]
