"""A numpy stand-in for the parts of `mlx.core` and `mlx_lm` that the reference's pure-host code
touches.

Used only by tests/golden/make_golden.py, in the build container, to execute the reference's
own Python (skinny_mlx/qmm.py `repack_for_skinny` and `config_for`; skinny_mlx/spec.py `greedy`,
`speculative`, `MTPDrafter` and skinny_mlx/rollback.py `HybridRollback` over the float64 oracle
model, oracle/model.py) and record golden vectors.  MLX and mlx-lm are not installable here;
nothing that needs Metal runs.
"""

from __future__ import annotations

import sys
import types

import numpy as np


class array(np.ndarray):
    """np.ndarray subclass so `isinstance(x, mx.array)` and `mx.array([...])` both work."""

    def __new__(cls, obj, dtype=None):
        return np.asarray(obj, dtype=dtype).view(cls)


def _noop(*_a, **_k):
    return None


def install(quantized_matmul=None, extra: dict | None = None) -> types.ModuleType:
    """Register fake `mlx`, `mlx.core` (and `mlx.nn`) modules in sys.modules."""
    core = types.ModuleType("mlx.core")
    core.array = array
    for name in ("float16", "float32", "int32", "uint32", "int64", "uint8"):
        setattr(core, name, getattr(np, name))
    core.bfloat16 = np.float32  # storage stand-in; never used for arithmetic here
    core.eval = _noop
    core.async_eval = _noop
    core.contiguous = lambda a: np.ascontiguousarray(a).view(array)
    core.argmax = lambda a, axis=None: np.asarray(np.argmax(a, axis=axis)).view(array)
    core.concatenate = lambda xs, axis=0: np.concatenate([np.asarray(x) for x in xs], axis=axis).view(array)
    core.zeros = lambda shape, dtype=np.float32: np.zeros(shape, dtype=dtype).view(array)
    core.fast = types.SimpleNamespace(metal_kernel=lambda **kw: None)
    if quantized_matmul is not None:
        core.quantized_matmul = quantized_matmul
    for k, v in (extra or {}).items():
        setattr(core, k, v)
    mlx = types.ModuleType("mlx")
    mlx.core = core
    nn = types.ModuleType("mlx.nn")

    class Module:
        pass

    nn.Module = Module
    mlx.nn = nn
    sys.modules["mlx"] = mlx
    sys.modules["mlx.core"] = core
    sys.modules["mlx.nn"] = nn
    return core


def install_mlx_lm(cache_mod, gated_delta_update) -> None:
    """Register fake `mlx_lm.models.cache` (KVCache, make_prompt_cache) and
    `mlx_lm.models.qwen3_5` (gated_delta_update), backed by the oracle's cache classes and
    recurrence.  make_prompt_cache(model) returns model.make_cache(), as mlx_lm does for models
    that define it."""
    lm = types.ModuleType("mlx_lm")
    models = types.ModuleType("mlx_lm.models")
    cache = types.ModuleType("mlx_lm.models.cache")
    cache.KVCache = cache_mod.KVCache
    cache.ArraysCache = cache_mod.ArraysCache
    cache.make_prompt_cache = lambda model, max_kv_size=None: model.make_cache()
    q35 = types.ModuleType("mlx_lm.models.qwen3_5")
    q35.gated_delta_update = gated_delta_update
    lm.models = models
    models.cache = cache
    models.qwen3_5 = q35
    sys.modules.update({"mlx_lm": lm, "mlx_lm.models": models, "mlx_lm.models.cache": cache,
                        "mlx_lm.models.qwen3_5": q35})
