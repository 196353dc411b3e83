"""ctypes binding of the C-ABI library (include/skinny_b200.h).

There is no fallback: if `_skinny_b200.so` is missing or does not load, every operation raises.
"""

from __future__ import annotations

import ctypes
from ctypes import c_int, c_size_t, c_uint32, c_void_p
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "_skinny_b200.so"
_lib = None

STATUS_NAMES = {
    0: "SKINNY_OK",
    -1: "SKINNY_ERR_INVALID_ARG",
    -2: "SKINNY_ERR_SHAPE",
    -3: "SKINNY_ERR_TOKENS",
    -4: "SKINNY_ERR_ALIGNMENT",
    -5: "SKINNY_ERR_WORKSPACE",
    -6: "SKINNY_ERR_CUDA",
    -7: "SKINNY_ERR_DEVICE",
    -8: "SKINNY_ERR_UNSUPPORTED",
    -9: "SKINNY_ERR_SCRATCH_LIMIT",
}

# name -> (restype, argtypes); mirrors include/skinny_b200.h
SIGNATURES = {
    "skinny_version": (c_int, []),
    "skinny_strerror": (ctypes.c_char_p, [c_int]),
    "skinny_last_cuda_error": (c_int, []),
    "skinny_repack_bytes": (c_size_t, [c_int, c_int]),
    "skinny_repack_w4g64": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "skinny_qmm_workspace_bytes": (c_size_t, [c_int, c_int]),
    "skinny_qmm_w4g64": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                 c_void_p, c_size_t, c_void_p]),
    "skinny_qmm_launch_config": (c_int, [c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "skinny_qmm_w4g64_grouped": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "skinny_xq_bytes": (c_size_t, [c_int, c_int]),
    "skinny_prep": (c_int, [c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int,
                            c_void_p, ctypes.c_float, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "skinny_gdn_fused": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 ctypes.c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                 c_int, c_void_p, c_void_p]),
    "skinny_attn_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "skinny_attn_fused": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, ctypes.c_float, c_void_p,
                                  c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
                                  c_void_p, c_void_p, c_void_p, c_void_p]),
    "skinny_qmm_w4g64_prepared": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                          c_size_t, c_void_p, c_int, c_void_p, c_void_p]),
    "skinny_dequant_w4g64": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_void_p]),
    "skinny_embed_w4g64": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int,
                                   c_void_p]),
    "skinny_ipc_alloc": (c_int, [c_size_t, c_void_p, c_void_p]),
    "skinny_ipc_open": (c_int, [c_void_p, c_void_p]),
    "skinny_ipc_close": (c_int, [c_void_p]),
    "skinny_ipc_free": (c_int, [c_void_p]),
    "skinny_spec_accept_workspace_bytes": (c_size_t, []),
    "skinny_spec_accept": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_size_t, c_void_p]),
    "skinny_gdn_recurrent": (c_int, [c_void_p] * 8 + [c_int] * 5 + [c_void_p]),
    "skinny_gdn_rollback": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_longlong,
                                    c_int, c_int, c_int, c_int, c_void_p]),
    "skinny_qmm_w4g64_noalloc": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int,
                                         c_int, c_void_p]),
    "skinny_qmm_w4g64_noalloc_errors": (c_int, [c_void_p, c_void_p]),
    "skinny_gdn_fused_tree": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      ctypes.c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                      c_int, c_void_p, c_void_p, c_void_p]),
    "skinny_attn_fused_tree": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, ctypes.c_float,
                                       c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                       c_size_t, c_void_p, c_void_p, c_void_p, c_void_p]),
    "skinny_spec_accept_tree": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_size_t, c_void_p]),
    "skinny_kv_compact": (c_int, [c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "skinny_gdn_rollback_tree": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_longlong, c_int,
                                         c_void_p, c_int, c_int, c_int, c_void_p]),
    "skinny_qmm_w4g64_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_size_t,
                                        c_void_p]),
}


class SkinnyError(RuntimeError):
    def __init__(self, fn: str, status: int, detail: str = ""):
        lib = _lib
        text = lib.skinny_strerror(status).decode() if lib is not None else STATUS_NAMES.get(status, "?")
        extra = ""
        if status == -6 and lib is not None:
            extra = f" (cudaError {lib.skinny_last_cuda_error()})"
        super().__init__(f"{fn}: {STATUS_NAMES.get(status, status)}: {text}{extra}{detail}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the library (once).  Raises if the CUDA extension was not built."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise RuntimeError(
                f"skinny_b200 CUDA library not built: {_LIB_PATH} is missing "
                "(run `python -m skinny_mlx_b200.build`)")
        handle = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(fn: str, status: int) -> None:
    if status != 0:
        raise SkinnyError(fn, status)


def call(name: str, *args) -> None:
    check(name, getattr(lib(), name)(*args))


class PeerSync(ctypes.Structure):
    """Mirror of skinny_peer_sync (include/skinny_b200.h): device pointers as integers."""

    _fields_ = [("epoch", c_void_p), ("wait_flags", c_void_p), ("counter", c_void_p),
                ("signal_flags", c_void_p * 8), ("err", c_void_p), ("n_ranks", c_int),
                ("mirror", c_void_p * 8), ("n_mirror", c_int)]


__all__ = ["lib", "call", "check", "SkinnyError", "SIGNATURES", "c_uint32", "PeerSync"]
