"""4-bit affine group-64 quantized matmul for 1..16 tokens per weight read, on B200.

Mirrors skinny_mlx/qmm.py (rachittshah/skinny-mlx):

* ``repack_for_skinny`` (qmm.py:96) relays MLX 4-bit packs once at load, here into the
  tcgen05 unit order (128 rows x 64 columns per 4608-byte unit, scales and biases folded in).
* ``skinny_qmm`` (qmm.py:132) runs the sm_100a kernel: x [M, K] @ dequant(W)[N, K]^T -> [M, N]
  in x's dtype, computing sum_g s * sum(x q) + b * sum(x) per 64-group in f32 (the affine
  identity of qmm.py:8-9).  The tensor-core products are exact integer dot products (tcgen05
  kind::i8): the nibbles as int8 16 (q - 8), x as two int8 digits of 16-bit fixed point per
  (token, group) with a power-of-two scale, so the only rounding before the f32 accumulation is
  x to 16 significant bits relative to its group maximum.
* ``qmm`` is the drop-in ``mx.quantized_matmul(x, w, scales, biases, transpose=True,
  group_size=64, bits=4)`` entry: MLX packing in, relayout cached per weight.
* ``quantize`` produces MLX's packing with the affine rule scale = (max - min) / 15,
  bias = min per 64-column group.

There is no CPU or library fallback: everything runs through the C-ABI in _skinny_b200.so.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass

import torch

from . import _lib

GROUP = 64
BITS = 4
MAX_TOKENS = 16
PREFILL_TOKENS = 64  # from this many tokens skinny_qmm dequantises once and runs a dense GEMM


# ---------------------------------------------------------------------------------------------
# quantization (MLX affine packing)
# ---------------------------------------------------------------------------------------------
def quantize(w: torch.Tensor, group_size: int = GROUP, bits: int = BITS):
    """w [N, K] float -> (w_packed uint32-as-int32 [N, K/8], scales bf16 [N, K/64], biases bf16).

    Per 64-column group: scale = (max - min) / 15, bias = min, both rounded to bf16, then
    q = clamp(round((w - bias) / scale), 0, 15) with round-half-even; a constant group
    (scale 0) gets q = 0.  Element k = 8j + i sits at bits 4i of word j, the order
    skinny_mlx/qmm.py:104 decodes.
    """
    if group_size != GROUP or bits != BITS:
        raise ValueError("only group_size=64, bits=4 is supported")
    n, k = w.shape
    if k % GROUP:
        raise ValueError(f"K={k} is not a multiple of {GROUP}")
    wg = w.float().reshape(n, k // GROUP, GROUP)
    wmax = wg.amax(-1)
    wmin = wg.amin(-1)
    scales = ((wmax - wmin) / 15.0).to(torch.bfloat16)
    biases = wmin.to(torch.bfloat16)
    s32 = scales.float().unsqueeze(-1)
    b32 = biases.float().unsqueeze(-1)
    safe = torch.where(s32 == 0, torch.ones_like(s32), s32)
    q = torch.round((wg - b32) / safe).clamp_(0, 15)
    q = torch.where(s32 == 0, torch.zeros_like(q), q).to(torch.int64).reshape(n, k // 8, 8)
    shifts = torch.arange(8, device=w.device, dtype=torch.int64) * 4
    words = (q << shifts).sum(-1)
    packed = words.to(torch.int64).bitwise_and(0xFFFFFFFF)
    packed = torch.where(packed >= 2**31, packed - 2**32, packed).to(torch.int32)
    return packed, scales, biases


def dequantize(w_packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor) -> torch.Tensor:
    """MLX packs -> float32 [N, K] (q * scale + bias)."""
    n, kw = w_packed.shape
    words = w_packed.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(8, device=w_packed.device, dtype=torch.int64) * 4
    q = ((words.unsqueeze(-1) >> shifts) & 0xF).reshape(n, kw * 8).float()
    s = scales.float().repeat_interleave(GROUP, dim=1)
    b = biases.float().repeat_interleave(GROUP, dim=1)
    return q * s + b


# ---------------------------------------------------------------------------------------------
# relaid weights
# ---------------------------------------------------------------------------------------------
@dataclass
class SkinnyWeight:
    """Relaid 4-bit weight: `w_tc` holds ceil(N/128) * (K/64) units of 4608 bytes."""

    w_tc: torch.Tensor
    N: int
    K: int

    @property
    def nbytes_mlx(self) -> int:
        """Bytes of the original MLX packing (nibbles + bf16 scales + bf16 biases)."""
        return self.N * self.K // 2 + self.N * (self.K // GROUP) * 4


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU fallback)")


def repack_for_skinny(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor) -> SkinnyWeight:
    """One-time relayout of MLX packs [N, K/8] + bf16 scales/biases [N, K/64] (C-ABI
    skinny_repack_w4g64; replaces skinny_mlx/qmm.py:96)."""
    for t, nm in ((w, "w"), (scales, "scales"), (biases, "biases")):
        _require_cuda(t, nm)
    n, kw = w.shape
    k = kw * 8
    if scales.shape != (n, k // GROUP) or biases.shape != (n, k // GROUP):
        raise ValueError(f"scales/biases must be [{n}, {k // GROUP}]")
    if scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
        raise ValueError("scales and biases must be bfloat16")
    w = w.contiguous()
    scales = scales.contiguous()
    biases = biases.contiguous()
    L = _lib.lib()
    nbytes = L.skinny_repack_bytes(n, k)
    if nbytes == 0:
        raise ValueError(f"unsupported shape N={n} K={k}")
    with torch.cuda.device(w.device):
        out = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
        _lib.call("skinny_repack_w4g64", w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                  out.data_ptr(), n, k, _stream_handle(w.device))
    return SkinnyWeight(out, n, k)


# ---------------------------------------------------------------------------------------------
# workspace (one per device and stream; zero-filled; grows on demand)
# ---------------------------------------------------------------------------------------------
_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def workspace_bytes(n: int, k: int) -> int:
    return int(_lib.lib().skinny_qmm_workspace_bytes(n, k))


def get_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           _stream_handle(device))
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(nbytes, 1 << 22)
            if ws is not None:
                size = max(size, 2 * ws.numel())
            ws = torch.zeros(size, dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def device_errors(device: torch.device | None = None) -> int:
    """OR of the error words of every workspace on `device` (synchronises)."""
    bits = 0
    with _ws_lock:
        for (dev, _), ws in _workspaces.items():
            if device is None or dev == (device.index or 0):
                bits |= int(ws[:4].view(torch.int32).item())
    return bits


def reset_workspaces() -> None:
    with _ws_lock:
        for ws in _workspaces.values():
            ws.zero_()


def config_for(m: int, k: int, n: int = 9728) -> tuple[int, int]:
    """The launch choice for M tokens of an N x K weight on the current device, as the pair the
    reference's heuristic returns (skinny_mlx/qmm.py:118 config_for(m, k) -> (RF, SK): row
    fragments per simdgroup, K-splits per threadgroup of the Metal kernel).  Here the two knobs
    are (token columns read back per 128 x 64 unit: 2, 4, 8 or 16; K-split per 128-row tile: 0 =
    the persistent stream-K grid, S >= 1 = S CTAs per tile summing S K-slices in a cluster).  The
    split depends on N and the device (how many tiles, how many clusters fit), so N is an argument
    (default: config 1's 9728).  Read from the library (skinny_qmm_launch_config), so it is what
    skinny_qmm actually launches; the reference's CONFIG_OVERRIDE has no B200 counterpart."""
    import ctypes

    tc, sp, ctas = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.call("skinny_qmm_launch_config", m, n, k, ctypes.byref(tc), ctypes.byref(sp), ctypes.byref(ctas))
    return tc.value, sp.value


def skinny_qmm(x: torch.Tensor, w: SkinnyWeight, out: torch.Tensor | None = None) -> torch.Tensor:
    """x [..., K] @ dequant(W)^T -> [..., N] through the tcgen05 kernel, in x's dtype (as the
    reference returns; the kernel reads bf16 activations and writes bf16, so other dtypes are cast
    on the way in and out).  `out`, when given, is a bf16 [M, N] buffer and is returned as is.

    Token counts above 16 are processed in 16-token chunks by the same kernel (each token's
    result does not depend on the chunking); from PREFILL_TOKENS tokens (a prompt) the weight is
    instead dequantised to bf16 once (skinny_dequant_w4g64) and multiplied by a dense GEMM, which
    rounds the weights to bf16 and so differs from the small-M results in the last bits.
    Replaces skinny_mlx/qmm.py:132.
    """
    _require_cuda(x, "x")
    if x.shape[-1] != w.K:
        raise ValueError(f"x has K={x.shape[-1]}, weight has K={w.K}")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, w.K)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    if not x2.is_contiguous() or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    m = x2.shape[0]
    cast = x.dtype if out is None and x.dtype != torch.bfloat16 else None
    if m == 0:
        return x.new_empty(*lead, w.N, dtype=cast or torch.bfloat16)
    dev = x2.device
    if out is None:
        out = torch.empty(m, w.N, dtype=torch.bfloat16, device=dev)
    elif out.shape != (m, w.N) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 [M, N] tensor")
    L = _lib.lib()
    if m >= PREFILL_TOKENS:
        with torch.cuda.device(dev):
            wd = torch.empty(w.N, w.K, dtype=torch.bfloat16, device=dev)
            _lib.check("skinny_dequant_w4g64", L.skinny_dequant_w4g64(
                w.w_tc.data_ptr(), w.N, w.K, wd.data_ptr(), w.K, _stream_handle(dev)))
            torch.matmul(x2, wd.t(), out=out)
        y = out.reshape(*lead, w.N)
        return y if cast is None else y.to(cast)
    with torch.cuda.device(dev):
        need = L.skinny_qmm_workspace_bytes(w.N, w.K)
        ws = get_workspace(dev, need)
        stream = _stream_handle(dev)
        for c0 in range(0, m, MAX_TOKENS):
            mc = min(MAX_TOKENS, m - c0)
            xs = x2[c0:c0 + mc]
            _lib.check("skinny_qmm_w4g64", L.skinny_qmm_w4g64(
                xs.data_ptr(), w.K, w.w_tc.data_ptr(), out[c0].data_ptr(), w.N, mc, w.N, w.K,
                ws.data_ptr(), ws.numel(), stream))
    y = out.reshape(*lead, w.N)
    return y if cast is None else y.to(cast)


MAX_GROUP = 192
MAX_GROUP_INPUTS = 8


def skinny_qmm_grouped(xs, weights, outs=None):
    """Many independent products at once: outs[i] = xs[i] @ dequant(weights[i])^T, one persistent
    launch over all matrices (C-ABI skinny_qmm_w4g64_grouped).  All xs share the token count
    (<= 16); at most 8 distinct x tensors.  Per-matrix results are bit-identical to skinny_qmm."""
    import ctypes

    n = len(weights)
    if n == 0:
        return []
    if n > MAX_GROUP:
        raise ValueError(f"at most {MAX_GROUP} matrices per grouped call")
    if len(xs) != n:
        raise ValueError("one x per weight")
    xs2 = []
    for x, w in zip(xs, weights):
        _require_cuda(x, "x")
        if x.shape[-1] != w.K:
            raise ValueError(f"x has K={x.shape[-1]}, weight has K={w.K}")
        x2 = x.reshape(-1, w.K)
        if x2.dtype != torch.bfloat16 or not x2.is_contiguous():
            x2 = x2.to(torch.bfloat16).contiguous()
        xs2.append(x2)
    m = xs2[0].shape[0]
    if any(x.shape[0] != m for x in xs2) or not 1 <= m <= MAX_TOKENS:
        raise ValueError(f"all inputs need the same token count in [1, {MAX_TOKENS}]")
    dev = xs2[0].device
    if outs is None:
        outs = [torch.empty(m, w.N, dtype=torch.bfloat16, device=dev) for w in weights]
    arr_p = ctypes.c_void_p * n
    arr_i = ctypes.c_int * n
    L = _lib.lib()
    with torch.cuda.device(dev):
        ws = get_workspace(dev, L.skinny_qmm_workspace_bytes(weights[0].N, weights[0].K))
        _lib.check("skinny_qmm_w4g64_grouped", L.skinny_qmm_w4g64_grouped(
            n, arr_p(*[x.data_ptr() for x in xs2]), arr_i(*[w.K for w in weights]),
            arr_p(*[w.w_tc.data_ptr() for w in weights]), arr_p(*[o.data_ptr() for o in outs]),
            arr_i(*[w.N for w in weights]), arr_i(*[w.N for w in weights]), arr_i(*[w.K for w in weights]),
            m, ws.data_ptr(), ws.numel(), _stream_handle(dev)))
    return outs


# ---------------------------------------------------------------------------------------------
# MLX-style drop-in entry
# ---------------------------------------------------------------------------------------------
# value: (relaid weight, the source tensors) -- the strong references keep a freed tensor's
# address from being reused under a stale key, as skinny_mlx/patch.py:66 does for its inputs.
_repack_cache: dict[tuple, tuple] = {}


def _cache_key(w, s, b):
    return tuple((t.data_ptr(), tuple(t.shape), t._version) for t in (w, s, b))


def qmm(x: torch.Tensor, w_packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
        group_size: int = GROUP, bits: int = BITS, transpose: bool = True) -> torch.Tensor:
    """Drop-in for ``mx.quantized_matmul(x, w, scales, biases, transpose=True, group_size=64,
    bits=4)`` (the call skinny_mlx/patch.py:35 and qmm.py:183 make) on MLX-packed weights.

    The relayout is done on first use and cached per (w, scales, biases) storage and version.
    Returns x's dtype, as mx.quantized_matmul does.
    """
    if group_size != GROUP or bits != BITS:
        raise ValueError("skinny qmm supports group_size=64, bits=4 only")
    if not transpose:
        raise ValueError("skinny qmm computes x @ W^T (transpose=True) only")
    key = _cache_key(w_packed, scales, biases)
    hit = _repack_cache.get(key)
    if hit is None:
        hit = (repack_for_skinny(w_packed, scales, biases), (w_packed, scales, biases))
        _repack_cache[key] = hit
    return skinny_qmm(x, hit[0])


__all__ = ["GROUP", "BITS", "MAX_TOKENS", "quantize", "dequantize", "SkinnyWeight",
           "repack_for_skinny", "skinny_qmm", "skinny_qmm_grouped", "qmm", "config_for",
           "device_errors", "reset_workspaces", "workspace_bytes"]
