"""TEST INFRASTRUCTURE ONLY -- float64 numpy restatement of the synthetic hybrid decoder and its
MTP draft head, shaped like the mlx_lm model the reference's host loops drive.

What it restates:
  * the decoder the reference patches (mlx_lm Qwen3.5, as built by skinny_mlx_b200.model from
    seeded weights): zero-centred RMSNorm (x / rms(x) * (1 + w)); Gated DeltaNet layers (fused
    in_proj_qkv / z / b / a, depthwise causal conv of kernel 4 + SiLU, L2-normalised q (scaled by
    Dk^-1/2) and k, g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b), the gated delta
    rule of oracle/gdn.py, gated RMSNorm norm(y) * silu(z), out_proj); full attention every 4th
    layer (gated query, per-head q/k RMSNorm, partial rotate-half RoPE, causal GQA softmax
    attention over a KV cache, output * sigmoid(gate), o_proj); SwiGLU MLP; tied quantized
    embedding / LM head.  Every projection is mx.quantized_matmul semantics (y = x @ (q s + b)^T,
    oracle/quant.py).  Arithmetic is float64; values are rounded to bf16 where the bf16 model
    stores an activation (projection outputs, norm outputs, residual sums, q/k/v of the
    recurrence and of attention), as the MLX model does;
  * the MTP head, skinny_mlx/mtp.py:64-67: norm(layer(fc(cat(norm_e(emb), norm_h(h))))) with one
    full-attention decoder layer (+ MLP) and the causal mask for T > 1.

Interface (what skinny_mlx/spec.py:23-156 and skinny_mlx/rollback.py:19-73 touch):
`model(ids [1, T], cache) -> logits [1, T, V]`, `model.language_model.model(ids, cache) -> h`,
`.embed_tokens(ids)`, `.embed_tokens.as_linear(h)`, `.embed_tokens.weight/scales/biases`,
`model.layers[i].is_linear`, `model.layers[i].linear_attn.conv1d` (a plain object whose class the
reference's rollback replaces to record conv inputs), `model.make_cache()` -> per layer an
`ArraysCache` ([conv window, recurrent state]) or a `KVCache` (offset, trim).  The recurrence is
called as `gdu.gated_delta_update(q, k, v, a, b, A_log, dt_bias, state, mask, use_kernel)` with
`gdu` looked up at call time, so the reference's HybridRollback can hook it as it hooks mlx_lm's.
Inputs and outputs carry a leading batch dimension of 1 like MLX's.  Nothing here mutates an
array it was given (the reference keeps references to pre-verify states).
"""

from __future__ import annotations

import math
import sys
from types import SimpleNamespace

import numpy as np

from . import quant

F64 = np.float64


def bf(a) -> np.ndarray:
    """Round float64 values to bf16 (8 significant bits, nearest even), kept as float64."""
    m, e = np.frexp(np.asarray(a, F64))
    return np.ldexp(np.rint(np.ldexp(m, 8)), e - 8)


def silu(x):
    return x / (1.0 + np.exp(-x))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def softplus(x):
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))


def rms_norm(x, w, eps):
    """Zero-centred RMSNorm over the last axis, output rounded to bf16."""
    x = np.asarray(x, F64)
    y = x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return bf(y * (1.0 + np.asarray(w, F64)))


class QLinear:
    """4-bit g64 projection: y = bf16(x @ (q s + b)^T) (mx.quantized_matmul, transpose=True)."""

    def __init__(self, packed, s_bits, b_bits):
        self.weight, self.scales, self.biases = packed, s_bits, b_bits
        self._w = None

    def deq(self) -> np.ndarray:
        if self._w is None:
            self._w = quant.dequantize(self.weight, self.scales, self.biases)
        return self._w

    def __call__(self, x):
        return bf(np.asarray(x, F64) @ self.deq().T)


def quantized_matmul(x, w, scales, biases, transpose=True, group_size=64, bits=4):
    """mx.quantized_matmul over MLX packs (scales / biases as bf16 bits), output bf16."""
    assert transpose and group_size == 64 and bits == 4
    return bf(np.asarray(x, F64) @ quant.dequantize(np.asarray(w), np.asarray(scales), np.asarray(biases)).T)


class Embedding:
    def __init__(self, packed, s_bits, b_bits):
        self.weight, self.scales, self.biases = packed, s_bits, b_bits
        self.group_size, self.bits = 64, 4
        self._lin = QLinear(packed, s_bits, b_bits)

    def __call__(self, ids):
        ids = np.asarray(ids, np.int64)
        rows = quant.dequantize(self.weight[ids.reshape(-1)], self.scales[ids.reshape(-1)],
                                self.biases[ids.reshape(-1)])
        return bf(rows).reshape(ids.shape + (-1,))

    def as_linear(self, h):
        return self._lin(h)


# ------------------------------------------------------------------------------------------------
# caches (the interface of mlx_lm's KVCache / ArraysCache that the reference touches)
# ------------------------------------------------------------------------------------------------
class KVCache:
    """keys / values [L, Hkv, D]; offset = cached tokens; trim(n) drops the last n."""

    def __init__(self):
        self.keys = None
        self.values = None
        self.offset = 0

    def update_and_fetch(self, k, v):
        if self.keys is None:
            self.keys, self.values = np.asarray(k, F64), np.asarray(v, F64)
        else:
            self.keys = np.concatenate([self.keys[:self.offset], k])
            self.values = np.concatenate([self.values[:self.offset], v])
        self.offset = self.keys.shape[0]
        return self.keys, self.values

    def trim(self, n: int) -> int:
        n = min(self.offset, n)
        self.offset -= n
        self.keys, self.values = self.keys[:self.offset], self.values[:self.offset]
        return n


class ArraysCache:
    """[conv window [1, W, C], recurrent state [1, Hv, Dv, Dk]] of one GDN layer."""

    def __init__(self, size: int = 2):
        self.cache = [None] * size

    def __getitem__(self, i):
        return self.cache[i]

    def __setitem__(self, i, v):
        self.cache[i] = v


# ------------------------------------------------------------------------------------------------
# the recurrence entry point (mlx_lm's gated_delta_update contract)
# ------------------------------------------------------------------------------------------------
def gated_delta_update(q, k, v, a, b, A_log, dt_bias, state=None, mask=None, use_kernel=True):
    """q, k [1, T, Hk, Dk]; v [1, T, Hv, Dv]; a, b [1, T, Hv]; state [1, Hv, Dv, Dk] or None ->
    (y [1, T, Hv, Dv], new state).  g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b),
    then S <- g S; S += beta (v - S k) k^T; y = S q (oracle/gdn.py), in float64."""
    from .gdn import recurrent

    q, k, v, a, b = (np.asarray(t, F64)[0] for t in (q, k, v, a, b))
    g = np.exp(-np.exp(np.asarray(A_log, F64)) * softplus(a + np.asarray(dt_bias, F64)))
    beta = sigmoid(b)
    Hv, Dv, Dk = v.shape[1], v.shape[2], k.shape[2]
    s0 = np.zeros((Hv, Dv, Dk)) if state is None else np.asarray(state, F64)[0]
    y, S, _ = recurrent(q, k, v, g, beta, s0)
    return y[None], S[None]


# ------------------------------------------------------------------------------------------------
# layers
# ------------------------------------------------------------------------------------------------
class Conv1d:
    """Depthwise causal conv, no bias: x [1, W + T, C] -> [1, T, C], out[t] = sum_j w[:, j] x[t + j]."""

    def __init__(self, w):
        self.weight = np.asarray(w, F64)  # [C, kernel]

    def __call__(self, x):
        x = np.asarray(x, F64)[0]
        kk = self.weight.shape[1]
        T = x.shape[0] - kk + 1
        out = np.zeros((T, x.shape[1]))
        for j in range(kk):
            out += self.weight[:, j] * x[j:j + T]
        return out[None]


def _rope(x, pos, rot, theta):
    """Rotate-half RoPE on the first `rot` dims of x [T, H, D]."""
    half = rot // 2
    inv = theta ** (-np.arange(half, dtype=F64) / half)
    ang = np.asarray(pos, F64)[:, None] * inv[None]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    x1, x2, rest = x[..., :half], x[..., half:rot], x[..., rot:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s, rest], -1)


class Attention:
    def __init__(self, p: dict, cfg: dict):
        self.cfg = cfg
        self.q_proj, self.k_proj, self.v_proj, self.o_proj = (QLinear(*p[n]) for n in ("q", "k", "v", "o"))
        self.qn, self.kn = np.asarray(p["q_norm"], F64), np.asarray(p["k_norm"], F64)

    def __call__(self, x, cache: KVCache):
        c = self.cfg
        T, D, nh, nkv = x.shape[0], c["head_dim"], c["n_heads"], c["n_kv_heads"]
        qg = self.q_proj(x).reshape(T, nh, 2 * D)
        q, gate = qg[..., :D], qg[..., D:]
        k = self.k_proj(x).reshape(T, nkv, D)
        v = self.v_proj(x).reshape(T, nkv, D)
        L0 = cache.offset
        pos = np.arange(L0, L0 + T)
        q = bf(_rope(rms_norm(q, self.qn, c["rms_eps"]), pos, c["rotary_dim"], c["rope_theta"]))
        k = bf(_rope(rms_norm(k, self.kn, c["rms_eps"]), pos, c["rotary_dim"], c["rope_theta"]))
        keys, values = cache.update_and_fetch(k, v)
        rep = nh // nkv
        K = np.repeat(keys, rep, axis=1)  # [L, nh, D]
        V = np.repeat(values, rep, axis=1)
        sc = np.einsum("thd,lhd->thl", q, K) / math.sqrt(D)
        causal = pos[:, None] >= np.arange(keys.shape[0])[None, :]
        sc = np.where(causal[:, None, :], sc, -np.inf)
        sc = np.exp(sc - sc.max(-1, keepdims=True))
        o = bf(np.einsum("thl,lhd->thd", sc / sc.sum(-1, keepdims=True), V))
        o = bf(o * sigmoid(gate))
        return self.o_proj(o.reshape(T, nh * D))


class GatedDeltaNet:
    def __init__(self, p: dict, cfg: dict, gdu):
        self.cfg, self.gdu = cfg, gdu
        self.in_proj_qkv, self.in_proj_z, self.in_proj_b, self.in_proj_a, self.out_proj = (
            QLinear(*p[n]) for n in ("qkv", "z", "b", "a", "out"))
        self.conv1d = Conv1d(p["conv_w"])
        self.A_log, self.dt_bias = np.asarray(p["A_log"], F64), np.asarray(p["dt_bias"], F64)
        self.norm_w = np.asarray(p["norm_w"], F64)

    def __call__(self, x, cache: ArraysCache):
        c = self.cfg
        T, dk = x.shape[0], c["gdn_dim"]
        Hk, Hv = c["gdn_k_heads"], c["gdn_v_heads"]
        qkv, z = self.in_proj_qkv(x), self.in_proj_z(x)
        b, a = self.in_proj_b(x), self.in_proj_a(x)
        W = c["conv_kernel"] - 1
        conv_state = np.zeros((1, W, qkv.shape[1])) if cache[0] is None else np.asarray(cache[0], F64)
        conv_in = np.concatenate([conv_state, qkv[None]], axis=1)  # [1, W + T, C]
        cache[0] = conv_in[:, -W:]
        conv = silu(self.conv1d(conv_in)[0])
        kd = Hk * dk
        q, k, v = conv[:, :kd], conv[:, kd:2 * kd], conv[:, 2 * kd:]
        q = q.reshape(T, Hk, dk)
        k = k.reshape(T, Hk, dk)
        q = bf(q / np.maximum(np.linalg.norm(q, axis=-1, keepdims=True), 1e-12) / math.sqrt(dk))
        k = bf(k / np.maximum(np.linalg.norm(k, axis=-1, keepdims=True), 1e-12))
        v = bf(v.reshape(T, Hv, dk))
        y, st = self.gdu.gated_delta_update(q[None], k[None], v[None], a[None], b[None], self.A_log, self.dt_bias,
                                            cache[1], None, True)
        cache[1] = st
        y = bf(np.asarray(y, F64)[0])
        o = bf(rms_norm(y, self.norm_w, c["rms_eps"]) * silu(z.reshape(T, Hv, dk)))
        return self.out_proj(o.reshape(T, Hv * dk))


class MLP:
    def __init__(self, p: dict):
        self.gate, self.up, self.down = QLinear(*p["gate"]), QLinear(*p["up"]), QLinear(*p["down"])

    def __call__(self, x):
        return self.down(bf(silu(self.gate(x)) * self.up(x)))


class DecoderLayer:
    def __init__(self, p: dict, cfg: dict, gdu):
        self.is_linear = p["kind"] == "gdn"
        if self.is_linear:
            self.linear_attn = GatedDeltaNet(p, cfg, gdu)
        else:
            self.self_attn = Attention(p, cfg)
        self.mlp = MLP(p)
        self.in_norm, self.post_norm, self.eps = p["in_norm"], p["post_norm"], cfg["rms_eps"]

    def __call__(self, x, cache):
        mixer = self.linear_attn if self.is_linear else self.self_attn
        h = bf(x + mixer(rms_norm(x, self.in_norm, self.eps), cache))
        return bf(h + self.mlp(rms_norm(h, self.post_norm, self.eps)))


class Inner:
    def __init__(self, w: dict, gdu):
        cfg = w["cfg"]
        self.cfg = cfg
        self.embed_tokens = Embedding(*w["embed"])
        self.layers = [DecoderLayer(p, cfg, gdu) for p in w["layers"]]
        self.norm_w = w["norm"]

    def __call__(self, ids, cache):
        ids = np.asarray(ids)
        x = self.embed_tokens(ids[0])
        for layer, c in zip(self.layers, cache):
            x = layer(x, c)
        return rms_norm(x, self.norm_w, self.cfg["rms_eps"])[None]


class HybridModel:
    """The mlx_lm-shaped float64 model; `gdu` supplies gated_delta_update (this module by
    default)."""

    def __init__(self, weights: dict, gdu=None):
        self.language_model = SimpleNamespace(model=Inner(weights, gdu or sys.modules[__name__]))
        self.layers = self.language_model.model.layers

    def make_cache(self):
        return [ArraysCache(2) if layer.is_linear else KVCache() for layer in self.layers]

    def __call__(self, inputs, cache=None):
        inner = self.language_model.model
        return inner.embed_tokens.as_linear(inner(inputs, cache if cache is not None else self.make_cache()))


class MTPHead:
    """skinny_mlx/mtp.py:53-67: h_next = norm(layer(fc([norm_e(emb), norm_h(h)])))."""

    def __init__(self, weights: dict):
        cfg = weights["cfg"]
        self.eps = cfg["rms_eps"]
        self.ne, self.nh, self.norm_w = weights["norm_e"], weights["norm_h"], weights["norm"]
        self.fc = QLinear(*weights["fc"])
        self.layer = DecoderLayer(weights["layer"], cfg, None)
        assert not self.layer.is_linear

    def __call__(self, emb, hidden, cache: KVCache):
        emb, hidden = np.asarray(emb, F64)[0], np.asarray(hidden, F64)[0]
        x = self.fc(np.concatenate([rms_norm(emb, self.ne, self.eps), rms_norm(hidden, self.nh, self.eps)], -1))
        return rms_norm(self.layer(x, cache), self.norm_w, self.eps)[None]


# ------------------------------------------------------------------------------------------------
# weights from the torch modules (duck-typed: reads tensors only)
# ------------------------------------------------------------------------------------------------
def _np(t):
    return t.detach().cpu().numpy()


def _bits(t):
    """bf16 tensor -> uint16 bits."""
    import torch

    return _np(t.contiguous().view(torch.int16)).view(np.uint16)


def _qlin(mod):
    return (_np(mod.weight).view(np.uint32), _bits(mod.scales), _bits(mod.biases))


def _f64(t):
    return _np(t.float()).astype(F64)


def _layer_weights(layer) -> dict:
    p = {"in_norm": _f64(layer.input_layernorm.weight), "post_norm": _f64(layer.post_attention_layernorm.weight),
         "gate": _qlin(layer.mlp.gate_proj), "up": _qlin(layer.mlp.up_proj), "down": _qlin(layer.mlp.down_proj)}
    if layer.is_linear:
        g = layer.linear_attn
        p.update(kind="gdn", qkv=_qlin(g.in_proj_qkv), z=_qlin(g.in_proj_z), b=_qlin(g.in_proj_b),
                 a=_qlin(g.in_proj_a), out=_qlin(g.out_proj), conv_w=_f64(g.conv_weight), A_log=_f64(g.A_log),
                 dt_bias=_f64(g.dt_bias), norm_w=_f64(g.norm.weight))
    else:
        a = layer.self_attn
        p.update(kind="attn", q=_qlin(a.q_proj), k=_qlin(a.k_proj), v=_qlin(a.v_proj), o=_qlin(a.o_proj),
                 q_norm=_f64(a.q_norm.weight), k_norm=_f64(a.k_norm.weight))
    return p


def _cfg(c) -> dict:
    return {k: getattr(c, k) for k in ("hidden", "head_dim", "n_heads", "n_kv_heads", "rotary_dim", "rope_theta",
                                       "rms_eps", "gdn_dim", "gdn_k_heads", "gdn_v_heads", "conv_kernel")}


def weights_from_torch(model) -> dict:
    """The weights of an UNPATCHED torch hybrid model (skinny_mlx_b200.model.HybridModel)."""
    e = model.embed_tokens
    return {"cfg": _cfg(model.cfg), "embed": _qlin(e), "norm": _f64(model.norm.weight),
            "layers": [_layer_weights(layer) for layer in model.layers]}


def head_weights_from_torch(head) -> dict:
    """The weights of an UNPATCHED torch MTP head (skinny_mlx_b200.mtp.MTPHead)."""
    return {"cfg": _cfg(head.cfg), "norm_e": _f64(head.pre_fc_norm_embedding.weight),
            "norm_h": _f64(head.pre_fc_norm_hidden.weight), "fc": _qlin(head.fc), "norm": _f64(head.norm.weight),
            "layer": _layer_weights(head.layer)}
