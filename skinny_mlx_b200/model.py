"""Synthetic Qwen3.5-style hybrid decoder (random weights, MLX 4-bit g64 packing) in PyTorch.

The reference patches mlx_lm's Qwen3.5 model (skinny_mlx/patch.py); that model and its
checkpoints are not available here, so this module builds the same architecture from seeded
random weights, with the module names the reference's FUSE_GROUPS match
(skinny_mlx/patch.py:23-27):

* Gated DeltaNet layers (`linear_attn`): in_proj_qkv, in_proj_z, in_proj_b, in_proj_a,
  depthwise causal conv1d (kernel 4) + SiLU, L2-normalised q/k, decay g = exp(-exp(A_log) *
  softplus(a + dt_bias)), beta = sigmoid(b), the gated delta recurrence
  (skinny_mlx_b200/gdn.py), gated RMSNorm (norm(y) * silu(z)), out_proj.
* Full attention every 4th layer (`self_attn`): gated query (q_proj emits query and gate),
  per-head q/k RMSNorm, partial RoPE (theta 1e6), grouped-query attention over a KV cache,
  output * sigmoid(gate), o_proj.  Config 3 uses this one consistent shape: 16 query heads x 128
  (+ gate) and 4 KV heads x 128 give the listed fused QKV width 5120, and o_proj is 2048 -> 2560.
* SwiGLU MLP (gate_proj, up_proj, down_proj), zero-centred RMSNorms (weight 1 + w), tied
  quantized embedding / LM head.

Quantized projections run as `QuantizedLinear` (dequantize + f32 matmul in torch, the semantics of
mx.quantized_matmul) until `skinny_mlx_b200.patch.patch_model` swaps them for the B200 kernel.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from .configs import HybridConfig
from .qmm import dequantize, quantize


# ---------------------------------------------------------------------------------------------
# configuration
# ---------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class ModelConfig:
    hidden: int = 2560
    layers: int = 32
    attn_every: int = 4
    vocab: int = 151936
    intermediate: int = 9728
    n_heads: int = 16
    n_kv_heads: int = 4
    head_dim: int = 128
    rotary_dim: int = 32          # partial RoPE: the first 32 of 128 dims of every head
    gdn_k_heads: int = 16
    gdn_v_heads: int = 16
    gdn_dim: int = 128            # key and value head dim of the GDN recurrence
    conv_kernel: int = 4
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    weight_std: float = 0.02

    def is_attention(self, i: int) -> bool:
        return i % self.attn_every == self.attn_every - 1

    @property
    def gdn_key_dim(self) -> int:
        return self.gdn_k_heads * self.gdn_dim

    @property
    def gdn_value_dim(self) -> int:
        return self.gdn_v_heads * self.gdn_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.gdn_key_dim + self.gdn_value_dim


def config3(cfg: HybridConfig | None = None) -> ModelConfig:
    """The config-3 model: the config-2 hybrid stack with one consistent attention shape."""
    c = cfg or HybridConfig()
    return ModelConfig(hidden=c.hidden, layers=c.layers, attn_every=c.attn_every, vocab=c.vocab,
                       intermediate=c.intermediate, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads,
                       head_dim=c.head_dim, gdn_k_heads=c.gdn_heads, gdn_v_heads=c.gdn_heads,
                       gdn_dim=c.gdn_k_dim, conv_kernel=c.conv_kernel, rope_theta=c.rope_theta,
                       rms_eps=c.rms_eps, weight_std=c.weight_std)


# Test-size model.  At this width projections with std 0.02 are too weak against the residual
# stream for next-token predictions to depend on the context, so the small model uses 0.05
# (the full-size configurations use BASELINE's 0.02).
SMALL = ModelConfig(hidden=512, layers=4, vocab=4096, intermediate=1024, n_heads=4, n_kv_heads=2,
                    gdn_k_heads=4, gdn_v_heads=4, weight_std=0.05)


# ---------------------------------------------------------------------------------------------
# quantized modules (the unpatched path)
# ---------------------------------------------------------------------------------------------
class QuantizedLinear(nn.Module):
    """y = x @ dequant(W)^T with MLX's 4-bit group-64 affine packing (bf16 out, f32 math).
    `accumulate` (class-wide) may be set to torch.float64 to measure rounding sensitivity."""

    accumulate = torch.float32

    def __init__(self, w_packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor):
        super().__init__()
        self.register_buffer("weight", w_packed)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.group_size, self.bits = 64, 4
        self._deq = None

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    def dequantized(self) -> torch.Tensor:
        if self._deq is None:
            self._deq = dequantize(self.weight, self.scales, self.biases).float()
        return self._deq

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        a = QuantizedLinear.accumulate
        return (x.to(a) @ self.dequantized().to(a).t()).to(torch.bfloat16)


class QuantizedEmbedding(nn.Module):
    """Quantized token embedding; `as_linear` is the tied LM head."""

    def __init__(self, w_packed, scales, biases):
        super().__init__()
        self.register_buffer("weight", w_packed)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.group_size, self.bits = 64, 4
        self.__dict__["_deq"] = None  # not a registered submodule or buffer

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        return dequantize(self.weight[ids], self.scales[ids], self.biases[ids]).to(torch.bfloat16)

    def as_linear(self, x: torch.Tensor) -> torch.Tensor:
        if self._deq is None:
            self.__dict__["_deq"] = dequantize(self.weight, self.scales, self.biases).float()
        a = QuantizedLinear.accumulate
        return (x.to(a) @ self._deq.to(a).t()).to(torch.bfloat16)


def _qlinear(n: int, k: int, gen: torch.Generator, std: float, dev) -> QuantizedLinear:
    w = torch.randn(n, k, generator=gen, device=dev) * std
    return QuantizedLinear(*quantize(w))


class RMSNorm(nn.Module):
    """Zero-centred RMSNorm: x / rms(x) * (1 + w), in f32."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(dim), requires_grad=False)
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * (1.0 + self.weight.float())).to(torch.bfloat16)


# ---------------------------------------------------------------------------------------------
# caches
# ---------------------------------------------------------------------------------------------
class AttnCache:
    """KV cache of one attention layer: preallocated tensors, a length; trim is a length update."""

    def __init__(self, cfg: ModelConfig, max_len: int, dev):
        self.k = torch.zeros(max_len, cfg.n_kv_heads, cfg.head_dim, dtype=torch.bfloat16, device=dev)
        self.v = torch.zeros_like(self.k)
        self.length = 0

    def trim(self, n: int) -> int:
        n = min(n, self.length)
        self.length -= n
        return n


class GDNCache:
    """Conv window, recurrent state and (while a verify is recorded) checkpoints of one GDN layer."""

    def __init__(self, cfg: ModelConfig, max_verify: int, dev):
        W = cfg.conv_kernel - 1
        self.conv = torch.zeros(W, cfg.conv_dim, dtype=torch.bfloat16, device=dev)
        self.state = torch.zeros(cfg.gdn_v_heads, cfg.gdn_dim, cfg.gdn_dim, dtype=torch.float32, device=dev)
        # the state after every verified token (a chain uses the first T - 1, a tree all T)
        self.ckpt = torch.zeros(max_verify, cfg.gdn_v_heads, cfg.gdn_dim, cfg.gdn_dim,
                                dtype=torch.float32, device=dev)
        self.conv_full = torch.zeros(W + max_verify, cfg.conv_dim, dtype=torch.bfloat16, device=dev)
        self.max_verify = max_verify
        self.recording = False
        self.fed = 0


class Cache:
    def __init__(self, model: "HybridModel", max_len: int = 4096, max_verify: int = 17):
        cfg, dev = model.cfg, model.device
        self.layers = [AttnCache(cfg, max_len, dev) if cfg.is_attention(i) else GDNCache(cfg, max_verify, dev)
                       for i in range(cfg.layers)]

    @property
    def offset(self) -> int:
        for c in self.layers:
            if isinstance(c, AttnCache):
                return c.length
        return 0

    def reset(self) -> None:
        """Empty the cache in place (same buffers: captured graphs that use it stay valid)."""
        for c in self.layers:
            if isinstance(c, AttnCache):
                c.length = 0
            else:
                c.conv.zero_()
                c.state.zero_()
                c.recording = False
                c.fed = 0


# ---------------------------------------------------------------------------------------------
# token trees (a speculative draft tree verified in one forward)
# ---------------------------------------------------------------------------------------------
def tree_paths(parent) -> list[list[int]]:
    """parent[t] of every node (parent[0] = -1, parent[t] < t) -> each node's path from the root
    (root first, the node last).  A chain is parent = [-1, 0, 1, ...]."""
    parent = [int(v) for v in parent]
    if not parent or parent[0] != -1 or any(not 0 <= parent[t] < t for t in range(1, len(parent))):
        raise ValueError("a token tree needs parent[0] = -1 and 0 <= parent[t] < t")
    paths = [[0]]
    for t in range(1, len(parent)):
        paths.append(paths[parent[t]] + [t])
    return paths


# ---------------------------------------------------------------------------------------------
# layers
# ---------------------------------------------------------------------------------------------
# Backends for the module path's attention: the memory-efficient kernel takes the explicit
# bottom-right causal mask; the cuDNN backend is left out because it builds a new execution plan
# for every new key length (tens of ms each time a decode loop's cache grows).
_SDPA_BACKENDS = [SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]


def _rope(x: torch.Tensor, pos: torch.Tensor, rot: int, theta: float) -> torch.Tensor:
    """Partial rotary embedding (rotate-half) on the first `rot` dims; x [T, H, D] f32."""
    half = rot // 2
    inv = theta ** (-torch.arange(0, half, device=x.device, dtype=torch.float32) / half)
    ang = pos.float()[:, None] * inv[None]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    x1, x2, rest = x[..., :half], x[..., half:rot], x[..., rot:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin, rest], dim=-1)


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig, gen, dev):
        super().__init__()
        H, D, std = cfg.hidden, cfg.head_dim, cfg.weight_std
        self.cfg = cfg
        self.q_proj = _qlinear(2 * cfg.n_heads * D, H, gen, std, dev)  # query and gate
        self.k_proj = _qlinear(cfg.n_kv_heads * D, H, gen, std, dev)
        self.v_proj = _qlinear(cfg.n_kv_heads * D, H, gen, std, dev)
        self.o_proj = _qlinear(H, cfg.n_heads * D, gen, std, dev)
        self.q_norm = RMSNorm(D, cfg.rms_eps)
        self.k_norm = RMSNorm(D, cfg.rms_eps)

    def forward(self, x: torch.Tensor, cache: AttnCache, tree=None) -> torch.Tensor:
        return self.o_proj(self.attend(self.q_proj(x), self.k_proj(x), self.v_proj(x), cache, tree))

    def attend(self, qg: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cache: AttnCache, tree=None) -> torch.Tensor:
        """Everything between the projections and o_proj: q/k norm, partial RoPE, KV append,
        causal GQA attention over the cache, output gate.  Returns o bf16 [T, n_heads * D].
        tree (parents of the T tokens, see tree_paths): token t sits at position L0 + depth(t)
        and sees the cache and its ancestors; its key / value go to slot L0 + t."""
        cfg = self.cfg
        T, D, nh, nkv = qg.shape[0], cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
        qg = qg.reshape(T, nh, 2 * D)
        q, gate = qg[..., :D], qg[..., D:]
        k = k.reshape(T, nkv, D)
        v = v.reshape(T, nkv, D)
        L0 = cache.length
        if tree is None:
            pos = torch.arange(L0, L0 + T, device=qg.device)
        else:
            paths = tree_paths(tree)
            pos = torch.tensor([L0 + len(pt) - 1 for pt in paths], device=qg.device)
        q = _rope(self.q_norm(q).float(), pos, cfg.rotary_dim, cfg.rope_theta)
        k = _rope(self.k_norm(k).float(), pos, cfg.rotary_dim, cfg.rope_theta)
        cache.k[L0:L0 + T] = k.to(torch.bfloat16)
        cache.v[L0:L0 + T] = v
        cache.length = L0 + T
        if tree is None:  # queries at positions L0 .. L0+T-1 after L0 cached keys: bottom-right causal
            causal = pos[:, None] >= torch.arange(L0 + T, device=qg.device)[None, :]
        else:
            causal = torch.zeros(T, L0 + T, dtype=torch.bool, device=qg.device)
            causal[:, :L0] = True
            for t, pt in enumerate(paths):
                causal[t, [L0 + j for j in pt]] = True
        with sdpa_kernel(_SDPA_BACKENDS):
            o = F.scaled_dot_product_attention(
                q.to(torch.bfloat16).transpose(0, 1)[None], cache.k[:L0 + T].transpose(0, 1)[None],
                cache.v[:L0 + T].transpose(0, 1)[None], attn_mask=causal, enable_gqa=True)[0].transpose(0, 1)
        o = o.float() * torch.sigmoid(gate.float())
        return o.reshape(T, nh * D).to(torch.bfloat16)


class GatedDeltaNet(nn.Module):
    # True: the recurrence runs in torch on CUDA too, so a module forward uses no kernel of this
    # library besides the patched projections (an independent reference for the fused step)
    torch_recurrence = False

    def __init__(self, cfg: ModelConfig, gen, dev):
        super().__init__()
        H, std = cfg.hidden, cfg.weight_std
        self.cfg = cfg
        self.in_proj_qkv = _qlinear(cfg.conv_dim, H, gen, std, dev)
        self.in_proj_z = _qlinear(cfg.gdn_value_dim, H, gen, std, dev)
        self.in_proj_b = _qlinear(cfg.gdn_v_heads, H, gen, std, dev)
        self.in_proj_a = _qlinear(cfg.gdn_v_heads, H, gen, std, dev)
        self.conv_weight = nn.Parameter(torch.randn(cfg.conv_dim, cfg.conv_kernel, generator=gen, device=dev) * 0.3,
                                        requires_grad=False)
        self.A_log = nn.Parameter(torch.log(torch.rand(cfg.gdn_v_heads, generator=gen, device=dev) * 15 + 1),
                                  requires_grad=False)
        self.dt_bias = nn.Parameter(torch.randn(cfg.gdn_v_heads, generator=gen, device=dev) * 0.1, requires_grad=False)
        self.norm = RMSNorm(cfg.gdn_dim, cfg.rms_eps)
        self.out_proj = _qlinear(H, cfg.gdn_value_dim, gen, std, dev)

    def forward(self, x: torch.Tensor, cache: GDNCache, tree=None) -> torch.Tensor:
        return self.out_proj(self.mix(self.in_proj_qkv(x), self.in_proj_z(x), self.in_proj_b(x),
                                      self.in_proj_a(x), cache, tree))

    def mix(self, qkv, z, b, a, cache: GDNCache, tree=None) -> torch.Tensor:
        """Everything between the input projections and out_proj (conv, gates, recurrence, gated
        norm).  Returns o bf16 [T, value_dim].  tree (parents, see tree_paths; needs a recording
        cache): each token's conv window and recurrence follow its ancestor path, the state after
        every token goes to the checkpoints, and the live state and window are left for the
        rollback to select."""
        cfg = self.cfg
        T, W, dk = qkv.shape[0], cfg.conv_kernel - 1, cfg.gdn_dim
        z = z.reshape(T, cfg.gdn_v_heads, dk)
        b = b.float()
        a = a.float()
        full = torch.cat([cache.conv, qkv], dim=0)                     # [W + T, C]
        if tree is not None and not cache.recording:
            raise ValueError("a tree verify needs a recording cache (HybridRollback.record)")
        if cache.recording:
            cache.conv_full[:W + T] = full
            cache.fed = T
        if tree is None:
            cache.conv.copy_(full[T:])
            # depthwise causal conv: out[t] = sum_j w[:, j] * full[t + j], then SiLU
            win = full.float().unfold(0, cfg.conv_kernel, 1)            # [T, C, kernel]
        else:
            rows = torch.tensor([tree_rows(tree, t, W) for t in range(T)], device=qkv.device)
            win = full.float()[rows].permute(0, 2, 1)                     # [T, C, kernel]
        conv = F.silu((win * self.conv_weight.float()[None]).sum(-1))
        q, k, v = torch.split(conv, [cfg.gdn_key_dim, cfg.gdn_key_dim, cfg.gdn_value_dim], dim=-1)
        q = F.normalize(q.view(T, cfg.gdn_k_heads, dk), dim=-1) / math.sqrt(dk)
        k = F.normalize(k.view(T, cfg.gdn_k_heads, dk), dim=-1)
        v = v.view(T, cfg.gdn_v_heads, dk)
        g = torch.exp(-torch.exp(self.A_log.float()) * F.softplus(a + self.dt_bias.float()))
        beta = torch.sigmoid(b)
        qb, kb, vb = (t.to(torch.bfloat16).contiguous() for t in (q, k, v))
        if tree is not None:  # (the module path's tree recurrence runs in torch)
            y = _recurrent_torch(qb, kb, vb, g, beta, cache, tree)
        elif qkv.is_cuda and not GatedDeltaNet.torch_recurrence:  # CPU runs (tests) use torch
            from .gdn import recurrent

            y = recurrent(qb, kb, vb, g.contiguous(), beta.contiguous(), cache.state,
                          cache.ckpt if cache.recording and T > 1 else None)
        else:
            y = _recurrent_torch(qb, kb, vb, g, beta, cache)
        o = self.norm(y).float() * F.silu(z.float())
        return o.reshape(T, cfg.gdn_value_dim).to(torch.bfloat16)


def tree_rows(tree, t: int, W: int) -> list[int]:
    """Rows of [conv window (W rows); the T inputs] that form input t's causal conv window along
    its ancestor path (the cached window above the root), oldest first, t's own row last."""
    path = tree_paths(tree)[t]
    seq = list(range(W)) + [W + j for j in path]
    return seq[-(W + 1):]


def _recurrent_torch(q, k, v, g, beta, cache: GDNCache, tree=None) -> torch.Tensor:
    """The same gated delta rule in torch (CPU runs and cross-checks).  tree: each token starts
    from its parent's state; the state after every token is checkpointed, the live state kept."""
    rep = v.shape[1] // q.shape[1]
    parent = [int(p) for p in tree] if tree is not None else None
    S = cache.state if tree is None else cache.state.clone()
    ys = []
    for t in range(q.shape[0]):
        if parent is not None and t > 0 and parent[t] != t - 1:
            S = cache.ckpt[parent[t]].clone()
        kt = k[t].float().repeat_interleave(rep, 0)
        qt = q[t].float().repeat_interleave(rep, 0)
        S.mul_(g[t][:, None, None])
        sk = torch.einsum("hvk,hk->hv", S, kt)
        S.add_(torch.einsum("hv,hk->hvk", beta[t][:, None] * (v[t].float() - sk), kt))
        ys.append(torch.einsum("hvk,hk->hv", S, qt))
        if cache.recording and (tree is not None or t + 1 < q.shape[0]):
            cache.ckpt[t].copy_(S)
    return torch.stack(ys).to(torch.bfloat16)


class MLP(nn.Module):
    def __init__(self, cfg: ModelConfig, gen, dev):
        super().__init__()
        H, I, std = cfg.hidden, cfg.intermediate, cfg.weight_std
        self.gate_proj = _qlinear(I, H, gen, std, dev)
        self.up_proj = _qlinear(I, H, gen, std, dev)
        self.down_proj = _qlinear(H, I, gen, std, dev)

    def forward(self, x):
        return self.down_proj((F.silu(self.gate_proj(x).float()) * self.up_proj(x).float()).to(torch.bfloat16))


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, i: int, gen, dev):
        super().__init__()
        self.is_linear = not cfg.is_attention(i)
        if self.is_linear:
            self.linear_attn = GatedDeltaNet(cfg, gen, dev)
        else:
            self.self_attn = Attention(cfg, gen, dev)
        self.mlp = MLP(cfg, gen, dev)
        self.input_layernorm = RMSNorm(cfg.hidden, cfg.rms_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden, cfg.rms_eps)

    def forward(self, x, cache, tree=None):
        mixer = self.linear_attn if self.is_linear else self.self_attn
        h = (x.float() + mixer(self.input_layernorm(x), cache, tree).float()).to(torch.bfloat16)
        return (h.float() + self.mlp(self.post_attention_layernorm(h)).float()).to(torch.bfloat16)


class HybridModel(nn.Module):
    """forward(ids [T] int64, cache) -> (final normed hidden [T, H] bf16, logits [T, V] bf16)."""

    def __init__(self, cfg: ModelConfig = SMALL, seed: int = 0, device="cuda", init_device=None):
        """init_device: where the seeded weights are drawn and quantized (default `device`).  The
        CPU generator gives the same weights on every machine, so a model drawn on "cpu" and moved
        to the GPU matches fixtures made from the same seed on a CPU-only host."""
        super().__init__()
        self.cfg = cfg
        self.device = torch.device(device)
        idev = torch.device(init_device) if init_device is not None else self.device
        gen = torch.Generator(device=idev).manual_seed(seed)
        ew = torch.randn(cfg.vocab, cfg.hidden, generator=gen, device=idev) * cfg.weight_std
        self.embed_tokens = QuantizedEmbedding(*quantize(ew))
        del ew
        self.layers = nn.ModuleList([DecoderLayer(cfg, i, gen, idev) for i in range(cfg.layers)])
        self.norm = RMSNorm(cfg.hidden, cfg.rms_eps)
        self.to(self.device)

    def make_cache(self, max_len: int = 4096, max_verify: int = 17) -> Cache:
        return Cache(self, max_len, max_verify)

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, cache: Cache, tree=None):
        """tree: parents of the input tokens (a draft tree, see tree_paths), or None (a chain)."""
        x = self.embed_tokens(ids)
        for layer, c in zip(self.layers, cache.layers):
            x = layer(x, c, tree)
        h = self.norm(x)
        return h, self.embed_tokens.as_linear(h)


__all__ = ["ModelConfig", "config3", "SMALL", "HybridModel", "QuantizedLinear", "QuantizedEmbedding", "tree_paths",
           "tree_rows",
           "Cache", "AttnCache", "GDNCache", "RMSNorm", "DecoderLayer", "Attention", "GatedDeltaNet", "MLP"]
