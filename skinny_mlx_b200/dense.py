"""a dense 4-bit g64 decoder, column-parallel over G GPUs.

64 layers, hidden 5120, 40 query / 8 KV heads x 128, SwiGLU 25600, vocab 151936 (random
weights).  Every projection is column-parallel: rank g holds rows [g N/G, (g+1) N/G) of each
packed matrix, so it streams 1/G of the weights, and an all-gather of the [M, N/G] outputs
rebuilds the full activation where the next step needs it:

* fused QKV: rank g holds its own heads (q heads 5g'..., their KV heads), so decode attention
  runs locally on the local KV shard; the attention output (M x 5120) is gathered;
* o_proj: gathered (M x 5120);  gate/up: matching slices, SwiGLU local, gathered (M x 25600);
* down: gathered (M x 5120);  LM head: gathered (M x 151936).

The exchange is torch.distributed all_gather_into_tensor (NCCL over NVLink on GPUs, gloo on CPU
for tests); nothing else crosses devices.  Weights are generated from per-block seeds (128-row
blocks for the layers, 16-row blocks for the head) so that every sharding reproduces exactly the
same model.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F
from torch.nn.attention import sdpa_kernel

from .configs import DenseConfig
from .model import _SDPA_BACKENDS, AttnCache, QuantizedLinear, RMSNorm, _rope
from .qmm import dequantize, quantize


def _blocks(n: int, k: int, rows: range, block: int, seed: int, std: float, dev) -> torch.Tensor:
    """Rows `rows` (a multiple of `block` at both ends) of an N x K matrix whose rows are generated
    block by block from seed (seed, block index)."""
    out = torch.empty(len(rows), k, device=dev)
    gen = torch.Generator(device=dev)
    for i, b0 in enumerate(range(rows.start, rows.stop, block)):
        gen.manual_seed(seed * 1000003 + b0 // block)
        out[i * block:(i + 1) * block] = torch.randn(block, k, generator=gen, device=dev) * std
    return out


class _Exchange:
    """all-gather of column shards [M, N/G] -> [M, N] (identity for G = 1)."""

    def __init__(self, world: int, group=None):
        self.world, self.group = world, group

    def gather(self, y: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return y
        m, n = y.shape
        buf = torch.empty(self.world * m, n, dtype=y.dtype, device=y.device)
        dist.all_gather_into_tensor(buf, y.contiguous(), group=self.group)
        return buf.view(self.world, m, n).transpose(0, 1).reshape(m, self.world * n)


class DenseLayer(nn.Module):
    def __init__(self, cfg: DenseConfig, li: int, rank: int, world: int, seed: int, dev):
        super().__init__()
        H, D, std = cfg.hidden, cfg.head_dim, cfg.weight_std
        nq, nkv = cfg.n_heads // world, cfg.n_kv_heads // world
        self.cfg, self.nq, self.nkv = cfg, nq, nkv
        s = seed + 97 * li
        q_rows = range(rank * nq * D, (rank + 1) * nq * D)
        kv_rows = range(rank * nkv * D, (rank + 1) * nkv * D)
        qkv = torch.cat([_blocks(cfg.n_heads * D, H, q_rows, 128, s + 1, std, dev),
                         _blocks(cfg.n_kv_heads * D, H, kv_rows, 128, s + 2, std, dev),
                         _blocks(cfg.n_kv_heads * D, H, kv_rows, 128, s + 3, std, dev)])
        self.qkv_proj = QuantizedLinear(*quantize(qkv))
        del qkv
        h_rows = range(rank * H // world, (rank + 1) * H // world)
        self.o_proj = QuantizedLinear(*quantize(_blocks(H, cfg.n_heads * D, h_rows, 128, s + 4, std, dev)))
        i_rows = range(rank * cfg.intermediate // world, (rank + 1) * cfg.intermediate // world)
        gu = torch.cat([_blocks(cfg.intermediate, H, i_rows, 128, s + 5, std, dev),
                        _blocks(cfg.intermediate, H, i_rows, 128, s + 6, std, dev)])
        self.gate_up_proj = QuantizedLinear(*quantize(gu))
        del gu
        self.down_proj = QuantizedLinear(*quantize(_blocks(H, cfg.intermediate, h_rows, 128, s + 7, std, dev)))
        self.q_norm = RMSNorm(D, cfg.rms_eps)
        self.k_norm = RMSNorm(D, cfg.rms_eps)
        self.input_layernorm = RMSNorm(H, cfg.rms_eps)
        self.post_attention_layernorm = RMSNorm(H, cfg.rms_eps)

    def forward(self, x: torch.Tensor, cache: AttnCache, ex: _Exchange) -> torch.Tensor:
        cfg, D, nq, nkv = self.cfg, self.cfg.head_dim, self.nq, self.nkv
        T = x.shape[0]
        qkv = self.qkv_proj(self.input_layernorm(x))
        q = qkv[:, :nq * D].reshape(T, nq, D)
        k = qkv[:, nq * D:(nq + nkv) * D].reshape(T, nkv, D)
        v = qkv[:, (nq + nkv) * D:].reshape(T, nkv, D)
        pos = torch.arange(cache.length, cache.length + T, device=x.device)
        q = _rope(self.q_norm(q).float(), pos, D, cfg.rope_theta).to(torch.bfloat16)
        k = _rope(self.k_norm(k).float(), pos, D, cfg.rope_theta).to(torch.bfloat16)
        L0 = cache.length
        cache.k[L0:L0 + T] = k
        cache.v[L0:L0 + T] = v
        cache.length = L0 + T
        causal = pos[:, None] >= torch.arange(L0 + T, device=x.device)[None, :]
        with sdpa_kernel(_SDPA_BACKENDS):
            o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], cache.k[:L0 + T].transpose(0, 1)[None],
                                               cache.v[:L0 + T].transpose(0, 1)[None], attn_mask=causal,
                                               enable_gqa=True)[0].transpose(0, 1).reshape(T, nq * D)
        o = ex.gather(o.to(torch.bfloat16))
        h = (x.float() + ex.gather(self.o_proj(o)).float()).to(torch.bfloat16)
        gu = self.gate_up_proj(self.post_attention_layernorm(h))
        half = gu.shape[1] // 2
        a = ex.gather((F.silu(gu[:, :half].float()) * gu[:, half:].float()).to(torch.bfloat16))
        return (h.float() + ex.gather(self.down_proj(a)).float()).to(torch.bfloat16)


class DenseModel(nn.Module):
    """Rank `rank` of a `world`-way column-parallel dense decoder.  forward(ids, caches) -> logits
    [T, vocab] bf16 (identical on every rank)."""

    def __init__(self, cfg: DenseConfig, rank: int = 0, world: int = 1, seed: int = 0, device="cuda",
                 group=None):
        super().__init__()
        assert cfg.n_kv_heads % world == 0 and cfg.hidden % (128 * world) == 0
        assert cfg.intermediate % (128 * world) == 0 and cfg.vocab % (16 * world) == 0
        self.cfg, self.rank, self.world = cfg, rank, world
        self.device = torch.device(device)
        self.ex = _Exchange(world, group)
        dev = self.device
        ew = _blocks(cfg.vocab, cfg.hidden, range(0, cfg.vocab), 16, seed + 11, cfg.weight_std, dev)
        self.embed = quantize(ew)  # replicated: the lookup needs every row
        v_rows = range(rank * cfg.vocab // world, (rank + 1) * cfg.vocab // world)
        self.lm_head = QuantizedLinear(*(t[v_rows.start:v_rows.stop].contiguous() for t in self.embed))
        del ew
        self.layers = nn.ModuleList([DenseLayer(cfg, i, rank, world, seed, dev) for i in range(cfg.layers)])
        self.norm = RMSNorm(cfg.hidden, cfg.rms_eps)
        self.to(dev)

    def make_cache(self, max_len: int = 4096) -> list[AttnCache]:
        c = self.cfg
        shard = type("C", (), {"n_kv_heads": c.n_kv_heads // self.world, "head_dim": c.head_dim})
        return [AttnCache(shard, max_len, self.device) for _ in range(c.layers)]

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, caches: list[AttnCache]) -> torch.Tensor:
        w, s, b = self.embed
        x = dequantize(w[ids], s[ids], b[ids]).to(torch.bfloat16)
        for layer, c in zip(self.layers, caches):
            x = layer(x, c, self.ex)
        return self.ex.gather(self.lm_head(self.norm(x)))


def small_dense() -> DenseConfig:
    """Test-size dense config (divisible for 1, 2, 4 and 8 ranks)."""
    return DenseConfig(name="dense-small", hidden=1024, layers=2, n_heads=8, n_kv_heads=8, head_dim=128,
                       intermediate=2048, vocab=4096, weight_std=0.05)


__all__ = ["DenseModel", "small_dense"]
