"""Multi-token-prediction draft head (skinny_mlx/mtp.py:53-84 on B200), random-initialised.

h_next = norm(layer(fc([norm_e(embed(tok_{t+1})), norm_h(h_t)])))   (mtp.py:64-67)

The reference range-fetches the head's weights from the Qwen3.5 checkpoint; there is no network
or checkpoint here, so the head is built from seeded random weights with the same structure: two
zero-centred RMSNorms, fc 2H -> H, one full-attention decoder layer with its MLP, a final norm,
all projections 4-bit g64.  It runs on the same qmm as the trunk once patched.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .model import AttnCache, DecoderLayer, HybridModel, RMSNorm, _qlinear


class MTPHead(nn.Module):
    def __init__(self, model: HybridModel, seed: int = 1):
        super().__init__()
        cfg = model.cfg
        gen = torch.Generator(device=model.device).manual_seed(seed)
        H = cfg.hidden
        self.cfg = cfg
        self.device = model.device
        self.pre_fc_norm_embedding = RMSNorm(H, cfg.rms_eps).to(model.device)
        self.pre_fc_norm_hidden = RMSNorm(H, cfg.rms_eps).to(model.device)
        self.fc = _qlinear(H, 2 * H, gen, cfg.weight_std, model.device)
        self.layer = DecoderLayer(cfg, cfg.attn_every - 1, gen, model.device)  # full attention
        assert not self.layer.is_linear
        self.norm = RMSNorm(H, cfg.rms_eps)
        self.to(model.device)

    @torch.no_grad()
    def forward(self, emb: torch.Tensor, hidden: torch.Tensor, cache: AttnCache) -> torch.Tensor:
        x = self.fc(torch.cat([self.pre_fc_norm_embedding(emb), self.pre_fc_norm_hidden(hidden)], -1))
        return self.norm(self.layer(x, cache))

    def make_cache(self, max_len: int = 4096) -> AttnCache:
        return AttnCache(self.cfg, max_len, self.device)


__all__ = ["MTPHead"]
