"""Multi-token-prediction draft head (skinny_mlx/mtp.py:53-84 on B200), random-initialised.

h_next = norm(layer(fc([norm_e(embed(tok_{t+1})), norm_h(h_t)])))   (mtp.py:64-67)

The reference range-fetches the head's weights from the Qwen3.5 checkpoint; there is no network
or checkpoint here, so the head is built from seeded random weights with the same structure: two
zero-centred RMSNorms, fc 2H -> H, one full-attention decoder layer with its MLP, a final norm,
all projections 4-bit g64.  It runs on the same qmm as the trunk once patched.
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn as nn

from . import _lib
from .fused import FusedOps, layer_entry
from .model import AttnCache, DecoderLayer, HybridModel, RMSNorm, _qlinear


class MTPHead(nn.Module):
    def __init__(self, model: HybridModel, seed: int = 1, init_device=None):
        """init_device: where the seeded weights are drawn (default the model's device)."""
        super().__init__()
        cfg = model.cfg
        idev = torch.device(init_device) if init_device is not None else model.device
        gen = torch.Generator(device=idev).manual_seed(seed)
        H = cfg.hidden
        self.cfg = cfg
        self.device = model.device
        self.pre_fc_norm_embedding = RMSNorm(H, cfg.rms_eps).to(model.device)
        self.pre_fc_norm_hidden = RMSNorm(H, cfg.rms_eps).to(model.device)
        self.fc = _qlinear(H, 2 * H, gen, cfg.weight_std, idev)
        self.layer = DecoderLayer(cfg, cfg.attn_every - 1, gen, idev)  # full attention
        assert not self.layer.is_linear
        self.norm = RMSNorm(H, cfg.rms_eps)
        self.to(model.device)

    @torch.no_grad()
    def forward(self, emb: torch.Tensor, hidden: torch.Tensor, cache: AttnCache) -> torch.Tensor:
        x = self.fc(torch.cat([self.pre_fc_norm_embedding(emb), self.pre_fc_norm_hidden(hidden)], -1))
        return self.norm(self.layer(x, cache))

    def make_cache(self, max_len: int = 4096) -> AttnCache:
        return AttnCache(self.cfg, max_len, self.device)


class FusedMTPHead(FusedOps):
    """MTPHead.forward for 1..16 tokens on the fused step's kernels: the two input norms write
    the digits of the two halves of fc's input, then fc, the decoder layer (prep, qkv, fused
    attention on the head's cache, o_proj, residual + norm, gate|up, SwiGLU, down) and the final
    residual + norm, 12 launches under programmatic dependent launch instead of the
    module-by-module forward.  More tokens (the prompt) run the module forward.  The result is a
    reused buffer, valid until the next call with the same token count."""

    def __init__(self, head: MTPHead, embed=None):
        """embed: the model's token embedding (QuantizedEmbedding), for step_ids."""
        from .patch import SkinnyQuantizedLinear

        if not isinstance(head.fc, SkinnyQuantizedLinear):
            raise ValueError("FusedMTPHead needs a patched head (skinny_mlx_b200.patch.patch_model(head))")
        self.head, self.cfg, self.embed = head, head.cfg, embed
        self.fc = head.fc.rweight
        self.ent = layer_entry(head.layer, head.cfg)
        self._attn_ws: dict = {}
        self._bufs: dict = {}

    def make_cache(self, max_len: int = 4096) -> AttnCache:
        return self.head.make_cache(max_len)

    def _buffers(self, m: int) -> dict:
        b = self._bufs.get(m)
        if b is None:
            cfg, dev, L = self.cfg, self.head.device, _lib.lib()
            H = cfg.hidden
            xq = lambda k: torch.empty(int(L.skinny_xq_bytes(m, k)), dtype=torch.uint8, device=dev)
            bf = lambda n: torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            b = {"emb": bf(H), "xq_fc": xq(2 * H), "xq_h": xq(H), "xq_o": xq(cfg.n_heads * cfg.head_dim),
                 "xq_i": xq(cfg.intermediate), "x": bf(H), "proj": bf(self.ent["proj"].N), "mix": bf(H),
                 "gu": bf(2 * cfg.intermediate), "down": bf(H), "h2": bf(H), "h3": bf(H), "out": bf(H),
                 "xb": int(L.skinny_xq_bytes(m, 64))}
            self._bufs[m] = b
        return b

    @torch.no_grad()
    def step_ids(self, ids: torch.Tensor, hidden: torch.Tensor, cache: AttnCache, len_dev=None) -> torch.Tensor:
        """The forward from token ids (int64, on the device): the embedding rows are gathered by
        one launch (skinny_embed_w4g64) into a reused buffer."""
        m = ids.numel()
        if m > 16:
            return self(self.embed(ids), hidden, cache)
        b = self._buffers(m)
        e = self.embed
        _lib.call("skinny_embed_w4g64", ctypes.c_void_p(ids.data_ptr()), m, ctypes.c_void_p(e.weight.data_ptr()),
                  ctypes.c_void_p(e.scales.data_ptr()), ctypes.c_void_p(e.biases.data_ptr()), e.weight.shape[0],
                  self.cfg.hidden, ctypes.c_void_p(b["emb"].data_ptr()), b["emb"].stride(0),
                  ctypes.c_void_p(torch.cuda.current_stream(self.head.device).cuda_stream))
        return self(b["emb"], hidden, cache, len_dev)

    @torch.no_grad()
    def __call__(self, emb: torch.Tensor, hidden: torch.Tensor, cache: AttnCache, len_dev=None) -> torch.Tensor:
        """len_dev: a device int32 holding cache.length when the launches run (graph replay); the
        caller then advances the host length itself."""
        m = emb.shape[0]
        if m > 16:
            return self.head(emb, hidden, cache)
        cfg, head, ent = self.cfg, self.head, self.ent
        H = cfg.hidden
        b = self._buffers(m)
        emb, hidden = emb.contiguous(), hidden.contiguous()
        stream = ctypes.c_void_p(torch.cuda.current_stream(head.device).cuda_stream)
        # fc input [norm_e(emb) | norm_h(hidden)]: digit groups [0, H/64) and [H/64, 2H/64)
        self._prep(0, emb, m, H, b["xq_fc"], stream, w=head.pre_fc_norm_embedding.weight)
        self._prep(0, hidden, m, H, b["xq_fc"][(H // 64) * b["xb"]:], stream, w=head.pre_fc_norm_hidden.weight)
        self._qmm(b["xq_fc"], self.fc, b["x"], m, stream)
        self._prep(0, b["x"], m, H, b["xq_h"], stream, w=ent["in_norm"])
        self._qmm(b["xq_h"], ent["proj"], b["proj"], m, stream)
        self._attention(ent, b["proj"], cache, m, b["xq_o"], stream, len_dev)
        self._qmm(b["xq_o"], ent["out"], b["mix"], m, stream)
        self._prep(0, b["x"], m, H, b["xq_h"], stream, d=b["mix"], h_out=b["h2"], w=ent["post_norm"])
        self._gate_up(ent, b["xq_h"], b["gu"], b["xq_i"], m, stream)
        self._qmm(b["xq_i"], ent["down"], b["down"], m, stream)
        self._prep(0, b["h2"], m, H, b["xq_h"], stream, d=b["down"], h_out=b["h3"], w=head.norm.weight,
                   a_out=b["out"])
        return b["out"]


__all__ = ["MTPHead", "FusedMTPHead"]
