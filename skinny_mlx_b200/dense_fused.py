"""One rank's verify step of the column-parallel dense model on the fused
kernels of the hybrid step (`skinny_mlx_b200.fused`), with the exchanges the sharding needs.

Per layer, rank g of G:

    prep     residual add (+ the gathered down output of the previous layer, read in its
             [G, M, H/G] all-gather layout) + input RMSNorm -> digits of the full hidden
    qmm      fused q | k | v rows of the rank's heads
    attn     q/k norm, RoPE (all 128 dims), KV append, GQA attention -> digits of the rank's
             heads' output: 2 nq 64-column groups, a contiguous slice of o_proj's input
    gather   all-gather of those digit blocks -> o_proj's full input
    qmm      o_proj rows [g H/G, (g+1) H/G)
    gather   all-gather of the [M, H/G] outputs
    prep     residual add (gathered layout) + post-attention RMSNorm -> digits
    qmm      gate | up rows of the rank's slice of the intermediate dimension
    prep     SwiGLU -> digits of the rank's I/G columns (a contiguous slice of down's input)
    gather   all-gather of those digit blocks -> down's full input
    qmm      down rows [g H/G, (g+1) H/G)
    gather   all-gather of the [M, H/G] outputs (added by the next layer's prep)

Every exchange is one NCCL all_gather_into_tensor on the job's process group (NVLink through
NVSwitch on a B200 node); nothing is transposed or copied around it: digit blocks concatenate in
rank order into the next matmul's input, and output shards are read in place by the next prep.
With G = 1 there are no gathers.  The logits come back as [G, M, V/G] (rank-major shards).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .dense import DenseModel
from .qmm import dequantize, get_workspace


def _p(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


class DenseFusedStep:
    def __init__(self, model: DenseModel):
        from .patch import SkinnyQuantizedLinear

        self.model, self.cfg, self.G = model, model.cfg, model.world
        self.group = model.ex.group
        cfg = self.cfg
        assert cfg.head_dim == 128
        self.layers = []
        for layer in model.layers:
            for lin in (layer.qkv_proj, layer.o_proj, layer.gate_up_proj, layer.down_proj):
                if not isinstance(lin, SkinnyQuantizedLinear):
                    raise ValueError("DenseFusedStep needs a patched model (skinny_mlx_b200.patch.patch_model)")
            self.layers.append({
                "qkv": layer.qkv_proj.rweight, "o": layer.o_proj.rweight, "gu": layer.gate_up_proj.rweight,
                "down": layer.down_proj.rweight, "in_norm": layer.input_layernorm.weight.float().contiguous(),
                "post_norm": layer.post_attention_layernorm.weight.float().contiguous(),
                "qn": layer.q_norm.weight.float().contiguous(), "kn": layer.k_norm.weight.float().contiguous()})
        self.nq, self.nkv = model.layers[0].nq, model.layers[0].nkv
        self.head = model.lm_head.rweight
        self.final_norm = model.norm.weight.float().contiguous()
        dev = model.device
        self.inv = (cfg.rope_theta ** (-torch.arange(0, 64, device=dev, dtype=torch.float32) / 64)).contiguous()
        self._bufs: dict[int, dict] = {}
        self._attn_ws: dict[int, torch.Tensor] = {}

    @property
    def device(self):
        return self.model.device

    def make_cache(self, *a, **k):
        return self.model.make_cache(*a, **k)

    def _buffers(self, m: int) -> dict:
        b = self._bufs.get(m)
        if b is None:
            cfg, G, dev = self.cfg, self.G, self.model.device
            L = _lib.lib()
            xq = lambda k: torch.zeros(int(L.skinny_xq_bytes(m, k)), dtype=torch.uint8, device=dev)
            bf = lambda *shape: torch.zeros(*shape, dtype=torch.bfloat16, device=dev)
            H, I, D = cfg.hidden, cfg.intermediate, cfg.head_dim
            b = {"h": [bf(m, H), bf(m, H)], "a": bf(m, H), "xq_h": xq(H),
                 "proj": bf(m, (self.nq + 2 * self.nkv) * D),
                 "xq_o": xq(cfg.n_heads * D), "o_all": bf(G, m, H // G),
                 "gu": bf(m, 2 * I // G), "xq_i": xq(I), "dn_all": bf(G, m, H // G),
                 "logits": bf(G, m, self.head.N)}
            if G > 1:  # the rank's own slices, gathered into the full buffers above
                b["xq_o_loc"] = xq(self.nq * D)
                b["xq_i_loc"] = xq(I // G)
                b["o_loc"] = bf(m, H // G)
                b["dn_loc"] = bf(m, H // G)
                b["logits_loc"] = bf(m, self.head.N)
            else:
                b["xq_o_loc"], b["xq_i_loc"] = b["xq_o"], b["xq_i"]
                b["o_loc"], b["dn_loc"], b["logits_loc"] = b["o_all"][0], b["dn_all"][0], b["logits"][0]
            self._bufs[m] = b
        return b

    def _gather(self, dst, src):
        if self.G > 1:
            dist.all_gather_into_tensor(dst, src, group=self.group)

    def _qmm(self, xq, w, out, m, stream):
        ws = get_workspace(out.device, int(_lib.lib().skinny_qmm_workspace_bytes(w.N, w.K)))
        _lib.call("skinny_qmm_w4g64_prepared", _p(xq), _p(w.w_tc), _p(out), out.stride(-2), m, w.N, w.K,
                  _p(ws), ws.numel(), stream)

    def _prep0(self, x, d_all, h_out, w, m, xq, stream, a_out=None):
        """Residual add of a gathered [G, m, H/G] output (or none) and RMSNorm -> digits."""
        H = self.cfg.hidden
        seg = H // self.G
        _lib.call("skinny_prep", 0, _p(x), H, _p(d_all), seg if d_all is not None else 0,
                  seg if d_all is not None else 0, m * seg if d_all is not None else 0,
                  _p(h_out if d_all is not None else None), H if d_all is not None else 0, _p(w), self.cfg.rms_eps,
                  m, H, _p(xq), _p(a_out), stream)

    @torch.no_grad()
    def __call__(self, ids: torch.Tensor, caches) -> torch.Tensor:
        """Logits [G, M, V/G] bf16 (rank-major shards of the vocabulary; a reused buffer)."""
        cfg, m = self.cfg, ids.shape[0]
        assert 1 <= m <= 16
        b = self._buffers(m)
        dev = self.model.device
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        w, s, bb = self.model.embed
        hs, cur = b["h"], 0
        hs[0].copy_(dequantize(w[ids], s[ids], bb[ids]).to(torch.bfloat16))
        d_all = None
        D = cfg.head_dim
        for ent, c in zip(self.layers, caches):
            nxt = 1 - cur if d_all is not None else cur
            self._prep0(hs[cur], d_all, hs[nxt], ent["in_norm"], m, b["xq_h"], stream)
            cur = nxt
            self._qmm(b["xq_h"], ent["qkv"], b["proj"], m, stream)
            max_len = c.k.shape[0]
            ws = self._attn_ws.get(max_len)
            if ws is None:
                n = int(_lib.lib().skinny_attn_workspace_bytes(16, self.nq, self.nkv, max_len))
                ws = self._attn_ws[max_len] = torch.zeros(n, dtype=torch.uint8, device=dev)
            _lib.call("skinny_attn_fused", _p(b["proj"]), b["proj"].stride(0), _p(ent["qn"]), _p(ent["kn"]),
                      _p(self.inv), D, 0, cfg.rms_eps, _p(c.k), _p(c.v), c.length, None, m, self.nq, self.nkv,
                      max_len, _p(ws), ws.numel(), _p(b["xq_o_loc"]), None, stream)
            c.length += m
            self._gather(b["xq_o"], b["xq_o_loc"])
            self._qmm(b["xq_o"], ent["o"], b["o_loc"], m, stream)
            self._gather(b["o_all"], b["o_loc"])
            self._prep0(hs[cur], b["o_all"], hs[1 - cur], ent["post_norm"], m, b["xq_h"], stream)
            cur = 1 - cur
            self._qmm(b["xq_h"], ent["gu"], b["gu"], m, stream)
            _lib.call("skinny_prep", 1, _p(b["gu"]), b["gu"].stride(0), None, 0, 0, 0, None, 0, None, 0.0, m,
                      cfg.intermediate // self.G, _p(b["xq_i_loc"]), None, stream)
            self._gather(b["xq_i"], b["xq_i_loc"])
            self._qmm(b["xq_i"], ent["down"], b["dn_loc"], m, stream)
            self._gather(b["dn_all"], b["dn_loc"])
            d_all = b["dn_all"]
        self._prep0(hs[cur], d_all, hs[1 - cur], self.final_norm, m, b["xq_h"], stream, a_out=b["a"])
        self._qmm(b["xq_h"], self.head, b["logits_loc"], m, stream)
        self._gather(b["logits"], b["logits_loc"])
        return b["logits"]


__all__ = ["DenseFusedStep"]
